// AdaLN-Zero modulated LayerNorm of 1024-wide rows, one warp per row:
//   y = (x - mean) * rstd * (1 + scale) + shift,  biased variance, eps 1e-6
// (src/flow/ops.cpp:94-104 over ggml_norm; flow_reference.py:174-179).
// Lane l owns columns 4 l + 128 i, i < 8.  Two-pass statistics in registers
// (mean, then the centred variance), every rounding step written out with
// explicit _rn intrinsics, so the standalone kernel (k_adaln) and the pass
// fused into the residual GEMM (gemm2.cuh) produce the same bits.
#pragma once

#include "common.cuh"
#include "kernels.h"

namespace lx {

__device__ __forceinline__ float adaln_warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float4 adaln_load4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 adaln_load4(const bf16* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const float2 fa = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.x));
  const float2 fb = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u.y));
  return make_float4(fa.x, fa.y, fb.x, fb.y);
}

__device__ __forceinline__ void adaln_store4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
__device__ __forceinline__ void adaln_store4(bf16* p, float4 v) {
  uint2 u;
  u.x = pack_bf16x2(v.x, v.y);
  u.y = pack_bf16x2(v.z, v.w);
  *reinterpret_cast<uint2*>(p) = u;
}

__device__ __forceinline__ float adaln_sum4(float4 v) { return __fadd_rn(__fadd_rn(v.x, v.y), __fadd_rn(v.z, v.w)); }

__device__ __forceinline__ float adaln_sq4(float4 v, float mean) {
  const float a = __fsub_rn(v.x, mean), b = __fsub_rn(v.y, mean), c = __fsub_rn(v.z, mean), d = __fsub_rn(v.w, mean);
  return __fadd_rn(__fadd_rn(__fmul_rn(a, a), __fmul_rn(b, b)), __fadd_rn(__fmul_rn(c, c), __fmul_rn(d, d)));
}

__device__ __forceinline__ float adaln_mod(float x, float mean, float rstd, float sc, float sh) {
  return __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(x, mean), rstd), __fadd_rn(1.0f, sc)), sh);
}

// NR rows per warp call, their loads issued together (rows < 0 are skipped).
template <int NR, typename Tin, typename Tout>
__device__ __forceinline__ void adaln_rows_warp(const Tin* __restrict__ x, Tout* __restrict__ y, const int (&rows)[NR],
                                                const float* __restrict__ shift, const float* __restrict__ scale,
                                                int lane) {
  float4 v[NR][8];
#pragma unroll
  for (int r = 0; r < NR; ++r) {
    if (rows[r] < 0) continue;
    const Tin* xr = x + static_cast<size_t>(rows[r]) * DIM;
#pragma unroll
    for (int i = 0; i < 8; ++i) v[r][i] = adaln_load4(xr + 4 * lane + 128 * i);
  }
#pragma unroll
  for (int r = 0; r < NR; ++r) {
    if (rows[r] < 0) continue;
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) s = __fadd_rn(s, adaln_sum4(v[r][i]));
    const float mean = __fmul_rn(adaln_warp_sum(s), 1.0f / DIM);
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) q = __fadd_rn(q, adaln_sq4(v[r][i], mean));
    const float var = __fmul_rn(adaln_warp_sum(q), 1.0f / DIM);
    const float rstd = __frcp_rn(__fsqrt_rn(__fadd_rn(var, 1e-6f)));
    Tout* yr = y + static_cast<size_t>(rows[r]) * DIM;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int c = 4 * lane + 128 * i;
      const float4 sc = __ldg(reinterpret_cast<const float4*>(scale + c));
      const float4 sh = __ldg(reinterpret_cast<const float4*>(shift + c));
      float4 o;
      o.x = adaln_mod(v[r][i].x, mean, rstd, sc.x, sh.x);
      o.y = adaln_mod(v[r][i].y, mean, rstd, sc.y, sh.y);
      o.z = adaln_mod(v[r][i].z, mean, rstd, sc.z, sh.z);
      o.w = adaln_mod(v[r][i].w, mean, rstd, sc.w, sh.w);
      adaln_store4(yr + c, o);
    }
  }
}

}  // namespace lx
