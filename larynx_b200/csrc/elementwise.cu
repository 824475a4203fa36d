// Row / element-wise kernels of the Flow path: AdaLN-Zero modulated
// LayerNorm, the CFG Euler update, layout gathers/scatters, the load-time
// time-embedding / modulation GEMVs, the once-per-utterance frontend, and the
// standalone fused ops timed by the microbench.
#include <cstdlib>

#include "common.cuh"
#include "kernels.h"

namespace lx {

namespace {

// Bring [p, p + bytes) into L2 (16-byte aligned, bytes a multiple of 16).
// Issued before pdl_wait by the standalone ops: L2 is coherent, so lines the
// previous kernel is still writing are read correctly after the wait, and
// inputs it does not write arrive early.
__device__ __forceinline__ void prefetch_l2_bulk(const void* p, uint32_t bytes) {
  if ((reinterpret_cast<uintptr_t>(p) & 15u) != 0 || (bytes & 15u) != 0) return;  // the bulk form's alignment rule
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <typename T>
__device__ __forceinline__ float4 load4(const T* p);
template <>
__device__ __forceinline__ float4 load4<float>(const float* p) {
  return *reinterpret_cast<const float4*>(p);
}
template <>
__device__ __forceinline__ float4 load4<bf16>(const bf16* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  const __nv_bfloat162 a = *reinterpret_cast<const __nv_bfloat162*>(&u.x);
  const __nv_bfloat162 b = *reinterpret_cast<const __nv_bfloat162*>(&u.y);
  const float2 fa = __bfloat1622float2(a);
  const float2 fb = __bfloat1622float2(b);
  return make_float4(fa.x, fa.y, fb.x, fb.y);
}

__device__ __forceinline__ void store4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
__device__ __forceinline__ void store4(bf16* p, float4 v) {
  uint2 u;
  u.x = pack_bf16x2(v.x, v.y);
  u.y = pack_bf16x2(v.z, v.w);
  *reinterpret_cast<uint2*>(p) = u;
}

// One warp per 1024-wide row; lane owns columns 4*lane + 128*i, i < 8.
// Biased variance, eps 1e-6, then (x - mean) * rstd * (1 + scale) + shift.
// The decode's instance (PF = false) takes two-pass statistics in registers
// (mean, then centred variance).  The standalone op instances (PF = true:
// the row is prefetched into L2 before the dependency wait) take both sums
// in one pass over x - K, K = the row's first element (the shifted-data
// variance: var = E[(x-K)^2] - E[x-K]^2, whose cancellation is bounded by
// (mean - K)^2 / var, small for a K drawn from the row), which saves one
// warp reduction on the latency chain of a launch that moves ~12 MB.
// REV visits the rows from the last one down (blocks are scheduled in index
// order, so the first blocks take the rows the previous kernel wrote last).
template <typename Tin, typename Tout, bool PF = false, bool REV = false>
__global__ void __launch_bounds__(512) k_adaln(const Tin* __restrict__ x, Tout* __restrict__ y,
                                                const float* __restrict__ shift, const float* __restrict__ scale,
                                                int R) {
  const int r0 = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int row = REV ? R - 1 - r0 : r0;
  const int lane = threadIdx.x & 31;
  if (PF && r0 < R && lane == 0) prefetch_l2_bulk(x + static_cast<size_t>(row) * DIM, DIM * sizeof(Tin));
  pdl_wait();
  pdl_launch_dependents();  // after the wait: at most one dependent launch ahead
  if (r0 >= R) return;  // r0 < R  <=>  0 <= row < R in either direction
  const Tin* xr = x + static_cast<size_t>(row) * DIM;
  float4 v[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = load4(xr + 4 * lane + 128 * i);
  float s = 0.f;
  if (!PF) {
#pragma unroll
    for (int i = 0; i < 8; ++i) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
  }
  float mean, var;
  if (PF) {
    const float K = __shfl_sync(0xffffffffu, v[0].x, 0);
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float a = v[i].x - K, b = v[i].y - K, c = v[i].z - K, d = v[i].w - K;
      s1 += (a + b) + (c + d);
      s2 += (a * a + b * b) + (c * c + d * d);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      s1 += __shfl_xor_sync(0xffffffffu, s1, o);
      s2 += __shfl_xor_sync(0xffffffffu, s2, o);
    }
    const float m1 = s1 * (1.0f / DIM);
    mean = K + m1;
    var = fmaxf(s2 * (1.0f / DIM) - m1 * m1, 0.f);
  } else {
    mean = warp_sum(s) * (1.0f / DIM);
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float a = v[i].x - mean, b = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
      q += (a * a + b * b) + (c * c + d * d);
    }
    var = warp_sum(q) * (1.0f / DIM);
  }
  const float rstd = 1.0f / sqrtf(var + 1e-6f);
  Tout* yr = y + static_cast<size_t>(row) * DIM;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int c = 4 * lane + 128 * i;
    const float4 sc = __ldg(reinterpret_cast<const float4*>(scale + c));
    const float4 sh = __ldg(reinterpret_cast<const float4*>(shift + c));
    float4 o;
    o.x = (v[i].x - mean) * rstd * (1.0f + sc.x) + sh.x;
    o.y = (v[i].y - mean) * rstd * (1.0f + sc.y) + sh.y;
    o.z = (v[i].z - mean) * rstd * (1.0f + sc.z) + sh.z;
    o.w = (v[i].w - mean) * rstd * (1.0f + sc.w) + sh.w;
    store4(yr + c, o);
  }
}

// CFG Euler step (src/flow/flow.cpp:257-259 order):
//   x += dt * ((1 + cfg) * d_cond - cfg * d_uncond)
__global__ void k_euler(float* __restrict__ xs, const float* __restrict__ dphi, const int2* __restrict__ rows,
                        bf16* __restrict__ xb, int F, float dt, float cfg) {
  pdl_launch_dependents();
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= F * MEL) return;
  const int f = i / MEL, c = i - f * MEL;
  const int2 r = __ldg(rows + f);
  const float dc = dphi[static_cast<size_t>(r.x) * MEL + c];
  const float du = dphi[static_cast<size_t>(r.y) * MEL + c];
  const float a = 1.0f + cfg;
  const float x = xs[i] + dt * (a * dc - cfg * du);
  xs[i] = x;
  const bf16 b = __float2bfloat16_rn(x);
  xb[static_cast<size_t>(r.x) * MEL + c] = b;
  xb[static_cast<size_t>(r.y) * MEL + c] = b;
}

__global__ void k_init_state(float* __restrict__ xs, const float* __restrict__ noise, const int2* __restrict__ rows,
                             const int2* __restrict__ src, bf16* __restrict__ xb, int F) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= F * MEL) return;
  const int f = i / MEL, c = i - f * MEL;
  const int2 sr = __ldg(src + f);
  const float x = noise[static_cast<size_t>(sr.x) + static_cast<size_t>(c) * sr.y];
  xs[i] = x;
  const int2 r = __ldg(rows + f);
  const bf16 b = __float2bfloat16_rn(x);
  xb[static_cast<size_t>(r.x) * MEL + c] = b;
  xb[static_cast<size_t>(r.y) * MEL + c] = b;
}

__global__ void k_gather_cond(bf16* __restrict__ a, const float* __restrict__ cond, const float* __restrict__ mu,
                              const float* __restrict__ spks, const int2* __restrict__ rows,
                              const int2* __restrict__ src, const int* __restrict__ utt, int F) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= F * MEL) return;
  const int f = i / MEL, c = i - f * MEL;
  const int2 sr = __ldg(src + f);
  const size_t off = static_cast<size_t>(sr.x) + static_cast<size_t>(c) * sr.y;
  bf16* ar = a + static_cast<size_t>(__ldg(rows + f).x) * COND_K;
  ar[c] = __float2bfloat16_rn(cond[off]);
  ar[MEL + c] = __float2bfloat16_rn(mu[off]);
  ar[2 * MEL + c] = __float2bfloat16_rn(spks[static_cast<size_t>(__ldg(utt + f)) * MEL + c]);
}

// Zero the staging rows that belong to no sequence (s2p < 0): they are the
// causal left padding of the conv-pos kernels and may hold rows of an earlier
// batch layout.
__global__ void k_zero_gap_rows(bf16* __restrict__ a, bf16* __restrict__ b, const int* __restrict__ s2p, int Rs) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= Rs || __ldg(s2p + row) >= 0) return;
  uint4* ra = reinterpret_cast<uint4*>(a + static_cast<size_t>(row) * DIM);
  uint4* rb = reinterpret_cast<uint4*>(b + static_cast<size_t>(row) * DIM);
  const uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    ra[lane + 32 * i] = z;
    rb[lane + 32 * i] = z;
  }
}

__global__ void k_scatter_mel(float* __restrict__ mel, const float* __restrict__ xs, const int2* __restrict__ src,
                              int F) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= F * MEL) return;
  const int f = i / MEL, c = i - f * MEL;
  const int2 sr = __ldg(src + f);
  mel[static_cast<size_t>(sr.x) + static_cast<size_t>(c) * sr.y] = xs[i];
}

template <typename T>
__global__ void k_gather_rows(float* __restrict__ dst, const T* __restrict__ src, const int* __restrict__ rows, int n,
                              int width) {
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<size_t>(n) * width) return;
  const int r = static_cast<int>(i / width), c = static_cast<int>(i % width);
  const int sr = rows[r];
  dst[i] = sr >= 0 ? static_cast<float>(src[static_cast<size_t>(sr) * width + c]) : 0.f;
}

// out[s][n] = act_out(sum_k act_in(in[s][k]) * W[n][k] + b[n]); warp per n.
template <int S>
__global__ void k_gemv_rows(const float* __restrict__ in, int K, const float* __restrict__ W,
                            const float* __restrict__ b, int N, float* __restrict__ out, int ldo, int act_in,
                            int act_out, int S_used) {
  const int n = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (n >= N) return;
  float acc[S];
#pragma unroll
  for (int s = 0; s < S; ++s) acc[s] = 0.f;
  const float* w = W + static_cast<size_t>(n) * K;
  for (int k = lane; k < K; k += 32) {
    const float wk = w[k];
#pragma unroll
    for (int s = 0; s < S; ++s) {
      if (s < S_used) {
        float xv = in[static_cast<size_t>(s) * K + k];
        if (act_in) xv = silu_f(xv);
        acc[s] = fmaf(xv, wk, acc[s]);
      }
    }
  }
#pragma unroll
  for (int s = 0; s < S; ++s) {
    if (s < S_used) {
      float v = warp_sum(acc[s]);
      if (lane == 0) {
        v += b ? b[n] : 0.f;
        if (act_out) v = silu_f(v);
        out[static_cast<size_t>(s) * ldo + n] = v;
      }
    }
  }
}

// SinusPositionEmbedding(256, scale 1000): emb[j] = sin(1000 t e^{-j ln(1e4)/127}),
// emb[j+128] = cos(.), j < 128 (src/flow/flow_matching.cpp:17-24).
__global__ void k_sinus(const float* __restrict__ t, int S, float* __restrict__ out) {
  const int s = blockIdx.x;
  const int j = threadIdx.x;
  if (s >= S || j >= 128) return;
  const float coeff = expf(-static_cast<float>(j) * (9.210340371976184f / 127.0f));
  const float ang = 1000.0f * t[s] * coeff;
  out[s * 256 + j] = sinf(ang);
  out[s * 256 + 128 + j] = cosf(ang);
}

__global__ void k_to_bf16(const float* __restrict__ src, bf16* __restrict__ dst, size_t n) {
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) dst[i] = __float2bfloat16_rn(src[i]);
}

// ---- frontend (flow.cpp:134-182, prelookahead.cpp:8-20, ops.cpp:106-122) --
__global__ void k_front_spk(const float* __restrict__ e, const float* __restrict__ w, const float* __restrict__ b,
                            float* __restrict__ spk) {
  __shared__ float red[32];
  __shared__ float en[192];
  const int t = threadIdx.x;  // 192 threads
  const float v = t < 192 ? e[t] : 0.f;
  float s = warp_sum(v * v);
  if ((t & 31) == 0) red[t >> 5] = s;
  __syncthreads();
  if (t == 0) {
    float tot = 0.f;
    for (int i = 0; i < 6; ++i) tot += red[i];
    red[0] = fmaxf(sqrtf(tot), 1e-12f);
  }
  __syncthreads();
  if (t < 192) en[t] = v / red[0];
  __syncthreads();
  if (t < MEL) {
    float acc = b[t];
    for (int k = 0; k < 192; ++k) acc = fmaf(w[t * 192 + k], en[k], acc);
    spk[t] = acc;
  }
}

__global__ void k_front_embed(const int* __restrict__ tok, int n, const float* __restrict__ table, int vocab,
                              float* __restrict__ out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n * MEL) return;
  const int t = i / MEL, c = i - t * MEL;
  int id = tok[t];
  id = id < 0 ? 0 : (id >= vocab ? vocab - 1 : id);
  out[i] = table[static_cast<size_t>(id) * MEL + c];
}

// conv1: [80 -> 1024, k=4] over the n_in rows of emb, zero beyond them, then
// LeakyReLU(0.01); n_out outputs (n_out = n_in: the finalize path, right
// padding 3; n_out = n_in - 3: the streaming path, the last 3 rows are context).
// emb [n_in][80] (time-major), w [1024][80][4], h [n_out][1024]
__global__ void k_front_conv1(const float* __restrict__ emb, int n_in, int n_out, const float* __restrict__ w,
                              const float* __restrict__ b, float* __restrict__ h) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n_out * DIM) return;
  const int t = i / DIM, o = i - t * DIM;
  float acc = b[o];
  for (int k = 0; k < 4; ++k) {
    const int ts = t + k;
    if (ts >= n_in) break;
    const float* e = emb + static_cast<size_t>(ts) * MEL;
    const float* wr = w + static_cast<size_t>(o) * MEL * 4 + k;
    for (int c = 0; c < MEL; ++c) acc = fmaf(wr[c * 4], e[c], acc);
  }
  h[i] = acc >= 0.f ? acc : 0.01f * acc;
}

// conv2: [1024 -> 80, k=3] over h padded left by 2, plus the residual emb.
__global__ void k_front_conv2(const float* __restrict__ h, const float* __restrict__ emb, int n,
                              const float* __restrict__ w, const float* __restrict__ b, float* __restrict__ out) {
  const int t = blockIdx.x;
  const int o = blockIdx.y * 8 + threadIdx.y;  // 8 outputs per block, 32 lanes split the reduction
  const int lane = threadIdx.x;
  if (t >= n) return;
  float acc = 0.f;
  for (int k = 0; k < 3; ++k) {
    const int ts = t + k - 2;
    if (ts < 0) continue;
    const float* hr = h + static_cast<size_t>(ts) * DIM;
    const float* wr = w + static_cast<size_t>(o) * DIM * 3 + k;
    for (int c = lane; c < DIM; c += 32) acc = fmaf(wr[c * 3], hr[c], acc);
  }
  acc = warp_sum(acc);
  if (lane == 0) out[t * MEL + o] = acc + b[o] + emb[t * MEL + o];
}

__global__ void k_front_mu_cond(const float* __restrict__ pre, int n_tok, const float* __restrict__ pf, int mel_len1,
                                float* __restrict__ mu, float* __restrict__ cond) {
  const int T = 2 * n_tok;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= T * MEL) return;
  const int c = i / T, t = i - c * T;
  mu[i] = pre[(t >> 1) * MEL + c];
  cond[i] = t < mel_len1 ? pf[t * MEL + c] : 0.f;
}

// ---- standalone fused ops -------------------------------
template <typename Tin>
__global__ void k_gate_res(float* __restrict__ x, const Tin* __restrict__ y, const float* __restrict__ gate,
                           size_t n4) {
  const size_t b0 = static_cast<size_t>(blockIdx.x) * blockDim.x;
  if (threadIdx.x == 0 && b0 + blockDim.x <= n4) {
    prefetch_l2_bulk(x + b0 * 4, blockDim.x * 16);
    prefetch_l2_bulk(y + b0 * 4, blockDim.x * 4 * sizeof(Tin));
  }
  pdl_wait();
  pdl_launch_dependents();  // after the wait: at most one dependent launch ahead
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n4) return;
  const int c = static_cast<int>((i * 4) % DIM);
  float4 xv = reinterpret_cast<float4*>(x)[i];
  const float4 yv = load4(y + i * 4);
  const float4 g = __ldg(reinterpret_cast<const float4*>(gate + c));
  xv.x += g.x * yv.x;
  xv.y += g.y * yv.y;
  xv.z += g.z * yv.z;
  xv.w += g.w * yv.w;
  reinterpret_cast<float4*>(x)[i] = xv;
}

// Partial rotary of one row per warp: lanes 0..15 rotate the pairs of
// channels 0..63 (lane l: pairs 2l, 2l+1), and every lane copies its share of
// the other channels.  Before the dependency wait the row of x and the table
// row of a speculative read of pos go into L2 (pos may still be being written
// by the previous kernel: the speculative value, read at L2 with __ldcg so no
// stale L1 line survives, only picks lines and the table address).  After the
// wait the table row is loaded at that address while pos is read again; a
// different pos reloads it.  The copies are stored first, the rotated chunk
// last.  The table itself is never written by a kernel (it is uploaded once
// by a blocking copy), so reading it early is safe.
template <typename Tin>
__global__ void __launch_bounds__(512) k_rotary(const Tin* __restrict__ x, float* __restrict__ y,
                                                 const int* __restrict__ pos, const float2* __restrict__ rope,
                                                 int R) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  int p_spec = 0;
  if (row < R) {
    const int p = __ldcg(pos + row);
    p_spec = p < 0 ? 0 : (p >= ROPE_MAX ? ROPE_MAX - 1 : p);
    if (lane == 0) {
      prefetch_l2_bulk(x + static_cast<size_t>(row) * DIM, DIM * sizeof(Tin));
      prefetch_l2_bulk(rope + static_cast<size_t>(p_spec) * 32, 32 * sizeof(float2));
    }
  }
  pdl_wait();
  pdl_launch_dependents();  // after the wait: at most one dependent launch ahead
  if (row >= R) return;
  const Tin* xr = x + static_cast<size_t>(row) * DIM;
  float* yr = y + static_cast<size_t>(row) * DIM;
  float4 v[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = load4(xr + 4 * lane + 128 * i);
  float2 t0 = make_float2(1.f, 0.f), t1 = make_float2(1.f, 0.f);
  int p = p_spec;
  if (lane < 16) {
    p = pos[row];
    const float2* cs = rope + static_cast<size_t>(p_spec) * 32 + 2 * lane;
    t0 = __ldg(cs);
    t1 = __ldg(cs + 1);
  }
#pragma unroll
  for (int i = 1; i < 8; ++i) store4(yr + 4 * lane + 128 * i, v[i]);
  if (lane < 16) {
    if (p != p_spec) {
      const float2* cs = rope + static_cast<size_t>(p) * 32 + 2 * lane;
      t0 = __ldg(cs);
      t1 = __ldg(cs + 1);
    }
    const float4 w = v[0];
    v[0] = make_float4(w.x * t0.x - w.y * t0.y, w.y * t0.x + w.x * t0.y, w.z * t1.x - w.w * t1.y,
                       w.w * t1.x + w.z * t1.y);
  }
  store4(yr + 4 * lane, v[0]);
}

// Two float4 per thread (block b covers 512 consecutive float4): one wave of
// ~7 blocks per SM at [2000, 1024], against two waves for one float4 per
// thread (measured: 0.88 / 0.78 vs 0.73 / 0.60 of HBM, fp32 / bf16 in).
constexpr int GELU_PER_THREAD = 2;
template <typename Tin>
__global__ void __launch_bounds__(256) k_gelu(const Tin* __restrict__ x, float* __restrict__ y, size_t n4) {
  const size_t b0 = static_cast<size_t>(blockIdx.x) * blockDim.x * GELU_PER_THREAD;
  if (threadIdx.x == 0) {
    const size_t span = static_cast<size_t>(blockDim.x) * GELU_PER_THREAD;
    const size_t cnt = n4 - b0 < span ? n4 - b0 : span;
    prefetch_l2_bulk(x + b0 * 4, static_cast<uint32_t>(cnt * 4 * sizeof(Tin)));
  }
  pdl_wait();
  pdl_launch_dependents();  // after the wait: at most one dependent launch ahead
  float4 v[GELU_PER_THREAD];
#pragma unroll
  for (int u = 0; u < GELU_PER_THREAD; ++u) {
    const size_t i = b0 + threadIdx.x + static_cast<size_t>(u) * blockDim.x;
    if (i < n4) v[u] = load4(x + i * 4);
  }
#pragma unroll
  for (int u = 0; u < GELU_PER_THREAD; ++u) {
    const size_t i = b0 + threadIdx.x + static_cast<size_t>(u) * blockDim.x;
    if (i < n4) {
      float4 w = v[u];
      w.x = gelu_tanh_fast(w.x);
      w.y = gelu_tanh_fast(w.y);
      w.z = gelu_tanh_fast(w.z);
      w.w = gelu_tanh_fast(w.w);
      reinterpret_cast<float4*>(y)[i] = w;
    }
  }
}

inline unsigned blocks_for(size_t n, unsigned t) { return static_cast<unsigned>((n + t - 1) / t); }

}  // namespace

void adaln_rows(const float* x, bf16* y, const float* shift, const float* scale, int R, cudaStream_t s, bool rev) {
  if (R <= 0) return;
  const dim3 grid((R + rows_per_block(R) - 1) / rows_per_block(R)), block(32 * rows_per_block(R));
  if (rev)
    launch_pdl(k_adaln<float, bf16, false, true>, grid, block, 0, s, x, y, shift, scale, R);
  else
    launch_pdl(k_adaln<float, bf16>, grid, block, 0, s, x, y, shift, scale, R);
}

bool row_order_alternates() {
  static const bool on = [] {
    const char* e = getenv("LX_FLOW_ROW_ORDER");
    return !(e && e[0] == '0');
  }();
  return on;
}
void euler_update(float* xs, const float* dphi, const int2* frame_rows, bf16* xb, int F, float dt, float cfg,
                  cudaStream_t s) {
  if (F > 0) launch_pdl(k_euler, dim3(blocks_for(static_cast<size_t>(F) * MEL, 256)), dim3(256), 0, s, xs, dphi, frame_rows, xb, F, dt, cfg);
}
void init_state(float* xs, const float* noise, const int2* frame_rows, const int2* frame_src, bf16* xb, int F,
                cudaStream_t s) {
  if (F > 0)
    k_init_state<<<blocks_for(static_cast<size_t>(F) * MEL, 256), 256, 0, s>>>(xs, noise, frame_rows, frame_src, xb, F);
}
void gather_cond(bf16* a_cond, const float* cond, const float* mu, const float* spks, const int2* frame_rows,
                 const int2* frame_src, const int* frame_utt, int F, cudaStream_t s) {
  if (F > 0)
    k_gather_cond<<<blocks_for(static_cast<size_t>(F) * MEL, 256), 256, 0, s>>>(a_cond, cond, mu, spks, frame_rows,
                                                                                 frame_src, frame_utt, F);
}
void zero_gap_rows(bf16* a, bf16* b, const int* s2p, int Rs, cudaStream_t s) {
  if (Rs > 0) k_zero_gap_rows<<<(Rs + 7) / 8, 256, 0, s>>>(a, b, s2p, Rs);
}
void scatter_mel(float* mel, const float* xs, const int2* frame_src, int F, cudaStream_t s) {
  if (F > 0) k_scatter_mel<<<blocks_for(static_cast<size_t>(F) * MEL, 256), 256, 0, s>>>(mel, xs, frame_src, F);
}
void gather_rows(float* dst, const float* src, const int* rows, int n, int width, cudaStream_t s) {
  if (n > 0)
    k_gather_rows<float><<<blocks_for(static_cast<size_t>(n) * width, 256), 256, 0, s>>>(dst, src, rows, n, width);
}
void gather_rows_bf16(float* dst, const bf16* src, const int* rows, int n, int width, cudaStream_t s) {
  if (n > 0)
    k_gather_rows<bf16><<<blocks_for(static_cast<size_t>(n) * width, 256), 256, 0, s>>>(dst, src, rows, n, width);
}
void gemv_rows(const float* in, int S, int K, const float* W, const float* b, int N, float* out, int ldo,
               int act_in, int act_out, cudaStream_t s) {
  if (S <= 0 || N <= 0) return;
  if (S <= 1)
    k_gemv_rows<1><<<(N + 7) / 8, 256, 0, s>>>(in, K, W, b, N, out, ldo, act_in, act_out, S);
  else
    k_gemv_rows<16><<<(N + 7) / 8, 256, 0, s>>>(in, K, W, b, N, out, ldo, act_in, act_out, S);
}
void sinus_embed(const float* t, int S, float* out, cudaStream_t s) {
  if (S > 0) k_sinus<<<S, 128, 0, s>>>(t, S, out);
}
void to_bf16(const float* src, bf16* dst, size_t n, cudaStream_t s) {
  if (n > 0) k_to_bf16<<<blocks_for(n, 256), 256, 0, s>>>(src, dst, n);
}

void frontend_spk(const float* emb192, const float* w, const float* b, float* spk80, cudaStream_t s) {
  k_front_spk<<<1, 192, 0, s>>>(emb192, w, b, spk80);
}
void frontend_embed(const int* tok, int n, const float* table, int vocab, float* out, cudaStream_t s) {
  if (n > 0) k_front_embed<<<blocks_for(static_cast<size_t>(n) * MEL, 256), 256, 0, s>>>(tok, n, table, vocab, out);
}
void frontend_conv1(const float* emb, int n_in, int n_out, const float* w, const float* b, float* h, cudaStream_t s) {
  if (n_out > 0)
    k_front_conv1<<<blocks_for(static_cast<size_t>(n_out) * DIM, 256), 256, 0, s>>>(emb, n_in, n_out, w, b, h);
}
void frontend_conv2(const float* h, const float* emb, int n, const float* w, const float* b, float* out,
                    cudaStream_t s) {
  if (n > 0) k_front_conv2<<<dim3(n, MEL / 8), dim3(32, 8), 0, s>>>(h, emb, n, w, b, out);
}
void frontend_mu_cond(const float* pre, int n_tok, const float* prompt_feat, int mel_len1, float* mu, float* cond,
                      cudaStream_t s) {
  const size_t n = static_cast<size_t>(2 * n_tok) * MEL;
  if (n > 0) k_front_mu_cond<<<blocks_for(n, 256), 256, 0, s>>>(pre, n_tok, prompt_feat, mel_len1, mu, cond);
}

void op_adaln_f32(const float* x, float* y, const float* shift, const float* scale, int R, cudaStream_t s) {
  if (R > 0) launch_pdl(k_adaln<float, float, true>, dim3((R + rows_per_block(R, 0) - 1) / rows_per_block(R, 0)), dim3(32 * rows_per_block(R, 0)), 0, s, x, y, shift, scale, R);
}
void op_adaln_bf16(const bf16* x, float* y, const float* shift, const float* scale, int R, cudaStream_t s) {
  if (R > 0) launch_pdl(k_adaln<bf16, float, true>, dim3((R + rows_per_block(R, 0) - 1) / rows_per_block(R, 0)), dim3(32 * rows_per_block(R, 0)), 0, s, x, y, shift, scale, R);
}
void op_gate_res_f32(float* x, const float* y, const float* gate, int R, cudaStream_t s) {
  const size_t n4 = static_cast<size_t>(R) * DIM / 4;
  if (n4) launch_pdl(k_gate_res<float>, dim3(blocks_for(n4, 256)), dim3(256), 0, s, x, y, gate, n4);
}
void op_gate_res_bf16(float* x, const bf16* y, const float* gate, int R, cudaStream_t s) {
  const size_t n4 = static_cast<size_t>(R) * DIM / 4;
  if (n4) launch_pdl(k_gate_res<bf16>, dim3(blocks_for(n4, 256)), dim3(256), 0, s, x, y, gate, n4);
}
void op_rotary_f32(const float* x, float* y, const int* pos, const float2* rope, int R, cudaStream_t s) {
  if (R > 0) launch_pdl(k_rotary<float>, dim3((R + rows_per_block(R, 0) - 1) / rows_per_block(R, 0)), dim3(32 * rows_per_block(R, 0)), 0, s, x, y, pos, rope, R);
}
void op_rotary_bf16(const bf16* x, float* y, const int* pos, const float2* rope, int R, cudaStream_t s) {
  if (R > 0) launch_pdl(k_rotary<bf16>, dim3((R + rows_per_block(R, 0) - 1) / rows_per_block(R, 0)), dim3(32 * rows_per_block(R, 0)), 0, s, x, y, pos, rope, R);
}
void op_gelu_f32(const float* x, float* y, size_t n, cudaStream_t s) {
  if (n >= 4) launch_pdl(k_gelu<float>, dim3(blocks_for(n / 4, 256 * GELU_PER_THREAD)), dim3(256), 0, s, x, y, n / 4);
}
void op_gelu_bf16(const bf16* x, float* y, size_t n, cudaStream_t s) {
  if (n >= 4) launch_pdl(k_gelu<bf16>, dim3(blocks_for(n / 4, 256 * GELU_PER_THREAD)), dim3(256), 0, s, x, y, n / 4);
}

}  // namespace lx
