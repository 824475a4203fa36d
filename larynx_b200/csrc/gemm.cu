// tcgen05 GEMM instantiations with the Flow-specific fused epilogues, the
// causal grouped conv-pos kernel, and tensor-map creation.
#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "gemm.cuh"
#include "gemm2.cuh"
#include "kernels.h"

namespace lx {

// ---------------------------------------------------------------------------
// device / tensor-map plumbing
// ---------------------------------------------------------------------------
int num_sms() {
  static int cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (cache[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

// Programmatic dependent launch.  Measured on the 64-utterance decode it costs
// ~2% of throughput (dependent CTAs park on SMs the running kernel's tail
// could use) and saves ~1 ms of the single-utterance latency, so by default
// the engine turns it on only for small batch plans (pdl_set_auto, per
// thread); LX_FLOW_PDL=1 / 0 forces it on / off everywhere.
namespace {
thread_local bool t_pdl_auto = false;
}

void pdl_set_auto(bool on) { t_pdl_auto = on; }

bool pdl_enabled() {
  static int env = -2;
  if (env == -2) {
    const char* e = getenv("LX_FLOW_PDL");
    env = (e && e[0] == '1') ? 1 : (e && e[0] == '0') ? 0 : -1;
  }
  return env >= 0 ? env != 0 : t_pdl_auto;
}

int rows_per_block(int R, int dflt) {
  static int fixed = -2;
  if (fixed == -2) {
    const char* e = getenv("LX_FLOW_ROWS_PER_BLOCK");
    fixed = e ? atoi(e) : -1;
  }
  const int v = fixed >= 0 ? fixed : dflt;
  if (v > 0) return v > 16 ? 16 : v;
  // 0: up to 16, few enough that a small batch spreads over every SM in one wave
  const int per_sm = (R + num_sms() - 1) / num_sms();
  return per_sm < 1 ? 1 : per_sm > 16 ? 16 : per_sm;
}

typedef CUresult (*PFN_encodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                    const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static PFN_encodeTiled get_encode() {
  static PFN_encodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_encodeTiled>(p);
  });
  return fn;
}

bool tmap_f32(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows,
              uint32_t box_cols) {
  PFN_encodeTiled enc = get_encode();
  if (!enc) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (ld * 4) % 16 != 0) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 4};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE,
                   box_cols * 4 == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool tmap_bf16(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows,
               uint32_t box_cols) {
  PFN_encodeTiled enc = get_encode();
  if (!enc) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0 || (ld * 2) % 16 != 0) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE,
                   box_cols * 2 == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// ---------------------------------------------------------------------------
// epilogues: called per (row, 16 consecutive columns) with fp32 accumulators
// ---------------------------------------------------------------------------
// 16 values to 32 contiguous bytes (32-byte aligned) of bf16 / fp16.
__device__ __forceinline__ void store_bf16x16(bf16* dst, const float (&v)[16]) {
  st_global_v8(dst, pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
               pack_bf16x2(v[6], v[7]), pack_bf16x2(v[8], v[9]), pack_bf16x2(v[10], v[11]),
               pack_bf16x2(v[12], v[13]), pack_bf16x2(v[14], v[15]));
}

__device__ __forceinline__ void store_f16x16(__half* dst, const float (&v)[16]) {
  st_global_v8(dst, pack_f16x2(v[0], v[1]), pack_f16x2(v[2], v[3]), pack_f16x2(v[4], v[5]), pack_f16x2(v[6], v[7]),
               pack_f16x2(v[8], v[9]), pack_f16x2(v[10], v[11]), pack_f16x2(v[12], v[13]),
               pack_f16x2(v[14], v[15]));
}

__device__ __forceinline__ void add_bias16(float (&v)[16], const float* bias) {
  const float4* b4 = reinterpret_cast<const float4*>(bias);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float4 b = __ldg(b4 + j);
    v[4 * j + 0] += b.x;
    v[4 * j + 1] += b.y;
    v[4 * j + 2] += b.z;
    v[4 * j + 3] += b.w;
  }
}

struct EpiQKV {
  // the pair kernel stages the q / k (bf16) and v (fp16) values and stores
  // them by TMA through one map over the three planes q, k, v (contiguous,
  // plane_rows rows apart)
  static constexpr bool kStageBf16 = true;
  const float* bias;
  bf16* q;
  bf16* k;
  __half* v;  // fp16 [M][1024]: the MN-major B operand of the attention PV MMA
  const int* pos;
  const float2* rope;  // [pos][32] (cos, sin)
  int plane_rows;      // rows between the q, k and v planes (0 when they are not one block)
  // bias, then the partial rotary of q and k (GPT-J pairs (2i, 2i+1) of
  // channels 0..63, angle pos * inv_freq[i])
  __device__ __forceinline__ void apply(int row, int col0, float (&v16)[16]) const {
    add_bias16(v16, bias + col0);
    const int c = col0 & (DIM - 1);
    if ((col0 >> 10) < 2 && c < HDIM) {
      const float2* cs = rope + static_cast<size_t>(__ldg(pos + row)) * 32 + (c >> 1);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float2 t = __ldg(cs + i);
        const float x0 = v16[2 * i], x1 = v16[2 * i + 1];
        v16[2 * i] = x0 * t.x - x1 * t.y;
        v16[2 * i + 1] = x1 * t.x + x0 * t.y;
      }
    }
  }
  __device__ __forceinline__ uint32_t pack2(int col0, float lo, float hi) const {
    return (col0 >> 10) < 2 ? pack_bf16x2(lo, hi) : pack_f16x2(lo, hi);
  }
  __device__ __forceinline__ void* out_ptr(int row, int col0) const {
    const int which = col0 >> 10;
    const size_t off = static_cast<size_t>(row) * DIM + (col0 & (DIM - 1));
    return which == 0 ? static_cast<void*>(q + off) : which == 1 ? static_cast<void*>(k + off)
                                                                 : static_cast<void*>(v + off);
  }
  __device__ __forceinline__ int store_x(int col0) const { return col0 & (DIM - 1); }
  __device__ __forceinline__ int store_y(int col0, int row) const { return (col0 >> 10) * plane_rows + row; }
  __device__ __forceinline__ void operator()(int row, int col0, float (&v16)[16]) const {
    apply(row, col0, v16);
    const int which = col0 >> 10;
    const int c = col0 & (DIM - 1);
    if (which < 2)
      store_bf16x16((which == 0 ? q : k) + static_cast<size_t>(row) * DIM + c, v16);
    else
      store_f16x16(v + static_cast<size_t>(row) * DIM + c, v16);
  }
};

struct EpiGateRes {
  const float* bias;
  const float* gate;
  float* x;
  __device__ __forceinline__ void operator()(int row, int col0, float (&v)[16]) const {
    float* xr = x + static_cast<size_t>(row) * DIM + col0;
    const float4* x4 = reinterpret_cast<const float4*>(xr);
    const float4* b4 = reinterpret_cast<const float4*>(bias + col0);
    const float4* g4 = reinterpret_cast<const float4*>(gate + col0);
    float o[16];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 xv = x4[j];
      const float4 b = __ldg(b4 + j);
      const float4 g = __ldg(g4 + j);
      o[4 * j + 0] = xv.x + g.x * (v[4 * j + 0] + b.x);
      o[4 * j + 1] = xv.y + g.y * (v[4 * j + 1] + b.y);
      o[4 * j + 2] = xv.z + g.z * (v[4 * j + 2] + b.z);
      o[4 * j + 3] = xv.w + g.w * (v[4 * j + 3] + b.w);
    }
    store_f32x16(xr, o);
  }
};

// x[row, col] = xin + gate[col] * (acc + bias[col]); xin is the residual tile
// the loader warp staged in shared memory (MODE_RESID)
struct EpiGateResSmem {
  static constexpr bool kStageBf16 = false;
  const float* bias;
  const float* gate;
  float* x;
  // o = xin + gate * (v + bias), the stored value, without the store (the
  // pair kernel writes it back into the residual box and stores it by TMA)
  __device__ __forceinline__ void apply(int col0, const float (&v)[16], const float (&xin)[16], float (&o)[16]) const {
    const float4* b4 = reinterpret_cast<const float4*>(bias + col0);
    const float4* g4 = reinterpret_cast<const float4*>(gate + col0);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 b = __ldg(b4 + j);
      const float4 g = __ldg(g4 + j);
      o[4 * j + 0] = xin[4 * j + 0] + g.x * (v[4 * j + 0] + b.x);
      o[4 * j + 1] = xin[4 * j + 1] + g.y * (v[4 * j + 1] + b.y);
      o[4 * j + 2] = xin[4 * j + 2] + g.z * (v[4 * j + 2] + b.z);
      o[4 * j + 3] = xin[4 * j + 3] + g.w * (v[4 * j + 3] + b.w);
    }
  }
  __device__ __forceinline__ void operator()(int row, int col0, float (&v)[16], const float (&xin)[16]) const {
    const float4* b4 = reinterpret_cast<const float4*>(bias + col0);
    const float4* g4 = reinterpret_cast<const float4*>(gate + col0);
    float o[16];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 b = __ldg(b4 + j);
      const float4 g = __ldg(g4 + j);
      o[4 * j + 0] = xin[4 * j + 0] + g.x * (v[4 * j + 0] + b.x);
      o[4 * j + 1] = xin[4 * j + 1] + g.y * (v[4 * j + 1] + b.y);
      o[4 * j + 2] = xin[4 * j + 2] + g.z * (v[4 * j + 2] + b.z);
      o[4 * j + 3] = xin[4 * j + 3] + g.w * (v[4 * j + 3] + b.w);
    }
    store_f32x16(x + static_cast<size_t>(row) * DIM + col0, o);
  }
};

struct EpiGelu {
  const float* bias;
  bf16* h;
  // the pair kernel stages GELU(acc + bias) as bf16 and stores it by TMA
  static constexpr bool kStageBf16 = true;
  __device__ __forceinline__ void* out_ptr(int row, int col0) const { return h + static_cast<size_t>(row) * FF + col0; }
  __device__ __forceinline__ int store_x(int col0) const { return col0; }
  __device__ __forceinline__ int store_y(int, int row) const { return row; }
  __device__ __forceinline__ uint32_t pack2(int, float lo, float hi) const { return pack_bf16x2(lo, hi); }
  __device__ __forceinline__ void apply(int, int col0, float (&v)[16]) const {
    add_bias16(v, bias + col0);
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
      const float2 g = gelu_tanh_fast2(make_float2(v[j], v[j + 1]));
      v[j] = g.x;
      v[j + 1] = g.y;
    }
  }
  __device__ __forceinline__ void operator()(int row, int col0, float (&v)[16]) const {
    add_bias16(v, bias + col0);
#pragma unroll
    for (int j = 0; j < 16; j += 2) {
      const float2 g = gelu_tanh_fast2(make_float2(v[j], v[j + 1]));
      v[j] = g.x;
      v[j + 1] = g.y;
    }
    store_bf16x16(h + static_cast<size_t>(row) * FF + col0, v);
  }
};

struct EpiF32 {
  static constexpr bool kStageBf16 = false;
  const float* bias;
  float* out;
  int ldo;
  __device__ __forceinline__ void operator()(int row, int col0, float (&v)[16]) const {
    if (bias) add_bias16(v, bias + col0);
    store_f32x16(out + static_cast<size_t>(row) * ldo + col0, v);
  }
};

struct EpiInProj {
  const float* cst;
  float* x;
  bf16* stage;
  const int* p2s;
  __device__ __forceinline__ void operator()(int row, int col0, float (&v)[16]) const {
    const float4* c4 = reinterpret_cast<const float4*>(cst + static_cast<size_t>(row) * DIM + col0);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 c = c4[j];
      v[4 * j + 0] += c.x;
      v[4 * j + 1] += c.y;
      v[4 * j + 2] += c.z;
      v[4 * j + 3] += c.w;
    }
    store_f32x16(x + static_cast<size_t>(row) * DIM + col0, v);
    const int srow = __ldg(p2s + row);
    if (srow >= 0) store_bf16x16(stage + static_cast<size_t>(srow) * DIM + col0, v);
  }
};

struct EpiConv {
  const float* bias;
  int second;
  bf16* out_stage;
  float* x;
  const int* s2p;
  __device__ __forceinline__ void operator()(int srow, int col0, float (&v)[16]) const {
    const int prow = __ldg(s2p + srow);
    if (prow < 0) return;  // zero gap rows of the staging layout stay zero
    add_bias16(v, bias + col0);
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = mish_f(v[j]);
    if (!second) {
      store_bf16x16(out_stage + static_cast<size_t>(srow) * DIM + col0, v);
    } else {
      float* xr = x + static_cast<size_t>(prow) * DIM + col0;
      const float4* x4 = reinterpret_cast<const float4*>(xr);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float4 xv = x4[j];
        v[4 * j + 0] += xv.x;
        v[4 * j + 1] += xv.y;
        v[4 * j + 2] += xv.z;
        v[4 * j + 3] += xv.w;
      }
      store_f32x16(xr, v);
    }
  }
};

// ---------------------------------------------------------------------------
// launch helper
// ---------------------------------------------------------------------------
template <int BN, int STAGES, int MODE, class Epi>
static void launch(const CUtensorMap& A, const CUtensorMap& B, int M, int N, int K, int b_off, const Epi& epi,
                   int* err, cudaStream_t s, const CUtensorMap* X = nullptr) {
  constexpr int smem = gemm_smem_bytes<BN, STAGES, MODE>();
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_done[dev & 63]) {
    cudaFuncSetAttribute(k_gemm<BN, STAGES, MODE, Epi>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    attr_done[dev & 63] = true;
  }
  const int tiles = ((M + GEMM_BM - 1) / GEMM_BM) * ((N + BN - 1) / BN);
  int grid = num_sms();
  if (tiles < grid) grid = tiles;
  if (grid <= 0) return;
  GemmShape sh{M, N, K, b_off, err};
  launch_pdl(k_gemm<BN, STAGES, MODE, Epi>, dim3(grid), dim3(gemm_threads(MODE)), smem, s, A, B, X ? *X : A, sh, epi);
}

// CTA-pair launch: persistent grid of up to num_sms() / 2 clusters of 2.
template <int STAGES, bool RES, int XS, class Epi>
static void launch_pair(const CUtensorMap& A, const CUtensorMap& B, int M, int N, int K, int b_off, const Epi& epi,
                        int* err, cudaStream_t s, const CUtensorMap* X = nullptr, const CUtensorMap* Xs = nullptr,
                        bool rev = false) {
  constexpr int smem = gemm2_smem_bytes<STAGES, RES, XS, Epi::kStageBf16>();
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_done[dev & 63]) {
    cudaFuncSetAttribute(k_gemm2<STAGES, RES, XS, Epi>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    attr_done[dev & 63] = true;
  }
  const int tiles = ((M + G2_BM - 1) / G2_BM) * (N / G2_BN);
  int pairs = num_sms() / 2;
  if (tiles < pairs) pairs = tiles;
  if (pairs <= 0) return;
  GemmShape sh{M, N, K, b_off, err, rev ? 1 : 0};
  launch_pdl(k_gemm2<STAGES, RES, XS, Epi>, dim3(2 * pairs), dim3(GEMM2_THREADS), smem, s, A, B, X ? *X : A,
             Xs ? *Xs : A, sh, epi);
}

template <class Epi>
static void launch_bn(int bn, const CUtensorMap& A, const CUtensorMap& B, int M, int N, int K, int b_off,
                      const Epi& e, int* err, cudaStream_t s) {
  if (bn == 256)
    launch<256, 4, MODE_GEMM>(A, B, M, N, K, b_off, e, err, s);
  else
    launch<128, 6, MODE_GEMM>(A, B, M, N, K, b_off, e, err, s);
}

int pick_bn(int M, int N) {
  if (N % 256 != 0) return 128;
  const long tiles256 = static_cast<long>((M + 127) / 128) * (N / 256);
  return tiles256 >= 2L * num_sms() ? 256 : 128;
}

void gemm_qkv(int bn, const CUtensorMap& A, const CUtensorMap& B, int M, int b_off, const float* bias, bf16* q,
              bf16* k, __half* v, const int* pos, const float2* rope, int* err, cudaStream_t s) {
  EpiQKV e{bias, q, k, v, pos, rope, 0};
  launch_bn(bn, A, B, M, QKV_N, DIM, b_off, e, err, s);
}

void gemm_gate_res(int bn, const CUtensorMap& A, const CUtensorMap& B, int M, int K, int b_off, const float* bias,
                   const float* gate, float* x, int* err, cudaStream_t s) {
  EpiGateRes e{bias, gate, x};
  launch_bn(bn, A, B, M, DIM, K, b_off, e, err, s);
}

void gemm_gate_res_tma(const CUtensorMap& A, const CUtensorMap& B, const CUtensorMap& X, int M, int K, int b_off,
                       const float* bias, const float* gate, float* x, int* err, cudaStream_t s) {
  EpiGateResSmem e{bias, gate, x};
  launch<128, 4, MODE_RESID>(A, B, M, DIM, K, b_off, e, err, s, &X);
}

void gemm_pair_qkv(const CUtensorMap& A, const CUtensorMap& B, const CUtensorMap& QKVs, int plane_rows, int M,
                   int b_off, const float* bias, bf16* q, bf16* k, __half* v, const int* pos, const float2* rope,
                   int* err, cudaStream_t s, bool rev) {
  EpiQKV e{bias, q, k, v, pos, rope, plane_rows};
  launch_pair<6, false, 0>(A, B, M, QKV_N, DIM, b_off, e, err, s, nullptr, &QKVs, rev);
}

void gemm_pair_gelu(const CUtensorMap& A, const CUtensorMap& B, const CUtensorMap& Hs, int M, int b_off,
                    const float* bias, bf16* h, int* err, cudaStream_t s, bool rev) {
  EpiGelu e{bias, h};
  launch_pair<6, false, 0>(A, B, M, FF, DIM, b_off, e, err, s, nullptr, &Hs, rev);
}

void gemm_pair_gate_res(const CUtensorMap& A, const CUtensorMap& B, const CUtensorMap& X, const CUtensorMap& Xs,
                        int M, int K, int b_off, const float* bias, const float* gate, float* x, int* err,
                        cudaStream_t s, bool rev) {
  EpiGateResSmem e{bias, gate, x};
  // 5 operand stages + 2 residual slots (same shared memory as 4 + 3):
  // measured FF2 -5.7%, the out projection unchanged
  launch_pair<5, true, 2>(A, B, M, DIM, K, b_off, e, err, s, &X, &Xs, rev);
}

void gemm_pair_f32(const CUtensorMap& A, const CUtensorMap& B, int M, int N, int K, const float* bias, float* out,
                   int ldo, int* err, cudaStream_t s) {
  EpiF32 e{bias, out, ldo};
  launch_pair<6, false, 0>(A, B, M, N, K, 0, e, err, s);
}

bool use_pair_gemm(int M, int N) {
  static int env = -1;
  if (env < 0) {
    const char* e = getenv("LX_FLOW_PAIR_GEMM");
    env = (e && e[0] == '0') ? 0 : (e && e[0] == '2') ? 2 : 1;
  }
  if (!env || N % G2_BN != 0) return false;
  if (env == 2) return true;
  const long pair_tiles = static_cast<long>((M + G2_BM - 1) / G2_BM) * (N / G2_BN);
  return pair_tiles >= 2L * (num_sms() / 2);
}

void gemm_gelu(int bn, const CUtensorMap& A, const CUtensorMap& B, int M, int b_off, const float* bias, bf16* h,
               int* err, cudaStream_t s) {
  EpiGelu e{bias, h};
  launch_bn(bn, A, B, M, FF, DIM, b_off, e, err, s);
}

void gemm_f32(int bn, const CUtensorMap& A, const CUtensorMap& B, int M, int N, int K, const float* bias,
              float* out, int ldo, int* err, cudaStream_t s) {
  EpiF32 e{bias, out, ldo};
  if (N == MEL)
    launch<80, 7, MODE_GEMM>(A, B, M, N, K, 0, e, err, s);
  else
    launch_bn(bn, A, B, M, N, K, 0, e, err, s);
}

void gemm_in_proj(int bn, const CUtensorMap& A, const CUtensorMap& B, int M, const float* cst, float* x,
                  bf16* stage, const int* p2s, int* err, cudaStream_t s) {
  EpiInProj e{cst, x, stage, p2s};
  launch_bn(bn, A, B, M, DIM, MEL, 0, e, err, s);
}

namespace {
template <int ROWT>
void launch_conv(const CUtensorMap& A, const CUtensorMap& B, const GemmShape& sh, const EpiConv& e, int items,
                 cudaStream_t s) {
  constexpr int smem = conv_win_smem_bytes(ROWT);
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_done[dev & 63]) {
    cudaFuncSetAttribute(k_conv_win<ROWT, EpiConv>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    attr_done[dev & 63] = true;
  }
  const int grid = items < num_sms() ? items : num_sms();
  launch_pdl(k_conv_win<ROWT, EpiConv>, dim3(grid), dim3(CONV_THREADS), smem, s, A, B, sh, e);
}
}  // namespace

// Row tiles per conv work item: the fewest waves of items, each weighted by
// the measured time of an item of ROWT tiles relative to ROWT one-tile items
// (1, 0.755, 0.65 per tile at 1, 2, 4 tiles on the config-3 decode).
static int conv_rowt(int Ms) {
  static const int rowts[3] = {1, 2, 4};
  static const double per_tile[3] = {1.0, 0.755, 0.65};
  int best = 1;
  double best_t = 1e300;
  for (int i = 0; i < 3; ++i) {
    const int rt = rowts[i];
    const long items = static_cast<long>((Ms + rt * GEMM_BM - 1) / (rt * GEMM_BM)) * (DIM / 64);
    const long waves = (items + num_sms() - 1) / num_sms();
    const double t = static_cast<double>(waves) * rt * per_tile[i];
    if (t < best_t - 1e-9) {
      best_t = t;
      best = rt;
    }
  }
  return best;
}

void conv_pos(const CUtensorMap& A, const CUtensorMap& B, int Ms, const float* bias, int second, bf16* out_stage,
              float* x, const int* s2p, int* err, cudaStream_t s) {
  if (Ms <= 0) return;
  EpiConv e{bias, second, out_stage, x, s2p};
  GemmShape sh{Ms, DIM, 0, 0, err};
  const int rt = conv_rowt(Ms);
  const int items = ((Ms + rt * GEMM_BM - 1) / (rt * GEMM_BM)) * (DIM / 64);
  if (rt == 4)
    launch_conv<4>(A, B, sh, e, items, s);
  else if (rt == 2)
    launch_conv<2>(A, B, sh, e, items, s);
  else
    launch_conv<1>(A, B, sh, e, items, s);
}

}  // namespace lx
