// Per-op entry points of the C ABI: the tcgen05 GEMM and the flash-attention
// kernel on caller-provided device buffers, for per-op parity and
// microbenchmarks.  These allocate small temporaries per call; the Flow hot
// path does not go through them.
#include <cstring>
#include <vector>

#include "../../include/larynx_flow.h"
#include "kernels.h"

using namespace lx;

namespace {

// v[R][1024] bf16 -> fp16 in the same layout (the attention's PV operand type).
__global__ void k_v_to_f16(const bf16* __restrict__ v, __half* __restrict__ vh, size_t n8) {
  for (size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x; i < n8;
       i += static_cast<size_t>(gridDim.x) * blockDim.x) {
    const uint4 a = reinterpret_cast<const uint4*>(v)[i];
    const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&a);
    uint4 o;
    __half2* h = reinterpret_cast<__half2*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) h[j] = __float22half2_rn(__bfloat1622float2(b[j]));
    reinterpret_cast<uint4*>(vh)[i] = o;
  }
}

// Waits for the call's work and reads its error word, in order on `s` (a
// plain cudaMemcpy would also wait for other blocking streams' work).
int sync_check(cudaStream_t s, int* d_err) {
  int e = 0;
  if (cudaMemcpyAsync(&e, d_err, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return LX_ERR_CUDA;
  return e ? LX_ERR_TIMEOUT : LX_OK;
}

}  // namespace

extern "C" {

// C[M,N] (fp32, row stride N) = A[M,K] * B[N,K]^T (+ bias[N]); A, B bf16
// row-major.  K % 8 == 0; N a multiple of 128, or N == 80.  Synchronous.
int lx_flow_op_gemm(int M, int N, int K, const void* A, const void* B, const float* bias, float* C, void* stream) {
  if (M <= 0 || K <= 0 || K % 8 != 0 || !A || !B || !C) return LX_ERR_ARG;
  if (!(N == MEL || (N > 0 && N % 128 == 0))) return LX_ERR_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool pair = N != MEL && K % 64 == 0 && use_pair_gemm(M, N);
  const int bn = N == MEL ? 128 : pair ? 128 : pick_bn(M, N);
  CUtensorMap ta, tb;
  if (!tmap_bf16(&ta, A, M, K, K, 128, 64)) return LX_ERR_ARG;
  if (!tmap_bf16(&tb, B, N, K, K, N == MEL ? MEL : bn, 64)) return LX_ERR_ARG;
  int* d_err = nullptr;
  if (cudaMalloc(&d_err, sizeof(int)) != cudaSuccess) return LX_ERR_OOM;
  cudaMemsetAsync(d_err, 0, sizeof(int), s);
  if (pair)
    gemm_pair_f32(ta, tb, M, N, K, bias, C, N, d_err, s);
  else
    gemm_f32(bn, ta, tb, M, N, K, bias, C, N, d_err, s);
  const int rc = sync_check(s, d_err);
  cudaFree(d_err);
  return rc;
}

// Flash attention over packed sequences.  q, k, v, out: bf16 [R][1024] device
// rows; sequence i occupies rows [start_i, start_i + len_i) with start_0 = 0
// and start_{i+1} = start_i + round_up(len_i, 8).  lengths is a host array.
// chunk > 0 applies the block-causal chunk mask.  Synchronous.
int lx_flow_op_attention(int n_seq, const int32_t* lengths, const void* q, const void* k, const void* v, void* out,
                         int chunk, void* stream) {
  if (n_seq <= 0 || !lengths || !q || !k || !v || !out || chunk < 0) return LX_ERR_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  std::vector<AttnTile> tiles;
  int R = 0;
  for (int i = 0; i < n_seq; ++i) {
    if (lengths[i] <= 0) return LX_ERR_ARG;
    for (int q0 = 0; q0 < lengths[i]; q0 += ATT_Q_ROWS) tiles.push_back(AttnTile{R, lengths[i], q0, 0});
    R += (lengths[i] + 7) / 8 * 8;
  }
  __half* vh = nullptr;
  AttnTile* d_tiles = nullptr;
  int* d_err = nullptr;
  int rc = LX_OK;
  if (cudaMalloc(&vh, static_cast<size_t>(R) * DIM * 2) != cudaSuccess ||
      cudaMalloc(&d_tiles, tiles.size() * sizeof(AttnTile)) != cudaSuccess ||
      cudaMalloc(&d_err, sizeof(int)) != cudaSuccess) {
    rc = LX_ERR_OOM;
  } else {
    cudaMemsetAsync(d_err, 0, sizeof(int), s);
    cudaMemcpyAsync(d_tiles, tiles.data(), tiles.size() * sizeof(AttnTile), cudaMemcpyHostToDevice, s);
    const size_t n8 = static_cast<size_t>(R) * DIM / 8;
    k_v_to_f16<<<static_cast<unsigned>((n8 + 255) / 256), 256, 0, s>>>(static_cast<const bf16*>(v), vh, n8);
    CUtensorMap tq, tk, tv;
    if (!tmap_bf16(&tq, q, R, DIM, DIM, 128, 64) || !tmap_bf16(&tk, k, R, DIM, DIM, 128, 64) ||
        !tmap_bf16(&tv, vh, R, DIM, DIM, 128, 64)) {
      rc = LX_ERR_ARG;
    } else {
      if (!attention(tq, tk, tv, d_tiles, static_cast<int>(tiles.size()), chunk, static_cast<bf16*>(out), d_err, s))
        rc = LX_ERR_CUDA;
      else
        rc = sync_check(s, d_err);
    }
  }
  if (vh) cudaFree(vh);
  if (d_tiles) cudaFree(d_tiles);
  if (d_err) cudaFree(d_err);
  return rc;
}

}  // extern "C"
