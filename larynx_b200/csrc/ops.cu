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

__global__ void k_transpose_v(const bf16* __restrict__ v, __half* __restrict__ vt, int R, int ldvt) {
  const int r = blockIdx.x * 32 + threadIdx.x;
  const int c = blockIdx.y * 32 + threadIdx.y;
  if (r < R && c < DIM)
    vt[static_cast<size_t>((c >> 6) * VT_ROWS + (c & 63)) * ldvt + r] =
        __float2half_rn(__bfloat162float(v[static_cast<size_t>(r) * DIM + c]));
}

int sync_check(cudaStream_t s, int* d_err) {
  if (cudaStreamSynchronize(s) != cudaSuccess) return LX_ERR_CUDA;
  int e = 0;
  if (cudaMemcpy(&e, d_err, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return LX_ERR_CUDA;
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
  const int bn = N == MEL ? 128 : pick_bn(M, N);
  CUtensorMap ta, tb;
  if (!tmap_bf16(&ta, A, M, K, K, 128, 64)) return LX_ERR_ARG;
  if (!tmap_bf16(&tb, B, N, K, K, N == MEL ? MEL : bn, 64)) return LX_ERR_ARG;
  int* d_err = nullptr;
  if (cudaMalloc(&d_err, sizeof(int)) != cudaSuccess) return LX_ERR_OOM;
  cudaMemsetAsync(d_err, 0, sizeof(int), s);
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
  const int Rv = (R + 7) / 8 * 8;
  __half* vt = nullptr;
  AttnTile* d_tiles = nullptr;
  int* d_err = nullptr;
  int rc = LX_OK;
  if (cudaMalloc(&vt, static_cast<size_t>(HEADS) * VT_ROWS * Rv * 2) != cudaSuccess ||
      cudaMalloc(&d_tiles, tiles.size() * sizeof(AttnTile)) != cudaSuccess ||
      cudaMalloc(&d_err, sizeof(int)) != cudaSuccess) {
    rc = LX_ERR_OOM;
  } else {
    cudaMemsetAsync(vt, 0, static_cast<size_t>(HEADS) * VT_ROWS * Rv * 2, s);
    cudaMemsetAsync(d_err, 0, sizeof(int), s);
    cudaMemcpyAsync(d_tiles, tiles.data(), tiles.size() * sizeof(AttnTile), cudaMemcpyHostToDevice, s);
    k_transpose_v<<<dim3((R + 31) / 32, DIM / 32), dim3(32, 32), 0, s>>>(static_cast<const bf16*>(v), vt, R, Rv);
    CUtensorMap tq, tk, tv;
    if (!tmap_bf16(&tq, q, R, DIM, DIM, 128, 64) || !tmap_bf16(&tk, k, R, DIM, DIM, 128, 64) ||
        !tmap_bf16(&tv, vt, static_cast<uint64_t>(HEADS) * VT_ROWS, Rv, Rv, VT_ROWS, 64)) {
      rc = LX_ERR_ARG;
    } else {
      attention(tq, tk, tv, d_tiles, static_cast<int>(tiles.size()), chunk, static_cast<bf16*>(out), d_err, s);
      rc = sync_check(s, d_err);
    }
  }
  if (vt) cudaFree(vt);
  if (d_tiles) cudaFree(d_tiles);
  if (d_err) cudaFree(d_err);
  return rc;
}

}  // extern "C"
