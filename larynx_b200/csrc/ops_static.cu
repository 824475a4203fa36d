// lx_flow_op_attention_static: the flash-attention entry point of ops.cu with
// every piece of device scratch held in file-scope __device__ arrays, so a call
// allocates no device memory at all (no cudaMalloc / cudaFree, no allocating
// library routine).
//
// Who needs it: callers that may not allocate device memory on the call path.
// cudaMalloc / cudaFree can block on, or synchronise with, work the caller has
// queued on other streams, and take unbounded time; an audio pipeline with a
// per-chunk deadline, or an embedder that hands the whole of HBM to its own
// pool allocator up front, cannot accept either.  lx_flow_op_attention
// allocates its fp16 copy of V, tile list and error word on every call; this
// entry point uses fixed static storage instead.
//
// Limit (checked on the host; a larger call returns LX_ERR_ARG before any
// device work is queued): packed rows R = sum_i round_up(len_i, 8) <=
// LX_STATIC_ATT_MAX_ROWS (4096).  Query tiles = sum_i ceil(len_i / 128) <= R / 8,
// so 512 tile slots always suffice.  The static storage is 8 MiB of fp16 V
// ([4096][1024]) + 8 KiB of tiles + one error word per device.
//
// Set-up: the first call on a device (with that device current) resolves the
// arrays' addresses with cudaGetSymbolAddress, which can load the module; make
// that first call before any stream capture begins.  The addresses are cached
// with the CUDA context they belong to; a call under another context (after a
// cudaDeviceReset, say) looks them up again.
//
// Zero state: only the error word must start at zero; each call clears it on
// the caller's stream before the kernels run.  Every V row the attention
// reads inside [0, R) is rewritten by the call's conversion, and keys past R
// come from the tensor map's zero fill, so nothing else needs clearing.
//
// Concurrency: the storage is shared by every call on a device.  Calls that
// overlap in time on one device (from two host threads, or from two streams)
// race on it and produce wrong results; serialise them.  Each call is
// synchronous on its stream, so calls made one after another from one thread
// are safe.
#include <cuda.h>

#include <mutex>

#include "../../include/larynx_flow.h"
#include "kernels.h"

using namespace lx;

namespace {

constexpr int kMaxRows = LX_STATIC_ATT_MAX_ROWS;
constexpr int kMaxTiles = kMaxRows / 8;
constexpr int kMaxDevices = 64;

__device__ __align__(256) __half g_v[static_cast<size_t>(kMaxRows) * DIM];
__device__ __align__(256) AttnTile g_tiles[kMaxTiles];
__device__ __align__(256) int g_err[1];

struct Scratch {
  __half* v = nullptr;
  AttnTile* tiles = nullptr;
  int* err = nullptr;
};

std::mutex g_setup_mu;
Scratch g_scratch[kMaxDevices];
CUcontext g_ctx[kMaxDevices] = {nullptr};

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

// The driver's cuCtxGetCurrent, found once through the runtime (the library
// does not link libcuda directly).
CtxGetCurrentFn ctx_get_current() {
  static CtxGetCurrentFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<CtxGetCurrentFn>(nullptr);
    return reinterpret_cast<CtxGetCurrentFn>(p);
  }();
  return fn;
}

// Resolves the static arrays of the current device, once per CUDA context.
int scratch_for_current_device(Scratch* out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return LX_ERR_CUDA;
  CtxGetCurrentFn get = ctx_get_current();
  CUcontext ctx = nullptr;
  if (!get || get(&ctx) != CUDA_SUCCESS) return LX_ERR_CUDA;
  if (!ctx) {
    // no context current on this thread yet: cudaSetDevice makes the
    // device's primary context current (CUDA 12 and later)
    if (cudaSetDevice(dev) != cudaSuccess || get(&ctx) != CUDA_SUCCESS || !ctx) return LX_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (g_ctx[dev] != ctx) {
    Scratch s;
    if (cudaGetSymbolAddress(reinterpret_cast<void**>(&s.v), g_v) != cudaSuccess ||
        cudaGetSymbolAddress(reinterpret_cast<void**>(&s.tiles), g_tiles) != cudaSuccess ||
        cudaGetSymbolAddress(reinterpret_cast<void**>(&s.err), g_err) != cudaSuccess)
      return LX_ERR_CUDA;
    g_scratch[dev] = s;
    g_ctx[dev] = ctx;
  }
  *out = g_scratch[dev];
  return LX_OK;
}

// v[R][1024] bf16 -> fp16 in the same layout (the attention's PV operand type).
__global__ void k_v_to_f16_static(const bf16* __restrict__ v, __half* __restrict__ vh, int n8) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n8) return;
  const uint4 a = reinterpret_cast<const uint4*>(v)[i];
  const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&a);
  uint4 o;
  __half2* h = reinterpret_cast<__half2*>(&o);
#pragma unroll
  for (int j = 0; j < 4; ++j) h[j] = __float22half2_rn(__bfloat1622float2(b[j]));
  reinterpret_cast<uint4*>(vh)[i] = o;
}

}  // namespace

extern "C" int lx_flow_op_attention_static(int n_seq, const int32_t* lengths, const void* q, const void* k,
                                           const void* v, void* out, int chunk, void* stream) {
  if (n_seq <= 0 || !lengths || !q || !k || !v || !out || chunk < 0) return LX_ERR_ARG;
  AttnTile tiles[kMaxTiles];
  int n_tiles = 0;
  long long R = 0;
  for (int i = 0; i < n_seq; ++i) {
    if (lengths[i] <= 0) return LX_ERR_ARG;
    for (int q0 = 0; q0 < lengths[i]; q0 += ATT_Q_ROWS) {
      if (n_tiles >= kMaxTiles) return LX_ERR_ARG;
      tiles[n_tiles++] = AttnTile{static_cast<int>(R), lengths[i], q0, 0};
    }
    R += (lengths[i] + 7) / 8 * 8;
    if (R > kMaxRows) return LX_ERR_ARG;
  }
  Scratch sc;
  if (int rc = scratch_for_current_device(&sc)) return rc;
  const int rows = static_cast<int>(R);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  CUtensorMap tq, tk, tv;
  if (!tmap_bf16(&tq, q, rows, DIM, DIM, 128, 64) || !tmap_bf16(&tk, k, rows, DIM, DIM, 128, 64) ||
      !tmap_bf16(&tv, sc.v, rows, DIM, DIM, 128, 64))
    return LX_ERR_ARG;
  if (cudaMemsetAsync(sc.err, 0, sizeof(int), s) != cudaSuccess ||
      cudaMemcpyAsync(sc.tiles, tiles, n_tiles * sizeof(AttnTile), cudaMemcpyHostToDevice, s) != cudaSuccess)
    return LX_ERR_CUDA;
  const int n8 = rows * (DIM / 8);
  k_v_to_f16_static<<<(n8 + 255) / 256, 256, 0, s>>>(static_cast<const bf16*>(v), sc.v, n8);
  if (!attention(tq, tk, tv, sc.tiles, n_tiles, chunk, static_cast<bf16*>(out), sc.err, s)) return LX_ERR_CUDA;
  if (cudaGetLastError() != cudaSuccess) return LX_ERR_CUDA;
  // read the error word in order on the caller's stream: a plain cudaMemcpy
  // would also wait for the work of every other blocking stream on the device
  int e = 0;
  if (cudaMemcpyAsync(&e, sc.err, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess)
    return LX_ERR_CUDA;
  return e ? LX_ERR_TIMEOUT : LX_OK;
}
