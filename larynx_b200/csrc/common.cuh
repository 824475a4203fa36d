// Device-side building blocks for the sm_100a Flow kernels: mbarriers with
// bounded waits, TMA tile loads, tcgen05 (UMMA + TMEM) wrappers and the
// shared-memory / instruction descriptor encodings.
//
// Every spin-wait in this library is bounded: a wait that exceeds
// LX_WAIT_TIMEOUT_NS records an error code in the launch's error word, raises
// the CTA's abort flag and returns false; callers then leave their loops, the
// CTA frees its tensor memory and returns, and the host reports
// LX_ERR_TIMEOUT.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace lx {

constexpr unsigned long long LX_WAIT_TIMEOUT_NS = 2000000000ull;  // 2 s

enum DeviceError : int {
  DEV_OK = 0,
  DEV_TIMEOUT_PRODUCER = 1,
  DEV_TIMEOUT_MMA = 2,
  DEV_TIMEOUT_EPILOGUE = 3,
  DEV_TIMEOUT_SOFTMAX = 4,
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait that may suspend the thread for up to `hint_ns` (it resumes as soon
// as the phase completes), so a waiting thread does not take issue slots from
// the working warps of its SM sub-partition.
__device__ __forceinline__ bool mbar_try_wait_hint(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

constexpr uint32_t LX_WAIT_SUSPEND_NS = 1000000u;  // 1 ms per suspended try

// Bounded wait for the phase of the given parity to complete.  Returns false
// (after recording `code` in *err and raising *abort) when the wait exceeds
// `limit_ns`, or when another role of the CTA has already aborted.
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, int* err, volatile int* abort_flag,
                                              int code, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (;;) {
    if (mbar_try_wait_hint(bar, parity, LX_WAIT_SUSPEND_NS)) return true;
    if (*abort_flag) return false;
    if (global_timer_ns() - t0 > limit_ns) {
      if (err) atomicCAS(err, 0, code);
      *abort_flag = 1;
      return false;
    }
  }
}

// The wait every kernel of the library uses: limit LX_WAIT_TIMEOUT_NS.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, volatile int* abort_flag,
                                          int code) {
  return mbar_wait_for(bar, parity, err, abort_flag, code, LX_WAIT_TIMEOUT_NS);
}

// ---------------------------------------------------------------------------
// TMA (every copy lands in the issuing CTA's own shared memory)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* tm) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tm)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* tm, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Tiled TMA store of this CTA's shared-memory box to global memory (rows and
// columns outside the tensor are not written), tracked as a bulk group.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* tm, const void* smem_src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(tm)),
               "r"(smem_u32(smem_src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// The shared-memory sources of every committed group have been read.
__device__ __forceinline__ void bulk_wait_group_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Every committed group has completed (its global writes done).
__device__ __forceinline__ void bulk_wait_group0() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// ---------------------------------------------------------------------------
// tcgen05: tensor memory and UMMA
// ---------------------------------------------------------------------------
// Warp-wide.  Writes the TMEM base address into *dst (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D(tmem) (+)= A(smem) * B(smem)^T, bf16/f16 inputs, f32 accumulate.
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D(tmem) (+)= A(tmem) * B(smem)^T: A is K-major in tensor memory (row m in
// lane m, two 16-bit K elements per 32-bit column).
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive (once) on the mbarrier when all previously issued tcgen05 ops of
// this thread have completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 bit, 16 consecutive columns per thread (thread i <-> lane i
// of the warp's 32-lane quarter).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor, K-major operand in the 128-byte swizzle
// canonical layout written by a TMA load with CU_TENSOR_MAP_SWIZZLE_128B and a
// 64-element (128-byte) inner box: rows of 128 bytes, 8-row atoms 1024 bytes
// apart (SBO = 1024), leading offset unused for swizzled K-major (encoded 1),
// descriptor version 1 (sm_100), layout type 2 = SWIZZLE_128B.
// Advancing K by 16 elements inside the atom adds 32 bytes to the start.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(1) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
         (static_cast<uint64_t>(2) << 61);
}

// Shared-memory matrix descriptor, MN-major operand in the 128-byte swizzle
// layout written by a TMA load with a 64-element (128-byte) inner box along
// MN: each K row is 128 contiguous bytes of 64 MN elements, 8-row atoms 1024
// bytes apart (SBO = 1024).  LBO (the stride between 64-element MN groups) is
// not used by a 64-wide operand.  Advancing K by 16 rows adds 2048 bytes.
__device__ __forceinline__ uint64_t sdesc_sw128_mn(uint32_t saddr) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(1024 >> 4) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
         (static_cast<uint64_t>(2) << 61);
}

// Instruction-descriptor bit selecting an MN-major B operand.
constexpr uint32_t IDESC_B_MN_MAJOR = 1u << 16;

// Instruction descriptor, kind::f16 with bf16 A/B, f32 D, both K-major.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N) {
  return (1u << 4)                                   // D format f32
         | (1u << 7)                                 // A format bf16
         | (1u << 10)                                // B format bf16
         | (static_cast<uint32_t>(N >> 3) << 17)     // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24);    // M / 16
}

// Instruction descriptor, kind::f16 with f16 A/B, f32 D, both K-major.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N) {
  return (1u << 4) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch.  pdl_launch_dependents lets the next kernel
// of the stream launch now; pdl_wait blocks until the previous kernel of the
// stream has finished and its memory is visible.  Every kernel of the decode
// calls both before its first global access, so when launched with the
// programmatic-serialization attribute (launch_pdl, opt-in) a dependent
// kernel's launch and prologue (barrier init, TMEM allocation, descriptor
// prefetch) overlap its predecessor's tail.  Both are no-ops otherwise.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ---------------------------------------------------------------------------
// 256-bit global stores: one full 32-byte sector per thread (the GEMM
// epilogues write rows per thread, so a warp store touches 32 rows; a 16-byte
// store would leave every sector half written by each instruction).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void st_global_v8(void* p, uint32_t a, uint32_t b, uint32_t c, uint32_t d, uint32_t e,
                                             uint32_t f, uint32_t g, uint32_t h) {
  asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(a), "r"(b), "r"(c), "r"(d), "r"(e),
               "r"(f), "r"(g), "r"(h)
               : "memory");
}

// 16 fp32 values to 64 contiguous bytes (32-byte aligned).
__device__ __forceinline__ void store_f32x16(float* dst, const float (&v)[16]) {
#pragma unroll
  for (int h = 0; h < 2; ++h)
    st_global_v8(dst + 8 * h, __float_as_uint(v[8 * h + 0]), __float_as_uint(v[8 * h + 1]),
                 __float_as_uint(v[8 * h + 2]), __float_as_uint(v[8 * h + 3]), __float_as_uint(v[8 * h + 4]),
                 __float_as_uint(v[8 * h + 5]), __float_as_uint(v[8 * h + 6]), __float_as_uint(v[8 * h + 7]));
}

// ---------------------------------------------------------------------------
// Small numerics helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// GELU, tanh form (nn.GELU(approximate="tanh")).
__device__ __forceinline__ float gelu_tanh_f(float x) {
  const float c1 = 0.7978845608028654f;
  const float c0 = 0.044715f;
  return 0.5f * x * (1.0f + tanhf(c1 * (x + c0 * x * x * x)));
}

// Same GELU with the hardware tanh approximation (one MUFU op; its error,
// ~2^-11 relative, is below the bf16 rounding of the GEMM epilogue output).
__device__ __forceinline__ float gelu_tanh_fast(float x) {
  const float c1 = 0.7978845608028654f;
  const float c0 = 0.044715f;
  float t;
  const float u = c1 * (x + c0 * x * x * x);
  asm("tanh.approx.f32 %0, %1;" : "=f"(t) : "f"(u));
  return 0.5f * x * (1.0f + t);
}

// The same GELU on a pair with packed fp32 arithmetic (fma / mul .f32x2):
// u = x (c1 + c1 c0 x^2), GELU = 0.5 x + 0.5 x tanh(u); five packed
// instructions and two MUFU tanh per pair instead of about twelve scalar ones.
__device__ __forceinline__ float2 gelu_tanh_fast2(float2 x) {
  const float c1 = 0.7978845608028654f;
  const float k1 = 0.7978845608028654f * 0.044715f;
  const float2 x2 = __fmul2_rn(x, x);
  const float2 u = __fmul2_rn(__ffma2_rn(x2, make_float2(k1, k1), make_float2(c1, c1)), x);
  float2 t;
  asm("tanh.approx.f32 %0, %1;" : "=f"(t.x) : "f"(u.x));
  asm("tanh.approx.f32 %0, %1;" : "=f"(t.y) : "f"(u.y));
  const float2 hx = __fmul2_rn(x, make_float2(0.5f, 0.5f));
  return __ffma2_rn(hx, t, hx);
}

// Mish = x * tanh(softplus(x)); softplus with torch's threshold 20.
// Mish x * tanh(softplus(x)) through the identity
//   tanh(log(1 + n)) = (n^2 + 2n) / (n^2 + 2n + 2),  n = e^x,
// one exponential and one division instead of exp, log1p and tanh (the
// conv-pos epilogue evaluates it for every output).  Above x = 20 the factor
// is 1 in fp32; far below 0, n -> 0 and the result -> x * n.
__device__ __forceinline__ float mish_f(float x) {
  if (x > 20.0f) return x;
  const float n = __expf(x);
  const float t = n * (n + 2.0f);
  return x * __fdividef(t, t + 2.0f);
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + expf(-x)); }

}  // namespace lx
