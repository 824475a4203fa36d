// Persistent warp-specialised tcgen05 GEMM on CTA pairs (cta_group::2).
//
//   D[M, N] = A[M, K] * B[N, K]^T      (A, B bf16, K-major; fp32 accumulate)
//
// Two CTAs of a 2-CTA cluster (one per SM of a TPC) compute one 256 x 256
// output tile with tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 16):
//   CTA rank r loads A rows [m0 + 128 r, +128) and B rows [n0 + 128 r, +128)
//   into its own shared memory; its tensor memory receives output rows
//   [m0 + 128 r, +128) x all 256 columns.
// Compared with one CTA per 128 x 256 tile, each SM moves 32 KB instead of
// 48 KB of operands through L2 per 64-deep K step for the same MMA work, and
// each issued MMA instruction carries twice the work.
//
// Roles (per CTA):
//   warp 0      TMA producer of this CTA's halves; the leader (rank 0) posts
//               the expected bytes of both CTAs on its own `full` barrier and
//               both CTAs' copies complete on it (.cta_group::2 form)
//   warp 1      TMEM allocation (cta_group::2, both CTAs); in the leader,
//               lane 0 issues the pair's MMAs and commits to the `empty`
//               barriers of both CTAs (one commit per CTA, to a mapped
//               shared::cluster address) and to both `tfull` barriers
//   warp 2      (RES only) residual loader: streams this CTA's fp32 residual
//               rows, two 128 x 32 boxes (one per epilogue column half) per
//               ring slot, XS slots ahead of the epilogue
//   warps 4..11 epilogue: warp w reads TMEM lane quarter w % 4 and column
//               half (w - 4) / 4 (two warps per SM sub-partition hide each
//               other's TMEM / global latencies); each warp arrives on the
//               leader's `tempty` barrier (8 local + 8 remote arrivals).
//               RES and Epi::kStageBf16 epilogues write their 32-row output
//               boxes in shared memory and store them with TMA copies; the
//               others store from registers.
// Every TMA copy in this file lands in the issuing CTA's own shared memory.
#pragma once

#include "common.cuh"
#include "gemm.cuh"

namespace lx {

constexpr int G2_BM = 256;   // output rows per CTA pair
constexpr int G2_BN = 256;   // output columns per CTA pair
constexpr int G2_HALF = 128; // rows of A and of B per CTA
constexpr int G2_BK = 64;

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// shared::cluster address of the variable at shared::cta address `a` in CTA `rank`
__device__ __forceinline__ uint32_t mapa_shared(uint32_t a, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
  return r;
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Bounded wait (acquire at cluster scope: the barrier receives remote arrivals).
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int* err, volatile int* abort_flag,
                                                  int code) {
  if (mbar_try_wait_cluster(bar, parity, 0u)) return true;
  const uint64_t t0 = global_timer_ns();
  for (;;) {
    if (mbar_try_wait_cluster(bar, parity, LX_WAIT_SUSPEND_NS)) return true;
    if (*abort_flag) return false;
    if (global_timer_ns() - t0 > LX_WAIT_TIMEOUT_NS) {
      if (err) atomicCAS(err, 0, code);
      *abort_flag = 1;
      return false;
    }
  }
}

// TMA tile load into this CTA's shared memory whose completion is signalled
// on `bar_cluster`, an mbarrier of this CTA or of its pair peer.
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* tm, uint32_t bar_cluster, int x,
                                                 int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void umma_pair_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on the mbarrier at shared::cluster address `bar_cluster` (this
// CTA's or the peer's) when the pair MMAs issued so far by this thread are done.
__device__ __forceinline__ void umma_pair_commit(uint32_t bar_cluster) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster)
               : "memory");
}

// 12 warps: 0 TMA, 1 MMA/TMEM, 2 residual loader (RES), 3 idle, 4..11 epilogue.
constexpr int GEMM2_THREADS = 384;
constexpr int G2_EPI_WARP0 = 4;
constexpr int G2_STEPS = G2_BN / 2 / 32;  // 32-column steps per epilogue column half

// 32 consecutive TMEM columns of this warp's 32 lanes, as two 16-column halves.
__device__ __forceinline__ void tmem_ld32x2(uint32_t taddr, float (&a)[16], float (&b)[16]) {
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
  for (int i = 0; i < 16; ++i) {
    a[i] = __uint_as_float(r[i]);
    b[i] = __uint_as_float(r[16 + i]);
  }
}

// 16 columns of the residual epilogue: xin from the 128B-swizzled 128 x 32
// fp32 box row `xrow` (row rt of the box), 16-byte units unit0 .. unit0 + 3.
template <class Epi>
__device__ __forceinline__ void epi_res_chunk(const Epi& epi, const uint8_t* xrow, int rt, int row, int col,
                                              int unit0, const GemmShape& sh, float (&v)[16]) {
  if (row >= sh.M) return;
  float xin[16];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float4 f = *reinterpret_cast<const float4*>(xrow + (((unit0 + j) ^ (rt & 7)) << 4));
    xin[4 * j + 0] = f.x;
    xin[4 * j + 1] = f.y;
    xin[4 * j + 2] = f.z;
    xin[4 * j + 3] = f.w;
  }
  epi(row, col, v, xin);
}

// One 32-column step of an epilogue warp: columns [col, col + 32) of `row`.
// RES: the step's residual box is the `half`-th 128 x 32 box of ring slot
// `slot`; the warp waits for it and releases it afterwards.
template <bool RES, class Epi>
__device__ __forceinline__ bool epi_step2(const Epi& epi, const uint8_t* sX, uint64_t* x_full, uint64_t* x_empty,
                                          int& slot, uint32_t& xph, int xs, int half, int rt, int row, int col,
                                          const GemmShape& sh, volatile int* abort_flag, float (&v0)[16],
                                          float (&v1)[16]) {
  constexpr int XBOX = G2_HALF * 32 * 4;
  if constexpr (RES) {
    const bool ok = mbar_wait(&x_full[slot], xph, sh.err, abort_flag, DEV_TIMEOUT_EPILOGUE);
    if (!__all_sync(0xffffffffu, ok)) return false;
    const uint8_t* xrow = sX + (2 * slot + half) * XBOX + rt * 128;
    epi_res_chunk(epi, xrow, rt, row, col, 0, sh, v0);
    epi_res_chunk(epi, xrow, rt, row, col + 16, 4, sh, v1);
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(&x_empty[slot]);
    if (++slot == xs) {
      slot = 0;
      xph ^= 1u;
    }
  } else {
    if (row < sh.M) {
      epi(row, col, v0);
      epi(row, col + 16, v1);
    }
  }
  return true;
}

// A box whose 32 rows reach past the last row is not stored by TMA (its
// tensor map spans the workspace's capacity, beyond M): each lane copies its
// own row, if it is a valid one, from the swizzled box to global memory.
__device__ __forceinline__ void copy_staged_row(const uint8_t* srow, int r, void* dst) {
#pragma unroll
  for (int u = 0; u < 8; ++u)
    reinterpret_cast<uint4*>(dst)[u] = *reinterpret_cast<const uint4*>(srow + ((u ^ (r & 7)) << 4));
}

// One 32-column residual step stored by TMA: the warp's 32 rows of the box
// are updated in place (o = epi.apply(v, x) written over x in the same
// swizzled positions), and lane 0 stores the warp's 32 x 32 sub-box with one
// bulk tensor copy (rows past the tensor are not written).  The slot is
// released once the copy has read shared memory.  Compared with each thread
// storing its row's 128 bytes, the LSU issues nothing for the output and the
// copy engine writes whole lines.
template <class Epi>
__device__ __forceinline__ bool epi_res_store_step(const Epi& epi, uint8_t* sX, uint64_t* x_full, uint64_t* x_empty,
                                                   int& slot, uint32_t& xph, int xs, int half, int q, int rt,
                                                   int row0, int col, const GemmShape& sh, const CUtensorMap* tmXs,
                                                   volatile int* abort_flag, const float (&v0)[16],
                                                   const float (&v1)[16]) {
  constexpr int XBOX = G2_HALF * 32 * 4;
  const bool ok = mbar_wait(&x_full[slot], xph, sh.err, abort_flag, DEV_TIMEOUT_EPILOGUE);
  if (!__all_sync(0xffffffffu, ok)) return false;
  uint8_t* box = sX + (2 * slot + half) * XBOX;
  uint8_t* xrow = box + rt * 128;
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    float xin[16], o[16];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 f = *reinterpret_cast<const float4*>(xrow + (((4 * c + j) ^ (rt & 7)) << 4));
      xin[4 * j + 0] = f.x;
      xin[4 * j + 1] = f.y;
      xin[4 * j + 2] = f.z;
      xin[4 * j + 3] = f.w;
    }
    epi.apply(col + 16 * c, c ? v1 : v0, xin, o);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      *reinterpret_cast<float4*>(xrow + (((4 * c + j) ^ (rt & 7)) << 4)) =
          make_float4(o[4 * j + 0], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
  }
  fence_proxy_async_smem();  // the generic-proxy writes, before the async-proxy read
  __syncwarp();
  const int y = row0 + 32 * q;  // first row of this warp's sub-box
  if (y + 32 <= sh.M) {
    if ((threadIdx.x & 31) == 0) {
      tma_store_2d(tmXs, box + q * 32 * 128, col, y);
      bulk_commit_group();
      bulk_wait_group_read0();
    }
  } else if (y + (rt & 31) < sh.M) {
    copy_staged_row(xrow, rt, epi.x + static_cast<size_t>(y + (rt & 31)) * DIM + col);
  }
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(&x_empty[slot]);
  if (++slot == xs) {
    slot = 0;
    xph ^= 1u;
  }
  return true;
}

// Half of a staged 64-column box: 32 columns of this thread's row (v0, v1)
// through epi.apply, packed to bf16 and written as 16-byte units u0 .. u0 + 3
// of the row in the 128-byte swizzle the box's TMA store reads.
// Rows at or past the last row (grow >= M) are never stored and are not
// passed through epi.apply, which may index per-row tables (the rotary
// position of a QKV row) that hold nothing valid there.
template <class Epi>
__device__ __forceinline__ void stage_bf16_half(const Epi& epi, uint8_t* stg, int r, int grow, int M, int col,
                                                float (&v0)[16], float (&v1)[16], int u0) {
  if (grow < M) {
    epi.apply(grow, col, v0);
    epi.apply(grow, col + 16, v1);
  }
  uint8_t* row = stg + r * 128;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const float* a = u < 2 ? v0 + 8 * u : v1 + 8 * (u - 2);
    *reinterpret_cast<uint4*>(row + (((u0 + u) ^ (r & 7)) << 4)) =
        make_uint4(epi.pack2(col, a[0], a[1]), epi.pack2(col, a[2], a[3]), epi.pack2(col, a[4], a[5]),
                   epi.pack2(col, a[6], a[7]));
  }
}

// 256-row block of work item `tile` (column tiles fastest).  With `rev` the
// blocks are visited from the last one down: the rows a kernel writes last
// are still in L2 when the next kernel starts, so the engine alternates the
// direction from kernel to kernel and the consumer reads those rows first.
__device__ __forceinline__ int g2_mblock(int tile, int tiles_n, int tiles_m, int rev) {
  const int mb = tile / tiles_n;
  return rev ? tiles_m - 1 - mb : mb;
}

// Staged bf16 epilogue (Epi::kStageBf16): each epilogue warp owns a 32-row x
// 64-column bf16 box (4 KB, 128-byte swizzle) in shared memory.
constexpr int G2_STAGE_BYTES = 32 * 128;

template <int STAGES, bool RES, int XS, bool STG = false>
__host__ __device__ constexpr int gemm2_smem_bytes() {
  return 1024 + STAGES * 2 * (G2_HALF * G2_BK * 2) + (RES ? XS * 2 * G2_HALF * 32 * 4 : 0) +
         (STG ? 8 * G2_STAGE_BYTES : 0) + 512;
}

template <int STAGES, bool RES, int XS, class Epi>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(GEMM2_THREADS, 1)
    k_gemm2(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
            const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmXs, GemmShape sh,
            Epi epi) {
  constexpr int A_BYTES = G2_HALF * G2_BK * 2;  // 16 KB
  constexpr int B_BYTES = G2_HALF * G2_BK * 2;  // 16 KB
  constexpr int XBOX = G2_HALF * 32 * 4;        // 16 KB: 128 rows x 32 fp32 columns
  constexpr int XSLOT = 2 * XBOX;               // one box per epilogue column half
  constexpr uint32_t TMEM_COLS = 2 * G2_BN;     // two accumulator stages
  constexpr uint32_t IDESC = idesc_bf16_f32(G2_BM, G2_BN);
  constexpr int XS_ = RES ? XS : 1;
  constexpr bool STG = Epi::kStageBf16;
  static_assert(!(STG && RES), "the staged bf16 epilogue has no residual");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint8_t* sX = sB + STAGES * B_BYTES;
  uint8_t* sStg = sX + (RES ? XS * XSLOT : 0);
  uint64_t* full = reinterpret_cast<uint64_t*>(sStg + (STG ? 8 * G2_STAGE_BYTES : 0));
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* x_full = tempty + 2;
  uint64_t* x_empty = x_full + XS_;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(x_empty + XS_);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 16);  // 8 epilogue warps of each CTA (used in the leader)
    }
    for (int s = 0; s < XS_; ++s) {
      mbar_init(&x_full[s], 1);
      mbar_init(&x_empty[s], 8);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (RES) tma_prefetch_desc(&tmX);
    if (RES || STG) tma_prefetch_desc(&tmXs);
  }
  __syncwarp();
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // barrier inits and the TMEM address visible pair-wide
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_launch_dependents();
  pdl_wait();

  const int tiles_n = sh.N / G2_BN;
  const int tiles_m = (sh.M + G2_BM - 1) / G2_BM;
  const int n_tiles = tiles_m * tiles_n;
  const int num_kb = sh.K / G2_BK;
  const int pair = blockIdx.x >> 1;
  const int n_pairs = gridDim.x >> 1;

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t full_leader = mapa_shared(smem_u32(full), 0);
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = pair; tile < n_tiles; tile += n_pairs) {
        const int m0 = g2_mblock(tile, tiles_n, tiles_m, sh.rev) * G2_BM + static_cast<int>(rank) * G2_HALF;
        const int n0 = (tile % tiles_n) * G2_BN + static_cast<int>(rank) * G2_HALF;
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, sh.err, abort_flag, DEV_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * (A_BYTES + B_BYTES));
          const uint32_t fb = full_leader + 8u * static_cast<uint32_t>(stage);
          tma_load_2d_pair(sA + stage * A_BYTES, &tmA, fb, kb * G2_BK, m0);
          tma_load_2d_pair(sB + stage * B_BYTES, &tmB, fb, kb * G2_BK, sh.b_off + n0);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    if (rank == 0 && lane == 0) {
      const uint64_t da0 = sdesc_sw128(smem_u32(sA));
      const uint64_t db0 = sdesc_sw128(smem_u32(sB));
      const uint32_t empty_own = mapa_shared(smem_u32(empty), 0);
      const uint32_t empty_peer = mapa_shared(smem_u32(empty), 1);
      const uint32_t tfull_own = mapa_shared(smem_u32(tfull), 0);
      const uint32_t tfull_peer = mapa_shared(smem_u32(tfull), 1);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int tile = pair; tile < n_tiles; tile += n_pairs) {
        if (!mbar_wait_cluster(&tempty[acc], acc_phase ^ 1u, sh.err, abort_flag, DEV_TIMEOUT_MMA)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * G2_BN);
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, sh.err, abort_flag, DEV_TIMEOUT_MMA)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = da0 + static_cast<uint64_t>((stage * A_BYTES) >> 4);
          const uint64_t db = db0 + static_cast<uint64_t>((stage * B_BYTES) >> 4);
#pragma unroll
          for (int k = 0; k < G2_BK / 16; ++k)
            umma_pair_ss(d_tmem, da + 2 * k, db + 2 * k, IDESC, (kb > 0 || k > 0) ? 1u : 0u);
          umma_pair_commit(empty_own + 8u * static_cast<uint32_t>(stage));
          umma_pair_commit(empty_peer + 8u * static_cast<uint32_t>(stage));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_pair_commit(tfull_own + 8u * static_cast<uint32_t>(acc));
        umma_pair_commit(tfull_peer + 8u * static_cast<uint32_t>(acc));
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
    }
  } else if (warp == 2) {
    if (RES && lane == 0) {
      // residual boxes of both column halves, step j: columns n0 + 32 j and n0 + 128 + 32 j
      int slot = 0;
      uint32_t xph = 0;
      for (int tile = pair; tile < n_tiles; tile += n_pairs) {
        const int m0 = g2_mblock(tile, tiles_n, tiles_m, sh.rev) * G2_BM + static_cast<int>(rank) * G2_HALF;
        const int n0 = (tile % tiles_n) * G2_BN;
        bool ok = true;
        for (int j = 0; j < G2_STEPS; ++j) {
          if (!mbar_wait(&x_empty[slot], xph ^ 1u, sh.err, abort_flag, DEV_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&x_full[slot], XSLOT);
          tma_load_2d(sX + slot * XSLOT, &tmX, &x_full[slot], n0 + 32 * j, m0);
          tma_load_2d(sX + slot * XSLOT + XBOX, &tmX, &x_full[slot], n0 + G2_BN / 2 + 32 * j, m0);
          if (++slot == XS_) {
            slot = 0;
            xph ^= 1u;
          }
        }
        if (!ok) break;
      }
    }
  } else if (warp >= G2_EPI_WARP0) {
    // epilogue warps 4..11: TMEM lane quarter warp % 4, column half (warp - 4) / 4
    const int q = warp & 3;
    const int half = (warp - G2_EPI_WARP0) >> 2;
    const int cb = half * (G2_BN / 2);
    const uint32_t tempty_leader = mapa_shared(smem_u32(tempty), 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    int slot = 0;
    uint32_t xph = 0;
    for (int tile = pair; tile < n_tiles; tile += n_pairs) {
      const int m0 = g2_mblock(tile, tiles_n, tiles_m, sh.rev) * G2_BM + static_cast<int>(rank) * G2_HALF;
      const int n0 = (tile % tiles_n) * G2_BN + cb;
      bool ok = mbar_wait(&tfull[acc], acc_phase, sh.err, abort_flag, DEV_TIMEOUT_EPILOGUE);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const int rt = q * 32 + lane;
      const int row = m0 + rt;
      const uint32_t t_row =
          tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * G2_BN + cb);
      float a0[16], a1[16], b0[16], b1[16];
      tmem_ld32x2(t_row, a0, a1);
      tmem_ld_wait();
      if constexpr (STG) {
        // two 32-column steps fill the warp's 32 x 64 box; one TMA store each
        uint8_t* stg = sStg + (warp - G2_EPI_WARP0) * G2_STAGE_BYTES;
        const int y = m0 + 32 * q;
#pragma unroll 1
        for (int j = 0; j < G2_STEPS; j += 2) {
          tmem_ld32x2(t_row + 32 * (j + 1), b0, b1);
          if (lane == 0) bulk_wait_group_read0();  // the previous box has been read
          __syncwarp();
          stage_bf16_half(epi, stg, lane, y + lane, sh.M, n0 + 32 * j, a0, a1, 0);
          tmem_ld_wait();
          if (j + 2 < G2_STEPS) tmem_ld32x2(t_row + 32 * (j + 2), a0, a1);
          stage_bf16_half(epi, stg, lane, y + lane, sh.M, n0 + 32 * (j + 1), b0, b1, 4);
          fence_proxy_async_smem();
          __syncwarp();
          if (y + 32 <= sh.M) {
            if (lane == 0) {
              tma_store_2d(&tmXs, stg, epi.store_x(n0 + 32 * j), epi.store_y(n0 + 32 * j, y));
              bulk_commit_group();
            }
          } else if (y + lane < sh.M) {
            copy_staged_row(stg + lane * 128, lane, epi.out_ptr(y + lane, n0 + 32 * j));
          }
          tmem_ld_wait();
        }
      }
#pragma unroll 1
      for (int j = 0; !STG && j < G2_STEPS && ok; j += 2) {
        // TMEM load of step j + 1 in flight while step j is processed
        tmem_ld32x2(t_row + 32 * (j + 1), b0, b1);
        if constexpr (RES)
          ok = epi_res_store_step(epi, sX, x_full, x_empty, slot, xph, XS_, half, q, rt, m0, n0 + 32 * j, sh, &tmXs,
                                  abort_flag, a0, a1);
        else
          ok = epi_step2<RES>(epi, sX, x_full, x_empty, slot, xph, XS_, half, rt, row, n0 + 32 * j, sh, abort_flag,
                              a0, a1);
        tmem_ld_wait();
        if (!ok) break;
        if (j + 2 < G2_STEPS) tmem_ld32x2(t_row + 32 * (j + 2), a0, a1);
        if constexpr (RES)
          ok = epi_res_store_step(epi, sX, x_full, x_empty, slot, xph, XS_, half, q, rt, m0, n0 + 32 * (j + 1), sh,
                                  &tmXs, abort_flag, b0, b1);
        else
          ok = epi_step2<RES>(epi, sX, x_full, x_empty, slot, xph, XS_, half, rt, row, n0 + 32 * (j + 1), sh,
                              abort_flag, b0, b1);
        tmem_ld_wait();
      }
      if (!ok) break;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (rank == 0)
          mbar_arrive(&tempty[acc]);
        else
          mbar_arrive_remote(tempty_leader + 8u * static_cast<uint32_t>(acc));
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
    // the TMA stores' global writes complete before the CTA exits
    if ((RES || STG) && lane == 0) bulk_wait_group0();
  }

  __syncwarp();
  tc_fence_before();
  cluster_sync_all();  // every MMA consumed, every epilogue done, in both CTAs
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

}  // namespace lx
