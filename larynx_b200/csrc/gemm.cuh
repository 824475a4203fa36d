// Persistent warp-specialised tcgen05 GEMM for sm_100a.
//
//   D[M, N] = A[M, K] * B[N, K]^T      (A, B bf16, K-major; fp32 accumulate)
//
// One CTA per SM walks a static list of 128 x BN output tiles.  Roles:
//   warp 0      TMA producer: 128x64 A box + BNx64 B box per stage
//               (128-byte swizzle) into a STAGES-deep shared-memory ring
//   warp 1      TMEM allocator; lane 0 issues tcgen05.mma (M=128, N=BN, K=16)
//               and tcgen05.commit to release ring slots / publish tiles
//   warps 2..9  epilogue: tcgen05.ld of a 32-row TMEM lane quarter each (two
//               warps per quarter, one per column half of the tile), fused
//               element-wise epilogue, direct global stores
// The fp32 accumulator is double-buffered in tensor memory (2 x BN columns),
// so the epilogue of tile i overlaps the MMAs of tile i+1.
//
// MODE_RESID has four epilogue warps (2..5) and a seventh warp that
// TMA-prefetches the fp32 residual tile
// (128 x BN, as 32-column 128B-swizzled boxes) into shared memory while the
// tile's MMAs run; the epilogue reads it from there instead of waiting on HBM.
//
// The causal grouped Conv1d of the DiT's position embedding runs in its own
// kernel below (k_conv_win): one A window per tile, taps as shifted views.
#pragma once

#include "common.cuh"
#include "kernels.h"

namespace lx {

enum GemmMode : int { MODE_GEMM = 0, MODE_RESID = 2 };

constexpr int GEMM_BM = 128;
constexpr int GEMM_BK = 64;
constexpr int CONV_TAPS = 31;

struct GemmShape {
  int M, N, K;
  int b_off;  // row offset into the B tensor (layer slice of stacked weights)
  int* err;   // device error word
  int rev;    // pair GEMM: nonzero visits the 256-row blocks from the last one down
};

__host__ __device__ constexpr int tmem_cols_for(int bn) {
  return (2 * bn) <= 32 ? 32 : (2 * bn) <= 64 ? 64 : (2 * bn) <= 128 ? 128 : (2 * bn) <= 256 ? 256 : 512;
}

// Epilogue warps: MODE_GEMM has eight (two per TMEM lane quarter, one per
// column half of the tile), so twice the rows' global traffic is in flight
// for epilogue-bound shapes (the K = 80 input projection, small batches);
// MODE_RESID has four beside its residual loader.
__host__ __device__ constexpr int gemm_epi_warps(int mode) { return mode == MODE_RESID ? 4 : 8; }
__host__ __device__ constexpr int gemm_threads(int mode) { return mode == MODE_RESID ? 224 : 64 + 32 * 8; }

template <int BN, int STAGES, int MODE = MODE_GEMM>
__host__ __device__ constexpr int gemm_smem_bytes() {
  return 1024 /*alignment slack*/ + STAGES * (GEMM_BM * GEMM_BK * 2 + BN * GEMM_BK * 2) +
         (MODE == MODE_RESID ? GEMM_BM * BN * 4 : 0) + 256 /*barriers*/;
}

// One 16-column chunk of the epilogue (residual from the swizzled smem tile
// when RES).
template <bool RES, class Epi>
__device__ __forceinline__ void epi_chunk(const Epi& epi, const uint8_t* sX, int rt, int row, int n0, int c0,
                                          const GemmShape& sh, float (&v)[16]) {
  constexpr int XBOX_BYTES = 128 * 32 * 4;
  if (row >= sh.M || n0 + c0 >= sh.N) return;
  if constexpr (RES) {
    float xin[16];
    const uint8_t* xrow = sX + (c0 / 32) * XBOX_BYTES + rt * 128;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int ch = ((c0 & 31) >> 2) + j;
      const float4 f = *reinterpret_cast<const float4*>(xrow + ((ch ^ (rt & 7)) << 4));
      xin[4 * j + 0] = f.x;
      xin[4 * j + 1] = f.y;
      xin[4 * j + 2] = f.z;
      xin[4 * j + 3] = f.w;
    }
    epi(row, n0 + c0, v, xin);
  } else {
    epi(row, n0 + c0, v);
  }
}

template <int BN, int STAGES, int MODE, class Epi>
__global__ void __launch_bounds__(gemm_threads(MODE), 1)
    k_gemm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
           const __grid_constant__ CUtensorMap tmX, GemmShape sh, Epi epi) {
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N for M=128 must be a multiple of 16 in [16,256]");
  static_assert(MODE != MODE_RESID || BN % 32 == 0, "residual boxes are 32 columns wide");
  constexpr bool RES = MODE == MODE_RESID;
  constexpr int A_BYTES = GEMM_BM * GEMM_BK * 2;
  constexpr int B_BYTES = BN * GEMM_BK * 2;
  constexpr int X_BYTES = RES ? GEMM_BM * BN * 4 : 0;
  constexpr int XBOX_BYTES = GEMM_BM * 32 * 4;  // 128 rows x 32 fp32 columns
  constexpr uint32_t TMEM_COLS = tmem_cols_for(BN);
  constexpr uint32_t IDESC = idesc_bf16_f32(GEMM_BM, BN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint8_t* sX = sB + STAGES * B_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sX + X_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* x_full = tempty + 2;
  uint64_t* x_empty = x_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(x_empty + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], gemm_epi_warps(MODE));
    }
    mbar_init(x_full, 1);
    mbar_init(x_empty, 4);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (RES) tma_prefetch_desc(&tmX);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_launch_dependents();
  pdl_wait();

  const int tiles_n = (sh.N + BN - 1) / BN;
  const int tiles_m = (sh.M + GEMM_BM - 1) / GEMM_BM;
  const int n_tiles = tiles_m * tiles_n;
  const int num_kb = (sh.K + GEMM_BK - 1) / GEMM_BK;

  if (warp == 0) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
        const int m0 = (tile / tiles_n) * GEMM_BM;
        const int n0 = (tile % tiles_n) * BN;
        bool ok = true;
        for (int kb = 0; kb < num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, sh.err, abort_flag, DEV_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[stage], A_BYTES + B_BYTES);
          tma_load_2d(sA + stage * A_BYTES, &tmA, &full[stage], kb * GEMM_BK, m0);
          tma_load_2d(sB + stage * B_BYTES, &tmB, &full[stage], kb * GEMM_BK, sh.b_off + n0);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // descriptors of stage 0; stage s and K step k add (s * bytes + 32 k) >> 4
      const uint64_t da0 = sdesc_sw128(smem_u32(sA));
      const uint64_t db0 = sdesc_sw128(smem_u32(sB));
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, sh.err, abort_flag, DEV_TIMEOUT_MMA)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
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
          for (int k = 0; k < GEMM_BK / 16; ++k)
            umma_ss(d_tmem, da + 2 * k, db + 2 * k, IDESC, (kb > 0 || k > 0) ? 1u : 0u);
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
    }
  } else if (RES && warp == 6) {
    // residual loader (MODE_RESID only): the 128 x BN fp32 tile of the residual
    if (RES && lane == 0) {
      uint32_t xph = 0;
      for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
        const int m0 = (tile / tiles_n) * GEMM_BM;
        const int n0 = (tile % tiles_n) * BN;
        if (!mbar_wait(x_empty, xph ^ 1u, sh.err, abort_flag, DEV_TIMEOUT_PRODUCER)) break;
        mbar_arrive_expect_tx(x_full, X_BYTES);
#pragma unroll
        for (int b = 0; b < BN / 32; ++b) tma_load_2d(sX + b * XBOX_BYTES, &tmX, x_full, n0 + 32 * b, m0);
        xph ^= 1u;
      }
    }
  } else {
    // epilogue warps 2.. -> TMEM lane quarters 2,3,0,1(,2,3,0,1); with eight
    // warps the second four take the right half of the tile's columns
    // (a BN whose half is not a multiple of 16 leaves the whole tile to the
    // first four, and the second four only keep the barrier protocol)
    constexpr bool SPLIT = gemm_epi_warps(MODE) == 8 && (BN / 2) % 16 == 0;
    constexpr int EPI_COLS = SPLIT ? BN / 2 : BN;
    const int q = warp & 3;
    const int grp = (warp - 2) >> 2;
    const int cb = grp * EPI_COLS;
    const bool has_cols = SPLIT || grp == 0;
    int acc = 0;
    uint32_t acc_phase = 0;
    uint32_t xph = 0;
    for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
      const int m0 = (tile / tiles_n) * GEMM_BM;
      const int n0 = (tile % tiles_n) * BN;
      bool ok = mbar_wait(&tfull[acc], acc_phase, sh.err, abort_flag, DEV_TIMEOUT_EPILOGUE);
      if (RES && ok) ok = mbar_wait(x_full, xph, sh.err, abort_flag, DEV_TIMEOUT_EPILOGUE);
      if (!__all_sync(0xffffffffu, ok)) break;  // warp-uniform exit before the .sync.aligned loads
      tc_fence_after();
      const int rt = q * 32 + lane;  // row inside the tile
      const int row = m0 + rt;
      const uint32_t t_row =
          tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * BN + cb);
      // software-pipelined: the TMEM load of chunk c+1 is in flight while
      // chunk c is processed (tcgen05.wait::ld waits for all of this thread's loads)
      float va[16], vb[16];
      if (has_cols) {
        tmem_ld16(t_row, va);
        tmem_ld_wait();
      }
#pragma unroll 1
      for (int c0 = 0; has_cols && c0 < EPI_COLS; c0 += 32) {
        if (c0 + 16 < EPI_COLS) tmem_ld16(t_row + c0 + 16, vb);
        epi_chunk<RES>(epi, sX, rt, row, n0, cb + c0, sh, va);
        tmem_ld_wait();
        if (c0 + 16 >= EPI_COLS) break;
        if (c0 + 32 < EPI_COLS) tmem_ld16(t_row + c0 + 32, va);
        epi_chunk<RES>(epi, sX, rt, row, n0, cb + c0 + 16, sh, vb);
        tmem_ld_wait();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&tempty[acc]);
        if (RES) mbar_arrive(x_empty);
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
      xph ^= 1u;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Causal grouped Conv1d of the DiT's position embedding (k = 31, 16 groups of
// 64 channels) with one A window per tile.  Tile = 128 staging rows x one
// group; the 31 taps read rows kb .. kb + 127 of a 160-row window loaded once
// from row m0 - 30 (TMA rows before the buffer read as zero; the staging
// layout's 32 zero rows before each sequence are the causal padding).  The
// 128B swizzle is applied on absolute shared-memory address bits, so a tap's
// operand is the window's descriptor advanced by kb rows (kb x 128 bytes).
// The per-tap [64 out x 64 in] weight slices stream through their own ring.
// A traffic per tile: 20 KB instead of 31 x 16 KB.
// A work item is ROWT consecutive tiles of one group: each weight slice feeds
// ROWT x 4 MMAs per barrier wait (a wait on an mbarrier costs about as long as
// the four N = 64 MMAs of one tile, which left the tensor pipe three quarters
// idle with one tile per item) and is read from L2 ROWT times less often.
// Measured on the config-3 decode: 18.8 ms (one tile), 14.2 (two), 12.8
// (three), 12.2 (four).  Fewer, longer items fill fewer SMs, so the host picks
// ROWT per launch from the row count (conv_pos, gemm.cu).
//   warp 0      TMA: A windows (2 slots x ROWT), weight slices (conv_bstages slots)
//   warp 1      TMEM allocator; lane 0 issues tcgen05.mma (M=128, N=64, K=16)
//   warps 2..17 epilogue, four per TMEM lane quarter, 16 columns each
// ---------------------------------------------------------------------------
constexpr int CONV_WIN_BYTES = CONV_WIN_ROWS * 128;
// ROWT = 128-row tiles per work item (1, 2 or 4), sharing each weight slice;
// the weight ring shrinks at 4 so that four pairs of windows fit.
__host__ __device__ constexpr int conv_bstages(int rowt) { return rowt >= 4 ? 6 : 12; }
constexpr int CONV_THREADS = 64 + 16 * 32;
__host__ __device__ constexpr int conv_win_smem_bytes(int rowt) {
  return 1024 + 2 * rowt * CONV_WIN_BYTES + conv_bstages(rowt) * 64 * 128 + 512;
}

template <int ROWT, class Epi>
__global__ void __launch_bounds__(CONV_THREADS, 1)
    k_conv_win(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, GemmShape sh,
               Epi epi) {
  constexpr int BN = 64;
  constexpr int B_BYTES = 64 * 128;
  constexpr int BSTAGES = conv_bstages(ROWT);
  constexpr int ACC_COLS = ROWT * BN;          // one accumulator set: ROWT tiles of 64 columns
  // two sets, double-buffered against the epilogue (allocated as a power of two)
  constexpr uint32_t TMEM_COLS = 2 * ACC_COLS <= 256 ? 256 : 512;
  static_assert(2 * ACC_COLS <= 512, "two accumulator sets fit in tensor memory");
  constexpr uint32_t IDESC = idesc_bf16_f32(GEMM_BM, BN);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;  // 2 slots x ROWT windows
  uint8_t* sB = smem + 2 * ROWT * CONV_WIN_BYTES;
  uint64_t* a_full = reinterpret_cast<uint64_t*>(sB + BSTAGES * B_BYTES);
  uint64_t* a_empty = a_full + 2;
  uint64_t* full = a_empty + 2;
  uint64_t* empty = full + BSTAGES;
  uint64_t* tfull = empty + BSTAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&a_full[i], 1);
      mbar_init(&a_empty[i], 1);
      mbar_init(&tfull[i], 1);
      mbar_init(&tempty[i], 16);
    }
    for (int i = 0; i < BSTAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_launch_dependents();
  pdl_wait();

  constexpr int ITEM_ROWS = ROWT * GEMM_BM;
  const int tiles_n = sh.N / BN;
  const int n_items = ((sh.M + ITEM_ROWS - 1) / ITEM_ROWS) * tiles_n;

  if (warp == 0) {
    if (lane == 0) {
      int as = 0, bs = 0;
      uint32_t aph = 0, bph = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < n_items; item += gridDim.x) {
        const int m0 = (item / tiles_n) * ITEM_ROWS;
        const int n0 = (item % tiles_n) * BN;  // group g = n0 / 64
        if (!(ok = mbar_wait(&a_empty[as], aph ^ 1u, sh.err, abort_flag, DEV_TIMEOUT_PRODUCER))) break;
        // a tile wholly past the last row is not loaded: its accumulator rows
        // are never stored
        const int nt = min(ROWT, (sh.M - m0 + GEMM_BM - 1) / GEMM_BM);
        mbar_arrive_expect_tx(&a_full[as], static_cast<uint32_t>(nt * CONV_WIN_BYTES));
        for (int r = 0; r < nt; ++r)
          tma_load_2d(sA + (as * ROWT + r) * CONV_WIN_BYTES, &tmA, &a_full[as], n0,
                      m0 + r * GEMM_BM - (CONV_TAPS - 1));
        if (++as == 2) {
          as = 0;
          aph ^= 1u;
        }
        for (int kb = 0; kb < CONV_TAPS; ++kb) {
          if (!(ok = mbar_wait(&empty[bs], bph ^ 1u, sh.err, abort_flag, DEV_TIMEOUT_PRODUCER))) break;
          mbar_arrive_expect_tx(&full[bs], B_BYTES);
          tma_load_2d(sB + bs * B_BYTES, &tmB, &full[bs], 0, sh.b_off + ((n0 / 64) * CONV_TAPS + kb) * 64);
          if (++bs == BSTAGES) {
            bs = 0;
            bph ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int as = 0, bs = 0, acc = 0;
      uint32_t aph = 0, bph = 0, acc_phase = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < n_items; item += gridDim.x) {
        if (!(ok = mbar_wait(&tempty[acc], acc_phase ^ 1u, sh.err, abort_flag, DEV_TIMEOUT_MMA))) break;
        if (!(ok = mbar_wait(&a_full[as], aph, sh.err, abort_flag, DEV_TIMEOUT_MMA))) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * ACC_COLS);
        const uint32_t wa = smem_u32(sA + as * ROWT * CONV_WIN_BYTES);
        for (int kb = 0; kb < CONV_TAPS; ++kb) {
          if (!(ok = mbar_wait(&full[bs], bph, sh.err, abort_flag, DEV_TIMEOUT_MMA))) break;
          tc_fence_after();
          const uint64_t db = sdesc_sw128(smem_u32(sB + bs * B_BYTES));
#pragma unroll
          for (int r = 0; r < ROWT; ++r) {
            const uint64_t da =
                sdesc_sw128(wa + static_cast<uint32_t>(r * CONV_WIN_BYTES) + static_cast<uint32_t>(kb) * 128u);
#pragma unroll
            for (int k = 0; k < GEMM_BK / 16; ++k)
              umma_ss(d_tmem + static_cast<uint32_t>(r * BN), da + 2 * k, db + 2 * k, IDESC,
                      (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty[bs]);
          if (++bs == BSTAGES) {
            bs = 0;
            bph ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&a_empty[as]);
        if (++as == 2) {
          as = 0;
          aph ^= 1u;
        }
        umma_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
    }
  } else {
    const int q = warp & 3;
    const int c0 = ((warp - 2) >> 2) * 16;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
      const int m0 = (item / tiles_n) * ITEM_ROWS;
      const int n0 = (item % tiles_n) * BN;
      const bool ok = mbar_wait(&tfull[acc], acc_phase, sh.err, abort_flag, DEV_TIMEOUT_EPILOGUE);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const int rt = q * 32 + lane;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc * ACC_COLS);
#pragma unroll
      for (int r = 0; r < ROWT; ++r) {
        float va[16];
        tmem_ld16(t_row + static_cast<uint32_t>(r * BN) + c0, va);
        tmem_ld_wait();
        epi_chunk<false>(epi, nullptr, rt, m0 + r * GEMM_BM + rt, n0, c0, sh, va);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

}  // namespace lx
