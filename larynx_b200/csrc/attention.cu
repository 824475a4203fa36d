// Fused flash attention for the DiT blocks on sm_100a (tcgen05 + TMEM).
//
// Persistent: two CTAs per SM (256 threads, 128 registers per thread at
// launch, 99 KB of shared memory and 256 tensor-memory columns each) walk the
// work items (128-query block, head), head_dim = 64; the host orders the
// blocks longest first and CTA c takes items c, c + grid, ...  Two resident
// CTAs keep the MUFU units busy: while one loads its scores, reduces the row
// max or stores P, the other one's exponentials run.  Within a CTA the next
// item's Q (double-buffered) and first QK^T run under the current item's last
// softmax step, so there is no per-item prologue or launch gap.
//
// Tensor memory (256 columns): S [0,128), P [128,192) (fp16 pairs), O [192,256).
//   warp 0      TMA: each item's Q tile (2 slots), then its K tiles [128 keys x
//               64] (bf16) through a 2-slot ring released as soon as QK^T has
//               read them
//   warp 2      TMA: the V tiles [128 keys x 64] (fp16, row-major as the QKV
//               GEMM wrote it; the PV MMA reads it as an MN-major operand, so
//               no transpose exists anywhere) through a 2-slot ring released
//               after PV.  Separate rings keep the K load of tile j+1 off the
//               softmax -> PV -> release chain of tile j-1.
//   warp 1      lane 0 issues the MMAs: S = Q K^T (M=128, N=128, K=64, bf16)
//               one key tile ahead of the softmax (across item boundaries),
//               then O += P V (M=128, N=64, K=128, fp16, P read from tensor
//               memory; an item's first PV waits until the softmax has read
//               the previous item's O)
//   warp 3      idle (warpgroup 0 lowers its registers with setmaxnreg)
//   warps 4..7  softmax: thread = query row; S row from TMEM into registers,
//               key-padding / block-causal mask on boundary tiles only,
//               online softmax in the exp2 domain (fp32 row sum), P written
//               as packed fp16 into its own TMEM columns (P never touches
//               shared memory, whose bandwidth the MMA operands need).  O is
//               rescaled in place only when a row's running max grows by more
//               than 2^8 (the reference max is otherwise kept, which is exact).
// No score matrix ever reaches HBM.
#include "common.cuh"
#include "kernels.h"

namespace lx {

namespace {

constexpr int ATT_THREADS = 256;  // warpgroup 0: K TMA, MMA, V TMA, idle; warpgroup 1: softmax
// Register split with setmaxnreg: the block is launched with 256 x 128 = 32768
// registers (two blocks per SM); warpgroup 0 drops to 48, warpgroup 1 rises
// to 208: 128 x 48 + 128 x 208 = 32768.  attention() checks the launch
// register count before the first launch, so the raise can always be met.
constexpr int ATT_LAUNCH_REGS = 128;
constexpr int REGS_PRODUCER = 48;
constexpr int REGS_SOFTMAX = 208;
static_assert(128 * REGS_PRODUCER + 128 * REGS_SOFTMAX <= ATT_THREADS * ATT_LAUNCH_REGS, "register split");
constexpr int ATT_STAGES = 2;
constexpr int Q_BYTES = 128 * 64 * 2;  // 16 KB
constexpr int K_BYTES = 128 * 64 * 2;  // 16 KB
constexpr int V_BYTES = 128 * 64 * 2;  // 16 KB: 128 keys x 64 fp16 values (MN-major B of PV)
constexpr int ATT_SMEM = 1024 + 2 * Q_BYTES + ATT_STAGES * (K_BYTES + V_BYTES) + 256;
constexpr uint32_t ATT_TMEM_COLS = 256;
constexpr uint32_t S_COL = 0, P_COL = 128, O_COL = 192;
constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units: P <= 2^8

// S = Q K^T from precomputed descriptors (start address advanced by 32 B = 2
// units per K=16 step; smem addresses stay below 2^18, so no carry leaves the
// 14-bit start-address field)
__device__ __forceinline__ void issue_s(uint32_t d, uint64_t dq, uint64_t dk) {
  constexpr uint32_t IDESC_S = idesc_bf16_f32(128, 128);
#pragma unroll
  for (int k = 0; k < 4; ++k) umma_ss(d, dq + 2 * k, dk + 2 * k, IDESC_S, k > 0 ? 1u : 0u);
}

// O (+)= P V: P (fp16, 128 keys = 64 TMEM columns) from TMEM, V (fp16, key
// rows of 64 values) from smem as an MN-major operand: K step kk = keys
// 16 kk .. 16 kk + 15 starts 16 rows x 128 B = 2048 B further
__device__ __forceinline__ void issue_pv(uint32_t d, uint32_t p_tmem, uint64_t dv, bool accumulate) {
  constexpr uint32_t IDESC_O = idesc_f16_f32(128, HDIM) | IDESC_B_MN_MAJOR;
#pragma unroll
  for (int kk = 0; kk < 8; ++kk)
    umma_ts(d, p_tmem + kk * 8, dv + static_cast<uint64_t>(kk * (2048 >> 4)), IDESC_O,
            (accumulate || kk > 0) ? 1u : 0u);
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]), "f"(v[8]),
      "f"(v[9]), "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15]), "f"(v[16]), "f"(v[17]),
      "f"(v[18]), "f"(v[19]), "f"(v[20]), "f"(v[21]), "f"(v[22]), "f"(v[23]), "f"(v[24]), "f"(v[25]), "f"(v[26]),
      "f"(v[27]), "f"(v[28]), "f"(v[29]), "f"(v[30]), "f"(v[31])
      : "memory");
}

__device__ __forceinline__ void tmem_st32u(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
      "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]),
      "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]),
      "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

template <int N>
__device__ __forceinline__ void regs_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void regs_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 2^x for a pair on the FMA pipe, for x <= 8 (the lazy-rescale bound; -inf
// allowed): x is clamped to -125 (2^-125 becomes 0 in fp16 and is negligible
// in the fp32 row sum), split as n + f with n = round(x) by the 1.5 * 2^23
// shifter and f in [-0.5, 0.5], 2^f from a cubic fitted to 2^f on [-0.5, 0.5]
// for minimum maximum relative error (weighted least squares, max relative
// error 7.5e-5, below the 4.9e-4 fp16 rounding of P), and 2^n added to the
// exponent field.  Its use offloads part of the exponentials from the MUFU
// units, which bound the softmax.
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  constexpr float SHIFT = 12582912.0f;  // 1.5 * 2^23
  x.x = fmaxf(x.x, -125.0f);
  x.y = fmaxf(x.y, -125.0f);
  const float2 t = __fadd2_rn(x, make_float2(SHIFT, SHIFT));
  const float2 n = __fadd2_rn(t, make_float2(-SHIFT, -SHIFT));
  const float2 f = __fadd2_rn(x, make_float2(-n.x, -n.y));
  float2 p = __ffma2_rn(make_float2(0.055171654f, 0.055171654f), f, make_float2(0.24261113f, 0.24261113f));
  p = __ffma2_rn(p, f, make_float2(0.69326097f, 0.69326097f));
  p = __ffma2_rn(p, f, make_float2(0.99992806f, 0.99992806f));
  // low 9 bits of the shifter's bit pattern hold n (two's complement)
  const uint32_t ex = __float_as_uint(t.x) << 23, ey = __float_as_uint(t.y) << 23;
  return make_float2(__uint_as_float(__float_as_uint(p.x) + ex), __uint_as_float(__float_as_uint(p.y) + ey));
}

// Pairs of a 32-score chunk whose exponentials run on the FMA pipe (bit i =
// pair i).  0: the softmax is bound by issue slots, not by the MUFU units, at
// this head size, so every exponential stays on MUFU.
constexpr uint32_t ATT_POLY_PAIRS = 0x0000u;

// p = 2^(s * sl2 - m) for 32 scores (packed f32x2 FMA, MUFU ex2 or the FMA
// polynomial), their fp32 sum added to (acc0, acc1), and the 32
// probabilities packed as 16 fp16 pairs.
__device__ __forceinline__ void exp_chunk32(const float* s, float sl2, float m, float2& acc0, float2& acc1,
                                            uint32_t* pk) {
  const float2 scale = make_float2(sl2, sl2);
  const float2 neg_m = make_float2(-m, -m);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float2 x = __ffma2_rn(make_float2(s[2 * i], s[2 * i + 1]), scale, neg_m);
    const float2 p = ((ATT_POLY_PAIRS >> i) & 1u) ? exp2_poly2(x) : make_float2(ex2(x.x), ex2(x.y));
    if (i & 1)
      acc1 = __fadd2_rn(acc1, p);
    else
      acc0 = __fadd2_rn(acc0, p);
    pk[i] = pack_f16x2(p.x, p.y);
  }
}

// One work item = (query block, head); items are numbered block-major (the
// host sorts blocks longest first) and CTA c takes items c, c + grid, ...
struct AttnItem {
  AttnTile t;
  int head, nq, nkv;
};

__device__ __forceinline__ AttnItem item_of(const AttnTile& t, int idx, int chunk) {
  AttnItem it;
  it.t = t;
  it.head = idx % HEADS;
  it.nq = min(128, it.t.seq_len - it.t.q0);
  // keys visible to the last query of the block
  int kv_end = it.t.seq_len;
  if (chunk > 0) kv_end = min(it.t.seq_len, ((it.t.q0 + it.nq - 1) / chunk + 1) * chunk);
  it.nkv = (kv_end + 127) / 128;
  return it;
}

// The query block of work item idx (or an empty one past the last item).  A
// role reads the next item's block while it works on the current one, so the
// global-memory latency of the read stays off the item boundary (measured:
// attention 2.8% faster at the same clock).
__device__ __forceinline__ AttnTile tile_of(const AttnTile* __restrict__ tiles, int idx, int n_items) {
  return idx < n_items ? tiles[idx / HEADS] : AttnTile{0, 1, 0, 0};
}

__global__ void __launch_bounds__(ATT_THREADS, 2)
    k_attention(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, const AttnTile* __restrict__ tiles, int n_items, int chunk,
                bf16* __restrict__ out, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;  // 2 slots: the next item's Q loads under the current item
  uint8_t* sK = sQ + 2 * Q_BYTES;
  uint8_t* sV = sK + ATT_STAGES * K_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + ATT_STAGES * V_BYTES);
  uint64_t* q_full = bars;       // [2]
  uint64_t* q_empty = bars + 2;  // [2]
  uint64_t* k_full = bars + 4;
  uint64_t* k_empty = k_full + ATT_STAGES;
  uint64_t* v_full = k_empty + ATT_STAGES;
  uint64_t* v_empty = v_full + ATT_STAGES;
  uint64_t* s_full = v_empty + ATT_STAGES;
  uint64_t* s_empty = s_full + 1;
  uint64_t* p_full = s_empty + 1;
  uint64_t* o_done = p_full + 1;
  uint64_t* o_free = o_done + 1;  // the softmax has read the finished O of an item
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_free + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int grid = gridDim.x;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    for (int s = 0; s < ATT_STAGES; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_empty, 4);
    mbar_init(p_full, 4);
    mbar_init(o_done, 1);
    mbar_init(o_free, 4);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, ATT_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_launch_dependents();
  pdl_wait();

  if (warp < 4) {
    regs_dec<REGS_PRODUCER>();
    if (warp == 0) {
      if (lane == 0) {
        // Q of every item, then its K tiles (global step g: ring slot g % 2)
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
        bool ok = true;
        int g = 0, n = 0;
        AttnTile next_t = tile_of(tiles, blockIdx.x, n_items);
        for (int idx = blockIdx.x; ok && idx < n_items; idx += grid, ++n) {
          const AttnItem it = item_of(next_t, idx, chunk);
          next_t = tile_of(tiles, idx + grid, n_items);
          const int qs = n & 1;
          if (!(ok = mbar_wait(&q_empty[qs], ((n >> 1) & 1) ^ 1u, err, abort_flag, DEV_TIMEOUT_PRODUCER))) break;
          mbar_arrive_expect_tx(&q_full[qs], Q_BYTES);
          tma_load_2d(sQ + qs * Q_BYTES, &tmQ, &q_full[qs], it.head * HDIM, it.t.seq_start + it.t.q0);
          for (int j = 0; j < it.nkv; ++j, ++g) {
            const int st = g & 1;
            if (!(ok = mbar_wait(&k_empty[st], ((g >> 1) & 1) ^ 1u, err, abort_flag, DEV_TIMEOUT_PRODUCER))) break;
            mbar_arrive_expect_tx(&k_full[st], K_BYTES);
            tma_load_2d(sK + st * K_BYTES, &tmK, &k_full[st], it.head * HDIM, it.t.seq_start + j * 128);
          }
        }
      }
    } else if (warp == 2) {
      if (lane == 0) {
        bool ok = true;
        int g = 0;
        AttnTile next_t = tile_of(tiles, blockIdx.x, n_items);
        for (int idx = blockIdx.x; ok && idx < n_items; idx += grid) {
          const AttnItem it = item_of(next_t, idx, chunk);
          next_t = tile_of(tiles, idx + grid, n_items);
          for (int j = 0; j < it.nkv; ++j, ++g) {
            const int st = g & 1;
            if (!(ok = mbar_wait(&v_empty[st], ((g >> 1) & 1) ^ 1u, err, abort_flag, DEV_TIMEOUT_PRODUCER))) break;
            mbar_arrive_expect_tx(&v_full[st], V_BYTES);
            tma_load_2d(sV + st * V_BYTES, &tmV, &v_full[st], it.head * HDIM, it.t.seq_start + j * 128);
          }
        }
      }
    } else if (warp == 1) {
      if (lane == 0) {
        // Global step g runs S_g = Q K_g^T, then PV_{g-1}: the QK^T of the next
        // key tile (or of the next item's first tile) is always in flight
        // while the softmax works on the current one.
        const uint64_t dq0 = sdesc_sw128(smem_u32(sQ));
        const uint64_t dk0 = sdesc_sw128(smem_u32(sK));
        const uint64_t dv0 = sdesc_sw128_mn(smem_u32(sV));
        const uint32_t s_t = tmem_base + S_COL;
        const uint32_t p_t = tmem_base + P_COL;
        const uint32_t o_t = tmem_base + O_COL;
        bool ok = true;
        int g = 0, n = 0, prev_j = 0, prev_n = 0;
        // PV of global step gp (key tile jp of the CTA's item np)
        auto issue_pv_step = [&](int gp, int jp, int np) -> bool {
          bool w = mbar_wait(p_full, static_cast<uint32_t>(gp & 1), err, abort_flag, DEV_TIMEOUT_MMA);
          if (w) w = mbar_wait(&v_full[gp & 1], static_cast<uint32_t>((gp >> 1) & 1), err, abort_flag, DEV_TIMEOUT_MMA);
          // the first PV of an item overwrites O: the previous item's O must have been read
          if (w && jp == 0 && np > 0)
            w = mbar_wait(o_free, static_cast<uint32_t>((np - 1) & 1), err, abort_flag, DEV_TIMEOUT_MMA);
          if (!w) return false;
          tc_fence_after();
          issue_pv(o_t, p_t, dv0 + static_cast<uint64_t>(((gp & 1) * V_BYTES) >> 4), jp > 0);
          umma_commit(o_done);
          umma_commit(&v_empty[gp & 1]);
          return true;
        };
        AttnTile next_t = tile_of(tiles, blockIdx.x, n_items);
        for (int idx = blockIdx.x; ok && idx < n_items; idx += grid, ++n) {
          const AttnItem it = item_of(next_t, idx, chunk);
          next_t = tile_of(tiles, idx + grid, n_items);
          const int qs = n & 1;
          const uint64_t dq = dq0 + static_cast<uint64_t>((qs * Q_BYTES) >> 4);
          if (!(ok = mbar_wait(&q_full[qs], static_cast<uint32_t>((n >> 1) & 1), err, abort_flag, DEV_TIMEOUT_MMA)))
            break;
          for (int j = 0; j < it.nkv; ++j, ++g) {
            ok = mbar_wait(&k_full[g & 1], static_cast<uint32_t>((g >> 1) & 1), err, abort_flag, DEV_TIMEOUT_MMA);
            // S_{g-1} must have been read by the softmax before S_g replaces it
            if (ok && g > 0) ok = mbar_wait(s_empty, static_cast<uint32_t>((g - 1) & 1), err, abort_flag, DEV_TIMEOUT_MMA);
            if (!ok) break;
            tc_fence_after();
            issue_s(s_t, dq, dk0 + static_cast<uint64_t>(((g & 1) * K_BYTES) >> 4));
            umma_commit(s_full);
            umma_commit(&k_empty[g & 1]);
            if (j == it.nkv - 1) umma_commit(&q_empty[qs]);
            if (g > 0 && !(ok = issue_pv_step(g - 1, prev_j, prev_n))) break;
            prev_j = j;
            prev_n = n;
          }
        }
        if (ok && g > 0) issue_pv_step(g - 1, prev_j, prev_n);
      }
    }
  } else {
    regs_inc<REGS_SOFTMAX>();
    const int q = warp & 3;       // TMEM lane quarter
    const int r = q * 32 + lane;  // row inside the query block
    const float sl2 = 0.125f * 1.4426950408889634f;  // 1/sqrt(64) * log2(e)
    const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
    bool ok = true;
    int g = 0, n = 0;
    AttnTile next_t = tile_of(tiles, blockIdx.x, n_items);
    for (int idx = blockIdx.x; ok && idx < n_items; idx += grid, ++n) {
      const AttnItem it = item_of(next_t, idx, chunk);
      next_t = tile_of(tiles, idx + grid, n_items);
      const int len = it.t.seq_len;
      const int qi = it.t.q0 + r;
      const int q_chunk = chunk > 0 ? qi / chunk : 0;
      float m_ref = -INFINITY;  // reference max, scaled (log2) units
      float l = 0.f;            // row sum of P relative to m_ref
      // a warp whose 32 rows all lie past the block's last query only keeps
      // the barrier protocol: its P rows feed O rows that are never stored
      const bool live = __any_sync(0xffffffffu, r < it.nq);
      for (int j = 0; j < it.nkv; ++j, ++g) {
        ok = mbar_wait(s_full, static_cast<uint32_t>(g & 1), err, abort_flag, DEV_TIMEOUT_SOFTMAX);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        if (!live) {
          __syncwarp();
          if (lane == 0) mbar_arrive(s_empty);
          // P_g may only be announced after PV_{g-1} retired, as on the live path
          if (g > 0) {
            ok = mbar_wait(o_done, static_cast<uint32_t>((g - 1) & 1), err, abort_flag, DEV_TIMEOUT_SOFTMAX);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(p_full);
          continue;
        }
        float s[128];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          float t[32];
          tmem_ld32(t_lane + S_COL + c * 32, t);
#pragma unroll
          for (int i = 0; i < 32; ++i) s[c * 32 + i] = t[i];
        }
        tmem_ld_wait();
        // the S columns may now be overwritten by the next QK^T
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(s_empty);

        // visible keys of this row form a prefix of the tile (key padding and
        // the block-causal rule both cut at an upper bound): mask past it
        const int key0 = j * 128;
        int vis_end = len;
        if (chunk > 0) vis_end = min(vis_end, (q_chunk + 1) * chunk);
        const int nvalid = vis_end - key0;
        if (nvalid < 128) {
#pragma unroll
          for (int c = 0; c < 128; ++c) s[c] = c < nvalid ? s[c] : -INFINITY;
        }
        // 32-key chunks past every row's visible prefix hold p = 0 exactly:
        // they are stored as zeros without running their exponentials
        const int nv_warp = __reduce_max_sync(0xffffffffu, nvalid);
        float mx[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) mx[k] = fmaxf(s[k], s[k + 8]);
#pragma unroll
        for (int c = 16; c < 128; c += 16) {
#pragma unroll
          for (int k = 0; k < 8; ++k) mx[k] = max3(mx[k], s[c + k], s[c + 8 + k]);
        }
        const float rmax = max3(max3(mx[0], mx[1], mx[2]), max3(mx[3], mx[4], mx[5]), fmaxf(mx[6], mx[7]));
        const float m_cand = rmax * sl2;
        const bool need = m_cand > m_ref + RESCALE_THRESHOLD;  // false when rmax == -inf
        bool waited = false;
        if (__any_sync(0xffffffffu, need)) {
          const float new_ref = need ? m_cand : m_ref;
          const float alpha = need ? ex2(m_ref - new_ref) : 1.0f;  // 0 from -inf
          if (j > 0) {
            // PV_{g-1} is the last update of O before this in-place rescale
            ok = mbar_wait(o_done, static_cast<uint32_t>((g - 1) & 1), err, abort_flag, DEV_TIMEOUT_SOFTMAX);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            tc_fence_after();
            waited = true;
#pragma unroll 1
            for (int h = 0; h < 2; ++h) {
              float t[32];
              tmem_ld32(t_lane + O_COL + h * 32, t);
              tmem_ld_wait();
#pragma unroll
              for (int i = 0; i < 32; ++i) t[i] *= alpha;
              tmem_st32(t_lane + O_COL + h * 32, t);
            }
            tmem_st_wait();
          }
          l *= alpha;
          m_ref = new_ref;
        }
        const float m_use = (m_ref == -INFINITY) ? 0.f : m_ref;
        // p = 2^(s*scale - m) in fp32, row sum in fp32, P packed as fp16
        // pairs; stored to TMEM in two 64-key halves
        float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t pk[32];
          if (64 * h < nv_warp) {
            exp_chunk32(s + 64 * h, sl2, m_use, acc0, acc1, pk);
          } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) pk[i] = 0u;
          }
          if (64 * h + 32 < nv_warp) {
            exp_chunk32(s + 64 * h + 32, sl2, m_use, acc0, acc1, pk + 16);
          } else {
#pragma unroll
            for (int i = 16; i < 32; ++i) pk[i] = 0u;
          }
          if (h == 0 && g > 0 && !waited) {
            // PV_{g-1} (possibly the previous item's last) must have read
            // P_{g-1} before P_g replaces it
            ok = mbar_wait(o_done, static_cast<uint32_t>((g - 1) & 1), err, abort_flag, DEV_TIMEOUT_SOFTMAX);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            tc_fence_after();
          }
          tmem_st32u(t_lane + P_COL + 32 * h, pk);
        }
        if (!ok) break;
        l += (acc0.x + acc0.y) + (acc1.x + acc1.y);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full);
      }
      if (!ok) break;
      // the item's O is final after its last PV (global step g - 1)
      ok = mbar_wait(o_done, static_cast<uint32_t>((g - 1) & 1), err, abort_flag, DEV_TIMEOUT_SOFTMAX);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      if (!live) {
        __syncwarp();
        if (lane == 0) mbar_arrive(o_free);
        continue;
      }
      float o[64];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float t[32];
        tmem_ld32(t_lane + O_COL + h * 32, t);
#pragma unroll
        for (int i = 0; i < 32; ++i) o[h * 32 + i] = t[i];
      }
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_free);
      const float inv = 1.0f / l;
      if (r < it.nq) {
        bf16* dst = out + static_cast<size_t>(it.t.seq_start + qi) * DIM + it.head * HDIM;
#pragma unroll
        for (int c = 0; c < 4; ++c)
          st_global_v8(dst + 16 * c, pack_bf16x2(o[16 * c + 0] * inv, o[16 * c + 1] * inv),
                       pack_bf16x2(o[16 * c + 2] * inv, o[16 * c + 3] * inv),
                       pack_bf16x2(o[16 * c + 4] * inv, o[16 * c + 5] * inv),
                       pack_bf16x2(o[16 * c + 6] * inv, o[16 * c + 7] * inv),
                       pack_bf16x2(o[16 * c + 8] * inv, o[16 * c + 9] * inv),
                       pack_bf16x2(o[16 * c + 10] * inv, o[16 * c + 11] * inv),
                       pack_bf16x2(o[16 * c + 12] * inv, o[16 * c + 13] * inv),
                       pack_bf16x2(o[16 * c + 14] * inv, o[16 * c + 15] * inv));
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, ATT_TMEM_COLS);
  }
}

}  // namespace

bool attention_ready() {
  static int checked[64] = {0};  // 0 unchecked, 1 ok, -1 unusable
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  int& state = checked[dev & 63];
  if (state == 0) {
    // setmaxnreg.inc waits for registers the block was launched with: refuse
    // to launch unless the launch register count covers the split
    cudaFuncAttributes fa;
    state = (cudaFuncGetAttributes(&fa, k_attention) == cudaSuccess && fa.numRegs >= ATT_LAUNCH_REGS &&
             cudaFuncSetAttribute(k_attention, cudaFuncAttributeMaxDynamicSharedMemorySize, ATT_SMEM) ==
                 cudaSuccess)
                ? 1
                : -1;
  }
  return state > 0;
}

bool attention(const CUtensorMap& Q, const CUtensorMap& K, const CUtensorMap& V, const AttnTile* tiles,
               int n_tiles, int chunk, bf16* out, int* err, cudaStream_t s) {
  if (n_tiles <= 0) return true;
  if (!attention_ready() || n_tiles > ATT_MAX_TILES) return false;
  // persistent: two CTAs per SM walk the (block, head) items
  const int n_items = n_tiles * HEADS;
  const int grid = n_items < 2 * num_sms() ? n_items : 2 * num_sms();
  launch_pdl(k_attention, dim3(grid), dim3(ATT_THREADS), ATT_SMEM, s, Q, K, V, tiles, n_items, chunk, out, err);
  return true;
}

}  // namespace lx
