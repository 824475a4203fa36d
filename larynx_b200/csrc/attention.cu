// Fused flash attention for the DiT blocks on sm_100a (tcgen05 + TMEM).
//
// One CTA = one (sequence, 256-query block, head), head_dim = 64, processed as
// two 128-row sub-tiles that ping-pong on the tensor core.  Warpgroup 0 is the
// producer (registers lowered with setmaxnreg), warpgroups 1 and 2 run the
// softmax of sub-tiles 0 and 1 (registers raised):
//   warp 0      TMA: both Q sub-tiles once, then per stage the K tile
//               [128 keys x 64] and the transposed fp16 V tile [64 x 128 keys]
//   warp 1      TMEM allocation; lane 0 issues, per key tile j and sub-tile i,
//               S_i = Q_i K_j^T (M=128, N=128, K=64, bf16) into TMEM and
//               O_i += P_i V_j (M=128, N=64, K=128, fp16) into TMEM, in the
//               order PV_0,j -> S_0,j+1 -> PV_1,j -> S_1,j+1 so that the
//               softmax of one sub-tile overlaps the MMAs of the other
//   warps 2..3  idle
//   warps 4..7  softmax of sub-tile 0, warps 8..11 softmax of sub-tile 1:
//               thread = query row; its S row is pulled from TMEM into
//               registers (releasing the S columns to the next QK^T at once),
//               key-padding /
//               block-causal mask on boundary tiles only, fp32 online softmax
//               in the exp2 domain, P written as fp16 into shared memory in
//               the 128B-swizzled K-major layout (P in [0, 256] and V^T are
//               the fp16 operands of the PV MMA).  O stays in TMEM; it is
//               rescaled only when a row's running max grows by more than
//               2^8 (the reference max is otherwise kept, which is exact).
// No score matrix ever reaches HBM.
#include "common.cuh"
#include "kernels.h"

namespace lx {

namespace {

constexpr int ATT_THREADS = 384;  // 3 warpgroups: producer (TMA, MMA, 2 idle), softmax 0, softmax 1
// Register split with setmaxnreg: the block is launched with 384 x 168 = 64512
// registers; producer warpgroup 128 x 56 + softmax warpgroups 256 x 224 = 64512.
constexpr int REGS_PRODUCER = 56;
constexpr int REGS_SOFTMAX = 224;
constexpr int ATT_STAGES = 3;
constexpr int Q_BYTES = 128 * 64 * 2;   // 16 KB per sub-tile
constexpr int K_BYTES = 128 * 64 * 2;   // 16 KB
constexpr int V_BYTES = 64 * 128 * 2;   // 16 KB (two 64-key boxes)
constexpr int P_BYTES = 128 * 128 * 2;  // 32 KB per sub-tile (two 64-key atoms)
constexpr int ATT_SMEM = 1024 + 2 * Q_BYTES + ATT_STAGES * (K_BYTES + V_BYTES) + 2 * P_BYTES + 512;
constexpr uint32_t ATT_TMEM_COLS = 512;
constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units: P <= 2^8

__device__ __forceinline__ uint32_t s_col(int i) { return static_cast<uint32_t>(i * 128); }
__device__ __forceinline__ uint32_t o_col(int i) { return static_cast<uint32_t>(256 + i * 64); }

__device__ __forceinline__ void issue_s(uint32_t d, uint32_t q_addr, uint32_t k_addr) {
  constexpr uint32_t IDESC_S = idesc_bf16_f32(128, 128);
#pragma unroll 1
  for (int k = 0; k < 4; ++k)
    umma_ss(d, sdesc_sw128(q_addr + k * 32), sdesc_sw128(k_addr + k * 32), IDESC_S, k > 0 ? 1u : 0u);
}

__device__ __forceinline__ void issue_pv(uint32_t d, uint32_t p_addr, uint32_t v_addr, bool accumulate) {
  constexpr uint32_t IDESC_O = idesc_f16_f32(128, 64);  // P, V^T in fp16
#pragma unroll 1
  for (int kk = 0; kk < 8; ++kk) {
    const uint32_t pa = p_addr + (kk >> 2) * (P_BYTES / 2) + (kk & 3) * 32;
    const uint32_t va = v_addr + (kk >> 2) * (V_BYTES / 2) + (kk & 3) * 32;
    umma_ss(d, sdesc_sw128(pa), sdesc_sw128(va), IDESC_O, (accumulate || kk > 0) ? 1u : 0u);
  }
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

// (a, b) = (a, b) * s + (c, c) with one packed f32x2 FMA
__device__ __forceinline__ void fma2(float& a, float& b, float s, float c) {
  asm("{\n\t.reg .b64 x, y, z, d;\n\t"
      "mov.b64 x, {%0, %1};\n\t"
      "mov.b64 y, {%2, %2};\n\t"
      "mov.b64 z, {%3, %3};\n\t"
      "fma.rn.f32x2 d, x, y, z;\n\t"
      "mov.b64 {%0, %1}, d;\n\t}"
      : "+f"(a), "+f"(b)
      : "f"(s), "f"(c));
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
template <int N>
__device__ __forceinline__ void regs_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void regs_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__global__ void __launch_bounds__(ATT_THREADS, 1)
    k_attention(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, const AttnTile* __restrict__ tiles, int chunk,
                bf16* __restrict__ out, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                                  // 2 sub-tiles
  uint8_t* sK = sQ + 2 * Q_BYTES;
  uint8_t* sV = sK + ATT_STAGES * K_BYTES;
  uint8_t* sP = sV + ATT_STAGES * V_BYTES;             // 2 sub-tiles
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * P_BYTES);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + ATT_STAGES;
  uint64_t* s_full = kv_empty + ATT_STAGES;  // [2]
  uint64_t* s_empty = s_full + 2;            // [2]
  uint64_t* p_full = s_empty + 2;            // [2]
  uint64_t* o_done = p_full + 2;             // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_done + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const AttnTile tile = tiles[blockIdx.x];
  const int head = blockIdx.y;
  const int len = tile.seq_len;
  const int nq0 = max(0, min(128, len - tile.q0));
  const int nq1 = max(0, min(128, len - tile.q0 - 128));
  const int n_sub = nq1 > 0 ? 2 : 1;
  // keys visible to the last query of the block
  int kv_end = len;
  if (chunk > 0) kv_end = min(len, ((tile.q0 + nq0 + nq1 - 1) / chunk + 1) * chunk);
  const int nkv = (kv_end + 127) / 128;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < ATT_STAGES; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 4);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_done[i], 1);
    }
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

  if (warp < 4) {
    regs_dec<REGS_PRODUCER>();
    if (warp == 0) {
      if (lane == 0) {
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
        mbar_arrive_expect_tx(q_full, Q_BYTES * n_sub);
        for (int i = 0; i < n_sub; ++i)
          tma_load_2d(sQ + i * Q_BYTES, &tmQ, q_full, head * HDIM, tile.seq_start + tile.q0 + 128 * i);
        int stage = 0;
        uint32_t phase = 0;
        for (int j = 0; j < nkv; ++j) {
          if (!mbar_wait(&kv_empty[stage], phase ^ 1u, err, abort_flag, DEV_TIMEOUT_PRODUCER)) break;
          mbar_arrive_expect_tx(&kv_full[stage], K_BYTES + V_BYTES);
          const int key0 = tile.seq_start + j * 128;
          tma_load_2d(sK + stage * K_BYTES, &tmK, &kv_full[stage], head * HDIM, key0);
          tma_load_2d(sV + stage * V_BYTES, &tmV, &kv_full[stage], key0, head * HDIM);
          tma_load_2d(sV + stage * V_BYTES + V_BYTES / 2, &tmV, &kv_full[stage], key0 + 64, head * HDIM);
          if (++stage == ATT_STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
    }
    } else if (warp == 1) {
      if (lane == 0) {
        bool ok = mbar_wait(q_full, 0, err, abort_flag, DEV_TIMEOUT_MMA);
        if (ok) ok = mbar_wait(&kv_full[0], 0, err, abort_flag, DEV_TIMEOUT_MMA);
        if (ok) {
          tc_fence_after();
          for (int i = 0; i < n_sub; ++i) {
            issue_s(tmem_base + s_col(i), smem_u32(sQ + i * Q_BYTES), smem_u32(sK));
            umma_commit(&s_full[i]);
          }
        }
        int stage = 0;
        uint32_t phase = 0;
        for (int j = 0; ok && j < nkv; ++j) {
          int st_n = stage + 1;
          uint32_t ph_n = phase;
          if (st_n == ATT_STAGES) {
            st_n = 0;
            ph_n ^= 1u;
          }
          for (int i = 0; ok && i < n_sub; ++i) {
            // O_i += P_i V_j once the softmax has published P_i (and rescaled O_i)
            ok = mbar_wait(&p_full[i], static_cast<uint32_t>(j & 1), err, abort_flag, DEV_TIMEOUT_MMA);
            if (!ok) break;
            tc_fence_after();
            issue_pv(tmem_base + o_col(i), smem_u32(sP + i * P_BYTES), smem_u32(sV + stage * V_BYTES), j > 0);
            umma_commit(&o_done[i]);
            if (i == n_sub - 1) umma_commit(&kv_empty[stage]);
            // S_i for the next key tile, once the softmax has pulled S_i into registers
            if (j + 1 < nkv) {
              if (i == 0) ok = mbar_wait(&kv_full[st_n], ph_n, err, abort_flag, DEV_TIMEOUT_MMA);
              if (ok) ok = mbar_wait(&s_empty[i], static_cast<uint32_t>(j & 1), err, abort_flag, DEV_TIMEOUT_MMA);
              if (!ok) break;
              tc_fence_after();
              issue_s(tmem_base + s_col(i), smem_u32(sQ + i * Q_BYTES), smem_u32(sK + st_n * K_BYTES));
              umma_commit(&s_full[i]);
            }
          }
          stage = st_n;
          phase = ph_n;
        }
      }
    }
  } else {
    regs_inc<REGS_SOFTMAX>();
    // softmax warpgroup `sub` (warps 4..7 -> sub-tile 0, warps 8..11 -> sub-tile 1)
    const int sub = (warp >> 2) - 1;
    const int q = warp & 3;       // TMEM lane quarter
    const int r = q * 32 + lane;  // row inside the sub-tile
    const int qi = tile.q0 + sub * 128 + r;
    const int q_chunk = chunk > 0 ? qi / chunk : 0;
    const float sl2 = 0.125f * 1.4426950408889634f;  // 1/sqrt(64) * log2(e)
    const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
    uint8_t* p_tile = sP + sub * P_BYTES;
    float m_ref = -INFINITY;  // reference max, scaled (log2) units
    float l = 0.f;
    bool ok = sub < n_sub;
    for (int j = 0; ok && j < nkv; ++j) {
      ok = mbar_wait(&s_full[sub], static_cast<uint32_t>(j & 1), err, abort_flag, DEV_TIMEOUT_SOFTMAX);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      float s[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float t[32];
        tmem_ld32(t_lane + s_col(sub) + c * 32, t);
#pragma unroll
        for (int i = 0; i < 32; ++i) s[c * 32 + i] = t[i];
      }
      tmem_ld_wait();
      // the S columns may now be overwritten by the next QK^T
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[sub]);

      // visible keys of this row form a prefix of the tile (key padding and the
      // block-causal rule both cut at an upper bound): mask past it
      const int key0 = j * 128;
      int vis_end = len;
      if (chunk > 0) vis_end = min(vis_end, (q_chunk + 1) * chunk);
      const int nvalid = vis_end - key0;
      if (nvalid < 128) {
#pragma unroll
        for (int c = 0; c < 128; ++c) s[c] = c < nvalid ? s[c] : -INFINITY;
      }
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
      // O_{sub} for key tile j-1 must be complete before it is rescaled and
      // before P_j overwrites the P tile that PV_{j-1} reads
      if (j > 0) {
        ok = mbar_wait(&o_done[sub], static_cast<uint32_t>((j - 1) & 1), err, abort_flag, DEV_TIMEOUT_SOFTMAX);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
      }
      if (__any_sync(0xffffffffu, need)) {
        const float new_ref = need ? m_cand : m_ref;
        const float alpha = need ? ex2(m_ref - new_ref) : 1.0f;  // 0 from -inf
        if (j > 0) {
#pragma unroll 1
          for (int h = 0; h < 2; ++h) {
            float t[32];
            tmem_ld32(t_lane + o_col(sub) + h * 32, t);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) t[i] *= alpha;
            tmem_st32(t_lane + o_col(sub) + h * 32, t);
          }
          tmem_st_wait();
        }
        l *= alpha;
        m_ref = new_ref;
      }
      const float m_use = (m_ref == -INFINITY) ? 0.f : m_ref;
      // p = 2^(s*scale - m), row sum, fp16 P into the swizzled tile
      float rs[4] = {0.f, 0.f, 0.f, 0.f};
      uint8_t* prow = p_tile + r * 128;
#pragma unroll
      for (int ch = 0; ch < 16; ++ch) {
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
          fma2(s[ch * 8 + i], s[ch * 8 + i + 1], sl2, -m_use);
          s[ch * 8 + i] = ex2(s[ch * 8 + i]);
          s[ch * 8 + i + 1] = ex2(s[ch * 8 + i + 1]);
          rs[(i >> 1) & 3] += s[ch * 8 + i] + s[ch * 8 + i + 1];
        }
        uint4 pk;
        pk.x = pack_f16x2(s[ch * 8 + 0], s[ch * 8 + 1]);
        pk.y = pack_f16x2(s[ch * 8 + 2], s[ch * 8 + 3]);
        pk.z = pack_f16x2(s[ch * 8 + 4], s[ch * 8 + 5]);
        pk.w = pack_f16x2(s[ch * 8 + 6], s[ch * 8 + 7]);
        *reinterpret_cast<uint4*>(prow + (ch >> 3) * (P_BYTES / 2) + (((ch & 7) ^ (r & 7)) << 4)) = pk;
      }
      l += (rs[0] + rs[1]) + (rs[2] + rs[3]);
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[sub]);
    }
    if (ok && sub < n_sub && nkv > 0) {
      ok = mbar_wait(&o_done[sub], static_cast<uint32_t>((nkv - 1) & 1), err, abort_flag, DEV_TIMEOUT_SOFTMAX);
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        tc_fence_after();
        const float inv = 1.0f / l;
        float o[64];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          float t[32];
          tmem_ld32(t_lane + o_col(sub) + h * 32, t);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[h * 32 + i] = t[i] * inv;
        }
        if (r < (sub == 0 ? nq0 : nq1)) {
          uint4* dst =
              reinterpret_cast<uint4*>(out + static_cast<size_t>(tile.seq_start + qi) * DIM + head * HDIM);
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            uint4 pk;
            pk.x = pack_bf16x2(o[c * 8 + 0], o[c * 8 + 1]);
            pk.y = pack_bf16x2(o[c * 8 + 2], o[c * 8 + 3]);
            pk.z = pack_bf16x2(o[c * 8 + 4], o[c * 8 + 5]);
            pk.w = pack_bf16x2(o[c * 8 + 6], o[c * 8 + 7]);
            dst[c] = pk;
          }
        }
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

void attention(const CUtensorMap& Q, const CUtensorMap& K, const CUtensorMap& Vt, const AttnTile* tiles,
               int n_tiles, int chunk, bf16* out, int* err, cudaStream_t s) {
  if (n_tiles <= 0) return;
  static bool attr_done[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!attr_done[dev & 63]) {
    cudaFuncSetAttribute(k_attention, cudaFuncAttributeMaxDynamicSharedMemorySize, ATT_SMEM);
    attr_done[dev & 63] = true;
  }
  dim3 grid(n_tiles, HEADS);
  k_attention<<<grid, ATT_THREADS, ATT_SMEM, s>>>(Q, K, Vt, tiles, chunk, out, err);
}

}  // namespace lx
