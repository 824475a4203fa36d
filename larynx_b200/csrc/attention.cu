// Fused flash attention for the DiT blocks on sm_100a (tcgen05 + TMEM).
//
// One CTA = one (sequence, 128-query tile, head).  head_dim = 64.
//   warp 0      TMA: Q tile once, then K tile [128 keys x 64] and the
//               transposed fp16 V tile [64 x 128 keys] per stage
//   warp 1      TMEM allocation; lane 0 issues S = Q K^T (M=128, N=128, K=64)
//               into TMEM columns [0,128) and O_j = P_j V_j (M=128, N=64,
//               K=128) into TMEM columns [128,192)
//   warps 2..5  softmax: thread = query row; reads its S row from TMEM,
//               applies the key-padding / block-causal mask, online softmax in
//               fp32 (exp2 domain), writes P_j as fp16 into shared memory in
//               the 128B-swizzled K-major layout (P in [0,1] and V^T are the
//               fp16 operands of the PV MMA: 8x finer than bf16 at no cost), accumulates O in registers
//               (o = o * alpha + O_j) and stores the normalised bf16 row.
// The next S MMA is issued as soon as the softmax warps have read S_j into
// registers, so QK^T of tile j+1 overlaps the softmax of tile j.  No score
// matrix ever reaches HBM.
#include "common.cuh"
#include "kernels.h"

namespace lx {

namespace {

constexpr int ATT_THREADS = 192;
constexpr int ATT_STAGES = 3;
constexpr int Q_BYTES = 128 * 64 * 2;   // 16 KB
constexpr int K_BYTES = 128 * 64 * 2;   // 16 KB
constexpr int V_BYTES = 64 * 128 * 2;   // 16 KB (two 64-key boxes)
constexpr int P_BYTES = 128 * 128 * 2;  // 32 KB (two 64-key atoms)
constexpr int ATT_SMEM = 1024 + Q_BYTES + ATT_STAGES * (K_BYTES + V_BYTES) + P_BYTES + 256;
constexpr uint32_t ATT_TMEM_COLS = 256;
constexpr uint32_t S_COL = 0;
constexpr uint32_t O_COL = 128;

__device__ __forceinline__ void issue_s(uint32_t d, uint32_t q_addr, uint32_t k_addr) {
  constexpr uint32_t IDESC_S = idesc_bf16_f32(128, 128);
#pragma unroll
  for (int k = 0; k < 4; ++k)
    umma_ss(d, sdesc_sw128(q_addr + k * 32), sdesc_sw128(k_addr + k * 32), IDESC_S, k > 0 ? 1u : 0u);
}

__global__ void __launch_bounds__(ATT_THREADS, 1)
    k_attention(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, const AttnTile* __restrict__ tiles, int chunk,
                bf16* __restrict__ out, int* err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + Q_BYTES;
  uint8_t* sV = sK + ATT_STAGES * K_BYTES;
  uint8_t* sP = sV + ATT_STAGES * V_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + P_BYTES);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + ATT_STAGES;
  uint64_t* s_full = kv_empty + ATT_STAGES;
  uint64_t* s_empty = s_full + 1;
  uint64_t* p_full = s_empty + 1;
  uint64_t* o_full = p_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_full + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const AttnTile tile = tiles[blockIdx.x];
  const int head = blockIdx.y;
  const int len = tile.seq_len;
  const int nq = min(128, len - tile.q0);
  // keys visible to the last query of the tile
  int kv_end = len;
  if (chunk > 0) kv_end = min(len, ((tile.q0 + nq - 1) / chunk + 1) * chunk);
  const int nkv = (kv_end + 127) / 128;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < ATT_STAGES; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_empty, 4);
    mbar_init(p_full, 4);
    mbar_init(o_full, 1);
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

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(q_full, Q_BYTES);
      tma_load_2d(sQ, &tmQ, q_full, head * HDIM, tile.seq_start + tile.q0);
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
      constexpr uint32_t IDESC_O = idesc_f16_f32(128, 64);  // P, V^T in fp16
      const uint32_t q_addr = smem_u32(sQ);
      const uint32_t p_addr = smem_u32(sP);
      bool ok = mbar_wait(q_full, 0, err, abort_flag, DEV_TIMEOUT_MMA);
      if (ok) ok = mbar_wait(&kv_full[0], 0, err, abort_flag, DEV_TIMEOUT_MMA);
      if (ok) {
        tc_fence_after();
        issue_s(tmem_base + S_COL, q_addr, smem_u32(sK));
        umma_commit(s_full);
      }
      int stage = 0;
      uint32_t phase = 0;
      for (int j = 0; ok && j < nkv; ++j) {
        const int st_j = stage;
        // S_{j+1}, once the softmax warps have pulled S_j into registers
        if (j + 1 < nkv) {
          int st_n = stage + 1;
          uint32_t ph_n = phase;
          if (st_n == ATT_STAGES) {
            st_n = 0;
            ph_n ^= 1u;
          }
          if (!mbar_wait(&kv_full[st_n], ph_n, err, abort_flag, DEV_TIMEOUT_MMA)) break;
          if (!mbar_wait(s_empty, static_cast<uint32_t>(j & 1), err, abort_flag, DEV_TIMEOUT_MMA)) break;
          tc_fence_after();
          issue_s(tmem_base + S_COL, q_addr, smem_u32(sK + st_n * K_BYTES));
          umma_commit(s_full);
        }
        // O_j = P_j V_j
        if (!mbar_wait(p_full, static_cast<uint32_t>(j & 1), err, abort_flag, DEV_TIMEOUT_MMA)) break;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sV + st_j * V_BYTES);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t pa = p_addr + (kk >> 2) * (P_BYTES / 2) + (kk & 3) * 32;
          const uint32_t va = v_addr + (kk >> 2) * (V_BYTES / 2) + (kk & 3) * 32;
          umma_ss(tmem_base + O_COL, sdesc_sw128(pa), sdesc_sw128(va), IDESC_O, kk > 0 ? 1u : 0u);
        }
        umma_commit(&kv_empty[st_j]);
        umma_commit(o_full);
        if (++stage == ATT_STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else {
    // softmax warps: TMEM lane quarter q holds rows q*32 .. q*32+31
    const int q = warp & 3;
    const int r = q * 32 + lane;  // row inside the tile
    const int qi = tile.q0 + r;   // query index inside the sequence
    const int q_chunk = chunk > 0 ? qi / chunk : 0;
    const float sl2 = 0.125f * 1.4426950408889634f;  // 1/sqrt(64) * log2(e)
    const uint32_t t_lane = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
    float m = -INFINITY, l = 0.f, a_prev = 1.f;
    float o[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) o[i] = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv; ++j) {
      ok = mbar_wait(s_full, static_cast<uint32_t>(j & 1), err, abort_flag, DEV_TIMEOUT_SOFTMAX);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      float s[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float t[32];
        tmem_ld32(t_lane + S_COL + c * 32, t);
#pragma unroll
        for (int i = 0; i < 32; ++i) s[c * 32 + i] = t[i];
      }
      tmem_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_empty);

      // mask + scale + row max
      const int key0 = j * 128;
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 128; ++c) {
        const int key = key0 + c;
        bool vis = key < len;
        if (chunk > 0) vis = vis && (key / chunk <= q_chunk);
        s[c] = vis ? s[c] * sl2 : -INFINITY;
        mx = fmaxf(mx, s[c]);
      }
      const float m_new = fmaxf(m, mx);
      const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
      const float alpha = exp2f(m - m_use);  // m == -inf -> 0
      float rs = 0.f;
#pragma unroll
      for (int c = 0; c < 128; ++c) {
        s[c] = exp2f(s[c] - m_use);
        rs += s[c];
      }
      l = l * alpha + rs;
      m = m_new;

      // PV_{j-1} must be complete before P_j overwrites the shared P tile
      if (j > 0) {
        ok = mbar_wait(o_full, static_cast<uint32_t>((j - 1) & 1), err, abort_flag, DEV_TIMEOUT_SOFTMAX);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
      }
      // P_j -> shared memory (bf16, 128B swizzle, K-major), row r
      {
        uint8_t* prow = sP + r * 128;
#pragma unroll
        for (int ch = 0; ch < 16; ++ch) {
          const int atom = ch >> 3;
          const int c16 = ch & 7;
          uint4 pk;
          pk.x = pack_f16x2(s[ch * 8 + 0], s[ch * 8 + 1]);
          pk.y = pack_f16x2(s[ch * 8 + 2], s[ch * 8 + 3]);
          pk.z = pack_f16x2(s[ch * 8 + 4], s[ch * 8 + 5]);
          pk.w = pack_f16x2(s[ch * 8 + 6], s[ch * 8 + 7]);
          *reinterpret_cast<uint4*>(prow + atom * (P_BYTES / 2) + ((c16 ^ (r & 7)) << 4)) = pk;
        }
      }
      // fold O_{j-1} (relative to the previous max) into the register
      // accumulator before PV_j may overwrite the O columns
      if (j > 0) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          float t[32];
          tmem_ld32(t_lane + O_COL + h * 32, t);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[h * 32 + i] = o[h * 32 + i] * a_prev + t[i];
        }
      }
      a_prev = alpha;
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    if (ok && nkv > 0) {
      ok = mbar_wait(o_full, static_cast<uint32_t>((nkv - 1) & 1), err, abort_flag, DEV_TIMEOUT_SOFTMAX);
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        tc_fence_after();
        const float inv = 1.0f / l;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          float t[32];
          tmem_ld32(t_lane + O_COL + h * 32, t);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[h * 32 + i] = (o[h * 32 + i] * a_prev + t[i]) * inv;
        }
        if (r < nq) {
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
