// Host-side interface of the Flow kernels (launchers).  All launches are
// asynchronous on the given stream; every kernel that waits on an mbarrier
// reports a timeout through the device error word `err`.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace lx {

typedef __nv_bfloat16 bf16;

constexpr int DIM = 1024;
constexpr int FF = 2048;
constexpr int MEL = 80;
constexpr int HEADS = 16;
constexpr int HDIM = 64;
constexpr int DEPTH = 22;
constexpr int QKV_N = 3 * DIM;
constexpr int MOD_N = 6 * DIM;
constexpr int CONV_K = 31;
constexpr int CONV_G = 16;
constexpr int COND_K = 3 * MEL;  // [cond, mu, spks] columns of the input projection
constexpr int PRE_LOOKAHEAD = 3;  // PreLookaheadLayer look-ahead tokens

// Number of SMs of the current device (cached per device).
int num_sms();

// Launch with programmatic stream serialization (see pdl_wait in common.cuh):
// the kernel may start while the previous kernel of the stream drains, and
// waits for it inside before touching memory.
// LX_FLOW_PDL=1 in the environment turns the attribute on (off by default).
bool pdl_enabled();
// Per-thread default of pdl_enabled() when LX_FLOW_PDL is unset.
void pdl_set_auto(bool on);
// Batch plans of at most this many packed rows launch with PDL by default
// (latency-bound: the single 20 s utterance is 2 x 1000 rows).
constexpr int PDL_AUTO_MAX_ROWS = 4096;
// Rows per block of the warp-per-row kernels: LX_FLOW_ROWS_PER_BLOCK when set,
// else `dflt` (the decode uses 8; the standalone ops 0); 0 = as many as
// spread the rows over every SM in one wave, at most 16.
int rows_per_block(int R, int dflt = 8);

template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                       Args... args) {
  if (!pdl_enabled()) {
    kernel<<<grid, block, smem, s>>>(static_cast<KArgs>(args)...);
    return;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// 2-D tensor map over 16-bit elements (bf16, or fp16 data: TMA copies bits):
// `rows` x `cols` elements, row stride `ld` elements, box = box_rows x
// box_cols (box_cols * 2 == 128 selects the 128B swizzle).
bool tmap_bf16(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows,
               uint32_t box_cols);
// same over fp32 elements (box_cols * 4 == 128 selects the 128B swizzle)
bool tmap_f32(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint64_t ld, uint32_t box_rows,
              uint32_t box_cols);

// Rows of the conv-pos A window (128 output rows + 30 taps, rounded to 8):
// the box height of the conv's staging tensor maps.
constexpr int CONV_WIN_ROWS = 160;

constexpr int ROPE_MAX = 16384;  // positions covered by the rotary tables

// Query rows per attention CTA.
constexpr int ATT_Q_ROWS = 128;

struct AttnTile {
  int seq_start;  // first packed row of the sequence
  int seq_len;    // valid frames of the sequence
  int q0;         // first query of this block (multiple of ATT_Q_ROWS), relative to seq_start
  int pad;
};

// Keys visible to the last query of tile t (the keys the attention CTA of t
// walks): the sequence length, or the end of that query's chunk.
inline int attn_tile_keys(const AttnTile& t, int chunk) {
  const int nq = t.seq_len - t.q0 < ATT_Q_ROWS ? t.seq_len - t.q0 : ATT_Q_ROWS;
  if (chunk <= 0) return t.seq_len;
  const int end = ((t.q0 + nq - 1) / chunk + 1) * chunk;
  return end < t.seq_len ? end : t.seq_len;
}

// ---- GEMMs (tcgen05) --------------------------------------------------------
// `bn` is the N tile (128 or 256; pick_bn chooses by wave count); the B tensor
// map's box must be bn x 64.  `b_off` selects the layer slice of stacked
// weights (row offset into B).
int pick_bn(int M, int N);
// q/k [M,1024] bf16 with bias + partial rotary on channels 0..63; v [M,1024]
// in fp16 (the MN-major PV operand of the attention).
void gemm_qkv(int bn, const CUtensorMap& A, const CUtensorMap& B, int M, int b_off, const float* bias, bf16* q,
              bf16* k, __half* v, const int* pos, const float2* rope, int* err, cudaStream_t s);
// x[M,1024] += gate[col] * (A*B^T + bias), residual tile prefetched by TMA
// through X (fp32 map of x, box 128 rows x 32 cols); B box 128 x 64.
void gemm_gate_res_tma(const CUtensorMap& A, const CUtensorMap& B, const CUtensorMap& X, int M, int K, int b_off,
                       const float* bias, const float* gate, float* x, int* err, cudaStream_t s);
// x[M,1024] += gate[col] * (A*B^T + bias)
void gemm_gate_res(int bn, const CUtensorMap& A, const CUtensorMap& B, int M, int K, int b_off, const float* bias,
                   const float* gate, float* x, int* err, cudaStream_t s);
// h[M,2048] = bf16(gelu_tanh(A*B^T + bias))
void gemm_gelu(int bn, const CUtensorMap& A, const CUtensorMap& B, int M, int b_off, const float* bias, bf16* h,
               int* err, cudaStream_t s);
// out[M,N] (row stride ldo) = A*B^T + bias (bias may be null).  N == 80 uses an
// 80-wide tile (B box 80 x 64) and ignores bn.
void gemm_f32(int bn, const CUtensorMap& A, const CUtensorMap& B, int M, int N, int K, const float* bias,
              float* out, int ldo, int* err, cudaStream_t s);
// x-part of the input projection: v = A*B^T + cst; x = v; stage[p2s[row]] = bf16(v)
void gemm_in_proj(int bn, const CUtensorMap& A, const CUtensorMap& B, int M, const float* cst, float* x,
                  bf16* stage, const int* p2s, int* err, cudaStream_t s);
// CTA-pair (cta_group::2) forms of the QKV, FF1 and residual GEMMs: 256 x 256
// tiles per pair of SMs; every B map has a 128 x 64 box, N % 256 == 0.
// use_pair_gemm decides by problem size (enough tiles for two waves of pairs);
// LX_FLOW_PAIR_GEMM=0 in the environment turns the pair path off, =2 uses it
// at every size (parity tests of small problems).
bool use_pair_gemm(int M, int N);
void gemm_pair_f32(const CUtensorMap& A, const CUtensorMap& B, int M, int N, int K, const float* bias, float* out,
                   int ldo, int* err, cudaStream_t s);
// The pair GEMMs' `rev` visits the 256-row blocks from the last one down (see
// row_order_alternates); the results do not depend on it.
// QKVs: q, k and v as one [3 x plane_rows][1024] block (k = q + plane_rows
// rows, v = q + 2 plane_rows rows; v's fp16 bits moved as 16-bit elements)
// with box 32 rows x 64 columns (the epilogue's TMA stores).
void gemm_pair_qkv(const CUtensorMap& A, const CUtensorMap& B, const CUtensorMap& QKVs, int plane_rows, int M,
                   int b_off, const float* bias, bf16* q, bf16* k, __half* v, const int* pos, const float2* rope,
                   int* err, cudaStream_t s, bool rev = false);
// Hs: h with box 32 rows x 64 columns (the epilogue's TMA stores).
void gemm_pair_gelu(const CUtensorMap& A, const CUtensorMap& B, const CUtensorMap& Hs, int M, int b_off,
                    const float* bias, bf16* h, int* err, cudaStream_t s, bool rev = false);
// X: the fp32 residual x with box 128 x 32 (loads); Xs: the same tensor with
// box 32 x 32 (the epilogue's TMA stores of each warp's 32 rows).
void gemm_pair_gate_res(const CUtensorMap& A, const CUtensorMap& B, const CUtensorMap& X, const CUtensorMap& Xs,
                        int M, int K, int b_off, const float* bias, const float* gate, float* x, int* err,
                        cudaStream_t s, bool rev = false);
// causal grouped conv (k=31, 16 groups) over the staged rows [0, Ms); B box 64 x 64.
// second == 0: out_stage[srow] = bf16(mish(conv + bias))  (rows with s2p >= 0)
// second == 1: x[s2p[srow]] += mish(conv + bias)
void conv_pos(const CUtensorMap& A, const CUtensorMap& B, int Ms, const float* bias, int second, bf16* out_stage,
              float* x, const int* s2p, int* err, cudaStream_t s);

// ---- attention (tcgen05 flash attention) -----------------------------------
// out[row, 64h..64h+63] for every valid query row of every tile; chunk > 0
// applies the block-causal chunk mask, keys >= seq_len are always masked.
// Q, K: bf16 [R][1024] maps, V: fp16 [R][1024] map; all boxes 128 rows x 64.
// Tiles in any order (longest first balances the last wave).  Returns false,
// launching nothing, when the kernel cannot be launched safely (see
// attention_ready) or n_tiles > ATT_MAX_TILES.
constexpr int ATT_MAX_TILES = 65535;
// True when the attention kernel's launch register count covers its
// setmaxnreg split on the current device (checked once per device).
bool attention_ready();
bool attention(const CUtensorMap& Q, const CUtensorMap& K, const CUtensorMap& V, const AttnTile* tiles,
               int n_tiles, int chunk, bf16* out, int* err, cudaStream_t s);

// ---- element-wise / row kernels -----------------------------------------
// y = bf16(LN(x) * (1 + scale) + shift), rows of 1024 fp32.
// rev: rows visited from the last one down (see row_order_alternates).
void adaln_rows(const float* x, bf16* y, const float* shift, const float* scale, int R, cudaStream_t s,
                bool rev = false);
// True unless LX_FLOW_ROW_ORDER=0: the decode alternates the row direction of
// consecutive row-streaming kernels (AdaLN, the pair GEMMs) so that each one
// starts on the rows its producer wrote last, which are still in L2.
bool row_order_alternates();
// x_state[f, c] += dt * (1.7 dphi[row_c] - 0.7 dphi[row_u]); xb rows <- bf16(x_state)
void euler_update(float* xs, const float* dphi, const int2* frame_rows, bf16* xb, int F, float dt, float cfg,
                  cudaStream_t s);
// x_state[f, c] = noise[src.x + c * src.y]; xb rows <- bf16
void init_state(float* xs, const float* noise, const int2* frame_rows, const int2* frame_src, bf16* xb, int F,
                cudaStream_t s);
// a_cond[row_c, 0:240] = bf16([cond, mu, spks]) from [u][80][T] inputs
void gather_cond(bf16* a_cond, const float* cond, const float* mu, const float* spks, const int2* frame_rows,
                 const int2* frame_src, const int* frame_utt, int F, cudaStream_t s);
// zero the staging rows with s2p < 0 in both conv staging buffers
void zero_gap_rows(bf16* a, bf16* b, const int* s2p, int Rs, cudaStream_t s);
// mel[src.x + c * src.y] = x_state[f, c]
void scatter_mel(float* mel, const float* xs, const int2* frame_src, int F, cudaStream_t s);
// copy fp32 rows of 1024 from packed rows to a [B, T, 1024] capture (row -> dst index)
void gather_rows(float* dst, const float* src, const int* rows, int n, int width, cudaStream_t s);
void gather_rows_bf16(float* dst, const bf16* src, const int* rows, int n, int width, cudaStream_t s);

// out[s][n] = act_out(sum_k act_in(in[s][k]) * W[n][k] + b[n]), S <= 16 rows, fp32.
// act: 0 none, 1 SiLU.
void gemv_rows(const float* in, int S, int K, const float* W, const float* b, int N, float* out, int ldo,
               int act_in, int act_out, cudaStream_t s);
// sinusoidal timestep embedding (256) of S timesteps.
void sinus_embed(const float* t, int S, float* out, cudaStream_t s);
// fp32 -> bf16 conversion
void to_bf16(const float* src, bf16* dst, size_t n, cudaStream_t s);

// ---- frontend (once per utterance) -----------------------------------------
void frontend_spk(const float* emb192, const float* w, const float* b, float* spk80, cudaStream_t s);
void frontend_embed(const int* tok, int n, const float* table, int vocab, float* out, cudaStream_t s);
// n_out = n_in (finalize: right zero padding) or n_in - 3 (streaming: the last 3 rows are context)
void frontend_conv1(const float* emb, int n_in, int n_out, const float* w, const float* b, float* h, cudaStream_t s);
void frontend_conv2(const float* h, const float* emb, int n, const float* w, const float* b, float* out,
                    cudaStream_t s);
// mu[c][2t + r] = pre[t][c]; cond[c][t] = t < mel_len1 ? prompt_feat[t][c] : 0
void frontend_mu_cond(const float* pre, int n_tok, const float* prompt_feat, int mel_len1, float* mu, float* cond,
                      cudaStream_t s);

// ---- standalone fused ops (microbench) ------------------
void op_adaln_f32(const float* x, float* y, const float* shift, const float* scale, int R, cudaStream_t s);
void op_adaln_bf16(const bf16* x, float* y, const float* shift, const float* scale, int R, cudaStream_t s);
void op_gate_res_f32(float* x, const float* y, const float* gate, int R, cudaStream_t s);
void op_gate_res_bf16(float* x, const bf16* y, const float* gate, int R, cudaStream_t s);
void op_rotary_f32(const float* x, float* y, const int* pos, const float2* rope, int R, cudaStream_t s);
void op_rotary_bf16(const bf16* x, float* y, const int* pos, const float2* rope, int R, cudaStream_t s);
void op_gelu_f32(const float* x, float* y, size_t n, cudaStream_t s);
void op_gelu_bf16(const bf16* x, float* y, size_t n, cudaStream_t s);

}  // namespace lx
