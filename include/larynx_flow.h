/*
 * larynx_flow.h -- C ABI of the B200 (sm_100a) Flow decoder.
 *
 * Drop-in replacement for the Flow decoder of hardenedlinux/larynx
 * (include/larynx/flow/flow.h, src/flow/*.cpp): the 22-block DiT estimator run
 * inside the 10-step classifier-free-guided CFM Euler loop, plus the flow.gguf
 * weight upload and the per-utterance frontend.  Plain C types only: host
 * pointers and sizes in, host pointers out, an int status back.  Device memory
 * is owned by the handle; all host buffers are owned by the caller.
 *
 * Threading: one handle per GPU; a handle is not thread-safe (same contract as
 * larynx::flow::FlowDecoder, which is non-copyable and used sequentially by
 * src/pipeline/pipeline.cpp:106-110).  Different handles may run concurrently.
 *
 * Data layouts follow the reference's PyTorch byte order:
 *   per-utterance mel-like tensors are [80][T] row-major (PyTorch (1, 80, T));
 *   prompt_feat is [mel_len1][80] (PyTorch (1, mel_len1, 80));
 *   batched tensors concatenate the utterances' [80][T_u] blocks in order.
 */
#ifndef LARYNX_FLOW_H
#define LARYNX_FLOW_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  The reference returns bool and logs to stderr
 * (src/flow/flow.cpp:75-77, src/flow/gguf.cpp:17); here every failure is a
 * distinct code and lx_flow_last_error() holds the message. */
#define LX_OK 0
#define LX_ERR_ARG 1     /* null pointer, bad count, buffer too small       */
#define LX_ERR_IO 2      /* file cannot be opened / read                    */
#define LX_ERR_FORMAT 3  /* malformed gguf or noise asset, missing tensor   */
#define LX_ERR_SHAPE 4   /* tensor or input of an unexpected shape          */
#define LX_ERR_OOM 5     /* device allocation failed                        */
#define LX_ERR_CUDA 6    /* CUDA runtime error / no sm_100 device           */
#define LX_ERR_TIMEOUT 7 /* a device-side wait exceeded its bound           */
#define LX_ERR_STATE 8   /* call order violated (e.g. infer before load)    */

#define LX_MEL_DIM 80
#define LX_SPK_EMBED_DIM 192
#define LX_DIM 1024
#define LX_DEPTH 22
#define LX_NOISE_MAX_FRAMES 15000

typedef struct lx_flow lx_flow;

/* Replaces FlowDecoder::FlowDecoder() + backend_init_best()
 * (include/larynx/flow/flow.h:41, include/larynx/backend.h:29-42): binds the
 * handle to CUDA device `device`; fails with LX_ERR_CUDA when it is not an
 * sm_100 part (there is no CPU fallback). */
int lx_flow_create(int device, lx_flow** out);

/* Replaces FlowDecoder::~FlowDecoder() (src/flow/flow.cpp:40-47). */
void lx_flow_destroy(lx_flow* h);

/* Message of the last failed call on this handle ("" if none). */
const char* lx_flow_last_error(const lx_flow* h);

/* Replaces FlowDecoder::load(gguf_path) (include/larynx/flow/flow.h:48;
 * src/flow/flow.cpp:49-60, src/flow/gguf.cpp:30-136): reads the 330 named
 * tensors of flow.gguf (F32/F16/BF16), uploads them in the device layout
 * (bf16 K-major GEMM operands, fused QKV, per-(group, tap) conv slices) and
 * precomputes the time embedding and AdaLN-Zero modulation tables for the
 * cosine 10-step schedule.  Idempotent like the reference. */
int lx_flow_load_gguf(lx_flow* h, const char* path);

/* Pre-laid-out weight cache (the flow.gguf -> device layout step done once;
 * the reference re-reads and converts the GGUF on every load,
 * src/flow/gguf.cpp:30-136).  lx_flow_save_layout writes the loaded model's
 * device layout (bf16 stacked projections, conv slices, rotary and
 * default-schedule modulation tables; ~1 GB) to `path`;
 * lx_flow_load_layout loads such a file instead of lx_flow_load_gguf (plain
 * copies: no GGUF parsing, conversion or table computation).  The file is
 * tied to this library's layout constants: another version returns
 * LX_ERR_FORMAT. */
int lx_flow_save_layout(lx_flow* h, const char* path);
int lx_flow_load_layout(lx_flow* h, const char* path);

/* Replaces FlowDecoder::load_noise (include/larynx/flow/flow.h:55;
 * src/flow/flow.cpp:70-108): the FNSE seed-noise bank (u32 magic 0x45534E46,
 * u32 version 1, u32 mel_dim 80, u64 max_frames 15000, f32[80][15000]). */
int lx_flow_load_noise(lx_flow* h, const char* path);

/* Optional per-stage captures of CFM step 1 (replaces larynx::flow::FlowDebug,
 * include/larynx/flow/flow.h:15-34: the same stages in the same order and the
 * same PyTorch byte layouts; FlowDebug::feat is mel_out itself).  Every
 * pointer may be NULL.  T = MEL_T; N = n_prompt + n_tokens token rows;
 * N_pre = N (finalize) or N - 3 (the streaming call).  In the [2][...] stages
 * row 0 is the conditional, row 1 the CFG-zeroed row.  conv_pos is taken as
 * input_embed - input_proj in fp32 (the conv output is added to the residual
 * in the conv kernel's epilogue, src/flow/dit.cpp:122). */
typedef struct lx_flow_debug {
  float* spk;          /* [80]                 (1, 80)           */
  float* token_embed;  /* [N][80]              (1, N, 80)        */
  float* prelookahead; /* [N_pre][80]          (1, N_pre, 80)    */
  float* mu;           /* [80][T]              (1, 80, T)        */
  float* cond;         /* [80][T]              (1, 80, T)        */
  float* time_embed;   /* [2][1024]            (2, 1024)         */
  float* input_proj;   /* [2][T][1024]         proj before conv-pos */
  float* conv_pos;     /* [2][T][1024]         conv-pos output   */
  float* input_embed;  /* [2][T][1024]                           */
  float* blocks;       /* [22][2][T][1024]     after each block  */
  float* norm_out;     /* [2][T][1024]                           */
  float* dphi;         /* [2][80][T]                             */
} lx_flow_debug;

/* Replaces both FlowDecoder::infer overloads (include/larynx/flow/flow.h:61-77;
 * src/flow/flow.cpp:110-308): token -> mel, whole sequence (finalize=True).
 * MEL_T = 2 * (n_prompt + n_tokens); mel_len1 = prompt_feat frames.
 * noise_z: [80][MEL_T], or NULL to slice the bank of lx_flow_load_noise
 * (the 6-argument form).  mel_out receives [80][MEL_T - mel_len1];
 * mel_cap is its capacity in floats. */
int lx_flow_infer(lx_flow* h, const int32_t* prompt_tokens, int n_prompt, const int32_t* tokens, int n_tokens,
                  const float* prompt_feat, int mel_len1, const float* spk_embedding, const float* noise_z,
                  float* mel_out, size_t mel_cap, lx_flow_debug* debug);

/* lx_flow_infer with the reference's `finalize` flag (flow_reference.py:531-563,
 * CosyVoice3 CausalMaskedDiffWithXvec.inference; the reference's C++ path
 * implements only finalize=True, src/flow/flow.cpp:110 / docs/FLOW.md §5).
 * finalize != 0 is lx_flow_infer.  finalize == 0 is the streaming call: the
 * last 3 tokens are PreLookahead look-ahead context (they replace its zero
 * padding and produce no frames), so MEL_T = 2 * (n_prompt + n_tokens - 3)
 * and mel_out receives [80][MEL_T - mel_len1].  The CFM noise is the first
 * MEL_T columns of noise_z (a [80][MEL_T] array) or of the noise bank.
 * chunk > 0 applies the block-causal chunk mask (as lx_flow_batch.chunk; the
 * streaming attention of upstream CosyVoice3 with static_chunk_size frames);
 * chunk == 0 is the reference's full attention.  Stage captures (debug) are
 * taken with full attention. */
int lx_flow_infer_ex(lx_flow* h, const int32_t* prompt_tokens, int n_prompt, const int32_t* tokens, int n_tokens,
                     const float* prompt_feat, int mel_len1, const float* spk_embedding, const float* noise_z,
                     int finalize, int chunk, float* mel_out, size_t mel_cap, lx_flow_debug* debug);

/* Batched decode at the estimator/CFM level (the north-star hot path;
 * extends FlowDecoder::infer's Euler loop, src/flow/flow.cpp:202-274, to many
 * utterances): each utterance u of T_u frames is decoded with its own
 * conditional row and a CFG-zeroed row, key-padding semantics (no frame
 * attends past its own utterance), optionally a block-causal chunk mask.
 * mel_out receives the final x of every frame ([80][T_u] per utterance, prompt
 * frames included; callers slice like flow.cpp:277-280). */
typedef struct lx_flow_batch {
  int n_utt;
  const int32_t* lengths; /* [n_utt] frames per utterance, >= 1          */
  const float* mu;        /* concat_u [80][T_u]                          */
  const float* cond;      /* concat_u [80][T_u] (zeros past the prompt)  */
  const float* spks;      /* [n_utt][80]                                 */
  const float* noise;     /* concat_u [80][T_u], or NULL = noise bank    */
  float* mel_out;         /* concat_u [80][T_u]                          */
  int chunk;              /* 0 = full attention; > 0 block-causal chunk   */
  int n_steps;            /* 0 = 10 (the reference's N_TIMESTEPS); 1..10 runs
                             the first n steps of that schedule        */
} lx_flow_batch;

/* Host buffers: uploads the inputs, decodes, downloads mel_out; returns when
 * the result is in mel_out. */
int lx_flow_decode(lx_flow* h, const lx_flow_batch* b);

/* Device buffers (pointers of this handle's GPU): enqueues the whole decode on
 * `stream` (a cudaStream_t, NULL = the handle's own stream) and returns
 * without synchronising.  `lengths` stays a host array. */
int lx_flow_decode_device(lx_flow* h, const lx_flow_batch* b, void* stream);

/* One estimator (DiT) forward, for per-stage parity (replaces the DiT graph
 * of src/flow/dit.cpp:83-145 as driven by tests/flow_dump.cpp): n_seq
 * independent sequences, all at the scalar timestep t.  x/mu/cond:
 * concat_s [80][T_s]; spks: [n_seq][80]; dphi_out: concat_s [80][T_s].
 * Optional captures (may be NULL), concat_s [T_s][1024]:
 * input_embed_out, block_out (after block `block_index`), norm_out. */
int lx_flow_estimator(lx_flow* h, int n_seq, const int32_t* lengths, const float* x, const float* mu,
                      const float* cond, const float* spks, float t, int chunk, float* dphi_out,
                      float* input_embed_out, float* block_out, int block_index, float* norm_out);

/* Diagnostic: runs lx_flow_decode_device without CUDA graphs, bracketing
 * every kernel with CUDA events on the launch stream, and returns per kernel
 * class the summed device milliseconds and launch counts (synchronous).
 * Classes (n_class >= 11): 0 input projection, 1 conv-pos, 2 AdaLN-mod,
 * 3 QKV GEMM, 4 attention, 5 out GEMM, 6 FF1 GEMM, 7 FF2 GEMM, 8 proj_out GEMM,
 * 9 Euler/CFG update, 10 other.  No reference counterpart (the reference has
 * no timers, per its own docs). */
int lx_flow_profile_decode(lx_flow* h, const lx_flow_batch* b, void* stream, double* ms_by_class,
                           int* launches_by_class, int n_class);

/* Total number of kernel launches enqueued by this handle so far. */
uint64_t lx_flow_launch_count(const lx_flow* h);

/* ---- standalone fused ops (BASELINE config 1 microbench) -----------------
 * Device pointers, rows of 1024 channels, asynchronous on `stream`.
 * in_bf16 != 0: the input x (and y for gate_res) is bf16, else fp32;
 * outputs are fp32.  op: 0 AdaLN-Zero modulated LayerNorm
 * (y = LN(x)(1+scale)+shift, src/flow/ops.cpp:94-104), 1 gate-residual
 * (x += gate * y, src/flow/dit.cpp:71,77), 2 partial rotary (channels 0..63,
 * pos[row], src/flow/ops.cpp:85-92), 3 GELU-tanh (src/flow/ops.cpp:73-83).
 * Launched with programmatic dependent launch: an op may begin while the
 * stream's previous kernel finishes and waits for it before reading memory. */
int lx_flow_op(int op, int in_bf16, int rows, const void* x, void* y, const float* shift, const float* scale,
               const float* gate, const int32_t* pos, void* stream);

/* ---- per-op kernels on caller buffers (parity tests, microbenchmarks) -----
 * Synchronous; they allocate small temporaries per call.
 * lx_flow_op_gemm: C[M][N] fp32 = A[M][K] * B[N][K]^T (+ bias[N]), A and B
 * bf16 row-major device arrays (the `linear` of src/flow/ops.cpp:20-26 on the
 * tensor cores); K % 8 == 0, N == 80 or a multiple of 128.
 * lx_flow_op_attention: softmax(q k^T / 8 + mask) v per head over packed
 * sequences (src/flow/dit.cpp:34-51 plus the key-padding / block-causal
 * masks); q, k, v, out bf16 [R][1024], sequence i at rows
 * [start_i, start_i + len_i), start_{i+1} = start_i + round_up(len_i, 8). */
int lx_flow_op_gemm(int M, int N, int K, const void* A, const void* B, const float* bias, float* C, void* stream);
int lx_flow_op_attention(int n_seq, const int32_t* lengths, const void* q, const void* k, const void* v, void* out,
                         int chunk, void* stream);

/* ---- lx_flow_op_attention without device allocation ----------------------
 * No counterpart in the reference: it exists for callers that may not
 * allocate device memory on the call path (cudaMalloc / cudaFree can stall on
 * other streams' work and take unbounded time; a deadline-bound audio loop or
 * an embedder owning all of HBM through its own pool cannot accept that).
 * Same arguments, result and synchronous behaviour as lx_flow_op_attention,
 * but all scratch (fp16 copy of V, tile list, error word) lives in fixed static
 * device storage (8 MiB + 8 KiB per device), so the call allocates nothing.
 * Limit: packed rows sum_i round_up(len_i, 8) <= LX_STATIC_ATT_MAX_ROWS,
 * else LX_ERR_ARG with no device work queued.  The first call on a device (with
 * that device current) looks the storage up with cudaGetSymbolAddress: make
 * it before any stream capture.  The storage is shared per device: calls that
 * overlap in time on one device (two threads, or two streams) race and give
 * wrong results, so serialise them. */
#define LX_STATIC_ATT_MAX_ROWS 4096
int lx_flow_op_attention_static(int n_seq, const int32_t* lengths, const void* q, const void* k, const void* v,
                                void* out, int chunk, void* stream);

/* ---- failure-path self test (no reference counterpart) ------------------
 * Runs one CTA whose consumer waits, through the library's bounded mbarrier
 * wait, for a producer that arrives only if producer_arrives != 0, with a
 * limit of limit_ms (0 < limit_ms <= 2000; the kernels themselves use 2 s).
 * Returns LX_OK when the wait completed, LX_ERR_TIMEOUT when it ran out (the
 * CTA then left through its abort flag and freed its tensor memory; the CUDA
 * context stays usable).  *device_code (may be NULL) receives the raw device
 * error code (0, or the role that gave up).  Synchronous on `stream`. */
int lx_flow_selftest_wait(int producer_arrives, double limit_ms, int* device_code, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LARYNX_FLOW_H */
