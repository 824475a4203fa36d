// Flow decoder engine (host side): device weights, batch plans, workspace,
// the per-step launch sequence and CUDA-graph replay.
#pragma once

#include <cstdint>
#include <map>
#include <string>
#include <vector>

#include "kernels.h"

namespace lx {

constexpr int N_STEPS_DEFAULT = 10;
constexpr float CFG_RATE = 0.7f;
constexpr int SEQ_ALIGN = 8;         // packed sequences start on 8-row boundaries (as lx_flow_op_attention)
constexpr int STAGE_GAP = 32;        // zero rows before each sequence in the conv staging layout (>= k-1 = 30)
constexpr int MAX_STEPS = 64;

struct Model {
  bf16 *wqkv = nullptr, *wo = nullptr, *w1 = nullptr, *w2 = nullptr;  // [22][N][K]
  float *bqkv = nullptr, *bo = nullptr, *b1 = nullptr, *b2 = nullptr;
  bf16 *win_x = nullptr, *win_c = nullptr;  // [1024][80], [1024][240]
  float* bin = nullptr;
  bf16 *wconv[2] = {nullptr, nullptr};      // [16][31][64][64]
  float* bconv[2] = {nullptr, nullptr};
  bf16* wout = nullptr;                     // [80][1024]
  float* bout = nullptr;
  float *adaln_w = nullptr, *adaln_b = nullptr;  // [22][6144][1024] fp32
  float *final_w = nullptr, *final_b = nullptr;  // [2048][1024]
  float *tmlp0_w = nullptr, *tmlp0_b = nullptr, *tmlp2_w = nullptr, *tmlp2_b = nullptr;
  float *emb = nullptr, *spk_w = nullptr, *spk_b = nullptr;
  float *pre1_w = nullptr, *pre1_b = nullptr, *pre2_w = nullptr, *pre2_b = nullptr;
  float* mod = nullptr;        // [n_sched][22][6144] for the schedule
  float* mod_final = nullptr;  // [n_sched][2048]
  float* temb = nullptr;       // [n_sched][1024]
  float* mod_x = nullptr;      // scratch: [22][6144] for an arbitrary t
  float* mod_final_x = nullptr;
  float* temb_x = nullptr;
  float* tscratch = nullptr;   // small scratch for the time MLP
  float2* rope = nullptr;      // [ROPE_MAX][32]
  int n_sched = 0;
  std::vector<float> sched_t, sched_dt;
  // B-operand tensor maps, one per (weight, N tile)
  CUtensorMap tm_wqkv[2], tm_wo[2], tm_w1[2], tm_w2[2], tm_winx[2], tm_winc[2];
  CUtensorMap tm_wconv[2], tm_wout;
};

// Pre-laid-out weight cache (layout.cu): write the device layout of a loaded
// model to `path`, or allocate (recorded in `allocs`) and fill the weight,
// rotary and default-schedule modulation buffers from such a file.  They
// return an LX_* status and put the message in *msg on failure.
int save_layout_file(Model& W, const std::string& gguf_path, const char* path, std::string* msg);
int load_layout_file(Model& W, std::vector<void*>& allocs, const char* path, std::string* msg);

// Packed variable-length layout of one batch.
struct Plan {
  int n_seq = 0;
  std::vector<int> seq_len, seq_start, seq_sstart;
  int R = 0, Rs = 0, F = 0;
  std::vector<int> pos, p2s, s2p, frame_utt;
  std::vector<int2> frame_rows, frame_src;
  std::vector<AttnTile> tiles;
  std::vector<int> seq_rows;  // per sequence-row capture index -> packed row (estimator captures)
  std::string key;
};

struct Workspace {
  int capR = 0, capRs = 0, capF = 0, capTiles = 0;
  size_t capIn = 0, capUtt = 0;
  float* x = nullptr;
  bf16 *xn = nullptr, *q = nullptr, *k = nullptr, *ao = nullptr, *h = nullptr;
  __half* v = nullptr;   // [R][1024] fp16 (attention values)
  bf16 *stage1 = nullptr, *stage2 = nullptr;
  float* cst = nullptr;
  bf16* a_cond = nullptr;
  bf16* xb = nullptr;
  float* dphi = nullptr;
  float* xs = nullptr;
  int *pos = nullptr, *p2s = nullptr, *s2p = nullptr, *frame_utt = nullptr, *seq_rows = nullptr;
  int2 *frame_rows = nullptr, *frame_src = nullptr;
  AttnTile* tiles = nullptr;
  float *in_mu = nullptr, *in_cond = nullptr, *in_noise = nullptr, *out_mel = nullptr, *in_spks = nullptr;
  float* cap = nullptr;  // capture scratch [R][1024]
  size_t capCap = 0;
  CUtensorMap tm_xn, tm_ao, tm_h, tm_xb, tm_acond, tm_stage1, tm_stage2, tm_q, tm_k, tm_v;
  CUtensorMap tm_x;   // fp32 residual stream, box 128 x 32
  CUtensorMap tm_xs;  // the same, box 32 x 32 (TMA stores of the residual GEMM epilogue)
  CUtensorMap tm_hs;  // FF hidden h, box 32 x 64 (TMA stores of the GELU GEMM epilogue)
  CUtensorMap tm_qkvs;  // q, k, v as one [3 capR][1024] block, box 32 x 64 (QKV GEMM epilogue stores)
  uint64_t generation = 0;
};

}  // namespace lx
