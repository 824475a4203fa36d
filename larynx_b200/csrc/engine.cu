// Flow decoder engine and the C ABI (include/larynx_flow.h).
//
// Hot path per CFM step (all on the device, captured once per batch plan as
// a CUDA graph covering every Euler step):
//   in_proj GEMM (x part, K=80) + per-utterance constant -> x, conv staging
//   conv-pos 1 (Mish) -> conv-pos 2 (Mish, + residual) -> x
//   22 x { AdaLN-mod -> QKV GEMM (+bias, partial rotary, fp16 V) -> flash attention
//          -> out GEMM (+bias, gate, residual) -> AdaLN-mod
//          -> FF1 GEMM (+bias, GELU-tanh) -> FF2 GEMM (+bias, gate, residual) }
//   final AdaLN-mod -> proj_out GEMM (N=80) -> CFG Euler update
// The reference runs the same steps as one GGML graph per Euler step with the
// Euler/CFG update on the host (src/flow/flow.cpp:240-274).
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <memory>
#include <string>
#include <thread>
#include <vector>

#include "../../include/larynx_flow.h"
#include "engine.h"
#include "gguf.h"

using namespace lx;

namespace {

// --------------------------------------------------------------------------
// host helpers
// --------------------------------------------------------------------------
inline uint16_t f2bf(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u) return static_cast<uint16_t>((u >> 16) | ((u & 0xFFFFu) ? 0x40u : 0u));
  const uint32_t r = ((u >> 16) & 1u) + 0x7FFFu;  // round to nearest even
  return static_cast<uint16_t>((u + r) >> 16);
}

void to_bf16_host(const float* src, uint16_t* dst, size_t n) {
  const unsigned nt = std::max(1u, std::min(16u, std::thread::hardware_concurrency()));
  if (n < (1u << 20) || nt == 1) {
    for (size_t i = 0; i < n; ++i) dst[i] = f2bf(src[i]);
    return;
  }
  std::vector<std::thread> th;
  const size_t chunk = (n + nt - 1) / nt;
  for (unsigned t = 0; t < nt; ++t) {
    const size_t a = t * chunk, b = std::min(n, a + chunk);
    if (a >= b) break;
    th.emplace_back([=] {
      for (size_t i = a; i < b; ++i) dst[i] = f2bf(src[i]);
    });
  }
  for (auto& t : th) t.join();
}

std::string blk(int i, const char* tail) {
  return "decoder.estimator.transformer_blocks." + std::to_string(i) + "." + tail;
}
const std::string EST = "decoder.estimator.";

}  // namespace

// --------------------------------------------------------------------------
// handle
// --------------------------------------------------------------------------
struct lx_flow {
  int device = 0;
  cudaStream_t stream = nullptr;
  std::string err;
  int* d_err = nullptr;
  uint64_t launches = 0;
  bool loaded = false;
  std::string gguf_path;     // the flow.gguf the model came from (recorded in layout files)
  std::vector<float> noise;  // [80][15000]
  bool noise_loaded = false;
  Model W;
  Workspace ws;
  std::vector<void*> allocs;  // model allocations
  struct GraphEntry {
    cudaGraphExec_t exec = nullptr;
    uint64_t nodes = 0;
  };
  std::map<std::string, GraphEntry> graphs;
  bool use_graphs = true;
  // per-kernel-class CUDA-event timing (lx_flow_profile_decode)
  struct ProfRec {
    int cls;
    cudaEvent_t a, b;
  };
  struct Prof {
    std::vector<cudaEvent_t> pool;
    size_t used = 0;
    std::vector<ProfRec> recs;
    cudaEvent_t get() {
      if (used == pool.size()) {
        cudaEvent_t e;
        cudaEventCreate(&e);
        pool.push_back(e);
      }
      return pool[used++];
    }
    ~Prof() {
      for (auto e : pool) cudaEventDestroy(e);
    }
  };
  Prof* prof = nullptr;
  // last plan uploaded to the workspace (skips rebuilding an identical layout)
  Plan cached_plan;
  uint64_t cached_gen = 0;
  bool cached_valid = false;
  // frontend scratch
  float *f_spk_in = nullptr, *f_spk = nullptr, *f_emb = nullptr, *f_h = nullptr, *f_pre = nullptr,
        *f_mu = nullptr, *f_cond = nullptr, *f_pf = nullptr;
  int* f_tok = nullptr;
  int f_cap = 0;

  int fail(int code, const std::string& msg) {
    err = msg;
    return code;
  }
};

namespace {

// kernel classes reported by lx_flow_profile_decode
enum KClass : int {
  K_INPROJ = 0, K_CONV = 1, K_ADALN = 2, K_QKV = 3, K_ATTN = 4, K_OUT = 5, K_FF1 = 6, K_FF2 = 7,
  K_PROJOUT = 8, K_EULER = 9, K_OTHER = 10, K_NCLASS = 11
};

// Bracket one launch with events when profiling (never inside a graph capture).
template <class F>
inline void timed(lx_flow* h, int cls, cudaStream_t s, F&& launch) {
  if (h->prof) {
    cudaEvent_t a = h->prof->get();
    cudaEventRecord(a, s);
    launch();
    cudaEvent_t b = h->prof->get();
    cudaEventRecord(b, s);
    h->prof->recs.push_back({cls, a, b});
  } else {
    launch();
  }
}

int cuda_fail(lx_flow* h, cudaError_t e, const char* what) {
  return h->fail(e == cudaErrorMemoryAllocation ? LX_ERR_OOM : LX_ERR_CUDA,
                 std::string(what) + ": " + cudaGetErrorString(e));
}

#define CK(expr)                                          \
  do {                                                    \
    cudaError_t e_ = (expr);                              \
    if (e_ != cudaSuccess) return cuda_fail(h, e_, #expr); \
  } while (0)

template <typename T>
int dev_alloc(lx_flow* h, T** p, size_t n, bool track = true) {
  void* v = nullptr;
  cudaError_t e = cudaMalloc(&v, std::max<size_t>(n, 1) * sizeof(T));
  if (e != cudaSuccess) return cuda_fail(h, e, "cudaMalloc");
  *p = static_cast<T*>(v);
  if (track) h->allocs.push_back(v);
  return LX_OK;
}

template <typename T>
int upload(lx_flow* h, T** p, const T* src, size_t n) {
  int rc = dev_alloc(h, p, n);
  if (rc) return rc;
  CK(cudaMemcpy(*p, src, n * sizeof(T), cudaMemcpyHostToDevice));
  return LX_OK;
}

int upload_bf16(lx_flow* h, bf16** p, const std::vector<float>& src) {
  std::vector<uint16_t> tmp(src.size());
  to_bf16_host(src.data(), tmp.data(), src.size());
  return upload(h, reinterpret_cast<uint16_t**>(p), tmp.data(), tmp.size());
}

void wsfree(void*& p) {
  if (p) cudaFree(p);
  p = nullptr;
}

void clear_graphs(lx_flow* h) {
  for (auto& kv : h->graphs)
    if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
  h->graphs.clear();
}

// --------------------------------------------------------------------------
// schedule: t_span = 1 - cos(linspace(0,1,n+1) * pi/2) in fp32 and the
// accumulated (t, dt) pairs of src/flow/flow.cpp:202-207, 235-273
// --------------------------------------------------------------------------
void make_schedule(int n, std::vector<float>& ts, std::vector<float>& dts) {
  const float PI = 3.14159265358979323846f;
  std::vector<float> span(n + 1);
  for (int i = 0; i <= n; ++i) span[i] = 1.0f - cosf((static_cast<float>(i) / static_cast<float>(n)) * 0.5f * PI);
  ts.assign(n, 0.f);
  dts.assign(n, 0.f);
  float t = span[0], dt = span[1] - span[0];
  for (int step = 1; step <= n; ++step) {
    ts[step - 1] = t;
    dts[step - 1] = dt;
    t += dt;
    if (step < n) dt = span[step + 1] - t;
  }
}

// time embedding + AdaLN-Zero modulation for S timesteps (device arrays)
void modulation_tables(lx_flow* h, const float* d_t, int S, float* temb, float* mod, float* mod_final,
                       cudaStream_t s) {
  Model& W = h->W;
  float* sin_buf = W.tscratch;               // [S][256]
  float* hid = W.tscratch + 16 * 256;        // [S][1024]
  sinus_embed(d_t, S, sin_buf, s);
  gemv_rows(sin_buf, S, 256, W.tmlp0_w, W.tmlp0_b, DIM, hid, DIM, 0, 1, s);
  gemv_rows(hid, S, DIM, W.tmlp2_w, W.tmlp2_b, DIM, temb, DIM, 0, 0, s);
  for (int l = 0; l < DEPTH; ++l)
    gemv_rows(temb, S, DIM, W.adaln_w + static_cast<size_t>(l) * MOD_N * DIM, W.adaln_b + static_cast<size_t>(l) * MOD_N,
              MOD_N, mod + static_cast<size_t>(l) * MOD_N, DEPTH * MOD_N, 1, 0, s);
  gemv_rows(temb, S, DIM, W.final_w, W.final_b, 2 * DIM, mod_final, 2 * DIM, 1, 0, s);
  h->launches += 4 + DEPTH;
}

int build_model_maps(lx_flow* h) {
  Model& W = h->W;
  bool ok = true;
  const int bns[2] = {128, 256};
  for (int i = 0; i < 2; ++i) {
    const uint32_t bn = bns[i];
    ok &= tmap_bf16(&W.tm_wqkv[i], W.wqkv, static_cast<uint64_t>(DEPTH) * QKV_N, DIM, DIM, bn, 64);
    ok &= tmap_bf16(&W.tm_wo[i], W.wo, static_cast<uint64_t>(DEPTH) * DIM, DIM, DIM, bn, 64);
    ok &= tmap_bf16(&W.tm_w1[i], W.w1, static_cast<uint64_t>(DEPTH) * FF, DIM, DIM, bn, 64);
    ok &= tmap_bf16(&W.tm_w2[i], W.w2, static_cast<uint64_t>(DEPTH) * DIM, FF, FF, bn, 64);
    ok &= tmap_bf16(&W.tm_winx[i], W.win_x, DIM, MEL, MEL, bn, 64);
    ok &= tmap_bf16(&W.tm_winc[i], W.win_c, DIM, COND_K, COND_K, bn, 64);
  }
  for (int c = 0; c < 2; ++c)
    ok &= tmap_bf16(&W.tm_wconv[c], W.wconv[c], static_cast<uint64_t>(CONV_G) * CONV_K * 64, 64, 64, 64, 64);
  ok &= tmap_bf16(&W.tm_wout, W.wout, MEL, DIM, DIM, MEL, 64);
  if (!ok) return h->fail(LX_ERR_CUDA, "cuTensorMapEncodeTiled failed for a weight tensor");
  return LX_OK;
}

// --------------------------------------------------------------------------
// weight load (src/flow/gguf.cpp:30-136 names; internal.h:50-93 shapes)
// --------------------------------------------------------------------------
int load_model(lx_flow* h, const char* path) {
  GgufFile g;
  int rc = g.open(path);
  if (rc) return h->fail(rc, g.error());
  Model& W = h->W;
  std::vector<float> a, b, c;
  auto rd = [&](const std::string& name, std::vector<int64_t> shape, std::vector<float>& out) -> int {
    int r = g.read_f32(name, shape, out);
    if (r) h->err = g.error();
    return r;
  };

  // stacked per-block projection weights
  std::vector<float> qkv(static_cast<size_t>(DEPTH) * QKV_N * DIM), bqkv(static_cast<size_t>(DEPTH) * QKV_N);
  std::vector<float> wo(static_cast<size_t>(DEPTH) * DIM * DIM), bo(static_cast<size_t>(DEPTH) * DIM);
  std::vector<float> w1(static_cast<size_t>(DEPTH) * FF * DIM), b1(static_cast<size_t>(DEPTH) * FF);
  std::vector<float> w2(static_cast<size_t>(DEPTH) * DIM * FF), b2(static_cast<size_t>(DEPTH) * DIM);
  std::vector<float> adw(static_cast<size_t>(DEPTH) * MOD_N * DIM), adb(static_cast<size_t>(DEPTH) * MOD_N);
  const size_t DD = static_cast<size_t>(DIM) * DIM;
  for (int l = 0; l < DEPTH; ++l) {
    const char* qn[3] = {"attn.to_q.", "attn.to_k.", "attn.to_v."};
    for (int j = 0; j < 3; ++j) {
      if ((rc = rd(blk(l, (std::string(qn[j]) + "weight").c_str()), {DIM, DIM}, a))) return rc;
      if ((rc = rd(blk(l, (std::string(qn[j]) + "bias").c_str()), {DIM}, b))) return rc;
      std::memcpy(&qkv[(static_cast<size_t>(l) * 3 + j) * DD], a.data(), DD * 4);
      std::memcpy(&bqkv[(static_cast<size_t>(l) * 3 + j) * DIM], b.data(), DIM * 4);
    }
    if ((rc = rd(blk(l, "attn.to_out.0.weight"), {DIM, DIM}, a))) return rc;
    std::memcpy(&wo[l * DD], a.data(), DD * 4);
    if ((rc = rd(blk(l, "attn.to_out.0.bias"), {DIM}, b))) return rc;
    std::memcpy(&bo[static_cast<size_t>(l) * DIM], b.data(), DIM * 4);
    if ((rc = rd(blk(l, "ff.ff.0.0.weight"), {FF, DIM}, a))) return rc;
    std::memcpy(&w1[l * 2 * DD], a.data(), 2 * DD * 4);
    if ((rc = rd(blk(l, "ff.ff.0.0.bias"), {FF}, b))) return rc;
    std::memcpy(&b1[static_cast<size_t>(l) * FF], b.data(), FF * 4);
    if ((rc = rd(blk(l, "ff.ff.2.weight"), {DIM, FF}, a))) return rc;
    std::memcpy(&w2[l * 2 * DD], a.data(), 2 * DD * 4);
    if ((rc = rd(blk(l, "ff.ff.2.bias"), {DIM}, b))) return rc;
    std::memcpy(&b2[static_cast<size_t>(l) * DIM], b.data(), DIM * 4);
    if ((rc = rd(blk(l, "attn_norm.linear.weight"), {MOD_N, DIM}, a))) return rc;
    std::memcpy(&adw[l * 6 * DD], a.data(), 6 * DD * 4);
    if ((rc = rd(blk(l, "attn_norm.linear.bias"), {MOD_N}, b))) return rc;
    std::memcpy(&adb[static_cast<size_t>(l) * MOD_N], b.data(), MOD_N * 4);
  }
  if ((rc = upload_bf16(h, &W.wqkv, qkv)) || (rc = upload(h, &W.bqkv, bqkv.data(), bqkv.size()))) return rc;
  if ((rc = upload_bf16(h, &W.wo, wo)) || (rc = upload(h, &W.bo, bo.data(), bo.size()))) return rc;
  if ((rc = upload_bf16(h, &W.w1, w1)) || (rc = upload(h, &W.b1, b1.data(), b1.size()))) return rc;
  if ((rc = upload_bf16(h, &W.w2, w2)) || (rc = upload(h, &W.b2, b2.data(), b2.size()))) return rc;
  if ((rc = upload(h, &W.adaln_w, adw.data(), adw.size())) || (rc = upload(h, &W.adaln_b, adb.data(), adb.size())))
    return rc;
  qkv.clear(); qkv.shrink_to_fit();
  w1.clear(); w1.shrink_to_fit();
  w2.clear(); w2.shrink_to_fit();
  adw.clear(); adw.shrink_to_fit();

  // input projection: columns [x | cond | mu | spks] (src/flow/dit.cpp:109)
  if ((rc = rd(EST + "input_embed.proj.weight", {DIM, 4 * MEL}, a))) return rc;
  if ((rc = rd(EST + "input_embed.proj.bias", {DIM}, b))) return rc;
  {
    std::vector<float> wx(static_cast<size_t>(DIM) * MEL), wc(static_cast<size_t>(DIM) * COND_K);
    for (int o = 0; o < DIM; ++o) {
      std::memcpy(&wx[static_cast<size_t>(o) * MEL], &a[static_cast<size_t>(o) * 4 * MEL], MEL * 4);
      std::memcpy(&wc[static_cast<size_t>(o) * COND_K], &a[static_cast<size_t>(o) * 4 * MEL + MEL], COND_K * 4);
    }
    if ((rc = upload_bf16(h, &W.win_x, wx)) || (rc = upload_bf16(h, &W.win_c, wc)) ||
        (rc = upload(h, &W.bin, b.data(), b.size())))
      return rc;
  }
  // conv-pos: [1024 out][64 in][31 k] -> [group][tap][64 out][64 in]
  for (int cv = 0; cv < 2; ++cv) {
    const std::string p = EST + "input_embed.conv_pos_embed.conv" + std::to_string(cv + 1) + ".0.";
    if ((rc = rd(p + "weight", {DIM, 64, CONV_K}, a))) return rc;
    if ((rc = rd(p + "bias", {DIM}, b))) return rc;
    std::vector<float> r(static_cast<size_t>(DIM) * 64 * CONV_K);
    for (int gidx = 0; gidx < CONV_G; ++gidx)
      for (int k = 0; k < CONV_K; ++k)
        for (int o = 0; o < 64; ++o)
          for (int i = 0; i < 64; ++i)
            r[((static_cast<size_t>(gidx) * CONV_K + k) * 64 + o) * 64 + i] =
                a[(static_cast<size_t>(gidx * 64 + o) * 64 + i) * CONV_K + k];
    if ((rc = upload_bf16(h, &W.wconv[cv], r)) || (rc = upload(h, &W.bconv[cv], b.data(), b.size()))) return rc;
  }
  if ((rc = rd(EST + "proj_out.weight", {MEL, DIM}, a))) return rc;
  if ((rc = rd(EST + "proj_out.bias", {MEL}, b))) return rc;
  if ((rc = upload_bf16(h, &W.wout, a)) || (rc = upload(h, &W.bout, b.data(), b.size()))) return rc;
  // fp32 small weights
  struct F32W {
    std::string name;
    std::vector<int64_t> shape;
    float** dst;
  };
  std::vector<F32W> f32w = {
      {EST + "norm_out.linear.weight", {2 * DIM, DIM}, &W.final_w},
      {EST + "norm_out.linear.bias", {2 * DIM}, &W.final_b},
      {EST + "time_embed.time_mlp.0.weight", {DIM, 256}, &W.tmlp0_w},
      {EST + "time_embed.time_mlp.0.bias", {DIM}, &W.tmlp0_b},
      {EST + "time_embed.time_mlp.2.weight", {DIM, DIM}, &W.tmlp2_w},
      {EST + "time_embed.time_mlp.2.bias", {DIM}, &W.tmlp2_b},
      {"input_embedding.weight", {6561, MEL}, &W.emb},
      {"spk_embed_affine_layer.weight", {MEL, 192}, &W.spk_w},
      {"spk_embed_affine_layer.bias", {MEL}, &W.spk_b},
      {"pre_lookahead_layer.conv1.weight", {DIM, MEL, 4}, &W.pre1_w},
      {"pre_lookahead_layer.conv1.bias", {DIM}, &W.pre1_b},
      {"pre_lookahead_layer.conv2.weight", {MEL, DIM, 3}, &W.pre2_w},
      {"pre_lookahead_layer.conv2.bias", {MEL}, &W.pre2_b},
  };
  for (auto& f : f32w) {
    if ((rc = rd(f.name, f.shape, a))) return rc;
    if ((rc = upload(h, f.dst, a.data(), a.size()))) return rc;
  }

  // rotary table: angle = fp32(p * inv_freq[i]), inv_freq = 1 / 10000^(2i/64)
  {
    std::vector<float2> rope(static_cast<size_t>(ROPE_MAX) * 32);
    for (int i = 0; i < 32; ++i) {
      const float inv = 1.0f / powf(10000.0f, static_cast<float>(2 * i) / 64.0f);
      for (int p = 0; p < ROPE_MAX; ++p) {
        const float ang = static_cast<float>(p) * inv;
        rope[static_cast<size_t>(p) * 32 + i] =
            make_float2(static_cast<float>(cos(static_cast<double>(ang))), static_cast<float>(sin(static_cast<double>(ang))));
      }
    }
    if ((rc = upload(h, &W.rope, rope.data(), rope.size()))) return rc;
  }

  // modulation tables for the 10-step cosine schedule
  make_schedule(N_STEPS_DEFAULT, W.sched_t, W.sched_dt);
  W.n_sched = N_STEPS_DEFAULT;
  if ((rc = dev_alloc(h, &W.mod, static_cast<size_t>(MAX_STEPS) * DEPTH * MOD_N)) ||
      (rc = dev_alloc(h, &W.mod_final, static_cast<size_t>(MAX_STEPS) * 2 * DIM)) ||
      (rc = dev_alloc(h, &W.temb, static_cast<size_t>(MAX_STEPS) * DIM)) ||
      (rc = dev_alloc(h, &W.mod_x, static_cast<size_t>(DEPTH) * MOD_N)) ||
      (rc = dev_alloc(h, &W.mod_final_x, 2 * DIM)) || (rc = dev_alloc(h, &W.temb_x, DIM)) ||
      (rc = dev_alloc(h, &W.tscratch, 16 * 256 + 16 * DIM + 64)))
    return rc;
  float* d_t = W.tscratch + 16 * 256 + 16 * DIM;
  CK(cudaMemcpy(d_t, W.sched_t.data(), W.n_sched * sizeof(float), cudaMemcpyHostToDevice));
  modulation_tables(h, d_t, W.n_sched, W.temb, W.mod, W.mod_final, h->stream);
  CK(cudaStreamSynchronize(h->stream));
  return build_model_maps(h);
}

// --------------------------------------------------------------------------
// batch plan
// --------------------------------------------------------------------------
std::string plan_key(int n_utt, const int32_t* lengths, bool cfg_pairs, int chunk, int steps);
// cfg_pairs: every utterance contributes a conditional and a CFG-zeroed
// sequence (decode); otherwise each input is one sequence (estimator).
Plan make_plan(int n_utt, const int32_t* lengths, bool cfg_pairs, int chunk, int steps) {
  Plan p;
  const int per = cfg_pairs ? 2 : 1;
  p.n_seq = n_utt * per;
  p.seq_len.resize(p.n_seq);
  p.seq_start.resize(p.n_seq);
  p.seq_sstart.resize(p.n_seq);
  int r = 0, sr = 0;
  for (int s = 0; s < p.n_seq; ++s) {
    const int L = lengths[s / per];
    p.seq_len[s] = L;
    sr += STAGE_GAP;
    p.seq_sstart[s] = sr;
    sr += L;
  }
  // Packed rows: longest sequences first when the row direction alternates.
  // Attention works longest first, so the rows it writes last (the shortest
  // sequences) are the highest ones, which the out projection then reads
  // first (it runs from the last row block down); see enqueue_dit.
  std::vector<int> ord(p.n_seq);
  for (int s = 0; s < p.n_seq; ++s) ord[s] = s;
  if (row_order_alternates())
    std::stable_sort(ord.begin(), ord.end(), [&p](int a, int b) { return p.seq_len[a] > p.seq_len[b]; });
  for (const int s : ord) {
    p.seq_start[s] = r;
    r += (p.seq_len[s] + SEQ_ALIGN - 1) / SEQ_ALIGN * SEQ_ALIGN;
  }
  p.R = std::max(r, 1);
  p.Rs = std::max(sr, 1);
  p.pos.assign(p.R, 0);
  p.p2s.assign(p.R, -1);
  p.s2p.assign(p.Rs, -1);
  for (int s = 0; s < p.n_seq; ++s)
    for (int t = 0; t < p.seq_len[s]; ++t) {
      p.pos[p.seq_start[s] + t] = t;
      p.p2s[p.seq_start[s] + t] = p.seq_sstart[s] + t;
      p.s2p[p.seq_sstart[s] + t] = p.seq_start[s] + t;
    }
  int f = 0;
  for (int u = 0; u < n_utt; ++u) f += lengths[u];
  p.F = f;
  p.frame_rows.resize(f);
  p.frame_src.resize(f);
  p.frame_utt.resize(f);
  p.seq_rows.resize(f);
  int fo = 0;
  for (int u = 0; u < n_utt; ++u) {
    const int L = lengths[u];
    const int sc = u * per, su = u * per + (per - 1);
    for (int t = 0; t < L; ++t) {
      p.frame_rows[fo + t] = make_int2(p.seq_start[sc] + t, p.seq_start[su] + t);
      p.frame_src[fo + t] = make_int2(MEL * fo + t, L);
      p.frame_utt[fo + t] = u;
      p.seq_rows[fo + t] = p.seq_start[sc] + t;
    }
    fo += L;
  }
  for (int s = 0; s < p.n_seq; ++s)
    for (int q0 = 0; q0 < p.seq_len[s]; q0 += ATT_Q_ROWS)
      p.tiles.push_back(AttnTile{p.seq_start[s], p.seq_len[s], q0, 0});
  // longest query blocks first: the shortest CTAs fill the last wave
  std::stable_sort(p.tiles.begin(), p.tiles.end(), [chunk](const AttnTile& a, const AttnTile& b) {
    return attn_tile_keys(a, chunk) > attn_tile_keys(b, chunk);
  });
  p.key = plan_key(n_utt, lengths, cfg_pairs, chunk, steps);
  return p;
}

int ensure_workspace(lx_flow* h, const Plan& p, size_t in_floats, int n_utt) {
  Workspace& w = h->ws;
  if (p.tiles.size() > static_cast<size_t>(ATT_MAX_TILES))
    return h->fail(LX_ERR_SHAPE, "batch too large: more than 65535 attention query blocks");
  const bool grow = p.R > w.capR || p.Rs > w.capRs || p.F > w.capF ||
                    static_cast<int>(p.tiles.size()) > w.capTiles || in_floats > w.capIn ||
                    static_cast<size_t>(n_utt) > w.capUtt;
  if (grow) {
    clear_graphs(h);
    // q, k and v are one block (k and v point into it)
    w.k = nullptr;
    w.v = nullptr;
    void** ptrs[] = {(void**)&w.x,       (void**)&w.xn,        (void**)&w.q,
                     (void**)&w.ao,        (void**)&w.h,        (void**)&w.stage1,
                     (void**)&w.stage2,  (void**)&w.cst,       (void**)&w.a_cond,   (void**)&w.xb,
                     (void**)&w.dphi,    (void**)&w.xs,        (void**)&w.pos,      (void**)&w.p2s,
                     (void**)&w.s2p,     (void**)&w.frame_utt, (void**)&w.seq_rows, (void**)&w.frame_rows,
                     (void**)&w.frame_src, (void**)&w.tiles,   (void**)&w.in_mu,    (void**)&w.in_cond,
                     (void**)&w.in_noise, (void**)&w.out_mel,  (void**)&w.in_spks,  (void**)&w.cap};
    for (void** pp : ptrs) wsfree(*pp);
    w.capCap = 0;
    // grow with headroom so that nearby shapes reuse the allocation
    w.capR = std::max(p.R, w.capR) + 256;
    w.capRs = std::max(p.Rs, w.capRs) + 256;
    w.capF = std::max(p.F, w.capF) + 256;
    w.capTiles = std::max(static_cast<int>(p.tiles.size()), w.capTiles) + 64;
    w.capIn = std::max(in_floats, w.capIn) + 256 * MEL;
    w.capUtt = std::max(static_cast<size_t>(n_utt), w.capUtt) + 16;
    const size_t R = w.capR, Rs = w.capRs, F = w.capF;
    int rc;
    if ((rc = dev_alloc(h, &w.x, R * DIM, false)) || (rc = dev_alloc(h, &w.xn, R * DIM, false)) ||
        (rc = dev_alloc(h, &w.q, 3 * R * DIM, false)) ||
        (rc = dev_alloc(h, &w.ao, R * DIM, false)) || (rc = dev_alloc(h, &w.h, R * FF, false)) ||
        (rc = dev_alloc(h, &w.stage1, Rs * DIM, false)) || (rc = dev_alloc(h, &w.stage2, Rs * DIM, false)) ||
        (rc = dev_alloc(h, &w.cst, R * DIM, false)) || (rc = dev_alloc(h, &w.a_cond, R * COND_K, false)) ||
        (rc = dev_alloc(h, &w.xb, R * MEL, false)) || (rc = dev_alloc(h, &w.dphi, R * MEL, false)) ||
        (rc = dev_alloc(h, &w.xs, F * MEL, false)) || (rc = dev_alloc(h, &w.pos, R, false)) ||
        (rc = dev_alloc(h, &w.p2s, R, false)) || (rc = dev_alloc(h, &w.s2p, Rs, false)) ||
        (rc = dev_alloc(h, &w.frame_utt, F, false)) || (rc = dev_alloc(h, &w.seq_rows, F, false)) ||
        (rc = dev_alloc(h, &w.frame_rows, F, false)) || (rc = dev_alloc(h, &w.frame_src, F, false)) ||
        (rc = dev_alloc(h, &w.tiles, static_cast<size_t>(w.capTiles), false)) ||
        (rc = dev_alloc(h, &w.in_mu, w.capIn, false)) || (rc = dev_alloc(h, &w.in_cond, w.capIn, false)) ||
        (rc = dev_alloc(h, &w.in_noise, w.capIn, false)) || (rc = dev_alloc(h, &w.out_mel, w.capIn, false)) ||
        (rc = dev_alloc(h, &w.in_spks, w.capUtt * MEL, false)))
      return rc;
    w.k = w.q + R * DIM;
    w.v = reinterpret_cast<__half*>(w.q + 2 * R * DIM);
    // every buffer starts finite: rows that no kernel writes (alignment gaps,
    // rows past the last sequence, staging gap rows) are read as operands
    CK(cudaMemset(w.x, 0, R * DIM * 4));
    CK(cudaMemset(w.xn, 0, R * DIM * 2));
    CK(cudaMemset(w.q, 0, 3 * R * DIM * 2));
    CK(cudaMemset(w.ao, 0, R * DIM * 2));
    CK(cudaMemset(w.h, 0, R * FF * 2));
    CK(cudaMemset(w.stage1, 0, Rs * DIM * 2));
    CK(cudaMemset(w.stage2, 0, Rs * DIM * 2));
    CK(cudaMemset(w.xb, 0, R * MEL * 2));
    CK(cudaMemset(w.pos, 0, R * sizeof(int)));
    bool ok = true;
    ok &= tmap_bf16(&w.tm_xn, w.xn, R, DIM, DIM, 128, 64);
    ok &= tmap_bf16(&w.tm_ao, w.ao, R, DIM, DIM, 128, 64);
    ok &= tmap_bf16(&w.tm_h, w.h, R, FF, FF, 128, 64);
    ok &= tmap_bf16(&w.tm_hs, w.h, R, FF, FF, 32, 64);
    ok &= tmap_bf16(&w.tm_xb, w.xb, R, MEL, MEL, 128, 64);
    ok &= tmap_bf16(&w.tm_acond, w.a_cond, R, COND_K, COND_K, 128, 64);
    ok &= tmap_bf16(&w.tm_stage1, w.stage1, Rs, DIM, DIM, CONV_WIN_ROWS, 64);
    ok &= tmap_bf16(&w.tm_stage2, w.stage2, Rs, DIM, DIM, CONV_WIN_ROWS, 64);
    ok &= tmap_bf16(&w.tm_q, w.q, R, DIM, DIM, 128, 64);
    ok &= tmap_bf16(&w.tm_k, w.k, R, DIM, DIM, 128, 64);
    ok &= tmap_bf16(&w.tm_v, w.v, R, DIM, DIM, 128, 64);
    ok &= tmap_bf16(&w.tm_qkvs, w.q, 3 * R, DIM, DIM, 32, 64);
    ok &= tmap_f32(&w.tm_x, w.x, R, DIM, DIM, 128, 32);
    ok &= tmap_f32(&w.tm_xs, w.x, R, DIM, DIM, 32, 32);
    if (!ok) return h->fail(LX_ERR_CUDA, "cuTensorMapEncodeTiled failed for a workspace tensor");
    ++w.generation;
  }
  return LX_OK;
}

int upload_plan(lx_flow* h, const Plan& p, cudaStream_t s) {
  Workspace& w = h->ws;
  h->cached_valid = false;
  CK(cudaMemcpyAsync(w.pos, p.pos.data(), p.R * sizeof(int), cudaMemcpyHostToDevice, s));
  CK(cudaMemcpyAsync(w.p2s, p.p2s.data(), p.R * sizeof(int), cudaMemcpyHostToDevice, s));
  CK(cudaMemcpyAsync(w.s2p, p.s2p.data(), p.Rs * sizeof(int), cudaMemcpyHostToDevice, s));
  CK(cudaMemcpyAsync(w.frame_rows, p.frame_rows.data(), p.F * sizeof(int2), cudaMemcpyHostToDevice, s));
  CK(cudaMemcpyAsync(w.frame_src, p.frame_src.data(), p.F * sizeof(int2), cudaMemcpyHostToDevice, s));
  CK(cudaMemcpyAsync(w.frame_utt, p.frame_utt.data(), p.F * sizeof(int), cudaMemcpyHostToDevice, s));
  CK(cudaMemcpyAsync(w.seq_rows, p.seq_rows.data(), p.F * sizeof(int), cudaMemcpyHostToDevice, s));
  CK(cudaMemcpyAsync(w.tiles, p.tiles.data(), p.tiles.size() * sizeof(AttnTile), cudaMemcpyHostToDevice, s));
  // conditioning rows that the gather does not write must read as zero
  CK(cudaMemsetAsync(w.a_cond, 0, static_cast<size_t>(p.R) * COND_K * 2, s));
  // the conv staging gaps (causal left padding) must be zero for this layout
  zero_gap_rows(w.stage1, w.stage2, w.s2p, p.Rs, s);
  ++h->launches;
  return LX_OK;
}

// --------------------------------------------------------------------------
// launch sequences
// --------------------------------------------------------------------------
struct StepIO {
  const float* mu;
  const float* cond;
  const float* spks;
  const float* noise;  // or x for the estimator
  float* out;          // mel (decode) or dphi (estimator)
};

// setup shared by decode and estimator: per-row constant of the input
// projection (cond, mu, spks columns + bias) and the initial state.
void enqueue_setup(lx_flow* h, const Plan& p, const StepIO& io, cudaStream_t s) {
  Workspace& w = h->ws;
  Model& W = h->W;
  gather_cond(w.a_cond, io.cond, io.mu, io.spks, w.frame_rows, w.frame_src, w.frame_utt, p.F, s);
  gemm_f32(pick_bn(p.R, DIM), w.tm_acond, W.tm_winc[pick_bn(p.R, DIM) == 256], p.R, DIM, COND_K, W.bin, w.cst, DIM,
           h->d_err, s);
  init_state(w.xs, io.noise, w.frame_rows, w.frame_src, w.xb, p.F, s);
  h->launches += 3;
}

// One DiT forward on the current xb rows with the given modulation tables.
// Optional capture callbacks after input_embed / a block / norm_out.
struct Captures {
  float* input_embed = nullptr;
  float* block = nullptr;       // the block `block_index` only
  int block_index = -1;
  float* blocks_all = nullptr;  // every block, [22][F][1024]
  float* norm_out = nullptr;
};

void enqueue_dit(lx_flow* h, const Plan& p, const float* mod, const float* mod_final, int chunk, cudaStream_t s,
                 const Captures* cap) {
  Workspace& w = h->ws;
  Model& W = h->W;
  const int R = p.R;
  const int bn1024 = pick_bn(R, DIM), bnq = pick_bn(R, QKV_N), bnf = pick_bn(R, FF);
  const int i1024 = bn1024 == 256, iq = bnq == 256, iff = bnf == 256;
  const bool pair_q = use_pair_gemm(R, QKV_N), pair_f = use_pair_gemm(R, FF), pair_d = use_pair_gemm(R, DIM);
  // Row direction per kernel: each row-streaming kernel starts on the rows its
  // producer wrote last (still in L2).  attention (longest sequences, the
  // lowest rows, first) -> out (down) -> AdaLN (up) -> FF1 (down) -> FF2 (up)
  // -> AdaLN (down) -> QKV (up).
  const bool alt = row_order_alternates();
  int* err = h->d_err;
  timed(h, K_INPROJ, s, [&] { gemm_in_proj(bn1024, w.tm_xb, W.tm_winx[i1024], R, w.cst, w.x, w.stage1, w.p2s, err, s); });
  timed(h, K_CONV, s, [&] { conv_pos(w.tm_stage1, W.tm_wconv[0], p.Rs, W.bconv[0], 0, w.stage2, w.x, w.s2p, err, s); });
  timed(h, K_CONV, s, [&] { conv_pos(w.tm_stage2, W.tm_wconv[1], p.Rs, W.bconv[1], 1, nullptr, w.x, w.s2p, err, s); });
  h->launches += 3;
  if (cap && cap->input_embed) {
    gather_rows(cap->input_embed, w.x, w.seq_rows, p.F, DIM, s);
    ++h->launches;
  }
  for (int l = 0; l < DEPTH; ++l) {
    // modulation chunks: shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp
    const float* m = mod + static_cast<size_t>(l) * MOD_N;
    timed(h, K_ADALN, s, [&] { adaln_rows(w.x, w.xn, m + 0 * DIM, m + 1 * DIM, R, s, alt); });
    timed(h, K_QKV, s, [&] {
      if (pair_q)
        gemm_pair_qkv(w.tm_xn, W.tm_wqkv[0], w.tm_qkvs, static_cast<int>(w.capR), R, l * QKV_N,
                      W.bqkv + static_cast<size_t>(l) * QKV_N, w.q, w.k, w.v, w.pos, W.rope, err, s);
      else
        gemm_qkv(bnq, w.tm_xn, W.tm_wqkv[iq], R, l * QKV_N, W.bqkv + static_cast<size_t>(l) * QKV_N, w.q, w.k, w.v,
                 w.pos, W.rope, err, s);
    });
    timed(h, K_ATTN, s,
          [&] { attention(w.tm_q, w.tm_k, w.tm_v, w.tiles, static_cast<int>(p.tiles.size()), chunk, w.ao, err, s); });
    timed(h, K_OUT, s, [&] {
      if (pair_d)
        gemm_pair_gate_res(w.tm_ao, W.tm_wo[0], w.tm_x, w.tm_xs, R, DIM, l * DIM, W.bo + static_cast<size_t>(l) * DIM,
                           m + 2 * DIM, w.x, err, s, alt);
      else
        gemm_gate_res_tma(w.tm_ao, W.tm_wo[0], w.tm_x, R, DIM, l * DIM, W.bo + static_cast<size_t>(l) * DIM,
                          m + 2 * DIM, w.x, err, s);
    });
    timed(h, K_ADALN, s, [&] { adaln_rows(w.x, w.xn, m + 3 * DIM, m + 4 * DIM, R, s); });
    timed(h, K_FF1, s, [&] {
      if (pair_f)
        gemm_pair_gelu(w.tm_xn, W.tm_w1[0], w.tm_hs, R, l * FF, W.b1 + static_cast<size_t>(l) * FF, w.h, err, s,
                       alt);
      else
        gemm_gelu(bnf, w.tm_xn, W.tm_w1[iff], R, l * FF, W.b1 + static_cast<size_t>(l) * FF, w.h, err, s);
    });
    timed(h, K_FF2, s, [&] {
      if (pair_d)
        gemm_pair_gate_res(w.tm_h, W.tm_w2[0], w.tm_x, w.tm_xs, R, FF, l * DIM, W.b2 + static_cast<size_t>(l) * DIM,
                           m + 5 * DIM, w.x, err, s);
      else
        gemm_gate_res_tma(w.tm_h, W.tm_w2[0], w.tm_x, R, FF, l * DIM, W.b2 + static_cast<size_t>(l) * DIM,
                          m + 5 * DIM, w.x, err, s);
    });
    h->launches += 7;
    if (cap && cap->block && cap->block_index == l) {
      gather_rows(cap->block, w.x, w.seq_rows, p.F, DIM, s);
      ++h->launches;
    }
    if (cap && cap->blocks_all) {
      gather_rows(cap->blocks_all + static_cast<size_t>(l) * p.F * DIM, w.x, w.seq_rows, p.F, DIM, s);
      ++h->launches;
    }
  }
  // AdaLayerNormZero_Final: chunk order scale, shift (flow_reference.py:192)
  timed(h, K_ADALN, s, [&] { adaln_rows(w.x, w.xn, mod_final + DIM, mod_final, R, s, alt); });
  timed(h, K_PROJOUT, s, [&] { gemm_f32(128, w.tm_xn, W.tm_wout, R, MEL, DIM, W.bout, w.dphi, MEL, err, s); });
  h->launches += 2;
  if (cap && cap->norm_out) {
    gather_rows_bf16(cap->norm_out, w.xn, w.seq_rows, p.F, DIM, s);
    ++h->launches;
  }
}

void enqueue_decode_steps(lx_flow* h, const Plan& p, int steps, int chunk, cudaStream_t s) {
  struct PdlScope {
    explicit PdlScope(bool on) { pdl_set_auto(on); }
    ~PdlScope() { pdl_set_auto(false); }
  } pdl_scope(p.R <= PDL_AUTO_MAX_ROWS);
  Model& W = h->W;
  for (int st = 0; st < steps; ++st) {
    enqueue_dit(h, p, W.mod + static_cast<size_t>(st) * DEPTH * MOD_N, W.mod_final + static_cast<size_t>(st) * 2 * DIM,
                chunk, s, nullptr);
    timed(h, K_EULER, s,
          [&] { euler_update(h->ws.xs, h->ws.dphi, h->ws.frame_rows, h->ws.xb, p.F, W.sched_dt[st], CFG_RATE, s); });
    ++h->launches;
  }
}

int check_device_error(lx_flow* h, cudaStream_t s) {
  CK(cudaGetLastError());
  CK(cudaStreamSynchronize(s));
  int e = 0;
  CK(cudaMemcpy(&e, h->d_err, sizeof(int), cudaMemcpyDeviceToHost));
  if (e != 0) {
    cudaMemset(h->d_err, 0, sizeof(int));
    return h->fail(LX_ERR_TIMEOUT, "device-side wait exceeded its bound (code " + std::to_string(e) + ")");
  }
  return LX_OK;
}

int validate_batch(lx_flow* h, const lx_flow_batch* b, size_t* total) {
  if (!b || b->n_utt <= 0 || !b->lengths || !b->mu || !b->cond || !b->spks || !b->mel_out)
    return h->fail(LX_ERR_ARG, "lx_flow_batch: null pointer or n_utt <= 0");
  if (b->chunk < 0) return h->fail(LX_ERR_ARG, "chunk must be >= 0");
  const int steps = b->n_steps == 0 ? N_STEPS_DEFAULT : b->n_steps;
  if (steps < 1 || steps > h->W.n_sched)
    return h->fail(LX_ERR_ARG, "n_steps must be 1..10 (a prefix of the 10-step cosine schedule)");
  size_t tot = 0;
  for (int u = 0; u < b->n_utt; ++u) {
    if (b->lengths[u] <= 0 || b->lengths[u] >= ROPE_MAX)
      return h->fail(LX_ERR_SHAPE, "utterance length out of range [1, 16383]");
    tot += static_cast<size_t>(b->lengths[u]);
  }
  if (!b->noise && !h->noise_loaded) return h->fail(LX_ERR_STATE, "no noise given and no noise bank loaded");
  if (!b->noise)
    for (int u = 0; u < b->n_utt; ++u)
      if (b->lengths[u] > LX_NOISE_MAX_FRAMES) return h->fail(LX_ERR_SHAPE, "utterance longer than the noise bank");
  *total = tot;
  return LX_OK;
}

std::string plan_key(int n_utt, const int32_t* lengths, bool cfg_pairs, int chunk, int steps) {
  std::string k = std::string(cfg_pairs ? "D" : "E") + ":" + std::to_string(chunk) + ":" + std::to_string(steps) + ":";
  for (int u = 0; u < n_utt; ++u) k += std::to_string(lengths[u]) + ",";
  return k;
}

// decode with inputs already on the device
int run_decode(lx_flow* h, const lx_flow_batch* b, const float* mu, const float* cond, const float* spks,
               const float* noise, float* out, cudaStream_t s) {
  const int steps = b->n_steps == 0 ? h->W.n_sched : b->n_steps;
  int rc;
  const std::string key = plan_key(b->n_utt, b->lengths, true, b->chunk, steps);
  if (!(h->cached_valid && h->cached_plan.key == key && h->cached_gen == h->ws.generation)) {
    Plan np_ = make_plan(b->n_utt, b->lengths, true, b->chunk, steps);
    if ((rc = ensure_workspace(h, np_, static_cast<size_t>(np_.F) * MEL, b->n_utt))) return rc;
    if ((rc = upload_plan(h, np_, s))) return rc;
    h->cached_plan = std::move(np_);
    h->cached_gen = h->ws.generation;
    h->cached_valid = true;
  }
  const Plan& p = h->cached_plan;
  StepIO io{mu, cond, spks, noise, out};
  enqueue_setup(h, p, io, s);
  if (h->use_graphs && !h->prof) {
    char ptrs[64];
    std::snprintf(ptrs, sizeof ptrs, "|g%llu", static_cast<unsigned long long>(h->ws.generation));
    const std::string key = p.key + ptrs;
    auto it = h->graphs.find(key);
    if (it == h->graphs.end()) {
      cudaStream_t cs;
      CK(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking));
      const uint64_t before = h->launches;
      cudaGraph_t g = nullptr;
      cudaError_t e = cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal);
      if (e == cudaSuccess) {
        enqueue_decode_steps(h, p, steps, b->chunk, cs);
        e = cudaStreamEndCapture(cs, &g);
      }
      cudaStreamDestroy(cs);
      h->launches = before;  // counted at replay
      if (e != cudaSuccess) {
        if (g) cudaGraphDestroy(g);
        return cuda_fail(h, e, "graph capture");
      }
      lx_flow::GraphEntry ge;
      size_t n = 0;
      cudaGraphGetNodes(g, nullptr, &n);
      ge.nodes = n;
      e = cudaGraphInstantiate(&ge.exec, g, 0);
      cudaGraphDestroy(g);
      if (e != cudaSuccess) return cuda_fail(h, e, "graph instantiate");
      it = h->graphs.emplace(key, ge).first;
    }
    CK(cudaGraphLaunch(it->second.exec, s));
    h->launches += it->second.nodes;
  } else {
    enqueue_decode_steps(h, p, steps, b->chunk, s);
  }
  scatter_mel(out, h->ws.xs, h->ws.frame_src, p.F, s);
  ++h->launches;
  CK(cudaGetLastError());
  return LX_OK;
}

}  // namespace

// ==========================================================================
// C ABI
// ==========================================================================
extern "C" {

int lx_flow_create(int device, lx_flow** out) {
  if (!out) return LX_ERR_ARG;
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return LX_ERR_CUDA;
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess || prop.major != 10) return LX_ERR_CUDA;
  if (cudaSetDevice(device) != cudaSuccess) return LX_ERR_CUDA;
  if (!attention_ready()) return LX_ERR_CUDA;
  std::unique_ptr<lx_flow> h(new lx_flow());
  h->device = device;
  if (cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking) != cudaSuccess) return LX_ERR_CUDA;
  if (cudaMalloc(&h->d_err, sizeof(int)) != cudaSuccess) return LX_ERR_OOM;
  cudaMemset(h->d_err, 0, sizeof(int));
  const char* g = std::getenv("LX_FLOW_GRAPHS");
  if (g && std::strcmp(g, "0") == 0) h->use_graphs = false;
  *out = h.release();
  return LX_OK;
}

void lx_flow_destroy(lx_flow* h) {
  if (!h) return;
  cudaSetDevice(h->device);
  cudaStreamSynchronize(h->stream);
  clear_graphs(h);
  Workspace& w = h->ws;
  // (w.k and w.v point into w.q's block)
  void* ws_ptrs[] = {w.x,        w.xn,       w.q,          w.ao,       w.h,
                     w.stage1,   w.stage2,   w.cst,        w.a_cond,    w.xb,        w.dphi,     w.xs,
                     w.pos,      w.p2s,      w.s2p,        w.frame_utt, w.seq_rows,  w.frame_rows, w.frame_src,
                     w.tiles,    w.in_mu,    w.in_cond,    w.in_noise,  w.out_mel,   w.in_spks,  w.cap,
                     h->f_spk_in, h->f_spk,  h->f_emb,     h->f_h,      h->f_pre,    h->f_mu,    h->f_cond,
                     h->f_pf,    h->f_tok};
  for (void* p : ws_ptrs)
    if (p) cudaFree(p);
  for (void* p : h->allocs) cudaFree(p);
  if (h->d_err) cudaFree(h->d_err);
  if (h->stream) cudaStreamDestroy(h->stream);
  delete h;
}

const char* lx_flow_last_error(const lx_flow* h) { return h ? h->err.c_str() : "null handle"; }

uint64_t lx_flow_launch_count(const lx_flow* h) { return h ? h->launches : 0; }

int lx_flow_load_gguf(lx_flow* h, const char* path) {
  if (!h || !path) return LX_ERR_ARG;
  if (h->loaded) return LX_OK;
  CK(cudaSetDevice(h->device));
  int rc = load_model(h, path);
  if (rc) {
    for (void* p : h->allocs) cudaFree(p);
    h->allocs.clear();
    h->W = Model();
    return rc;
  }
  h->gguf_path = path;
  h->loaded = true;
  return LX_OK;
}

int lx_flow_save_layout(lx_flow* h, const char* path) {
  if (!h || !path) return LX_ERR_ARG;
  if (!h->loaded) return h->fail(LX_ERR_STATE, "no model loaded");
  CK(cudaSetDevice(h->device));
  CK(cudaStreamSynchronize(h->stream));
  std::string msg;
  const int rc = save_layout_file(h->W, h->gguf_path, path, &msg);
  return rc ? h->fail(rc, msg) : LX_OK;
}

int lx_flow_load_layout(lx_flow* h, const char* path) {
  if (!h || !path) return LX_ERR_ARG;
  if (h->loaded) return LX_OK;
  CK(cudaSetDevice(h->device));
  Model& W = h->W;
  std::string msg;
  int rc = load_layout_file(W, h->allocs, path, &msg);
  if (!rc)
    rc = (dev_alloc(h, &W.mod_x, static_cast<size_t>(DEPTH) * MOD_N)) ||
                 (dev_alloc(h, &W.mod_final_x, 2 * DIM)) || (dev_alloc(h, &W.temb_x, DIM)) ||
                 (dev_alloc(h, &W.tscratch, 16 * 256 + 16 * DIM + 64))
             ? LX_ERR_OOM
             : LX_OK;
  else
    h->fail(rc, msg);
  if (!rc) {
    make_schedule(N_STEPS_DEFAULT, W.sched_t, W.sched_dt);
    W.n_sched = N_STEPS_DEFAULT;
    rc = build_model_maps(h);
  }
  if (rc) {
    for (void* p : h->allocs) cudaFree(p);
    h->allocs.clear();
    h->W = Model();
    return rc;
  }
  h->gguf_path.clear();
  h->loaded = true;
  return LX_OK;
}

int lx_flow_load_noise(lx_flow* h, const char* path) {
  if (!h || !path) return LX_ERR_ARG;
  if (h->noise_loaded) return LX_OK;
  FILE* f = std::fopen(path, "rb");
  if (!f) return h->fail(LX_ERR_IO, std::string("cannot open noise asset ") + path);
  uint32_t magic = 0, version = 0, mel = 0;
  uint64_t maxf = 0;
  bool ok = std::fread(&magic, 4, 1, f) == 1 && std::fread(&version, 4, 1, f) == 1 &&
            std::fread(&mel, 4, 1, f) == 1 && std::fread(&maxf, 8, 1, f) == 1;
  if (!ok || magic != 0x45534E46u || version != 1 || mel != MEL || maxf != LX_NOISE_MAX_FRAMES) {
    std::fclose(f);
    return h->fail(LX_ERR_FORMAT, std::string("bad noise asset header in ") + path);
  }
  std::vector<float> buf(static_cast<size_t>(MEL) * LX_NOISE_MAX_FRAMES);
  ok = std::fread(buf.data(), 4, buf.size(), f) == buf.size();
  std::fclose(f);
  if (!ok) return h->fail(LX_ERR_FORMAT, std::string("short read on noise asset ") + path);
  h->noise.swap(buf);
  h->noise_loaded = true;
  return LX_OK;
}

int lx_flow_decode_device(lx_flow* h, const lx_flow_batch* b, void* stream) {
  if (!h) return LX_ERR_ARG;
  if (!h->loaded) return h->fail(LX_ERR_STATE, "lx_flow_load_gguf has not succeeded");
  size_t tot = 0;
  int rc = validate_batch(h, b, &tot);
  if (rc) return rc;
  if (!b->noise) return h->fail(LX_ERR_ARG, "lx_flow_decode_device needs explicit device noise");
  CK(cudaSetDevice(h->device));
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : h->stream;
  return run_decode(h, b, b->mu, b->cond, b->spks, b->noise, b->mel_out, s);
}

int lx_flow_profile_decode(lx_flow* h, const lx_flow_batch* b, void* stream, double* ms_by_class,
                           int* launches_by_class, int n_class) {
  if (!h || !ms_by_class || !launches_by_class || n_class < K_NCLASS) return LX_ERR_ARG;
  if (!h->loaded) return h->fail(LX_ERR_STATE, "lx_flow_load_gguf has not succeeded");
  size_t tot = 0;
  int rc = validate_batch(h, b, &tot);
  if (rc) return rc;
  if (!b->noise) return h->fail(LX_ERR_ARG, "lx_flow_profile_decode needs explicit device noise");
  CK(cudaSetDevice(h->device));
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : h->stream;
  lx_flow::Prof prof;
  h->prof = &prof;
  rc = run_decode(h, b, b->mu, b->cond, b->spks, b->noise, b->mel_out, s);
  h->prof = nullptr;
  if (rc) return rc;
  if ((rc = check_device_error(h, s))) return rc;
  for (int c = 0; c < n_class; ++c) {
    ms_by_class[c] = 0.0;
    launches_by_class[c] = 0;
  }
  for (auto& r : prof.recs) {
    float ms = 0.f;
    cudaEventElapsedTime(&ms, r.a, r.b);
    ms_by_class[r.cls] += ms;
    launches_by_class[r.cls] += 1;
  }
  return LX_OK;
}

int lx_flow_decode(lx_flow* h, const lx_flow_batch* b) {
  if (!h) return LX_ERR_ARG;
  if (!h->loaded) return h->fail(LX_ERR_STATE, "lx_flow_load_gguf has not succeeded");
  size_t tot = 0;
  int rc = validate_batch(h, b, &tot);
  if (rc) return rc;
  CK(cudaSetDevice(h->device));
  cudaStream_t s = h->stream;
  // make room for the inputs (plan sizes are recomputed inside run_decode)
  Plan p0 = make_plan(b->n_utt, b->lengths, true, b->chunk, h->W.n_sched);
  if ((rc = ensure_workspace(h, p0, tot * MEL, b->n_utt))) return rc;
  Workspace& w = h->ws;
  const size_t nb = tot * MEL * sizeof(float);
  CK(cudaMemcpyAsync(w.in_mu, b->mu, nb, cudaMemcpyHostToDevice, s));
  CK(cudaMemcpyAsync(w.in_cond, b->cond, nb, cudaMemcpyHostToDevice, s));
  CK(cudaMemcpyAsync(w.in_spks, b->spks, static_cast<size_t>(b->n_utt) * MEL * sizeof(float), cudaMemcpyHostToDevice, s));
  if (b->noise) {
    CK(cudaMemcpyAsync(w.in_noise, b->noise, nb, cudaMemcpyHostToDevice, s));
  } else {
    // slice the bank per utterance: [c][t] of the first T_u columns
    std::vector<float> nz(tot * MEL);
    size_t off = 0;
    for (int u = 0; u < b->n_utt; ++u) {
      const int L = b->lengths[u];
      for (int c = 0; c < MEL; ++c)
        std::memcpy(&nz[off + static_cast<size_t>(c) * L], &h->noise[static_cast<size_t>(c) * LX_NOISE_MAX_FRAMES],
                    L * sizeof(float));
      off += static_cast<size_t>(L) * MEL;
    }
    CK(cudaMemcpyAsync(w.in_noise, nz.data(), nb, cudaMemcpyHostToDevice, s));
    CK(cudaStreamSynchronize(s));
  }
  rc = run_decode(h, b, w.in_mu, w.in_cond, w.in_spks, w.in_noise, w.out_mel, s);
  if (rc) return rc;
  CK(cudaMemcpyAsync(b->mel_out, w.out_mel, nb, cudaMemcpyDeviceToHost, s));
  return check_device_error(h, s);
}

int lx_flow_estimator(lx_flow* h, int n_seq, const int32_t* lengths, const float* x, const float* mu,
                      const float* cond, const float* spks, float t, int chunk, float* dphi_out,
                      float* input_embed_out, float* block_out, int block_index, float* norm_out) {
  if (!h) return LX_ERR_ARG;
  if (!h->loaded) return h->fail(LX_ERR_STATE, "lx_flow_load_gguf has not succeeded");
  if (n_seq <= 0 || !lengths || !x || !mu || !cond || !spks || !dphi_out || chunk < 0)
    return h->fail(LX_ERR_ARG, "lx_flow_estimator: bad argument");
  if (block_out && (block_index < 0 || block_index >= DEPTH)) return h->fail(LX_ERR_ARG, "block_index out of range");
  size_t tot = 0;
  for (int i = 0; i < n_seq; ++i) {
    if (lengths[i] <= 0 || lengths[i] >= ROPE_MAX) return h->fail(LX_ERR_SHAPE, "sequence length out of range");
    tot += lengths[i];
  }
  CK(cudaSetDevice(h->device));
  cudaStream_t s = h->stream;
  Plan p = make_plan(n_seq, lengths, false, chunk, 1);
  int rc = ensure_workspace(h, p, tot * MEL, n_seq);
  if (rc) return rc;
  Workspace& w = h->ws;
  if (w.capCap < 3 * tot * DIM) {
    wsfree(reinterpret_cast<void*&>(w.cap));
    if ((rc = dev_alloc(h, &w.cap, 3 * tot * DIM, false))) return rc;
    w.capCap = 3 * tot * DIM;
  }
  const size_t nb = tot * MEL * sizeof(float);
  CK(cudaMemcpyAsync(w.in_mu, mu, nb, cudaMemcpyHostToDevice, s));
  CK(cudaMemcpyAsync(w.in_cond, cond, nb, cudaMemcpyHostToDevice, s));
  CK(cudaMemcpyAsync(w.in_noise, x, nb, cudaMemcpyHostToDevice, s));
  CK(cudaMemcpyAsync(w.in_spks, spks, static_cast<size_t>(n_seq) * MEL * sizeof(float), cudaMemcpyHostToDevice, s));
  if ((rc = upload_plan(h, p, s))) return rc;
  // modulation for this t
  float* d_t = h->W.tscratch + 16 * 256 + 16 * DIM;
  CK(cudaMemcpyAsync(d_t, &t, sizeof(float), cudaMemcpyHostToDevice, s));
  CK(cudaStreamSynchronize(s));
  modulation_tables(h, d_t, 1, h->W.temb_x, h->W.mod_x, h->W.mod_final_x, s);
  StepIO io{w.in_mu, w.in_cond, w.in_spks, w.in_noise, nullptr};
  enqueue_setup(h, p, io, s);
  Captures cap;
  cap.input_embed = input_embed_out ? w.cap : nullptr;
  cap.block = block_out ? w.cap + tot * DIM : nullptr;
  cap.block_index = block_index;
  cap.norm_out = norm_out ? w.cap + 2 * tot * DIM : nullptr;
  enqueue_dit(h, p, h->W.mod_x, h->W.mod_final_x, chunk, s, &cap);
  // dphi rows -> [80][T] per sequence: gather rows then transpose on the host
  std::vector<float> rows(static_cast<size_t>(p.F) * MEL);
  {
    // reuse gather_rows with width 80 over the cond rows
    gather_rows(w.out_mel, w.dphi, w.seq_rows, p.F, MEL, s);
    ++h->launches;
    CK(cudaMemcpyAsync(rows.data(), w.out_mel, rows.size() * sizeof(float), cudaMemcpyDeviceToHost, s));
  }
  if (input_embed_out) CK(cudaMemcpyAsync(input_embed_out, cap.input_embed, tot * DIM * 4, cudaMemcpyDeviceToHost, s));
  if (block_out) CK(cudaMemcpyAsync(block_out, cap.block, tot * DIM * 4, cudaMemcpyDeviceToHost, s));
  if (norm_out) CK(cudaMemcpyAsync(norm_out, cap.norm_out, tot * DIM * 4, cudaMemcpyDeviceToHost, s));
  if ((rc = check_device_error(h, s))) return rc;
  size_t off = 0;
  for (int i = 0; i < n_seq; ++i) {
    const int L = lengths[i];
    for (int tt = 0; tt < L; ++tt)
      for (int c = 0; c < MEL; ++c) dphi_out[off * MEL + static_cast<size_t>(c) * L + tt] = rows[(off + tt) * MEL + c];
    off += L;
  }
  return LX_OK;
}

int lx_flow_infer(lx_flow* h, const int32_t* prompt_tokens, int n_prompt, const int32_t* tokens, int n_tokens,
                  const float* prompt_feat, int mel_len1, const float* spk_embedding, const float* noise_z,
                  float* mel_out, size_t mel_cap, lx_flow_debug* debug) {
  return lx_flow_infer_ex(h, prompt_tokens, n_prompt, tokens, n_tokens, prompt_feat, mel_len1, spk_embedding, noise_z,
                          1, 0, mel_out, mel_cap, debug);
}

int lx_flow_infer_ex(lx_flow* h, const int32_t* prompt_tokens, int n_prompt, const int32_t* tokens, int n_tokens,
                     const float* prompt_feat, int mel_len1, const float* spk_embedding, const float* noise_z,
                     int finalize, int chunk, float* mel_out, size_t mel_cap, lx_flow_debug* debug) {
  if (!h) return LX_ERR_ARG;
  if (chunk < 0) return h->fail(LX_ERR_ARG, "lx_flow_infer_ex: chunk < 0");
  if (!h->loaded) return h->fail(LX_ERR_STATE, "lx_flow_load_gguf has not succeeded");
  if (n_prompt < 0 || n_tokens < 0 || (n_prompt > 0 && !prompt_tokens) || (n_tokens > 0 && !tokens) ||
      !spk_embedding || !mel_out || mel_len1 < 0 || (mel_len1 > 0 && !prompt_feat))
    return h->fail(LX_ERR_ARG, "lx_flow_infer: bad argument");
  const int n_tok = n_prompt + n_tokens;
  // streaming call: the last PRE_LOOKAHEAD tokens are PreLookahead context only
  const int n_pre = finalize ? n_tok : n_tok - PRE_LOOKAHEAD;
  if (!finalize && n_pre <= 0) return h->fail(LX_ERR_SHAPE, "a streaming call needs more tokens than the look-ahead");
  const int T = 2 * n_pre;
  if (T <= 0 || mel_len1 > T) return h->fail(LX_ERR_SHAPE, "prompt_feat longer than the mel sequence");
  if (!noise_z && !h->noise_loaded) return h->fail(LX_ERR_STATE, "lx_flow_load_noise has not succeeded");
  if (!noise_z && T > LX_NOISE_MAX_FRAMES) return h->fail(LX_ERR_SHAPE, "sequence longer than the noise bank");
  const size_t out_n = static_cast<size_t>(MEL) * (T - mel_len1);
  if (mel_cap < out_n) return h->fail(LX_ERR_ARG, "mel_out too small");
  CK(cudaSetDevice(h->device));
  cudaStream_t s = h->stream;
  Model& W = h->W;
  int rc;
  if (n_tok > h->f_cap) {
    void** fp[] = {(void**)&h->f_spk_in, (void**)&h->f_spk, (void**)&h->f_emb, (void**)&h->f_h, (void**)&h->f_pre,
                   (void**)&h->f_mu,     (void**)&h->f_cond, (void**)&h->f_pf, (void**)&h->f_tok};
    for (void** p : fp) wsfree(*p);
    const size_t cap = static_cast<size_t>(n_tok) + 64;
    if ((rc = dev_alloc(h, &h->f_spk_in, 192, false)) || (rc = dev_alloc(h, &h->f_spk, MEL, false)) ||
        (rc = dev_alloc(h, &h->f_emb, cap * MEL, false)) || (rc = dev_alloc(h, &h->f_h, cap * DIM, false)) ||
        (rc = dev_alloc(h, &h->f_pre, cap * MEL, false)) || (rc = dev_alloc(h, &h->f_mu, 2 * cap * MEL, false)) ||
        (rc = dev_alloc(h, &h->f_cond, 2 * cap * MEL, false)) || (rc = dev_alloc(h, &h->f_pf, 2 * cap * MEL, false)) ||
        (rc = dev_alloc(h, &h->f_tok, cap, false)))
      return rc;
    h->f_cap = static_cast<int>(cap);
  }
  std::vector<int32_t> tok(n_tok);
  for (int i = 0; i < n_prompt; ++i) tok[i] = prompt_tokens[i];
  for (int i = 0; i < n_tokens; ++i) tok[n_prompt + i] = tokens[i];
  CK(cudaMemcpyAsync(h->f_tok, tok.data(), n_tok * sizeof(int), cudaMemcpyHostToDevice, s));
  CK(cudaMemcpyAsync(h->f_spk_in, spk_embedding, 192 * sizeof(float), cudaMemcpyHostToDevice, s));
  if (mel_len1 > 0)
    CK(cudaMemcpyAsync(h->f_pf, prompt_feat, static_cast<size_t>(mel_len1) * MEL * sizeof(float),
                       cudaMemcpyHostToDevice, s));
  // frontend (flow.cpp:134-182): spk affine, embedding, PreLookahead, x2 repeat, cond pad
  frontend_spk(h->f_spk_in, W.spk_w, W.spk_b, h->f_spk, s);
  frontend_embed(h->f_tok, n_tok, W.emb, 6561, h->f_emb, s);
  frontend_conv1(h->f_emb, n_tok, n_pre, W.pre1_w, W.pre1_b, h->f_h, s);
  frontend_conv2(h->f_h, h->f_emb, n_pre, W.pre2_w, W.pre2_b, h->f_pre, s);
  frontend_mu_cond(h->f_pre, n_pre, h->f_pf, mel_len1, h->f_mu, h->f_cond, s);
  h->launches += 5;
  // noise
  Plan p0 = make_plan(1, &T, true, 0, W.n_sched);
  if ((rc = ensure_workspace(h, p0, static_cast<size_t>(T) * MEL, 1))) return rc;
  Workspace& w = h->ws;
  if (noise_z) {
    CK(cudaMemcpyAsync(w.in_noise, noise_z, static_cast<size_t>(T) * MEL * sizeof(float), cudaMemcpyHostToDevice, s));
  } else {
    for (int c = 0; c < MEL; ++c)
      CK(cudaMemcpyAsync(w.in_noise + static_cast<size_t>(c) * T, &h->noise[static_cast<size_t>(c) * LX_NOISE_MAX_FRAMES],
                         T * sizeof(float), cudaMemcpyHostToDevice, s));
  }
  if (debug) {
    if (debug->spk) CK(cudaMemcpyAsync(debug->spk, h->f_spk, MEL * 4, cudaMemcpyDeviceToHost, s));
    if (debug->mu) CK(cudaMemcpyAsync(debug->mu, h->f_mu, static_cast<size_t>(T) * MEL * 4, cudaMemcpyDeviceToHost, s));
    if (debug->cond)
      CK(cudaMemcpyAsync(debug->cond, h->f_cond, static_cast<size_t>(T) * MEL * 4, cudaMemcpyDeviceToHost, s));
    if (debug->token_embed)
      CK(cudaMemcpyAsync(debug->token_embed, h->f_emb, static_cast<size_t>(n_tok) * MEL * 4, cudaMemcpyDeviceToHost, s));
    if (debug->prelookahead)
      CK(cudaMemcpyAsync(debug->prelookahead, h->f_pre, static_cast<size_t>(n_pre) * MEL * 4, cudaMemcpyDeviceToHost,
                         s));
    // both CFG rows run at the same t, so the two rows of time_embed are equal
    if (debug->time_embed)
      for (int r = 0; r < 2; ++r)
        CK(cudaMemcpyAsync(debug->time_embed + r * DIM, W.temb, DIM * 4, cudaMemcpyDeviceToHost, s));
  }
  lx_flow_batch b{};
  b.n_utt = 1;
  b.lengths = &T;
  b.mu = h->f_mu;
  b.cond = h->f_cond;
  b.spks = h->f_spk;
  b.noise = w.in_noise;
  b.mel_out = w.out_mel;
  b.chunk = chunk;
  b.n_steps = 0;
  const bool want_stages = debug && (debug->input_proj || debug->conv_pos || debug->input_embed || debug->blocks ||
                                     debug->norm_out || debug->dphi);
  if (want_stages) {
    // step-1 captures: one estimator pass on [x; x] rows with the step-1 modulation
    Plan p = make_plan(1, &T, true, 0, 1);
    if ((rc = upload_plan(h, p, s))) return rc;
    const size_t rows2 = static_cast<size_t>(2) * T;
    const size_t need = (2 + static_cast<size_t>(DEPTH)) * rows2 * DIM;
    if (w.capCap < need) {
      wsfree(reinterpret_cast<void*&>(w.cap));
      if ((rc = dev_alloc(h, &w.cap, need, false))) return rc;
      w.capCap = need;
    }
    StepIO io{h->f_mu, h->f_cond, h->f_spk, w.in_noise, nullptr};
    enqueue_setup(h, p, io, s);
    // capture rows: cond rows then uncond rows
    std::vector<int> crow(rows2);
    for (int t = 0; t < T; ++t) {
      crow[t] = p.seq_start[0] + t;
      crow[T + t] = p.seq_start[1] + t;
    }
    CK(cudaMemcpyAsync(w.seq_rows, crow.data(), rows2 * sizeof(int), cudaMemcpyHostToDevice, s));
    h->cached_valid = false;
    Plan pc = p;
    pc.F = static_cast<int>(rows2);
    // conv_pos = input_embed - input_proj: both are fetched when it is asked for
    std::vector<float> proj_tmp, embed_tmp;
    float* proj_dst = debug->input_proj;
    float* embed_dst = debug->input_embed;
    if (debug->conv_pos && !proj_dst) {
      proj_tmp.resize(rows2 * DIM);
      proj_dst = proj_tmp.data();
    }
    if (debug->conv_pos && !embed_dst) {
      embed_tmp.resize(rows2 * DIM);
      embed_dst = embed_tmp.data();
    }
    if (proj_dst) {
      // input_proj = x after the in-proj GEMM, before the conv-pos residual
      gemm_in_proj(pick_bn(p.R, DIM), w.tm_xb, W.tm_winx[pick_bn(p.R, DIM) == 256], p.R, w.cst, w.x, w.stage1, w.p2s,
                   h->d_err, s);
      gather_rows(w.cap, w.x, w.seq_rows, static_cast<int>(rows2), DIM, s);
      CK(cudaMemcpyAsync(proj_dst, w.cap, rows2 * DIM * 4, cudaMemcpyDeviceToHost, s));
      h->launches += 2;
    }
    {
      Captures cap;
      cap.input_embed = embed_dst ? w.cap : nullptr;
      cap.norm_out = debug->norm_out ? w.cap + rows2 * DIM : nullptr;
      cap.blocks_all = debug->blocks ? w.cap + 2 * rows2 * DIM : nullptr;
      enqueue_dit(h, pc, W.mod, W.mod_final, 0, s, &cap);
      if (cap.input_embed) CK(cudaMemcpyAsync(embed_dst, cap.input_embed, rows2 * DIM * 4, cudaMemcpyDeviceToHost, s));
      if (cap.norm_out) CK(cudaMemcpyAsync(debug->norm_out, cap.norm_out, rows2 * DIM * 4, cudaMemcpyDeviceToHost, s));
      if (cap.blocks_all)
        CK(cudaMemcpyAsync(debug->blocks, cap.blocks_all, static_cast<size_t>(DEPTH) * rows2 * DIM * 4,
                           cudaMemcpyDeviceToHost, s));
      CK(cudaStreamSynchronize(s));
      if (debug->conv_pos)
        for (size_t i = 0; i < rows2 * DIM; ++i) debug->conv_pos[i] = embed_dst[i] - proj_dst[i];
    }
    if (debug->dphi) {
      std::vector<float> rows(rows2 * MEL);
      gather_rows(w.out_mel, w.dphi, w.seq_rows, static_cast<int>(rows2), MEL, s);
      CK(cudaMemcpyAsync(rows.data(), w.out_mel, rows.size() * 4, cudaMemcpyDeviceToHost, s));
      CK(cudaStreamSynchronize(s));
      for (int r = 0; r < 2; ++r)
        for (int t = 0; t < T; ++t)
          for (int c = 0; c < MEL; ++c)
            debug->dphi[(static_cast<size_t>(r) * MEL + c) * T + t] = rows[(static_cast<size_t>(r) * T + t) * MEL + c];
    }
    if ((rc = check_device_error(h, s))) return rc;
  }
  if ((rc = run_decode(h, &b, b.mu, b.cond, b.spks, b.noise, w.out_mel, s))) return rc;
  // feat = x[:, :, mel_len1:] (flow.cpp:277-280)
  std::vector<float> full(static_cast<size_t>(T) * MEL);
  CK(cudaMemcpyAsync(full.data(), w.out_mel, full.size() * 4, cudaMemcpyDeviceToHost, s));
  if ((rc = check_device_error(h, s))) return rc;
  const int OUT = T - mel_len1;
  for (int c = 0; c < MEL; ++c)
    std::memcpy(mel_out + static_cast<size_t>(c) * OUT, &full[static_cast<size_t>(c) * T + mel_len1], OUT * 4);
  return LX_OK;
}

int lx_flow_op(int op, int in_bf16, int rows, const void* x, void* y, const float* shift, const float* scale,
               const float* gate, const int32_t* pos, void* stream) {
  if (rows < 0 || !x || !y) return LX_ERR_ARG;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Programmatic dependent launch (unless LX_FLOW_PDL=0): the op may start
  // while the previous kernel of the stream drains; its blocks wait inside
  // before touching memory, so any predecessor is safe.  In a chain of short
  // ops one launch's ramp then overlaps the last one's tail.
  struct PdlOn {
    PdlOn() { pdl_set_auto(true); }
    ~PdlOn() { pdl_set_auto(false); }
  } pdl_on;
  switch (op) {
    case 0:
      if (!shift || !scale) return LX_ERR_ARG;
      if (in_bf16)
        op_adaln_bf16(static_cast<const bf16*>(x), static_cast<float*>(y), shift, scale, rows, s);
      else
        op_adaln_f32(static_cast<const float*>(x), static_cast<float*>(y), shift, scale, rows, s);
      break;
    case 1:  // x (fp32, in/out) += gate * y  -- here `x` is the residual, `y` the branch
      if (!gate) return LX_ERR_ARG;
      if (in_bf16)
        op_gate_res_bf16(static_cast<float*>(const_cast<void*>(x)), static_cast<const bf16*>(y), gate, rows, s);
      else
        op_gate_res_f32(static_cast<float*>(const_cast<void*>(x)), static_cast<const float*>(y), gate, rows, s);
      break;
    case 2: {
      if (!pos) return LX_ERR_ARG;
      // per-device rotary table, built once
      static float2* tables[64] = {nullptr};
      int dev = 0;
      cudaGetDevice(&dev);
      if (!tables[dev & 63]) {
        std::vector<float2> rope(static_cast<size_t>(ROPE_MAX) * 32);
        for (int i = 0; i < 32; ++i) {
          const float inv = 1.0f / powf(10000.0f, static_cast<float>(2 * i) / 64.0f);
          for (int p = 0; p < ROPE_MAX; ++p) {
            const float ang = static_cast<float>(p) * inv;
            rope[static_cast<size_t>(p) * 32 + i] = make_float2(static_cast<float>(cos(static_cast<double>(ang))),
                                                                static_cast<float>(sin(static_cast<double>(ang))));
          }
        }
        float2* d = nullptr;
        if (cudaMalloc(&d, rope.size() * sizeof(float2)) != cudaSuccess) return LX_ERR_OOM;
        if (cudaMemcpy(d, rope.data(), rope.size() * sizeof(float2), cudaMemcpyHostToDevice) != cudaSuccess)
          return LX_ERR_CUDA;
        tables[dev & 63] = d;
      }
      if (in_bf16)
        op_rotary_bf16(static_cast<const bf16*>(x), static_cast<float*>(y), pos, tables[dev & 63], rows, s);
      else
        op_rotary_f32(static_cast<const float*>(x), static_cast<float*>(y), pos, tables[dev & 63], rows, s);
      break;
    }
    case 3:
      if (in_bf16)
        op_gelu_bf16(static_cast<const bf16*>(x), static_cast<float*>(y), static_cast<size_t>(rows) * DIM, s);
      else
        op_gelu_f32(static_cast<const float*>(x), static_cast<float*>(y), static_cast<size_t>(rows) * DIM, s);
      break;
    default:
      return LX_ERR_ARG;
  }
  return cudaGetLastError() == cudaSuccess ? LX_OK : LX_ERR_CUDA;
}

}  // extern "C"
