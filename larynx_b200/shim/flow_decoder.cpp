// larynx::flow::FlowDecoder implemented over the B200 library's C ABI.
//
// This is the reference-side binding: it implements the unchanged interface
// of include/larynx/flow/flow.h (FlowDecoder, FlowDebug, module_name) by
// forwarding to include/larynx_flow.h, so src/pipeline/pipeline.cpp and
// tests/flow_dump.cpp of the reference compile and link against it as they
// are.  A maintainer drops src/flow/*.cpp from the flow target and adds this
// file (include path: this repository's include/; link:
// larynx_b200/liblarynx_flow.so).
//
// Behaviour kept from src/flow/flow.cpp: bool results, errors printed to
// stderr, `load` and `load_noise` idempotent, `mel` resized by the callee to
// 80 x (MEL_T - mel_len1), FlowDebug filled in PyTorch byte order, the
// 6-argument infer fed from the load_noise bank.  The decoder binds CUDA
// device 0 (the reference's backend_init_best() picks the first GPU).
#include <cstdio>
#include <string>
#include <vector>

#include "larynx/flow/flow.h"
#include "larynx_flow.h"

namespace larynx::flow {

std::string module_name() { return "flow (B200 sm_100a: tcgen05 DiT + CFM, liblarynx_flow)"; }

struct FlowDecoder::Impl {
  lx_flow* h = nullptr;
};

FlowDecoder::FlowDecoder() : impl_(new Impl()) {
  if (lx_flow_create(0, &impl_->h) != LX_OK) {
    std::fprintf(stderr, "flow: no usable sm_100 GPU (lx_flow_create failed)\n");
    impl_->h = nullptr;
  }
}

FlowDecoder::~FlowDecoder() {
  if (impl_->h) lx_flow_destroy(impl_->h);
  delete impl_;
}

namespace {

bool report(lx_flow* h, int rc, const char* what) {
  if (rc == LX_OK) return true;
  std::fprintf(stderr, "flow: %s failed (status %d): %s\n", what, rc, lx_flow_last_error(h));
  return false;
}

bool run_infer(lx_flow* h, const std::vector<int32_t>& prompt_tokens, const std::vector<int32_t>& tokens,
               const std::vector<float>& prompt_feat, const std::vector<float>& spk_embedding, const float* noise,
               std::vector<float>& mel, FlowDebug* dbg) {
  const int n_tok = static_cast<int>(prompt_tokens.size() + tokens.size());
  const int T = 2 * n_tok;
  const int mel_len1 = static_cast<int>(prompt_feat.size() / LX_MEL_DIM);
  if (spk_embedding.size() != LX_SPK_EMBED_DIM || mel_len1 > T) {
    std::fprintf(stderr, "flow: infer: bad input sizes\n");
    return false;
  }
  mel.resize(static_cast<size_t>(LX_MEL_DIM) * (T - mel_len1));
  lx_flow_debug d{};
  std::vector<float> blocks;
  if (dbg) {
    const size_t row2 = static_cast<size_t>(2) * T * LX_DIM;
    dbg->spk.resize(LX_MEL_DIM);
    dbg->token_embed.resize(static_cast<size_t>(n_tok) * LX_MEL_DIM);
    dbg->prelookahead.resize(static_cast<size_t>(n_tok) * LX_MEL_DIM);
    dbg->mu.resize(static_cast<size_t>(LX_MEL_DIM) * T);
    dbg->cond.resize(static_cast<size_t>(LX_MEL_DIM) * T);
    dbg->time_embed.resize(2 * LX_DIM);
    dbg->input_proj.resize(row2);
    dbg->conv_pos.resize(row2);
    dbg->input_embed.resize(row2);
    dbg->norm_out.resize(row2);
    dbg->dphi.resize(static_cast<size_t>(2) * LX_MEL_DIM * T);
    blocks.resize(LX_DEPTH * row2);
    d.spk = dbg->spk.data();
    d.token_embed = dbg->token_embed.data();
    d.prelookahead = dbg->prelookahead.data();
    d.mu = dbg->mu.data();
    d.cond = dbg->cond.data();
    d.time_embed = dbg->time_embed.data();
    d.input_proj = dbg->input_proj.data();
    d.conv_pos = dbg->conv_pos.data();
    d.input_embed = dbg->input_embed.data();
    d.blocks = blocks.data();
    d.norm_out = dbg->norm_out.data();
    d.dphi = dbg->dphi.data();
  }
  const int rc = lx_flow_infer(h, prompt_tokens.data(), static_cast<int>(prompt_tokens.size()), tokens.data(),
                               static_cast<int>(tokens.size()), prompt_feat.data(), mel_len1, spk_embedding.data(),
                               noise, mel.data(), mel.size(), dbg ? &d : nullptr);
  if (!report(h, rc, "infer")) return false;
  if (dbg) {
    const size_t row2 = static_cast<size_t>(2) * T * LX_DIM;
    dbg->blocks.assign(LX_DEPTH, {});
    for (int i = 0; i < LX_DEPTH; ++i)
      dbg->blocks[i].assign(blocks.begin() + i * row2, blocks.begin() + (i + 1) * row2);
    dbg->feat = mel;
  }
  return true;
}

}  // namespace

bool FlowDecoder::load(const std::string& gguf_path) {
  return impl_->h && report(impl_->h, lx_flow_load_gguf(impl_->h, gguf_path.c_str()), "load");
}

bool FlowDecoder::load_noise(const std::string& noise_path) {
  return impl_->h && report(impl_->h, lx_flow_load_noise(impl_->h, noise_path.c_str()), "load_noise");
}

bool FlowDecoder::infer(const std::vector<int32_t>& prompt_tokens, const std::vector<int32_t>& tokens,
                        const std::vector<float>& prompt_feat, const std::vector<float>& spk_embedding,
                        const std::vector<float>& noise_z, std::vector<float>& mel, FlowDebug* debug) {
  if (!impl_->h) return false;
  const size_t need = static_cast<size_t>(LX_MEL_DIM) * 2 * (prompt_tokens.size() + tokens.size());
  if (noise_z.size() < need) {
    std::fprintf(stderr, "flow: infer: noise_z has %zu floats, %zu needed\n", noise_z.size(), need);
    return false;
  }
  return run_infer(impl_->h, prompt_tokens, tokens, prompt_feat, spk_embedding, noise_z.data(), mel, debug);
}

bool FlowDecoder::infer(const std::vector<int32_t>& prompt_tokens, const std::vector<int32_t>& tokens,
                        const std::vector<float>& prompt_feat, const std::vector<float>& spk_embedding,
                        std::vector<float>& mel, FlowDebug* debug) {
  if (!impl_->h) return false;
  return run_infer(impl_->h, prompt_tokens, tokens, prompt_feat, spk_embedding, nullptr, mel, debug);
}

}  // namespace larynx::flow
