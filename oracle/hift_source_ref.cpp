// C entry points over the reference's own host-side HiFT stages
// (src/hift/source.cpp: f0_predict, source_stft, istft), compiled from the
// reference's source file where it lies, for the oracle tests (TEST
// INFRASTRUCTURE ONLY: oracle/Makefile builds it into oracle/_ref/, the
// product never loads it).  Each wrapper copies plain arrays into the
// std::vector / HiFTWeights arguments the reference functions take
// (src/hift/internal.h:150-168) and copies the results out.
#include <cstring>
#include <vector>

#include "internal.h"

using namespace larynx::hift;

extern "C" {

// mel [80][T] float64 -> f0 [T] float64.  f0_w[i] / f0_b[i]: condnet convs
// 0, 2, 4, 6, 8 ([512][80][4], then [512][512][3]); cls_w [512], cls_b [1].
void hiftref_f0_predict(const double* mel, int T, const double* const* f0_w, const double* const* f0_b,
                        const double* cls_w, const double* cls_b, double* f0_out) {
  HiFTWeights w;
  for (int i = 0; i < 5; ++i) {
    const size_t nw = static_cast<size_t>(BASE_CH) * (i == 0 ? IN_CH * 4 : BASE_CH * 3);
    w.f0_w[i].assign(f0_w[i], f0_w[i] + nw);
    w.f0_b[i].assign(f0_b[i], f0_b[i] + BASE_CH);
  }
  w.f0_cls_w.assign(cls_w, cls_w + BASE_CH);
  w.f0_cls_b.assign(cls_b, cls_b + 1);
  std::vector<double> m(mel, mel + static_cast<size_t>(IN_CH) * T), f0;
  f0_predict(f0, m, w);
  std::memcpy(f0_out, f0.data(), f0.size() * sizeof(double));
}

// f0 [T] float32, rand_ini [9], sine_waves [T*480][9] -> s_stft [18][T*120+1],
// sine_wavs [T*480][9], sine_merge [T*480].
void hiftref_source_stft(const float* f0, int T, const float* rand_ini, const float* sine_waves,
                         const float* m_source_w, const float* m_source_b, float* s_stft_out, float* sine_wavs_out,
                         float* sine_merge_out) {
  HiFTWeights w;
  w.m_source_w.assign(m_source_w, m_source_w + NB_HARM + 1);
  w.m_source_b.assign(m_source_b, m_source_b + 1);
  const size_t ls = static_cast<size_t>(T) * TOTAL_SCALE;
  std::vector<float> f(f0, f0 + T), ri(rand_ini, rand_ini + NB_HARM + 1);
  std::vector<float> sw(sine_waves, sine_waves + ls * (NB_HARM + 1));
  std::vector<float> st, wavs, merge;
  source_stft(f, ri, sw, w, st, &wavs, &merge);
  std::memcpy(s_stft_out, st.data(), st.size() * sizeof(float));
  std::memcpy(sine_wavs_out, wavs.data(), wavs.size() * sizeof(float));
  std::memcpy(sine_merge_out, merge.data(), merge.size() * sizeof(float));
}

// magnitude / phase [9][n_frames] -> audio [(n_frames - 1) * 4].
void hiftref_istft(const float* magnitude, const float* phase, int n_frames, float* audio_out) {
  const size_t n = static_cast<size_t>(N_BINS) * n_frames;
  std::vector<float> m(magnitude, magnitude + n), p(phase, phase + n), a;
  istft(m, p, a);
  std::memcpy(audio_out, a.data(), a.size() * sizeof(float));
}

}  // extern "C"
