// HiFT vocoder (CosyVoice3 CausalHiFTGenerator, finalize=True) on sm_100a.
//
// Every stage runs on the device.  Reference: hardenedlinux/larynx
// src/hift/{hift,source,ops,gguf}.cpp, include/larynx/hift/hift.h.
//
//   f0 predictor   k_f0_conv / k_f0_cls: float64, one thread per output, the
//                  reference's accumulation order (bias, then ic-major, k
//                  inner, products and sums rounded separately: no FMA), so
//                  f0 matches source.cpp:18-96 bit for bit up to exp() in ELU
//   SineGen2       k_sine_cumsum (9 serial float32 prefix sums over frames,
//                  the order of source.cpp:131-139), k_source (one thread per
//                  sample: phase, sin, uv/noise mix, m_source tanh)
//   STFT           k_stft: one thread per frame, 16-point DFT with the
//                  reference's tables and order (source.cpp:168-193)
//   conv network   k_hconv: float32 implicit-GEMM conv on the CUDA cores
//                  (time-major [T][C] activations; 128 time rows x 64/128
//                  output channels per CTA, 8 x 4 / 8 x 8 outputs per thread,
//                  16-channel K slices staged through shared memory, double
//                  buffered).  The input activation (leaky ReLU or Snake), the
//                  nearest upsample and the causal zero padding are applied
//                  while the input slice is staged; bias and the residual add
//                  in the epilogue.  float32 throughout: the reference pins
//                  this network to fp32 (TF32 disabled), which a single-pass
//                  bf16/tf32 tensor-core product would not meet.
//                  k_conv_direct: the 18-channel convs (strided source
//                  downsampling) and conv_post's tail, one thread per output
//   ISTFT          k_istft_frames (exp/sin split, clip, inverse DFT x window)
//                  + k_istft_ola (overlap-add in frame order, envelope
//                  normalisation, clamp)
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "../../include/larynx_hift.h"
#include "common.cuh"
#include "gguf.h"
#include "kernels.h"

namespace lx {
namespace hift {

constexpr int IN_CH = 80;
constexpr int BASE_CH = 512;
constexpr int NB_HARM = 8;
constexpr int HARM = NB_HARM + 1;
constexpr int SAMPLE_RATE = 24000;
constexpr float NSF_ALPHA = 0.1f;
constexpr float NSF_SIGMA = 0.003f;
constexpr float NSF_VOICED = 10.0f;
constexpr int UPSAMPLE_RATES[3] = {8, 5, 3};
constexpr int UPSAMPLE_KERNELS[3] = {16, 11, 7};
constexpr int N_FFT = 16;
constexpr int HOP = 4;
constexpr int N_BINS = 9;
constexpr int OUT_CH = 18;
constexpr int RESBLOCK_KERNELS[3] = {3, 7, 11};
constexpr int RESBLOCK_DILATIONS[3] = {1, 3, 5};
constexpr int SRC_RB_KERNELS[3] = {7, 7, 11};
constexpr int SRC_DOWN_KERNELS[3] = {30, 6, 1};
constexpr int SRC_DOWN_STRIDES[3] = {15, 3, 1};
constexpr float LRELU_SLOPE = 0.1f;
constexpr float AUDIO_LIMIT = 0.99f;
constexpr int CONV_PRE_LOOK_RIGHT = 4;
constexpr int TOTAL_SCALE = 8 * 5 * 3 * HOP;  // 480
constexpr float SNAKE_EPS = 1e-9f;
constexpr long long SINE_MAX_SAMPLES = 300LL * SAMPLE_RATE;
constexpr double PI_D = 3.14159265358979323846;

inline int stage_channels(int i) { return BASE_CH >> (i + 1); }

// ---------------------------------------------------------------------------
// f0 predictor (float64, channel-major [C][T])
// ---------------------------------------------------------------------------
// out[oc][t] = b[oc] + sum_ic sum_k W[oc][ic][k] x[ic][t + k - pad_left]
// (source.cpp:18-35), then ELU when `elu`.  Each output keeps the
// reference's order (bias, ic ascending, k ascending, out-of-range taps
// skipped) with separately rounded products and sums.  Block: 64 t x 32 oc,
// thread = one t and 8 oc; 8-channel slices of x and W staged in shared
// memory so each x value feeds 8 outputs and each W value 64.
constexpr int F0_BT = 64, F0_BO = 32, F0_BC = 8;

template <int K>
__global__ void __launch_bounds__(256) k_f0_conv(const double* __restrict__ x, int L, int IC,
                                                 const double* __restrict__ W, const double* __restrict__ b,
                                                 int pad_left, int elu, double* __restrict__ out) {
  constexpr int WR = F0_BT + K - 1;
  __shared__ double xs[F0_BC][WR];
  __shared__ __align__(16) double ws[F0_BC][K][F0_BO];
  const int tid = threadIdx.x, tx = tid & 63, ty = tid >> 6;  // ty: 8-oc group 0..3
  const int t0 = blockIdx.x * F0_BT, oc0 = blockIdx.y * F0_BO;
  const int t = t0 + tx;
  double acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = b[oc0 + ty * 8 + j];
  bool valid[K];
#pragma unroll
  for (int k = 0; k < K; ++k) valid[k] = t + k - pad_left >= 0 && t + k - pad_left < L;
  for (int ic0 = 0; ic0 < IC; ic0 += F0_BC) {
    const int nc = min(F0_BC, IC - ic0);
    for (int i = tid; i < F0_BC * WR; i += 256) {
      const int c = i / WR, r = i - c * WR;
      const int src = t0 + r - pad_left;
      xs[c][r] = (c < nc && src >= 0 && src < L) ? x[static_cast<size_t>(ic0 + c) * L + src] : 0.0;
    }
    // W[oc][ic0 .. ic0+7][0 .. K-1] is contiguous per oc: 8K doubles
    for (int i = tid; i < F0_BO * F0_BC * K; i += 256) {
      const int o = i / (F0_BC * K), e = i - o * (F0_BC * K), c = e / K, k = e - c * K;
      ws[c][k][o] = c < nc ? W[(static_cast<size_t>(oc0 + o) * IC + ic0) * K + e] : 0.0;
    }
    __syncthreads();
    for (int c = 0; c < nc; ++c) {
#pragma unroll
      for (int k = 0; k < K; ++k) {
        if (!valid[k]) continue;
        const double xv = xs[c][tx + k];
        const double2* wp = reinterpret_cast<const double2*>(&ws[c][k][ty * 8]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const double2 wv = wp[j];
          acc[2 * j] = __dadd_rn(acc[2 * j], __dmul_rn(wv.x, xv));
          acc[2 * j + 1] = __dadd_rn(acc[2 * j + 1], __dmul_rn(wv.y, xv));
        }
      }
    }
    __syncthreads();
  }
  if (t >= L) return;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    double v = acc[j];
    if (elu && v <= 0.0) v = exp(v) - 1.0;
    out[static_cast<size_t>(oc0 + ty * 8 + j) * L + t] = v;
  }
}

// f0[t] = |b + sum_ic w[ic] y[ic][t]| (source.cpp:89-95), cast to float32;
// also the float64 mel input conversion's counterpart for the debug capture.
__global__ void k_f0_cls(const double* __restrict__ y, int L, const double* __restrict__ w, double b,
                         float* __restrict__ f0) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= L) return;
  double acc = b;
  for (int ic = 0; ic < BASE_CH; ++ic) acc = __dadd_rn(acc, __dmul_rn(w[ic], y[static_cast<size_t>(ic) * L + t]));
  f0[t] = static_cast<float>(fabs(acc));
}

__global__ void k_mel_prep(const float* __restrict__ mel, int T, double* __restrict__ mel_d,
                           float* __restrict__ melT) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= IN_CH * T) return;
  const int c = i / T, t = i - c * T;
  const float v = mel[i];
  mel_d[i] = static_cast<double>(v);
  melT[static_cast<size_t>(t) * IN_CH + c] = v;
}

// ---------------------------------------------------------------------------
// SineGen2 + m_source (float32, source.cpp:98-166)
// ---------------------------------------------------------------------------
__device__ __forceinline__ float rad_at(const float* f0, const float* rand_ini, int i, int h) {
  const float fn = __fmul_rn(f0[i / TOTAL_SCALE], static_cast<float>(h + 1));
  float r = fmodf(__fdiv_rn(fn, static_cast<float>(SAMPLE_RATE)), 1.0f);
  if (i == 0) r = __fadd_rn(r, rand_ini[h]);
  return r;
}

// rad_down[i][h]: the linear x(1/480) downsample of rad, align_corners=False
// (source.cpp:117-129), one thread per (frame, harmonic).
__global__ void k_rad_down(const float* __restrict__ f0, const float* __restrict__ rand_ini, int T,
                           float* __restrict__ rd) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= T * HARM) return;
  const int i = idx / HARM, h = idx - i * HARM;
  const int L_S = T * TOTAL_SCALE;
  const float src = __fsub_rn(__fmul_rn(__fadd_rn(static_cast<float>(i), 0.5f), static_cast<float>(L_S / T)), 0.5f);
  const int f = static_cast<int>(floorf(src));
  const int c = min(f + 1, L_S - 1);
  const float frac = __fsub_rn(src, static_cast<float>(f));
  rd[idx] = __fadd_rn(__fmul_rn(rad_at(f0, rand_ini, f, h), __fsub_rn(1.0f, frac)),
                      __fmul_rn(rad_at(f0, rand_ini, c, h), frac));
}

// Per harmonic the running sum over frames, serially in frame order
// (source.cpp:131-139), in place.
__global__ void k_sine_cumsum(float* __restrict__ cums, int T) {
  const int h = threadIdx.x;
  if (h >= HARM) return;
  float acc = 0.0f;
  for (int i = 0; i < T; ++i) {
    acc = __fadd_rn(acc, cums[i * HARM + h]);
    cums[i * HARM + h] = acc;
  }
}

// One thread per sample: sine_wavs[i][h] and s[i] = tanh(m_source(sine_wavs[i])).
__global__ void k_source(const float* __restrict__ f0, const float* __restrict__ cums,
                         const float* __restrict__ bank, const float* __restrict__ msw, float msb, int T,
                         float* __restrict__ s, float* __restrict__ sine_wavs) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int L_S = T * TOTAL_SCALE;
  if (i >= L_S) return;
  const int t = i / TOTAL_SCALE;
  const float fu = f0[t];
  const float uv = fu > NSF_VOICED ? 1.0f : 0.0f;
  const float noise_amp = __fadd_rn(__fmul_rn(uv, NSF_SIGMA), __fdiv_rn(__fmul_rn(__fsub_rn(1.0f, uv), NSF_ALPHA), 3.0f));
  float acc = msb;
#pragma unroll
  for (int h = 0; h < HARM; ++h) {
    float p = cums[t * HARM + h];
    p = __fmul_rn(p, 2.0f);
    p = __fmul_rn(p, static_cast<float>(PI_D));
    p = __fmul_rn(p, static_cast<float>(TOTAL_SCALE));
    const float sn = __fmul_rn(sinf(p), NSF_ALPHA);
    const float noise = __fmul_rn(noise_amp, bank[static_cast<size_t>(i) * HARM + h]);
    const float sw = __fadd_rn(__fmul_rn(sn, uv), noise);
    if (sine_wavs) sine_wavs[static_cast<size_t>(i) * HARM + h] = sw;
    acc = __fadd_rn(acc, __fmul_rn(msw[h], sw));
  }
  s[i] = tanhf(acc);
}

struct DftConst {
  float c[N_FFT][N_FFT];
  float s[N_FFT][N_FFT];
  float win[N_FFT];
};
__constant__ DftConst g_dft;

// One thread per STFT frame: center reflect-pad 8, periodic Hann window,
// onesided 9 bins; out [N][18] time-major (real bins 0..8, imaginary 9..17).
__global__ void k_stft(const float* __restrict__ s, int L_S, float* __restrict__ out) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  const int n_frames = L_S / HOP + 1;
  if (t >= n_frames) return;
  float seg[N_FFT];
#pragma unroll
  for (int n = 0; n < N_FFT; ++n) {
    int j = t * HOP + n - N_FFT / 2;  // index into s before the reflect pad
    if (j < 0) j = -j;
    if (j >= L_S) j = 2 * (L_S - 1) - j;
    seg[n] = __fmul_rn(s[j], g_dft.win[n]);
  }
  float* o = out + static_cast<size_t>(t) * OUT_CH;
#pragma unroll
  for (int k = 0; k < N_BINS; ++k) {
    float re = 0.0f, im = 0.0f;
#pragma unroll
    for (int n = 0; n < N_FFT; ++n) {
      re = __fadd_rn(re, __fmul_rn(seg[n], g_dft.c[k][n]));
      im = __fsub_rn(im, __fmul_rn(seg[n], g_dft.s[k][n]));
    }
    o[k] = re;
    o[N_BINS + k] = im;
  }
}

// ---------------------------------------------------------------------------
// ISTFT (source.cpp:198-239): per frame the windowed inverse DFT, then the
// overlap-add per sample in frame order and the envelope normalisation.
// ---------------------------------------------------------------------------
__global__ void k_istft_frames(const float* __restrict__ post, int n_frames, float* __restrict__ vw,
                               float* __restrict__ mag_out, float* __restrict__ pha_out) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= n_frames) return;
  const float* x = post + static_cast<size_t>(t) * OUT_CH;
  float Xr[N_FFT], Xi[N_FFT];
#pragma unroll
  for (int k = 0; k < N_BINS; ++k) {
    const float mg = expf(x[k]);
    const float ph = sinf(x[N_BINS + k]);
    if (mag_out) mag_out[static_cast<size_t>(k) * n_frames + t] = mg;
    if (pha_out) pha_out[static_cast<size_t>(k) * n_frames + t] = ph;
    const float m = mg > 100.0f ? 100.0f : mg;
    Xr[k] = __fmul_rn(m, cosf(ph));
    Xi[k] = __fmul_rn(m, sinf(ph));
  }
#pragma unroll
  for (int k = 1; k < N_FFT / 2; ++k) {
    Xr[N_FFT - k] = Xr[k];
    Xi[N_FFT - k] = -Xi[k];
  }
  float* o = vw + static_cast<size_t>(t) * N_FFT;
#pragma unroll
  for (int n = 0; n < N_FFT; ++n) {
    float v = 0.0f;
#pragma unroll
    for (int k = 0; k < N_FFT; ++k)
      v = __fadd_rn(v, __fsub_rn(__fmul_rn(Xr[k], g_dft.c[k][n]), __fmul_rn(Xi[k], g_dft.s[k][n])));
    v = __fdiv_rn(v, static_cast<float>(N_FFT));
    o[n] = __fmul_rn(v, g_dft.win[n]);
  }
}

__global__ void k_istft_ola(const float* __restrict__ vw, int n_frames, float* __restrict__ raw,
                            float* __restrict__ audio) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int L_S = (n_frames - 1) * HOP;
  if (i >= L_S) return;
  const int j = i + N_FFT / 2;  // position in the untrimmed overlap-add buffer
  int t0 = (j - N_FFT + HOP) / HOP;  // first frame t with t*HOP + 15 >= j
  if (t0 < 0) t0 = 0;
  const int t1 = min(j / HOP, n_frames - 1);
  float acc = 0.0f, env = 0.0f;
  for (int t = t0; t <= t1; ++t) {
    const int n = j - t * HOP;
    acc = __fadd_rn(acc, vw[static_cast<size_t>(t) * N_FFT + n]);
    env = __fadd_rn(env, __fmul_rn(g_dft.win[n], g_dft.win[n]));
  }
  if (env < 1e-8f) env = 1e-8f;
  const float v = __fdiv_rn(acc, env);
  if (raw) raw[i] = v;
  audio[i] = fminf(fmaxf(v, -AUDIO_LIMIT), AUDIO_LIMIT);
}

// ---------------------------------------------------------------------------
// Conv network (float32, time-major [L][C])
// ---------------------------------------------------------------------------
enum Act : int { ACT_NONE = 0, ACT_LRELU = 1, ACT_SNAKE = 2 };

struct ConvArgs {
  const float* in;         // [L_in][C_in]
  int L_in, C_in;
  int up;                  // nearest upsample factor applied to the input (1 = none)
  const float* wt;         // [K][C_in][C_out_pad], zero past C_out
  const float* bias;       // [C_out_pad]
  int C_out, C_out_pad, K, dil, pad_left;
  int act;                 // activation of the input, applied as it is staged
  float slope;             // ACT_LRELU
  const float* alpha;      // ACT_SNAKE: [C_in]
  const float* inv_alpha;  // ACT_SNAKE: [C_in], 1 / (alpha + 1e-9)
  const float* res;        // [L_out][C_out] added after the bias, or null (may alias out)
  float* out;              // [L_out][C_out]
  int L_out;
};

__device__ __forceinline__ float act_apply(float x, int act, float slope, const float* alpha, const float* inv,
                                           int c) {
  if (act == ACT_LRELU) return x > 0.0f ? x : __fmul_rn(x, slope);
  if (act == ACT_SNAKE) {
    // x + (1/(alpha + eps)) * sin(x alpha)^2 (ops.cpp snake)
    const float s = sinf(__fmul_rn(x, alpha[c]));
    return __fadd_rn(x, __fmul_rn(inv[c], __fmul_rn(s, s)));
  }
  return x;
}

// out[t][oc] = bias[oc] + sum_{k, ic} act(in_up[t + k*dil - pad_left][ic]) W[oc][ic][k]
// (+ res[t][oc]), in_up[u] = in[u / up] for 0 <= u < L_in*up and 0 elsewhere.
// K loop: (tap, 16-channel slice) pairs; A slices are staged transposed
// ([c][row]) so each thread reads its 8 rows as two float4.
constexpr int HC_BC = 16, HC_THREADS = 256;

// BT time rows x BO output channels per CTA; thread (ty, tx) of a 16 x 16
// grid owns rows ty*TM .. +TM-1 and channels tx*4 .. +3 (+ 64 for BO = 128).
template <int BT, int BO>
__global__ void __launch_bounds__(HC_THREADS) k_hconv(ConvArgs a) {
  constexpr int TM = BT / 16;       // rows per thread (4 or 8)
  constexpr int TN = BO / 16;       // output channels per thread (4 or 8)
  constexpr int NA = BT / 64;       // float4 A loads per thread per slice
  constexpr int NB = BO / 64;       // float4 B loads per thread per slice
  constexpr int AP = BT + 4;
  __shared__ __align__(16) float As[2][HC_BC][AP];
  __shared__ __align__(16) float Bs[2][HC_BC][BO];
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const int t0 = blockIdx.x * BT, oc0 = blockIdx.y * BO;
  const int n_cb = a.C_in / HC_BC;
  const int n_it = a.K * n_cb;
  const int Lu = a.L_in * a.up;
  float4 ra[NA], rb[NB];

  auto load_a = [&](int it) {
    const int k = it / n_cb, cb = it - k * n_cb;
#pragma unroll
    for (int q = 0; q < NA; ++q) {
      const int idx = tid + HC_THREADS * q, r = idx >> 2, c4 = idx & 3;
      const int u = t0 + r + k * a.dil - a.pad_left;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (u >= 0 && u < Lu) {
        const int src = a.up == 1 ? u : u / a.up;
        const int c = cb * HC_BC + c4 * 4;
        v = __ldg(reinterpret_cast<const float4*>(a.in + static_cast<size_t>(src) * a.C_in + c));
        if (a.act != ACT_NONE) {
          v.x = act_apply(v.x, a.act, a.slope, a.alpha, a.inv_alpha, c);
          v.y = act_apply(v.y, a.act, a.slope, a.alpha, a.inv_alpha, c + 1);
          v.z = act_apply(v.z, a.act, a.slope, a.alpha, a.inv_alpha, c + 2);
          v.w = act_apply(v.w, a.act, a.slope, a.alpha, a.inv_alpha, c + 3);
        }
      }
      ra[q] = v;
    }
  };
  auto store_a = [&](int buf) {
#pragma unroll
    for (int q = 0; q < NA; ++q) {
      const int idx = tid + HC_THREADS * q, r = idx >> 2, c4 = idx & 3;
      As[buf][c4 * 4 + 0][r] = ra[q].x;
      As[buf][c4 * 4 + 1][r] = ra[q].y;
      As[buf][c4 * 4 + 2][r] = ra[q].z;
      As[buf][c4 * 4 + 3][r] = ra[q].w;
    }
  };
  auto load_b = [&](int it) {
    const int k = it / n_cb, cb = it - k * n_cb;
    const float* base = a.wt + (static_cast<size_t>(k) * a.C_in + cb * HC_BC) * a.C_out_pad + oc0;
#pragma unroll
    for (int q = 0; q < NB; ++q) {
      const int idx = tid + HC_THREADS * q, c = idx / (BO / 4), o4 = idx % (BO / 4);
      rb[q] = __ldg(reinterpret_cast<const float4*>(base + static_cast<size_t>(c) * a.C_out_pad + o4 * 4));
    }
  };
  auto store_b = [&](int buf) {
#pragma unroll
    for (int q = 0; q < NB; ++q) {
      const int idx = tid + HC_THREADS * q, c = idx / (BO / 4), o4 = idx % (BO / 4);
      *reinterpret_cast<float4*>(&Bs[buf][c][o4 * 4]) = rb[q];
    }
  };

  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.0f;

  load_a(0);
  load_b(0);
  store_a(0);
  store_b(0);
  __syncthreads();
  for (int it = 0; it < n_it; ++it) {
    const int buf = it & 1;
    if (it + 1 < n_it) {
      load_a(it + 1);
      load_b(it + 1);
    }
#pragma unroll
    for (int c = 0; c < HC_BC; ++c) {
      float av[TM];
#pragma unroll
      for (int g = 0; g < TM / 4; ++g) {
        const float4 x = *reinterpret_cast<const float4*>(&As[buf][c][ty * TM + 4 * g]);
        av[4 * g + 0] = x.x;
        av[4 * g + 1] = x.y;
        av[4 * g + 2] = x.z;
        av[4 * g + 3] = x.w;
      }
      float bv[TN];
#pragma unroll
      for (int g = 0; g < TN / 4; ++g) {
        const float4 b = *reinterpret_cast<const float4*>(&Bs[buf][c][g * 64 + tx * 4]);
        bv[g * 4 + 0] = b.x;
        bv[g * 4 + 1] = b.y;
        bv[g * 4 + 2] = b.z;
        bv[g * 4 + 3] = b.w;
      }
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(av[i], bv[j], acc[i][j]);
    }
    if (it + 1 < n_it) {
      store_a(buf ^ 1);
      store_b(buf ^ 1);
    }
    __syncthreads();
  }

  const bool vec = (a.C_out & 3) == 0;
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int t = t0 + ty * TM + i;
    if (t >= a.L_out) continue;
#pragma unroll
    for (int g = 0; g < TN / 4; ++g) {
      const int ocb = oc0 + g * 64 + tx * 4;
      if (ocb >= a.C_out) continue;
      float v[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) v[e] = __fadd_rn(acc[i][g * 4 + e], a.bias[ocb + e]);
      const size_t o = static_cast<size_t>(t) * a.C_out + ocb;
      if (vec) {
        if (a.res) {
          const float4 r = *reinterpret_cast<const float4*>(a.res + o);
          v[0] = __fadd_rn(v[0], r.x);
          v[1] = __fadd_rn(v[1], r.y);
          v[2] = __fadd_rn(v[2], r.z);
          v[3] = __fadd_rn(v[3], r.w);
        }
        *reinterpret_cast<float4*>(a.out + o) = make_float4(v[0], v[1], v[2], v[3]);
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          if (ocb + e >= a.C_out) break;
          float w = v[e];
          if (a.res) w = __fadd_rn(w, a.res[o + e]);
          a.out[o + e] = w;
        }
      }
    }
  }
}

// Direct conv for few input channels (the strided source downsampling of the
// 18-channel STFT): one thread per (row, 4 output channels), C_out % 4 == 0.
__global__ void k_conv_direct(const float* __restrict__ in, int L_in, int C_in, const float* __restrict__ wt,
                              const float* __restrict__ bias, int C_out, int C_out_pad, int K, int stride,
                              int pad_left, float* __restrict__ out, int L_out) {
  const int c4 = C_out / 4;
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<size_t>(L_out) * c4) return;
  const int t = static_cast<int>(i / c4), oc = static_cast<int>(i % c4) * 4;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int k = 0; k < K; ++k) {
    const int src = t * stride + k - pad_left;
    if (src < 0 || src >= L_in) continue;
    const float* x = in + static_cast<size_t>(src) * C_in;
    const float* w = wt + static_cast<size_t>(k) * C_in * C_out_pad + oc;
    for (int ic = 0; ic < C_in; ++ic) {
      const float xv = x[ic];
      const float4 wv = __ldg(reinterpret_cast<const float4*>(w + static_cast<size_t>(ic) * C_out_pad));
      acc.x = fmaf(xv, wv.x, acc.x);
      acc.y = fmaf(xv, wv.y, acc.y);
      acc.z = fmaf(xv, wv.z, acc.z);
      acc.w = fmaf(xv, wv.w, acc.w);
    }
  }
  const float4 bv = *reinterpret_cast<const float4*>(bias + oc);
  *reinterpret_cast<float4*>(out + static_cast<size_t>(t) * C_out + oc) =
      make_float4(__fadd_rn(acc.x, bv.x), __fadd_rn(acc.y, bv.y), __fadd_rn(acc.z, bv.z), __fadd_rn(acc.w, bv.w));
}

__global__ void k_add(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ o, size_t n4) {
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n4) return;
  const float4 x = reinterpret_cast<const float4*>(a)[i], y = reinterpret_cast<const float4*>(b)[i];
  reinterpret_cast<float4*>(o)[i] =
      make_float4(__fadd_rn(x.x, y.x), __fadd_rn(x.y, y.y), __fadd_rn(x.z, y.z), __fadd_rn(x.w, y.w));
}

// x = ((r0 + r1) + r2) * (1/3): the resblock sum of a stage (hift.cpp:237-244)
__global__ void k_combine3(const float* __restrict__ r0, const float* __restrict__ r1, const float* __restrict__ r2,
                           float* __restrict__ o, size_t n4) {
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n4) return;
  const float4 a = reinterpret_cast<const float4*>(r0)[i], b = reinterpret_cast<const float4*>(r1)[i],
               c = reinterpret_cast<const float4*>(r2)[i];
  const float s = 1.0f / 3.0f;
  reinterpret_cast<float4*>(o)[i] = make_float4(__fmul_rn(__fadd_rn(__fadd_rn(a.x, b.x), c.x), s),
                                                __fmul_rn(__fadd_rn(__fadd_rn(a.y, b.y), c.y), s),
                                                __fmul_rn(__fadd_rn(__fadd_rn(a.z, b.z), c.z), s),
                                                __fmul_rn(__fadd_rn(__fadd_rn(a.w, b.w), c.w), s));
}

// nn.ReflectionPad1d((1, 0)) of rows 1.. of p: row 0 = row 2 (the unpadded row 1)
__global__ void k_reflect_row0(float* p, int C) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c < C) p[c] = p[2 * C + c];
}

// [L][C] -> [C][L] with an optional activation (debug captures)
__global__ void k_transpose(const float* __restrict__ in, int L, int C, int act, float slope, float* __restrict__ out) {
  __shared__ float tile[32][33];
  const int l0 = blockIdx.x * 32, c0 = blockIdx.y * 32;
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int l = l0 + r, c = c0 + threadIdx.x;
    float v = (l < L && c < C) ? in[static_cast<size_t>(l) * C + c] : 0.0f;
    if (act == ACT_LRELU) v = v > 0.0f ? v : __fmul_rn(v, slope);
    tile[r][threadIdx.x] = v;
  }
  __syncthreads();
  for (int r = threadIdx.y; r < 32; r += blockDim.y) {
    const int c = c0 + r, l = l0 + threadIdx.x;
    if (c < C && l < L) out[static_cast<size_t>(c) * L + l] = tile[threadIdx.x][r];
  }
}

// ---------------------------------------------------------------------------
// Tensor-core conv with a 3-term bf16 split (tcgen05, 1 CTA per SM)
// ---------------------------------------------------------------------------
// fp32 products to ~2^-17 relative on the bf16 tensor cores: each operand is
// split v = hi + lo (hi = bf16(v), lo = bf16(v - hi)) and
//   D = A_hi B_hi + A_hi B_lo + A_lo B_hi      (A_lo B_lo ~ 2^-18 |AB| dropped)
// with fp32 accumulation.  A = the activation rows (time) of one tap and 64
// channels, B = that tap's [BN out x 64 in] weight slice.  Per 16-wide K step
// two MMAs: A_hi x [B_hi; B_lo] (N = 2 BN, into accumulator columns
// [0, 2BN): hh | hl) and A_lo x B_hi (N = BN, added into [0, BN)); the
// epilogue sums the two halves.  Per (tile, 64-channel slice) one A window
// of 128 + (K-1)*dil rows is loaded (from row m0 - pad_left; TMA rows outside
// the tensor read as zero: the causal padding) and tap t reads it from row
// t*dil on, so the activations cross L2 once per slice instead of once per
// tap; the taps' weight slices stream through their own ring.
//   warp 0      TMA: A_hi, A_lo windows (2 slots) and per tap B_hi, B_lo
//               (BN x 64, adjacent in shared memory; 6 / 3 slots)
//   warp 1      TMEM allocator; lane 0 issues the MMAs
//   warps 2..17 epilogue, four warps per TMEM lane quarter (each a quarter
//               of the columns): TMEM -> registers, hh+lh + hl + bias
//               (+ residual), fp32 stores and / or the next conv's split
//               operands (the Snake of the next conv makes this the heavy
//               part for the short convs, hence the many warps)
constexpr int TC_THREADS = 576;  // warp 0 TMA, warp 1 MMA, warps 2..17 epilogue

struct TcConvArgs {
  int L_out, C_out, K_taps, dil, pad_left, n_cb;
  int wrows;          // rows of an A window: 128 + (K_taps - 1) * dil rounded up to 8 (<= TC_WROWS_MAX)
  int ldo;            // real output channels (<= C_out, the 64-padded tile count): row stride of res / out
  const float* bias;  // [C_out]
  const float* res;   // [L_out][ldo] or null (may alias out)
  float* out;         // [L_out][ldo], or null when only the split output is needed
  int* err;
  // optional: the next conv's A operands, split(act(out)) as bf16 hi / lo
  // [L_out][ldo] (ldo % 16 == 0)
  bf16* nhi;
  bf16* nlo;
  int nact;
  float nslope;
  const float* nalpha;
  const float* ninv;
};

// (hi pair, lo pair) of two values: hi = bf16(a), lo = bf16(a - hi)
__device__ __forceinline__ uint2 split_pair(float a0, float a1) {
  const bf16 h0 = __float2bfloat16_rn(a0), h1 = __float2bfloat16_rn(a1);
  const bf16 l0 = __float2bfloat16_rn(__fsub_rn(a0, __bfloat162float(h0)));
  const bf16 l1 = __float2bfloat16_rn(__fsub_rn(a1, __bfloat162float(h1)));
  return make_uint2(
      static_cast<uint32_t>(__bfloat16_as_ushort(h0)) | (static_cast<uint32_t>(__bfloat16_as_ushort(h1)) << 16),
      static_cast<uint32_t>(__bfloat16_as_ushort(l0)) | (static_cast<uint32_t>(__bfloat16_as_ushort(l1)) << 16));
}

constexpr int TC_WROWS_MAX = 184;  // A window rows: 128 + (K - 1) * dil, rounded up to 8 (K = 11, dil = 5)
constexpr int TC_A_HALF = TC_WROWS_MAX * 128;  // one bf16 plane of a window (23 KB, 1024-aligned)
constexpr int TC_A_SLOT = 2 * TC_A_HALF;       // hi + lo

template <int BN>
__host__ __device__ constexpr int tc_bslots() { return BN == 64 ? 6 : 3; }
template <int BN>
__host__ __device__ constexpr int tc_smem_bytes() {
  return 1024 + 2 * TC_A_SLOT + tc_bslots<BN>() * 2 * BN * 128 + 256;
}

template <int BN>
__global__ void __launch_bounds__(TC_THREADS, 1)
    k_hconv_tc(const __grid_constant__ CUtensorMap tmAh, const __grid_constant__ CUtensorMap tmAl,
               const __grid_constant__ CUtensorMap tmBh, const __grid_constant__ CUtensorMap tmBl, TcConvArgs a) {
  constexpr int NBS = tc_bslots<BN>();
  constexpr int B_BYTES = BN * 128;
  constexpr int B_SLOT = 2 * B_BYTES;
  constexpr uint32_t ACC_COLS = 2 * BN;
  constexpr uint32_t TMEM_COLS = 4 * BN;  // two accumulators
  constexpr uint32_t IDESC_HH_HL = idesc_bf16_f32(128, 2 * BN);
  constexpr uint32_t IDESC_LH = idesc_bf16_f32(128, BN);
  static_assert(2 * BN <= 256 && TMEM_COLS <= 512, "accumulator layout");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + 2 * TC_A_SLOT;
  uint64_t* a_full = reinterpret_cast<uint64_t*>(sB + NBS * B_SLOT);
  uint64_t* a_empty = a_full + 2;
  uint64_t* b_full = a_empty + 2;
  uint64_t* b_empty = b_full + NBS;
  uint64_t* tfull = b_empty + NBS;
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
    for (int i = 0; i < NBS; ++i) {
      mbar_init(&b_full[i], 1);
      mbar_init(&b_empty[i], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmAh);
    tma_prefetch_desc(&tmAl);
    tma_prefetch_desc(&tmBh);
    tma_prefetch_desc(&tmBl);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int tiles_n = a.C_out / BN;
  const int n_tiles = ((a.L_out + 127) / 128) * tiles_n;

  if (warp == 0) {
    if (lane == 0) {
      // per (tile, 64-channel slice): one A window (hi, lo) of wrows rows from
      // row m0 - pad_left, then the K taps' weight slices through the B ring
      int as = 0, bs = 0;
      uint32_t aph = 0, bph = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x) {
        const int m0 = (tile / tiles_n) * 128, n0 = (tile % tiles_n) * BN;
        for (int c = 0; ok && c < a.n_cb; ++c) {
          if (!(ok = mbar_wait(&a_empty[as], aph ^ 1u, a.err, abort_flag, DEV_TIMEOUT_PRODUCER))) break;
          uint8_t* wa = sA + as * TC_A_SLOT;
          mbar_arrive_expect_tx(&a_full[as], 2 * a.wrows * 128);
          tma_load_2d(wa, &tmAh, &a_full[as], c * 64, m0 - a.pad_left);
          tma_load_2d(wa + TC_A_HALF, &tmAl, &a_full[as], c * 64, m0 - a.pad_left);
          if (++as == 2) {
            as = 0;
            aph ^= 1u;
          }
          for (int t = 0; t < a.K_taps; ++t) {
            if (!(ok = mbar_wait(&b_empty[bs], bph ^ 1u, a.err, abort_flag, DEV_TIMEOUT_PRODUCER))) break;
            uint8_t* wb = sB + bs * B_SLOT;
            mbar_arrive_expect_tx(&b_full[bs], B_SLOT);
            tma_load_2d(wb, &tmBh, &b_full[bs], c * 64, t * a.C_out + n0);
            tma_load_2d(wb + B_BYTES, &tmBl, &b_full[bs], c * 64, t * a.C_out + n0);
            if (++bs == NBS) {
              bs = 0;
              bph ^= 1u;
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int as = 0, bs = 0, acc = 0;
      uint32_t aph = 0, bph = 0, acc_phase = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < n_tiles; tile += gridDim.x) {
        if (!(ok = mbar_wait(&tempty[acc], acc_phase ^ 1u, a.err, abort_flag, DEV_TIMEOUT_MMA))) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc) * ACC_COLS;
        bool first = true;
        for (int c = 0; ok && c < a.n_cb; ++c) {
          if (!(ok = mbar_wait(&a_full[as], aph, a.err, abort_flag, DEV_TIMEOUT_MMA))) break;
          const uint32_t wa = smem_u32(sA + as * TC_A_SLOT);
          for (int t = 0; t < a.K_taps; ++t) {
            if (!(ok = mbar_wait(&b_full[bs], bph, a.err, abort_flag, DEV_TIMEOUT_MMA))) break;
            tc_fence_after();
            // tap t reads the window from row t * dil: the 128B swizzle is a
            // function of the absolute shared-memory address, so a view that
            // starts at any 128-byte row is a valid operand (base offset 0)
            const uint32_t shift = static_cast<uint32_t>(t * a.dil) * 128u;
            const uint64_t dah = sdesc_sw128(wa + shift);
            const uint64_t dal = sdesc_sw128(wa + TC_A_HALF + shift);
            const uint64_t dbh = sdesc_sw128(smem_u32(sB + bs * B_SLOT));
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              umma_ss(d_tmem, dah + 2 * k, dbh + 2 * k, IDESC_HH_HL, (first && k == 0) ? 0u : 1u);
              umma_ss(d_tmem, dal + 2 * k, dbh + 2 * k, IDESC_LH, 1u);
            }
            first = false;
            umma_commit(&b_empty[bs]);
            if (++bs == NBS) {
              bs = 0;
              bph ^= 1u;
            }
          }
          umma_commit(&a_empty[as]);
          if (++as == 2) {
            as = 0;
            aph ^= 1u;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
    }
  } else {
    // epilogue warps 2..17 -> TMEM lane quarter warp % 4; warps 2..5 take
    // columns [0, BN/4), 6..9 [BN/4, BN/2), ...  The residual rows of the
    // next tile are loaded into registers while this tile is finished, so
    // their latency is off the epilogue's path (the next tile's output rows
    // are written only by this warp, later, so an in-place residual is safe).
    constexpr int NCH = BN / 64;  // 16-column chunks per warp
    const int q = warp & 3;
    const int cbeg = ((warp - 2) >> 2) * (BN / 4);
    const bool vec = a.res && (a.ldo & 3) == 0;
    float4 rres[NCH][4];
    auto load_res = [&](int tile_) {
      if (!vec || tile_ >= n_tiles) return;
      const int row_ = (tile_ / tiles_n) * 128 + q * 32 + lane;
      const int n0_ = (tile_ % tiles_n) * BN;
#pragma unroll
      for (int ch = 0; ch < NCH; ++ch) {
        const int col_ = n0_ + cbeg + 16 * ch;
        if (row_ < a.L_out && col_ + 16 <= a.ldo) {
          const float4* rp = reinterpret_cast<const float4*>(a.res + static_cast<size_t>(row_) * a.ldo + col_);
#pragma unroll
          for (int j = 0; j < 4; ++j) rres[ch][j] = rp[j];
        }
      }
    };
    load_res(blockIdx.x);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
      const int m0 = (tile / tiles_n) * 128, n0 = (tile % tiles_n) * BN;
      const bool ok = mbar_wait(&tfull[acc], acc_phase, a.err, abort_flag, DEV_TIMEOUT_EPILOGUE);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const int row = m0 + q * 32 + lane;
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(acc) * ACC_COLS;
#pragma unroll
      for (int ch = 0; ch < NCH; ++ch) {
        const int c0 = cbeg + 16 * ch;
        float u[16], v[16];
        tmem_ld16(t_row + c0, u);
        tmem_ld16(t_row + BN + c0, v);
        tmem_ld_wait();
        const int col = n0 + c0;
        if (row < a.L_out && (col + 16 > a.ldo || (a.ldo & 3))) {
          // ragged last columns (conv_post's 18 outputs): scalar stores
          const size_t o = static_cast<size_t>(row) * a.ldo + col;
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            if (col + e < a.ldo) {
              float w = __fadd_rn(__fadd_rn(u[e], v[e]), a.bias[col + e]);
              if (a.res) w = __fadd_rn(w, a.res[o + e]);
              a.out[o + e] = w;
            }
          }
        } else if (row < a.L_out) {
          const size_t o = static_cast<size_t>(row) * a.ldo + col;
          float w[16];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float4 r = vec ? rres[ch][j] : make_float4(0.f, 0.f, 0.f, 0.f);
            const float4 b = *reinterpret_cast<const float4*>(a.bias + col + 4 * j);
            w[4 * j + 0] = __fadd_rn(__fadd_rn(__fadd_rn(u[4 * j + 0], v[4 * j + 0]), b.x), r.x);
            w[4 * j + 1] = __fadd_rn(__fadd_rn(__fadd_rn(u[4 * j + 1], v[4 * j + 1]), b.y), r.y);
            w[4 * j + 2] = __fadd_rn(__fadd_rn(__fadd_rn(u[4 * j + 2], v[4 * j + 2]), b.z), r.z);
            w[4 * j + 3] = __fadd_rn(__fadd_rn(__fadd_rn(u[4 * j + 3], v[4 * j + 3]), b.w), r.w);
            if (a.out)
              *reinterpret_cast<float4*>(a.out + o + 4 * j) =
                  make_float4(w[4 * j + 0], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
          }
          if (a.nhi) {
            uint32_t hi[8], lo[8];
#pragma unroll
            for (int e = 0; e < 16; e += 2) {
              const float a0 = act_apply(w[e], a.nact, a.nslope, a.nalpha, a.ninv, col + e);
              const float a1 = act_apply(w[e + 1], a.nact, a.nslope, a.nalpha, a.ninv, col + e + 1);
              const uint2 p = split_pair(a0, a1);
              hi[e / 2] = p.x;
              lo[e / 2] = p.y;
            }
            st_global_v8(a.nhi + o, hi[0], hi[1], hi[2], hi[3], hi[4], hi[5], hi[6], hi[7]);
            st_global_v8(a.nlo + o, lo[0], lo[1], lo[2], lo[3], lo[4], lo[5], lo[6], lo[7]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[acc]);
      load_res(tile + gridDim.x);
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

// act(in_up) split into bf16 hi / lo planes [L_in*up][C] (the A operands of
// k_hconv_tc), 8 channels per thread.
__global__ void k_split(const float* __restrict__ in, int L_in, int C, int up, int act, float slope,
                        const float* __restrict__ alpha, const float* __restrict__ inv, bf16* __restrict__ hi,
                        bf16* __restrict__ lo) {
  const size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int c8 = C / 8;
  if (i >= static_cast<size_t>(L_in) * up * c8) return;
  const int u = static_cast<int>(i / c8), c = static_cast<int>(i % c8) * 8;
  const int src = up == 1 ? u : u / up;
  const float4* p = reinterpret_cast<const float4*>(in + static_cast<size_t>(src) * C + c);
  const float4 x0 = __ldg(p), x1 = __ldg(p + 1);
  float v[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
  uint32_t h[4], l[4];
#pragma unroll
  for (int e = 0; e < 8; e += 2) {
    const float a0 = act_apply(v[e], act, slope, alpha, inv, c + e);
    const float a1 = act_apply(v[e + 1], act, slope, alpha, inv, c + e + 1);
    const uint2 p = split_pair(a0, a1);
    h[e / 2] = p.x;
    l[e / 2] = p.y;
  }
  const size_t o = static_cast<size_t>(u) * C + c;
  *reinterpret_cast<uint4*>(hi + o) = make_uint4(h[0], h[1], h[2], h[3]);
  *reinterpret_cast<uint4*>(lo + o) = make_uint4(l[0], l[1], l[2], l[3]);
}

// ---------------------------------------------------------------------------
// Device model
// ---------------------------------------------------------------------------
struct ConvW {
  float* wt = nullptr;  // [K][C_in][C_out_pad]
  float* b = nullptr;   // [C_out_pad]
  int C_in = 0, C_out = 0, C_out_pad = 0, K = 0;
  // tensor-core form (C_in % 64 == 0, C_out % 64 == 0): bf16 hi / lo planes
  // of W as [K][C_out][C_in] and their tensor maps for BN = 64 / 128
  bf16* whi = nullptr;
  bf16* wlo = nullptr;
  bool tc = false;
  CUtensorMap tmh[2], tml[2];
};
struct SnakeW {
  float* alpha = nullptr;
  float* inv = nullptr;
};
struct ResW {
  ConvW c1[3], c2[3];
  SnakeW a1[3], a2[3];
};
struct Model {
  ConvW conv_pre, conv_post, ups[3], src_down[3];
  ResW src_rb[3], rb[9];
  double* f0_w[5] = {};
  double* f0_b[5] = {};
  double* cls_w = nullptr;
  double cls_b = 0.0;
  float* msw = nullptr;
  float msb = 0.0f;
};

// Per-call buffers, grown to the largest T seen.
struct Work {
  int cap_T = 0;
  bool cap_dbg = false;
  double *mel_d = nullptr, *y0 = nullptr, *y1 = nullptr;
  float *mel = nullptr, *melT = nullptr, *f0 = nullptr, *cums = nullptr, *bank = nullptr, *rand = nullptr;
  float *s = nullptr, *stft = nullptr, *post = nullptr, *vw = nullptr, *audio = nullptr;
  float* act[8] = {};  // X, F, S1, S2, R0, R1, R2, T1
  float *sine_wavs = nullptr, *mag = nullptr, *pha = nullptr, *raw = nullptr, *stage = nullptr;
  bf16 *ahi = nullptr, *alo = nullptr;  // split A operands of the tensor-core convs
  bf16 *bhi = nullptr, *blo = nullptr;  // second set (resblocks ping-pong between the two)
  int* err = nullptr;
};

}  // namespace hift
}  // namespace lx

struct lx_hift {
  int device = 0;
  cudaStream_t stream = nullptr;
  bool loaded = false, source_loaded = false;
  lx::hift::Model m;
  std::vector<void*> allocs;
  float* d_rand_ini = nullptr;  // [9]
  float* d_bank = nullptr;      // [SINE_MAX_SAMPLES][9]
  lx::hift::Work ws;
  // whole-vocode CUDA graphs (no debug captures), keyed by T and the source
  // buffers; dropped whenever the workspace is reallocated
  std::map<std::string, cudaGraphExec_t> graphs;
  bool use_graphs = true;
  std::string err;
  int fail(int code, const std::string& msg) {
    err = msg;
    return code;
  }
};

namespace lx {
namespace hift {
namespace {

int cuda_fail(lx_hift* h, cudaError_t e, const char* what) {
  return h->fail(e == cudaErrorMemoryAllocation ? LX_ERR_OOM : LX_ERR_CUDA,
                 std::string(what) + ": " + cudaGetErrorString(e));
}

#define HCK(expr)                                          \
  do {                                                     \
    cudaError_t e_ = (expr);                               \
    if (e_ != cudaSuccess) return cuda_fail(h, e_, #expr); \
  } while (0)

template <typename T>
int dalloc(lx_hift* h, T** p, size_t n) {
  void* v = nullptr;
  cudaError_t e = cudaMalloc(&v, std::max<size_t>(n, 1) * sizeof(T));
  if (e != cudaSuccess) return cuda_fail(h, e, "cudaMalloc");
  h->allocs.push_back(v);
  *p = static_cast<T*>(v);
  return LX_OK;
}

template <typename T>
int dupload(lx_hift* h, T** p, const T* src, size_t n) {
  if (int rc = dalloc(h, p, n)) return rc;
  HCK(cudaMemcpy(*p, src, n * sizeof(T), cudaMemcpyHostToDevice));
  return LX_OK;
}

int read_t(lx_hift* h, GgufFile& g, const std::string& name, std::vector<int64_t> shape, std::vector<float>& out) {
  int rc = g.read_f32(name, shape, out);
  if (rc) return h->fail(rc, "hift: " + g.error());
  return LX_OK;
}

// float -> bf16 bits, round to nearest even (finite inputs)
uint16_t bf16_bits(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  return static_cast<uint16_t>((u + (((u >> 16) & 1u) + 0x7FFFu)) >> 16);
}

// Conv weight W[oc][ic][k] (PyTorch) -> wt[k][ic][oc], oc padded to a
// multiple of 64 with zeros.
int load_conv(lx_hift* h, GgufFile& g, const std::string& name, int C_out, int C_in, int K, ConvW* out) {
  std::vector<float> w, b;
  if (int rc = read_t(h, g, name + ".weight", {C_out, C_in, K}, w)) return rc;
  if (int rc = read_t(h, g, name + ".bias", {C_out}, b)) return rc;
  const int pad = (C_out + 63) / 64 * 64;
  std::vector<float> wt(static_cast<size_t>(K) * C_in * pad, 0.0f), bp(pad, 0.0f);
  for (int oc = 0; oc < C_out; ++oc)
    for (int ic = 0; ic < C_in; ++ic)
      for (int k = 0; k < K; ++k)
        wt[(static_cast<size_t>(k) * C_in + ic) * pad + oc] = w[(static_cast<size_t>(oc) * C_in + ic) * K + k];
  for (int oc = 0; oc < C_out; ++oc) bp[oc] = b[oc];
  out->C_in = C_in;
  out->C_out = C_out;
  out->C_out_pad = pad;
  out->K = K;
  if (int rc = dupload(h, &out->wt, wt.data(), wt.size())) return rc;
  if (int rc = dupload(h, &out->b, bp.data(), bp.size())) return rc;
  if (C_in % 64 == 0) {
    // hi = bf16(w), lo = bf16(w - hi), tap-major rows [k][oc] of C_in, oc
    // padded to `pad` with zero rows
    std::vector<uint16_t> hb(static_cast<size_t>(K) * pad * C_in, 0), lb(hb.size(), 0);
    for (int oc = 0; oc < C_out; ++oc)
      for (int ic = 0; ic < C_in; ++ic)
        for (int k = 0; k < K; ++k) {
          const float v = w[(static_cast<size_t>(oc) * C_in + ic) * K + k];
          const size_t o = (static_cast<size_t>(k) * pad + oc) * C_in + ic;
          hb[o] = bf16_bits(v);
          const uint32_t bits = static_cast<uint32_t>(hb[o]) << 16;
          float hv;
          std::memcpy(&hv, &bits, 4);
          lb[o] = bf16_bits(v - hv);
        }
    if (int rc = dupload(h, reinterpret_cast<uint16_t**>(&out->whi), hb.data(), hb.size())) return rc;
    if (int rc = dupload(h, reinterpret_cast<uint16_t**>(&out->wlo), lb.data(), lb.size())) return rc;
    const uint64_t rows = static_cast<uint64_t>(K) * pad;
    bool ok = tmap_bf16(&out->tmh[0], out->whi, rows, C_in, C_in, 64, 64) &&
              tmap_bf16(&out->tml[0], out->wlo, rows, C_in, C_in, 64, 64);
    if (ok && pad % 128 == 0)
      ok = tmap_bf16(&out->tmh[1], out->whi, rows, C_in, C_in, 128, 64) &&
           tmap_bf16(&out->tml[1], out->wlo, rows, C_in, C_in, 128, 64);
    if (!ok) return h->fail(LX_ERR_CUDA, "hift: tensor map of " + name);
    out->tc = true;
  }
  return LX_OK;
}

int load_snake(lx_hift* h, GgufFile& g, const std::string& name, int C, SnakeW* out) {
  std::vector<float> a;
  if (int rc = read_t(h, g, name, {C}, a)) return rc;
  std::vector<float> inv(C);
  for (int c = 0; c < C; ++c) inv[c] = 1.0f / (a[c] + SNAKE_EPS);  // gguf.cpp:24-33
  if (int rc = dupload(h, &out->alpha, a.data(), a.size())) return rc;
  return dupload(h, &out->inv, inv.data(), inv.size());
}

int load_resblock(lx_hift* h, GgufFile& g, const std::string& p, int C, int K, ResW* out) {
  for (int j = 0; j < 3; ++j) {
    const std::string s = std::to_string(j);
    if (int rc = load_conv(h, g, p + ".convs1." + s, C, C, K, &out->c1[j])) return rc;
    if (int rc = load_conv(h, g, p + ".convs2." + s, C, C, K, &out->c2[j])) return rc;
    if (int rc = load_snake(h, g, p + ".activations1." + s + ".alpha", C, &out->a1[j])) return rc;
    if (int rc = load_snake(h, g, p + ".activations2." + s + ".alpha", C, &out->a2[j])) return rc;
  }
  return LX_OK;
}

int load_f64(lx_hift* h, GgufFile& g, const std::string& name, std::vector<int64_t> shape, double** out) {
  std::vector<float> v;
  if (int rc = read_t(h, g, name, shape, v)) return rc;
  std::vector<double> d(v.begin(), v.end());
  return dupload(h, out, d.data(), d.size());
}

int load_model(lx_hift* h, const char* path) {
  GgufFile g;
  if (int rc = g.open(path)) return h->fail(rc, "hift: " + g.error());
  Model& m = h->m;
  if (int rc = load_conv(h, g, "conv_pre", BASE_CH, IN_CH, 5, &m.conv_pre)) return rc;
  if (int rc = load_conv(h, g, "conv_post", OUT_CH, 64, 7, &m.conv_post)) return rc;
  int cin = BASE_CH;
  for (int i = 0; i < 3; ++i) {
    const int ch = stage_channels(i);
    const std::string s = std::to_string(i);
    if (int rc = load_conv(h, g, "ups." + s, ch, cin, UPSAMPLE_KERNELS[i], &m.ups[i])) return rc;
    if (int rc = load_conv(h, g, "source_downs." + s, ch, OUT_CH, SRC_DOWN_KERNELS[i], &m.src_down[i])) return rc;
    if (int rc = load_resblock(h, g, "source_resblocks." + s, ch, SRC_RB_KERNELS[i], &m.src_rb[i])) return rc;
    cin = ch;
  }
  for (int i = 0; i < 9; ++i)
    if (int rc = load_resblock(h, g, "resblocks." + std::to_string(i), stage_channels(i / 3), RESBLOCK_KERNELS[i % 3],
                               &m.rb[i]))
      return rc;
  std::vector<float> v;
  if (int rc = read_t(h, g, "m_source.l_linear.weight", {1, HARM}, v)) return rc;
  if (int rc = dupload(h, &m.msw, v.data(), v.size())) return rc;
  if (int rc = read_t(h, g, "m_source.l_linear.bias", {1}, v)) return rc;
  m.msb = v[0];
  if (int rc = load_f64(h, g, "f0_predictor.condnet.0.weight", {BASE_CH, IN_CH, 4}, &m.f0_w[0])) return rc;
  if (int rc = load_f64(h, g, "f0_predictor.condnet.0.bias", {BASE_CH}, &m.f0_b[0])) return rc;
  for (int i = 1; i < 5; ++i) {
    const std::string s = std::to_string(2 * i);
    if (int rc = load_f64(h, g, "f0_predictor.condnet." + s + ".weight", {BASE_CH, BASE_CH, 3}, &m.f0_w[i])) return rc;
    if (int rc = load_f64(h, g, "f0_predictor.condnet." + s + ".bias", {BASE_CH}, &m.f0_b[i])) return rc;
  }
  if (int rc = load_f64(h, g, "f0_predictor.classifier.weight", {1, BASE_CH}, &m.cls_w)) return rc;
  if (int rc = read_t(h, g, "f0_predictor.classifier.bias", {1}, v)) return rc;
  m.cls_b = static_cast<double>(v[0]);
  return LX_OK;
}

void wfree(void*& p) {
  if (p) cudaFree(p);
  p = nullptr;
}

void free_work(Work& w) {
  void** ptrs[] = {reinterpret_cast<void**>(&w.mel_d), reinterpret_cast<void**>(&w.y0), reinterpret_cast<void**>(&w.y1),
                   reinterpret_cast<void**>(&w.mel),   reinterpret_cast<void**>(&w.melT), reinterpret_cast<void**>(&w.f0),
                   reinterpret_cast<void**>(&w.cums),  reinterpret_cast<void**>(&w.bank), reinterpret_cast<void**>(&w.rand),
                   reinterpret_cast<void**>(&w.s),     reinterpret_cast<void**>(&w.stft), reinterpret_cast<void**>(&w.post),
                   reinterpret_cast<void**>(&w.vw),    reinterpret_cast<void**>(&w.audio),
                   reinterpret_cast<void**>(&w.sine_wavs), reinterpret_cast<void**>(&w.mag),
                   reinterpret_cast<void**>(&w.pha),   reinterpret_cast<void**>(&w.raw), reinterpret_cast<void**>(&w.stage),
                   reinterpret_cast<void**>(&w.ahi),   reinterpret_cast<void**>(&w.alo), reinterpret_cast<void**>(&w.err),
                   reinterpret_cast<void**>(&w.bhi),   reinterpret_cast<void**>(&w.blo)};
  for (void** p : ptrs) wfree(*p);
  for (float*& p : w.act) {
    void* v = p;
    wfree(v);
    p = nullptr;
  }
  w.cap_T = 0;
  w.cap_dbg = false;
}

size_t act_floats(int T) { return static_cast<size_t>(7680) * T + 64; }
// largest tensor-core A operand: the x3 upsampled 128-channel input of ups.2
size_t split_elems(int T) { return static_cast<size_t>(15360) * T + 64; }

void clear_graphs(lx_hift* h) {
  for (auto& kv : h->graphs) cudaGraphExecDestroy(kv.second);
  h->graphs.clear();
}

int ensure_work(lx_hift* h, int T, bool dbg) {
  Work& w = h->ws;
  if (w.cap_T >= T && (w.cap_dbg || !dbg)) return LX_OK;
  cudaStreamSynchronize(h->stream);
  clear_graphs(h);
  const int nT = std::max(T, w.cap_T);
  const bool nd = dbg || w.cap_dbg;
  free_work(w);
  const size_t L_S = static_cast<size_t>(nT) * TOTAL_SCALE, N = L_S / HOP + 1;
  auto A = [&](auto** p, size_t n) -> bool {
    return cudaMalloc(reinterpret_cast<void**>(p), std::max<size_t>(n, 1) * sizeof(**p)) == cudaSuccess;
  };
  bool ok = A(&w.mel_d, static_cast<size_t>(IN_CH) * nT) && A(&w.y0, static_cast<size_t>(BASE_CH) * nT) &&
            A(&w.y1, static_cast<size_t>(BASE_CH) * nT) && A(&w.mel, static_cast<size_t>(IN_CH) * nT) &&
            A(&w.melT, static_cast<size_t>(IN_CH) * nT) && A(&w.f0, nT) && A(&w.cums, static_cast<size_t>(HARM) * nT) &&
            A(&w.bank, L_S * HARM) && A(&w.rand, HARM) && A(&w.s, L_S) && A(&w.stft, N * OUT_CH) &&
            A(&w.post, N * OUT_CH) && A(&w.vw, N * N_FFT) && A(&w.audio, L_S) && A(&w.ahi, split_elems(nT)) &&
            A(&w.alo, split_elems(nT)) && A(&w.bhi, act_floats(nT)) && A(&w.blo, act_floats(nT)) && A(&w.err, 1);
  for (int i = 0; ok && i < 8; ++i) ok = A(&w.act[i], act_floats(nT));
  if (ok && nd)
    ok = A(&w.sine_wavs, L_S * HARM) && A(&w.mag, N * N_BINS) && A(&w.pha, N * N_BINS) && A(&w.raw, L_S) &&
         A(&w.stage, act_floats(nT));
  if (!ok) {
    free_work(w);
    cudaGetLastError();
    return h->fail(LX_ERR_OOM, "hift: workspace allocation failed");
  }
  w.cap_T = nT;
  w.cap_dbg = nd;
  return LX_OK;
}

inline unsigned nblk(size_t n, unsigned t) { return static_cast<unsigned>((n + t - 1) / t); }

int num_sms_hift() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  }
  return n;
}

// LX_HIFT_TC=0 keeps every conv on the fp32 CUDA-core kernel (A/B switch);
// by default the convs with 64-multiple channel counts use k_hconv_tc.
bool use_tc() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("LX_HIFT_TC");
    v = (e && std::strcmp(e, "0") == 0) ? 0 : 1;
  }
  return v == 1;
}

// The next conv's A operands, written by a tensor-core conv's epilogue.
struct NextSplit {
  bf16* hi = nullptr;
  bf16* lo = nullptr;
  int act = ACT_NONE;
  float slope = 0.f;
  const SnakeW* sn = nullptr;
};

void split(cudaStream_t s, const float* in, int L_in, int C, int up, int act, float slope, const SnakeW* sn, bf16* hi,
           bf16* lo) {
  const size_t n8 = static_cast<size_t>(L_in) * up * C / 8;
  k_split<<<nblk(n8, 256), 256, 0, s>>>(in, L_in, C, up, act, slope, sn ? sn->alpha : nullptr, sn ? sn->inv : nullptr,
                                        hi, lo);
}

// Tensor-core conv over already split A operands (rows_a rows of C_in).
// out may be null when nx carries the only consumer.  False when a tensor
// map cannot be encoded.
bool tc_conv(cudaStream_t s, const Work& ws, const bf16* ahi, const bf16* alo, size_t rows_a, int C_in, const ConvW& w,
             int dil, int pad_left, const float* res, float* out, int L_out, const NextSplit* nx) {
  const int sms = num_sms_hift();
  const int wrows = (128 + (w.K - 1) * dil + 7) / 8 * 8;
  if (wrows > TC_WROWS_MAX) return false;
  CUtensorMap ah, al;
  if (!tmap_bf16(&ah, ahi, rows_a, C_in, C_in, wrows, 64) || !tmap_bf16(&al, alo, rows_a, C_in, C_in, wrows, 64))
    return false;
  TcConvArgs ta;
  ta.wrows = wrows;
  ta.L_out = L_out;
  ta.C_out = w.C_out_pad;
  ta.ldo = w.C_out;
  ta.K_taps = w.K;
  ta.dil = dil;
  ta.pad_left = pad_left;
  ta.n_cb = C_in / 64;
  ta.bias = w.b;
  ta.res = res;
  ta.out = out;
  ta.err = ws.err;
  ta.nhi = nx ? nx->hi : nullptr;
  ta.nlo = nx ? nx->lo : nullptr;
  ta.nact = nx ? nx->act : ACT_NONE;
  ta.nslope = nx ? nx->slope : 0.f;
  ta.nalpha = nx && nx->sn ? nx->sn->alpha : nullptr;
  ta.ninv = nx && nx->sn ? nx->sn->inv : nullptr;
  const int tiles_m = static_cast<int>(nblk(static_cast<size_t>(L_out), 128));
  if (w.C_out_pad % 128 == 0 && tiles_m * (w.C_out_pad / 128) >= sms) {
    const int tiles = tiles_m * (w.C_out_pad / 128);
    k_hconv_tc<128><<<std::min(tiles, sms), TC_THREADS, tc_smem_bytes<128>(), s>>>(ah, al, w.tmh[1], w.tml[1], ta);
  } else {
    const int tiles = tiles_m * (w.C_out_pad / 64);
    k_hconv_tc<64><<<std::min(tiles, sms), TC_THREADS, tc_smem_bytes<64>(), s>>>(ah, al, w.tmh[0], w.tml[0], ta);
  }
  return true;
}

// One conv of the network (see ConvArgs for the semantics).  Returns false
// when a tensor map cannot be encoded.
bool hconv(cudaStream_t s, const Work& ws, const float* in, int L_in, int C_in, int up, const ConvW& w, int dil,
           int pad_left, int act, float slope, const SnakeW* sn, const float* res, float* out, int L_out) {
  const int sms = num_sms_hift();
  if (use_tc() && w.tc && C_in % 64 == 0) {
    split(s, in, L_in, C_in, up, act, slope, sn, ws.ahi, ws.alo);
    return tc_conv(s, ws, ws.ahi, ws.alo, static_cast<size_t>(L_in) * up, C_in, w, dil, pad_left, res, out, L_out,
                   nullptr);
  }
  ConvArgs a;
  a.in = in;
  a.L_in = L_in;
  a.C_in = C_in;
  a.up = up;
  a.wt = w.wt;
  a.bias = w.b;
  a.C_out = w.C_out;
  a.C_out_pad = w.C_out_pad;
  a.K = w.K;
  a.dil = dil;
  a.pad_left = pad_left;
  a.act = act;
  a.slope = slope;
  a.alpha = sn ? sn->alpha : nullptr;
  a.inv_alpha = sn ? sn->inv : nullptr;
  a.res = res;
  a.out = out;
  a.L_out = L_out;
  // the largest tile that still gives two waves of CTAs, else the smallest
  const size_t waves2 = 2 * static_cast<size_t>(sms);
  const size_t g128 = nblk(static_cast<size_t>(L_out), 128), g64 = nblk(static_cast<size_t>(L_out), 64);
  if (w.C_out_pad % 128 == 0 && g128 * (w.C_out_pad / 128) >= waves2)
    k_hconv<128, 128><<<dim3(g128, w.C_out_pad / 128), HC_THREADS, 0, s>>>(a);
  else if (g128 * (w.C_out_pad / 64) >= waves2)
    k_hconv<128, 64><<<dim3(g128, w.C_out_pad / 64), HC_THREADS, 0, s>>>(a);
  else
    k_hconv<64, 64><<<dim3(g64, w.C_out_pad / 64), HC_THREADS, 0, s>>>(a);
  return true;
}

// resblock (hift.cpp:25-40): R = x after 3 x (snake1 -> conv1(d_j) -> snake2 -> conv2 + residual)
bool resblock(cudaStream_t s, const Work& ws, const ResW& w, int k, const float* X, float* R, float* T1, int C, int L) {
  if (use_tc() && w.c1[0].tc && C % 64 == 0) {
    // split(snake1_0(X)) once; afterwards every conv's epilogue writes the
    // next conv's split operands (conv1 -> snake2 of its output, no fp32
    // copy; conv2 -> the residual sum R and snake1_{j+1}(R)), ping-ponging
    // between the two split buffers
    split(s, X, L, C, 1, ACT_SNAKE, 0.f, &w.a1[0], ws.ahi, ws.alo);
    for (int j = 0; j < 3; ++j) {
      const int d = RESBLOCK_DILATIONS[j];
      NextSplit n1;
      n1.hi = ws.bhi;
      n1.lo = ws.blo;
      n1.act = ACT_SNAKE;
      n1.sn = &w.a2[j];
      if (!tc_conv(s, ws, ws.ahi, ws.alo, L, C, w.c1[j], d, d * (k - 1), nullptr, nullptr, L, &n1)) return false;
      NextSplit n2;
      n2.hi = ws.ahi;
      n2.lo = ws.alo;
      n2.act = ACT_SNAKE;
      n2.sn = j < 2 ? &w.a1[j + 1] : nullptr;
      if (!tc_conv(s, ws, ws.bhi, ws.blo, L, C, w.c2[j], 1, k - 1, j == 0 ? X : R, R, L, j < 2 ? &n2 : nullptr))
        return false;
    }
    return true;
  }
  for (int j = 0; j < 3; ++j) {
    const int d = RESBLOCK_DILATIONS[j];
    const float* src = j == 0 ? X : R;
    if (!hconv(s, ws, src, L, C, 1, w.c1[j], d, d * (k - 1), ACT_SNAKE, 0.f, &w.a1[j], nullptr, T1, L)) return false;
    if (!hconv(s, ws, T1, L, C, 1, w.c2[j], 1, k - 1, ACT_SNAKE, 0.f, &w.a2[j], src, R, L)) return false;
  }
  return true;
}

// Debug capture of a time-major device tensor into the caller's [C][L] buffer.
int capture(lx_hift* h, float* dst, const float* src, int L, int C, int act = ACT_NONE, float slope = 0.f) {
  if (!dst) return LX_OK;
  k_transpose<<<dim3(nblk(L, 32), nblk(C, 32)), dim3(32, 8), 0, h->stream>>>(src, L, C, act, slope, h->ws.stage);
  HCK(cudaMemcpyAsync(dst, h->ws.stage, static_cast<size_t>(L) * C * sizeof(float), cudaMemcpyDeviceToHost,
                      h->stream));
  HCK(cudaStreamSynchronize(h->stream));
  return LX_OK;
}

int copy_out(lx_hift* h, float* dst, const float* src, size_t n) {
  if (!dst) return LX_OK;
  HCK(cudaMemcpyAsync(dst, src, n * sizeof(float), cudaMemcpyDeviceToHost, h->stream));
  HCK(cudaStreamSynchronize(h->stream));
  return LX_OK;
}

// The whole vocoder on stream s: mel_dev [80][T] -> ws.audio [T*480].
// bank [T*480][9] and rand [9] are device buffers.  dbg (host pointers) makes
// the call synchronous at every captured stage.
int forward(lx_hift* h, const float* mel_dev, int T, const float* rand, const float* bank, cudaStream_t s,
            lx_hift_debug* dbg) {
  Work& w = h->ws;
  const Model& m = h->m;
  const int L_S = T * TOTAL_SCALE, N = L_S / HOP + 1;
  // f0 predictor (float64)
  k_mel_prep<<<nblk(static_cast<size_t>(IN_CH) * T, 256), 256, 0, s>>>(mel_dev, T, w.mel_d, w.melT);
  const dim3 f0_grid(nblk(T, F0_BT), BASE_CH / F0_BO);
  k_f0_conv<4><<<f0_grid, 256, 0, s>>>(w.mel_d, T, IN_CH, m.f0_w[0], m.f0_b[0], 0, 1, w.y0);
  double *ya = w.y0, *yb = w.y1;
  for (int i = 1; i < 5; ++i) {
    k_f0_conv<3><<<f0_grid, 256, 0, s>>>(ya, T, BASE_CH, m.f0_w[i], m.f0_b[i], 2, 1, yb);
    std::swap(ya, yb);
  }
  k_f0_cls<<<nblk(T, 128), 128, 0, s>>>(ya, T, m.cls_w, m.cls_b, w.f0);
  // SineGen2 + m_source + STFT
  k_rad_down<<<nblk(static_cast<size_t>(T) * HARM, 256), 256, 0, s>>>(w.f0, rand, T, w.cums);
  k_sine_cumsum<<<1, 32, 0, s>>>(w.cums, T);
  k_source<<<nblk(L_S, 256), 256, 0, s>>>(w.f0, w.cums, bank, m.msw, m.msb, T, w.s, dbg ? w.sine_wavs : nullptr);
  k_stft<<<nblk(N, 128), 128, 0, s>>>(w.s, L_S, w.stft);
  if (dbg) {
    if (int rc = copy_out(h, dbg->f0, w.f0, T)) return rc;
    if (int rc = copy_out(h, dbg->sine_wavs, w.sine_wavs, static_cast<size_t>(L_S) * HARM)) return rc;
    if (int rc = copy_out(h, dbg->sine_merge, w.s, L_S)) return rc;
    if (int rc = capture(h, dbg->s_stft, w.stft, N, OUT_CH)) return rc;
  }
  float *X = w.act[0], *F = w.act[1], *S1 = w.act[2], *S2 = w.act[3], *T1 = w.act[7];
  float* R[3] = {w.act[4], w.act[5], w.act[6]};
  // conv_pre: CausalConv1d(80 -> 512, k=5, right pad 4)
  auto bad_map = [h]() { return h->fail(LX_ERR_CUDA, "hift: tensor map encoding failed"); };
  HCK(cudaMemsetAsync(w.err, 0, sizeof(int), s));
  if (!hconv(s, w, w.melT, T, IN_CH, 1, m.conv_pre, 1, 0, ACT_NONE, 0.f, nullptr, nullptr, X, T)) return bad_map();
  if (dbg)
    if (int rc = capture(h, dbg->conv_pre, X, T, BASE_CH)) return rc;
  int L_prev = T, C_prev = BASE_CH;
  for (int i = 0; i < 3; ++i) {
    const int C = stage_channels(i), L = L_prev * UPSAMPLE_RATES[i];
    if (dbg)
      if (int rc = capture(h, dbg->ups_lrelu[i], X, L_prev, C_prev, ACT_LRELU, LRELU_SLOPE)) return rc;
    // CausalConv1dUpsample: leaky_relu -> nearest x rate -> left pad k-1 -> conv
    float* U = i == 2 ? F + C : F;
    if (!hconv(s, w, X, L_prev, C_prev, UPSAMPLE_RATES[i], m.ups[i], 1, UPSAMPLE_KERNELS[i] - 1, ACT_LRELU,
               LRELU_SLOPE, nullptr, nullptr, U, L))
      return bad_map();
    if (dbg)
      if (int rc = capture(h, dbg->ups[i], U, L, C)) return rc;
    int Lf = L;
    if (i == 2) {
      k_reflect_row0<<<nblk(C, 64), 64, 0, s>>>(F, C);
      Lf = L + 1;
      if (dbg)
        if (int rc = capture(h, dbg->reflection_pad, F, Lf, C)) return rc;
    }
    // source branch: CausalConv1dDownSample (left pad stride-1), resblock
    const int st = SRC_DOWN_STRIDES[i];
    const ConvW& sd = m.src_down[i];
    k_conv_direct<<<nblk(static_cast<size_t>(Lf) * C / 4, 256), 256, 0, s>>>(
        w.stft, N, OUT_CH, sd.wt, sd.b, C, sd.C_out_pad, sd.K, st, st == 1 ? 0 : st - 1, S1, Lf);
    if (dbg)
      if (int rc = capture(h, dbg->source_downs[i], S1, Lf, C)) return rc;
    if (!resblock(s, w, m.src_rb[i], SRC_RB_KERNELS[i], S1, S2, T1, C, Lf)) return bad_map();
    if (dbg)
      if (int rc = capture(h, dbg->source_resblocks[i], S2, Lf, C)) return rc;
    const size_t n4 = static_cast<size_t>(Lf) * C / 4;
    k_add<<<nblk(n4, 256), 256, 0, s>>>(F, S2, F, n4);
    if (dbg)
      if (int rc = capture(h, dbg->fusion[i], F, Lf, C)) return rc;
    for (int j = 0; j < 3; ++j) {
      if (!resblock(s, w, m.rb[3 * i + j], RESBLOCK_KERNELS[j], F, R[j], T1, C, Lf)) return bad_map();
      if (dbg)
        if (int rc = capture(h, dbg->resblocks[3 * i + j], R[j], Lf, C)) return rc;
    }
    k_combine3<<<nblk(n4, 256), 256, 0, s>>>(R[0], R[1], R[2], X, n4);
    if (dbg)
      if (int rc = capture(h, dbg->post_resblocks[i], X, Lf, C)) return rc;
    L_prev = Lf;
    C_prev = C;
  }
  // final leaky_relu (slope 0.01) -> conv_post (k=7, left pad 6)
  if (dbg)
    if (int rc = capture(h, dbg->final_lrelu, X, N, 64, ACT_LRELU, 0.01f)) return rc;
  if (!hconv(s, w, X, N, 64, 1, m.conv_post, 1, 6, ACT_LRELU, 0.01f, nullptr, nullptr, w.post, N)) return bad_map();
  if (dbg)
    if (int rc = capture(h, dbg->conv_post, w.post, N, OUT_CH)) return rc;
  k_istft_frames<<<nblk(N, 128), 128, 0, s>>>(w.post, N, w.vw, dbg ? w.mag : nullptr, dbg ? w.pha : nullptr);
  k_istft_ola<<<nblk(L_S, 256), 256, 0, s>>>(w.vw, N, dbg ? w.raw : nullptr, w.audio);
  if (dbg) {
    if (int rc = copy_out(h, dbg->magnitude, w.mag, static_cast<size_t>(N) * N_BINS)) return rc;
    if (int rc = copy_out(h, dbg->phase, w.pha, static_cast<size_t>(N) * N_BINS)) return rc;
    if (int rc = copy_out(h, dbg->istft, w.raw, L_S)) return rc;
    if (int rc = copy_out(h, dbg->speech, w.audio, L_S)) return rc;
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(h, e, "hift launch");
  return LX_OK;
}

// forward() on stream s, replayed from a CUDA graph when no debug capture is
// asked for (the ~120 launches of a call then cost one graph launch).  The
// graph reads mel from the workspace, so callers copy it there first.
int run_forward(lx_hift* h, int T, const float* rand, const float* bank, cudaStream_t s, lx_hift_debug* dbg) {
  if (dbg || !h->use_graphs) return forward(h, h->ws.mel, T, rand, bank, s, dbg);
  char key[96];
  std::snprintf(key, sizeof key, "%d|%p|%p", T, static_cast<const void*>(rand), static_cast<const void*>(bank));
  auto it = h->graphs.find(key);
  if (it == h->graphs.end()) {
    cudaStream_t cs;
    HCK(cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking));
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal);
    int rc = LX_OK;
    if (e == cudaSuccess) {
      rc = forward(h, h->ws.mel, T, rand, bank, cs, nullptr);
      e = cudaStreamEndCapture(cs, &g);
    }
    cudaStreamDestroy(cs);
    if (rc != LX_OK || e != cudaSuccess) {
      if (g) cudaGraphDestroy(g);
      cudaGetLastError();
      return rc != LX_OK ? rc : cuda_fail(h, e, "hift graph capture");
    }
    cudaGraphExec_t ex = nullptr;
    e = cudaGraphInstantiate(&ex, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return cuda_fail(h, e, "hift graph instantiate");
    it = h->graphs.emplace(key, ex).first;
  }
  HCK(cudaGraphLaunch(it->second, s));
  return LX_OK;
}

int upload_dft(lx_hift* h) {
  DftConst d;
  for (int f = 0; f < N_FFT; ++f)
    for (int n = 0; n < N_FFT; ++n) {
      const double a = 2.0 * PI_D * f * n / N_FFT;
      d.c[f][n] = static_cast<float>(std::cos(a));
      d.s[f][n] = static_cast<float>(std::sin(a));
    }
  // periodic Hann in float32 arithmetic, as source.cpp:47-50
  for (int n = 0; n < N_FFT; ++n)
    d.win[n] = 0.5f * (1.0f - std::cos(2.0f * static_cast<float>(PI_D) * static_cast<float>(n) / static_cast<float>(N_FFT)));
  HCK(cudaMemcpyToSymbol(g_dft, &d, sizeof(d)));
  return LX_OK;
}

}  // namespace
}  // namespace hift
}  // namespace lx

// ---------------------------------------------------------------------------
// C ABI
// ---------------------------------------------------------------------------
using lx::hift::TOTAL_SCALE;
using lx::hift::HARM;

extern "C" int lx_hift_create(int device, lx_hift** out) {
  if (!out) return LX_ERR_ARG;
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return LX_ERR_CUDA;
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess || prop.major != 10) return LX_ERR_CUDA;
  if (cudaSetDevice(device) != cudaSuccess) return LX_ERR_CUDA;
  std::unique_ptr<lx_hift> h(new lx_hift());
  h->device = device;
  const char* ge = std::getenv("LX_HIFT_GRAPHS");
  if (ge && std::strcmp(ge, "0") == 0) h->use_graphs = false;
  if (cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking) != cudaSuccess) return LX_ERR_CUDA;
  if (lx::hift::upload_dft(h.get()) != LX_OK) return LX_ERR_CUDA;
  if (cudaFuncSetAttribute(lx::hift::k_hconv_tc<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           lx::hift::tc_smem_bytes<64>()) != cudaSuccess ||
      cudaFuncSetAttribute(lx::hift::k_hconv_tc<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           lx::hift::tc_smem_bytes<128>()) != cudaSuccess)
    return LX_ERR_CUDA;
  *out = h.release();
  return LX_OK;
}

extern "C" void lx_hift_destroy(lx_hift* h) {
  if (!h) return;
  cudaSetDevice(h->device);
  cudaStreamSynchronize(h->stream);
  lx::hift::clear_graphs(h);
  lx::hift::free_work(h->ws);
  for (void* p : h->allocs) cudaFree(p);
  if (h->d_bank) cudaFree(h->d_bank);
  if (h->d_rand_ini) cudaFree(h->d_rand_ini);
  cudaStreamDestroy(h->stream);
  delete h;
}

extern "C" const char* lx_hift_last_error(const lx_hift* h) { return h ? h->err.c_str() : "null handle"; }

extern "C" int lx_hift_load_gguf(lx_hift* h, const char* path) {
  if (!h || !path) return LX_ERR_ARG;
  if (h->loaded) return LX_OK;
  cudaSetDevice(h->device);
  h->err.clear();
  const int rc = lx::hift::load_model(h, path);
  if (rc) {
    for (void* p : h->allocs) cudaFree(p);
    h->allocs.clear();
    h->m = lx::hift::Model();
    return rc;
  }
  h->loaded = true;
  return LX_OK;
}

extern "C" int lx_hift_load_source(lx_hift* h, const char* path) {
  if (!h || !path) return LX_ERR_ARG;
  if (h->source_loaded) return LX_OK;
  cudaSetDevice(h->device);
  FILE* f = std::fopen(path, "rb");
  if (!f) return h->fail(LX_ERR_IO, std::string("hift: cannot open source asset ") + path);
  uint32_t magic = 0, version = 0, dim = 0;
  uint64_t sine_max = 0;
  bool ok = std::fread(&magic, 4, 1, f) == 1 && std::fread(&version, 4, 1, f) == 1 && std::fread(&dim, 4, 1, f) == 1 &&
            std::fread(&sine_max, 8, 1, f) == 1;
  // hift.cpp:104-114: magic "HSRC", version 1, 9 harmonics, the full 300 s bank
  if (!ok || magic != 0x43525348u || version != 1 || dim != static_cast<uint32_t>(HARM) ||
      sine_max != static_cast<uint64_t>(lx::hift::SINE_MAX_SAMPLES)) {
    std::fclose(f);
    return h->fail(LX_ERR_FORMAT, std::string("hift: bad source asset header in ") + path);
  }
  std::vector<float> rand(HARM), bank(static_cast<size_t>(sine_max) * HARM);
  ok = std::fread(rand.data(), 4, HARM, f) == static_cast<size_t>(HARM) &&
       std::fread(bank.data(), 4, bank.size(), f) == bank.size();
  std::fclose(f);
  if (!ok) return h->fail(LX_ERR_FORMAT, std::string("hift: short read on source asset ") + path);
  if (cudaMalloc(&h->d_rand_ini, HARM * sizeof(float)) != cudaSuccess ||
      cudaMalloc(&h->d_bank, bank.size() * sizeof(float)) != cudaSuccess) {
    if (h->d_rand_ini) cudaFree(h->d_rand_ini);
    h->d_rand_ini = nullptr;
    return h->fail(LX_ERR_OOM, "hift: source bank allocation failed");
  }
  if (cudaMemcpy(h->d_rand_ini, rand.data(), HARM * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(h->d_bank, bank.data(), bank.size() * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess)
    return h->fail(LX_ERR_CUDA, "hift: source bank upload failed");
  h->source_loaded = true;
  return LX_OK;
}

extern "C" int lx_hift_vocode(lx_hift* h, const float* mel, int T, const float* rand_ini, const float* sine_waves,
                              float* audio, size_t audio_cap, lx_hift_debug* debug) {
  if (!h || !mel || !audio || T <= 0) return LX_ERR_ARG;
  if (!h->loaded) return h->fail(LX_ERR_STATE, "hift: vocode before load");
  if ((rand_ini == nullptr) != (sine_waves == nullptr))
    return h->fail(LX_ERR_ARG, "hift: rand_ini and sine_waves must both be given or both be NULL");
  const size_t L_S = static_cast<size_t>(T) * TOTAL_SCALE;
  if (audio_cap < L_S) return h->fail(LX_ERR_ARG, "hift: audio buffer too small");
  if (!rand_ini) {
    if (!h->source_loaded) return h->fail(LX_ERR_STATE, "hift: vocode without explicit buffers before load_source");
    if (L_S > static_cast<size_t>(lx::hift::SINE_MAX_SAMPLES))
      return h->fail(LX_ERR_SHAPE, "hift: utterance longer than the 300 s source bank");
  }
  cudaSetDevice(h->device);
  h->err.clear();
  if (int rc = lx::hift::ensure_work(h, T, debug != nullptr)) return rc;
  lx::hift::Work& w = h->ws;
  cudaStream_t s = h->stream;
#define VCK(expr)                                                                  \
  do {                                                                             \
    cudaError_t e_ = (expr);                                                       \
    if (e_ != cudaSuccess) return h->fail(LX_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(e_)); \
  } while (0)
  VCK(cudaMemcpyAsync(w.mel, mel, static_cast<size_t>(lx::hift::IN_CH) * T * sizeof(float), cudaMemcpyHostToDevice, s));
  const float *rand = h->d_rand_ini, *bank = h->d_bank;
  if (rand_ini) {
    VCK(cudaMemcpyAsync(w.rand, rand_ini, HARM * sizeof(float), cudaMemcpyHostToDevice, s));
    VCK(cudaMemcpyAsync(w.bank, sine_waves, L_S * HARM * sizeof(float), cudaMemcpyHostToDevice, s));
    rand = w.rand;
    bank = w.bank;
  }
  if (int rc = lx::hift::run_forward(h, T, rand, bank, s, debug)) return rc;
  VCK(cudaMemcpyAsync(audio, w.audio, L_S * sizeof(float), cudaMemcpyDeviceToHost, s));
  int dev_err = 0;
  VCK(cudaMemcpyAsync(&dev_err, w.err, sizeof(int), cudaMemcpyDeviceToHost, s));
  VCK(cudaStreamSynchronize(s));
#undef VCK
  if (dev_err) return h->fail(LX_ERR_TIMEOUT, "hift: a device-side wait exceeded its bound (code " +
                                                   std::to_string(dev_err) + ")");
  return LX_OK;
}

extern "C" int lx_hift_vocode_device(lx_hift* h, const float* mel_dev, int T, float* audio_dev, void* stream) {
  if (!h || !mel_dev || !audio_dev || T <= 0) return LX_ERR_ARG;
  if (!h->loaded) return h->fail(LX_ERR_STATE, "hift: vocode before load");
  if (!h->source_loaded) return h->fail(LX_ERR_STATE, "hift: vocode_device needs load_source");
  const size_t L_S = static_cast<size_t>(T) * TOTAL_SCALE;
  if (L_S > static_cast<size_t>(lx::hift::SINE_MAX_SAMPLES))
    return h->fail(LX_ERR_SHAPE, "hift: utterance longer than the 300 s source bank");
  cudaSetDevice(h->device);
  if (int rc = lx::hift::ensure_work(h, T, false)) return rc;
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : h->stream;
  if (cudaMemcpyAsync(h->ws.mel, mel_dev, static_cast<size_t>(lx::hift::IN_CH) * T * sizeof(float),
                      cudaMemcpyDeviceToDevice, s) != cudaSuccess)
    return h->fail(LX_ERR_CUDA, "hift: input copy failed");
  if (int rc = lx::hift::run_forward(h, T, h->d_rand_ini, h->d_bank, s, nullptr)) return rc;
  if (cudaMemcpyAsync(audio_dev, h->ws.audio, L_S * sizeof(float), cudaMemcpyDeviceToDevice, s) != cudaSuccess)
    return h->fail(LX_ERR_CUDA, "hift: output copy failed");
  return LX_OK;
}
