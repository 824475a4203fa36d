/*
 * larynx_hift.h -- C ABI of the B200 (sm_100a) HiFT vocoder.
 *
 * Drop-in replacement for larynx::hift::HiftVocoder of hardenedlinux/larynx
 * (include/larynx/hift/hift.h, src/hift/*.cpp): CosyVoice3's
 * CausalHiFTGenerator, whole-sequence (finalize=True) path, mel -> 24 kHz
 * PCM.  Every stage runs on the GPU: the float64 f0 predictor, SineGen2 +
 * m_source + the 16-point STFT, the conv network (conv_pre, three
 * upsample / source-fusion / resblock stages, conv_post) in float32, and the
 * ISTFT.  Plain C types only; status codes are those of larynx_flow.h.
 *
 * Layouts follow the reference's PyTorch byte order: mel is [80][T]
 * ((1, 80, T) row-major), sine_waves is [T*480][9], audio is [T*480].
 * Threading: one handle per GPU, not thread-safe (as HiftVocoder).
 */
#ifndef LARYNX_HIFT_H
#define LARYNX_HIFT_H

#include <stddef.h>
#include <stdint.h>

#include "larynx_flow.h"

#ifdef __cplusplus
extern "C" {
#endif

#define LX_HIFT_SAMPLES_PER_FRAME 480
#define LX_HIFT_HARMONICS 9
#define LX_HIFT_SINE_MAX_SAMPLES 7200000 /* 300 s at 24 kHz */

typedef struct lx_hift lx_hift;

/* Per-stage captures (replaces larynx::hift::HiFTDebug, include/larynx/hift/
 * hift.h:16-41).  Each non-NULL pointer receives that stage in the
 * reference's layout: [C][len] channel-major, len = T (conv_pre), 8T, 40T,
 * 120T (ups / source / fusion / resblock stages 0, 1, 2; stage 2 after the
 * reflection pad is 120T + 1), N = 120T + 1 (s_stft, conv_post, magnitude,
 * phase, reflection_pad, final_lrelu).  ups_lrelu[i] has the channel count
 * of the stage input (512, 256, 128).  resblocks[3 i + j] is stage i's j-th
 * resblock output. */
typedef struct lx_hift_debug {
  float* f0;                  /* [T]          */
  float* sine_wavs;           /* [T*480][9]   */
  float* sine_merge;          /* [T*480]      */
  float* s_stft;              /* [18][N]      */
  float* conv_pre;            /* [512][T]     */
  float* ups_lrelu[3];
  float* ups[3];
  float* source_downs[3];
  float* source_resblocks[3];
  float* fusion[3];
  float* resblocks[9];
  float* post_resblocks[3];
  float* reflection_pad;      /* [64][N]      */
  float* final_lrelu;         /* [64][N]      */
  float* conv_post;           /* [18][N]      */
  float* magnitude;           /* [9][N]       */
  float* phase;               /* [9][N]       */
  float* istft;               /* [T*480]      */
  float* speech;              /* [T*480]      */
} lx_hift_debug;

/* Replaces HiftVocoder() + backend_init_best() (hift.h:48-49, hift.cpp:55-57):
 * binds the handle to CUDA device `device` (an sm_100 part, no CPU fallback). */
int lx_hift_create(int device, lx_hift** out);

/* Replaces ~HiftVocoder() (src/hift/hift.cpp:59-66). */
void lx_hift_destroy(lx_hift* h);

/* Message of the last failed call on this handle ("" if none). */
const char* lx_hift_last_error(const lx_hift* h);

/* Replaces HiftVocoder::load (hift.h:55, hift.cpp:68-79, gguf.cpp:82-158):
 * reads the 246 named float32 tensors of hift.gguf (weight-norm folded),
 * checks every shape and uploads them (conv weights tap-major for the conv
 * kernels; the f0 predictor in float64).  Idempotent like the reference. */
int lx_hift_load_gguf(lx_hift* h, const char* path);

/* Replaces HiftVocoder::load_source (hift.h:63, hift.cpp:88-131): the
 * SineGen2 buffers from an "HSRC" v1 asset (magic 0x43525348, version 1,
 * harmonic_dim 9, sine_max 7,200,000, rand_ini[9], sine_waves[sine_max][9]);
 * the bank is kept in device memory (259 MB). */
int lx_hift_load_source(lx_hift* h, const char* path);

/* Replaces both HiftVocoder::vocode overloads (hift.h:76-87, hift.cpp:140-333).
 * mel: [80][T] host.  rand_ini ([9]) and sine_waves ([T*480][9]) are the
 * explicit SineGen2 buffers of the 5-argument form; pass both NULL for the
 * production form, which uses the loaded source (first T*480 rows of the
 * bank).  audio receives [T*480] floats (audio_cap is its capacity).  Host
 * buffers; synchronous.  debug may be NULL. */
int lx_hift_vocode(lx_hift* h, const float* mel, int T, const float* rand_ini, const float* sine_waves,
                   float* audio, size_t audio_cap, lx_hift_debug* debug);

/* The same on device buffers, enqueued on `stream` (a cudaStream_t, NULL =
 * the handle's stream) without synchronizing: mel_dev [80][T] float32,
 * audio_dev [T*480] float32; uses the loaded source.  No reference
 * counterpart (the reference's API is host vectors only). */
int lx_hift_vocode_device(lx_hift* h, const float* mel_dev, int T, float* audio_dev, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LARYNX_HIFT_H */
