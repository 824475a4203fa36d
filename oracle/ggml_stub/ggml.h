/* Declaration-only stand-in for the ggml headers (test infrastructure).
 *
 * The reference's src/hift/internal.h includes ggml.h, ggml-alloc.h,
 * ggml-backend.h, ggml-cpu.h and larynx/backend.h (which includes gguf.h), but
 * the host-side HiFT functions in src/hift/source.cpp (f0_predict,
 * source_stft, istft) use no ggml code: ggml appears only as opaque pointer
 * types in HiFTWeights and in inline helpers of backend.h that source.cpp
 * never calls.  These headers declare just those types and functions (names
 * and signatures of the ggml API), so source.cpp compiles from its own file
 * and links without ggml.  Nothing here is defined; any call would fail to
 * link, which is the point. */
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

struct ggml_tensor;
struct ggml_context;
struct ggml_cgraph;

struct ggml_tensor* ggml_get_tensor(struct ggml_context* ctx, const char* name);
size_t ggml_nbytes(const struct ggml_tensor* tensor);

#ifdef __cplusplus
}
#endif
