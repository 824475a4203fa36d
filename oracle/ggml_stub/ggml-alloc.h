/* Declaration-only stand-in (see ggml.h in this folder). */
#pragma once
#include "ggml-backend.h"

#ifdef __cplusplus
extern "C" {
#endif

ggml_backend_buffer_t ggml_backend_alloc_ctx_tensors(struct ggml_context* ctx, ggml_backend_t backend);

#ifdef __cplusplus
}
#endif
