/* Declaration-only stand-in (see ggml.h in this folder). */
#pragma once
#include "ggml.h"

#ifdef __cplusplus
extern "C" {
#endif

struct gguf_context;

size_t gguf_get_data_offset(const struct gguf_context* ctx);
int64_t gguf_get_n_tensors(const struct gguf_context* ctx);
const char* gguf_get_tensor_name(const struct gguf_context* ctx, int64_t tensor_id);
size_t gguf_get_tensor_offset(const struct gguf_context* ctx, int64_t tensor_id);

#ifdef __cplusplus
}
#endif
