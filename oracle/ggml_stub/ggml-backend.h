/* Declaration-only stand-in (see ggml.h in this folder). */
#pragma once
#include "ggml.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct ggml_backend* ggml_backend_t;
typedef struct ggml_backend_buffer* ggml_backend_buffer_t;

ggml_backend_t ggml_backend_init_best(void);
const char* ggml_backend_name(ggml_backend_t backend);
void ggml_backend_tensor_set(struct ggml_tensor* tensor, const void* data, size_t offset, size_t size);
void ggml_backend_tensor_memset(struct ggml_tensor* tensor, uint8_t value, size_t offset, size_t size);
void ggml_backend_buffer_free(ggml_backend_buffer_t buffer);

#ifdef __cplusplus
}
#endif
