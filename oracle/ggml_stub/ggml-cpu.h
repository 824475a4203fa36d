/* Declaration-only stand-in (see ggml.h in this folder). */
#pragma once
#include "ggml-backend.h"

#ifdef __cplusplus
extern "C" {
#endif

ggml_backend_t ggml_backend_cpu_init(void);

#ifdef __cplusplus
}
#endif
