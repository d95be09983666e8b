// Stand-in (test infrastructure; see ggml.h): host-memory "backend" buffers.
// Tensors of a context get host allocations; set/get are copies.
#pragma once
#include "ggml.h"

typedef struct ggml_backend *ggml_backend_t;
typedef struct ggml_backend_buffer *ggml_backend_buffer_t;
typedef struct ggml_backend_sched *ggml_backend_sched_t;

ggml_backend_buffer_t ggml_backend_alloc_ctx_tensors(struct ggml_context *ctx, ggml_backend_t be);
void ggml_backend_buffer_free(ggml_backend_buffer_t buf);
void ggml_backend_tensor_set(struct ggml_tensor *t, const void *data, size_t offset, size_t size);
void ggml_backend_tensor_get(const struct ggml_tensor *t, void *data, size_t offset, size_t size);
