/* ggml-backend.h -- the subset of ggml's backend API that sam3.cpp calls
 * (backend selection sam3.cpp:3279-3287, weight buffers sam3.cpp:3320,
 * tensor copies, graph compute sam3.cpp:1019-1030), with ggml's names. */
#pragma once

#include "ggml.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct ggml_backend_buffer_type *ggml_backend_buffer_type_t;
typedef struct ggml_backend_buffer *ggml_backend_buffer_t;
typedef struct ggml_backend *ggml_backend_t;
typedef struct ggml_backend_device *ggml_backend_dev_t;

enum ggml_backend_buffer_usage {
    GGML_BACKEND_BUFFER_USAGE_ANY = 0,
    GGML_BACKEND_BUFFER_USAGE_WEIGHTS = 1,
    GGML_BACKEND_BUFFER_USAGE_COMPUTE = 2,
};

/* buffer types and buffers */
const char *ggml_backend_buft_name(ggml_backend_buffer_type_t buft);
ggml_backend_buffer_t ggml_backend_buft_alloc_buffer(ggml_backend_buffer_type_t buft, size_t size);
size_t ggml_backend_buft_get_alignment(ggml_backend_buffer_type_t buft);
size_t ggml_backend_buft_get_alloc_size(ggml_backend_buffer_type_t buft, const struct ggml_tensor *tensor);
bool ggml_backend_buft_is_host(ggml_backend_buffer_type_t buft);
ggml_backend_dev_t ggml_backend_buft_get_device(ggml_backend_buffer_type_t buft);

void ggml_backend_buffer_free(ggml_backend_buffer_t buffer);
void *ggml_backend_buffer_get_base(ggml_backend_buffer_t buffer);
size_t ggml_backend_buffer_get_size(ggml_backend_buffer_t buffer);
enum ggml_status ggml_backend_buffer_init_tensor(ggml_backend_buffer_t buffer, struct ggml_tensor *tensor);
void ggml_backend_buffer_clear(ggml_backend_buffer_t buffer, uint8_t value);
void ggml_backend_buffer_set_usage(ggml_backend_buffer_t buffer, enum ggml_backend_buffer_usage usage);
enum ggml_backend_buffer_usage ggml_backend_buffer_get_usage(ggml_backend_buffer_t buffer);
ggml_backend_buffer_type_t ggml_backend_buffer_get_type(ggml_backend_buffer_t buffer);

/* backends */
const char *ggml_backend_name(ggml_backend_t backend);
void ggml_backend_free(ggml_backend_t backend);
ggml_backend_buffer_type_t ggml_backend_get_default_buffer_type(ggml_backend_t backend);
ggml_backend_buffer_t ggml_backend_alloc_buffer(ggml_backend_t backend, size_t size);
void ggml_backend_synchronize(ggml_backend_t backend);
enum ggml_status ggml_backend_graph_compute(ggml_backend_t backend, struct ggml_cgraph *cgraph);
bool ggml_backend_supports_op(ggml_backend_t backend, const struct ggml_tensor *op);
ggml_backend_dev_t ggml_backend_get_device(ggml_backend_t backend);
bool ggml_backend_dev_supports_op(ggml_backend_dev_t device, const struct ggml_tensor *op);

/* tensor data (tensor->buffer must be set) */
void ggml_backend_tensor_set(struct ggml_tensor *tensor, const void *data, size_t offset, size_t size);
void ggml_backend_tensor_get(const struct ggml_tensor *tensor, void *data, size_t offset, size_t size);
void ggml_backend_tensor_memset(struct ggml_tensor *tensor, uint8_t value, size_t offset, size_t size);

/* place every tensor of a no_alloc context in one new buffer */
ggml_backend_buffer_t ggml_backend_alloc_ctx_tensors_from_buft(struct ggml_context *ctx,
                                                               ggml_backend_buffer_type_t buft);
ggml_backend_buffer_t ggml_backend_alloc_ctx_tensors(struct ggml_context *ctx, ggml_backend_t backend);

#ifdef __cplusplus
}
#endif
