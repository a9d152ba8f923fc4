/* ggml-alloc.h -- the graph and tensor allocators sam3.cpp uses
 * (ggml_gallocr_new(ggml_backend_get_default_buffer_type(backend)) at
 * sam3.cpp:6101, ggml_tallocr for the memory bank), with ggml's names. */
#pragma once

#include "ggml-backend.h"

#ifdef __cplusplus
extern "C" {
#endif

struct ggml_tallocr {
    ggml_backend_buffer_t buffer;
    void *base;
    size_t alignment;
    size_t offset;
};

struct ggml_tallocr ggml_tallocr_new(ggml_backend_buffer_t buffer);
enum ggml_status ggml_tallocr_alloc(struct ggml_tallocr *talloc, struct ggml_tensor *tensor);

typedef struct ggml_gallocr *ggml_gallocr_t;

ggml_gallocr_t ggml_gallocr_new(ggml_backend_buffer_type_t buft);
void ggml_gallocr_free(ggml_gallocr_t galloc);
/* sizes a buffer for the graph's tensors that have no data; false on failure */
bool ggml_gallocr_reserve(ggml_gallocr_t galloc, struct ggml_cgraph *graph);
/* gives every node and leaf of the graph without data a place in that buffer (reserving first if
 * needed) and points every view at its source's data */
bool ggml_gallocr_alloc_graph(ggml_gallocr_t galloc, struct ggml_cgraph *graph);
size_t ggml_gallocr_get_buffer_size(ggml_gallocr_t galloc, int buffer_id);

#ifdef __cplusplus
}
#endif
