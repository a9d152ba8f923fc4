/* ggml-b200.h -- the B200 (sm_100a) ggml backend.  sam3.cpp selects it where
 * it selects Metal today (sam3.cpp:3279-3284):
 *
 *   #ifdef GGML_USE_B200
 *       if (params.use_gpu) model->backend = ggml_backend_b200_init(0);
 *   #endif
 *
 * Weights go into buffers of ggml_backend_b200_buffer_type(device) through
 * ggml_backend_alloc_ctx_tensors / ggml_backend_tensor_set as they do for any
 * backend; graphs run through ggml_backend_graph_compute. */
#pragma once

#include "ggml-backend.h"

#ifdef __cplusplus
extern "C" {
#endif

ggml_backend_t ggml_backend_b200_init(int device);
bool ggml_backend_is_b200(ggml_backend_t backend);
ggml_backend_buffer_type_t ggml_backend_b200_buffer_type(int device);
int ggml_backend_b200_get_device_count(void);
/* the sam3b200_backend (include/sam3_b200.h) behind a B200 ggml backend, for the encoder-level entries */
void *ggml_backend_b200_get_handle(ggml_backend_t backend);

#ifdef __cplusplus
}
#endif
