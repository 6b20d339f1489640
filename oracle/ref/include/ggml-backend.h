/* Test infrastructure: backend declarations used by the reference's sources
 * (see ggml.h in this folder).  Every function is a failing stub. */
#pragma once
#include "ggml.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct ggml_backend *ggml_backend_t;
typedef struct ggml_backend_buffer *ggml_backend_buffer_t;
typedef struct ggml_backend_buffer_type *ggml_backend_buffer_type_t;
typedef struct ggml_backend_sched *ggml_backend_sched_t;
typedef struct ggml_backend_device *ggml_backend_dev_t;

enum ggml_backend_dev_type { GGML_BACKEND_DEVICE_TYPE_CPU, GGML_BACKEND_DEVICE_TYPE_GPU, GGML_BACKEND_DEVICE_TYPE_IGPU,
                             GGML_BACKEND_DEVICE_TYPE_ACCEL };
enum ggml_backend_buffer_usage { GGML_BACKEND_BUFFER_USAGE_ANY, GGML_BACKEND_BUFFER_USAGE_WEIGHTS,
                                 GGML_BACKEND_BUFFER_USAGE_COMPUTE };

void ggml_backend_tensor_set(struct ggml_tensor *t, const void *data, size_t offset, size_t size);
void ggml_backend_tensor_get(const struct ggml_tensor *t, void *data, size_t offset, size_t size);
ggml_backend_sched_t ggml_backend_sched_new(ggml_backend_t *backends, ggml_backend_buffer_type_t *bufts, int n_backends,
                                            size_t graph_size, bool parallel, bool op_offload);
void ggml_backend_sched_free(ggml_backend_sched_t sched);
void ggml_backend_sched_reset(ggml_backend_sched_t sched);
bool ggml_backend_sched_alloc_graph(ggml_backend_sched_t sched, struct ggml_cgraph *graph);
enum ggml_status ggml_backend_sched_graph_compute(ggml_backend_sched_t sched, struct ggml_cgraph *graph);
ggml_backend_buffer_t ggml_backend_alloc_ctx_tensors(struct ggml_context *ctx, ggml_backend_t backend);
void ggml_backend_buffer_free(ggml_backend_buffer_t buffer);
void ggml_backend_buffer_set_usage(ggml_backend_buffer_t buffer, enum ggml_backend_buffer_usage usage);
void ggml_backend_buffer_clear(ggml_backend_buffer_t buffer, uint8_t value);
void ggml_backend_free(ggml_backend_t backend);
ggml_backend_t ggml_backend_init_by_type(enum ggml_backend_dev_type type, const char *params);
const char *ggml_backend_name(ggml_backend_t backend);
ggml_backend_dev_t ggml_backend_get_device(ggml_backend_t backend);
enum ggml_backend_dev_type ggml_backend_dev_type(ggml_backend_dev_t device);

#ifdef __cplusplus
}
#endif
