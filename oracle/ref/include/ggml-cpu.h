/* Test infrastructure: CPU-backend declarations used by the reference's
 * sources (see ggml.h in this folder).  Failing stubs. */
#pragma once
#include "ggml-backend.h"

#ifdef __cplusplus
extern "C" {
#endif

ggml_backend_t ggml_backend_cpu_init(void);
void ggml_backend_cpu_set_n_threads(ggml_backend_t backend, int n_threads);
enum ggml_status ggml_graph_compute_with_ctx(struct ggml_context *ctx, struct ggml_cgraph *cgraph, int n_threads);

#ifdef __cplusplus
}
#endif
