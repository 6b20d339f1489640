/*
 * Test infrastructure: declaration shim that lets the reference's scalar
 * text-decoder path (src/text-decoder.cpp, src/gguf-model.cpp,
 * src/ggml-backends.cpp of qwenasr.cpp) compile without GGML, which is an
 * empty git submodule in the reference tree.  Only the names those files use
 * are declared; graph and backend functions are stubs that return null /
 * failure (oracle/ref/ggml_shim.cpp), so only the scalar CPU functions work.
 * Written for this repository; not GGML source.
 */
#pragma once
#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GGML_MAX_DIMS 4
#define GGML_UNUSED(x) (void)(x)
#define GGML_ROPE_TYPE_NEOX 2

enum ggml_type { GGML_TYPE_F32 = 0, GGML_TYPE_F16 = 1, GGML_TYPE_I32 = 26, GGML_TYPE_BF16 = 30, GGML_TYPE_COUNT = 64 };
enum ggml_status { GGML_STATUS_ALLOC_FAILED = -2, GGML_STATUS_FAILED = -1, GGML_STATUS_SUCCESS = 0, GGML_STATUS_ABORTED = 1 };
enum ggml_prec { GGML_PREC_DEFAULT = 0, GGML_PREC_F32 = 10 };

struct ggml_context;
struct ggml_cgraph;

struct ggml_tensor {
    enum ggml_type type;
    int64_t ne[GGML_MAX_DIMS];
    size_t nb[GGML_MAX_DIMS];
    void *data;
    char name[64];
};

struct ggml_init_params {
    size_t mem_size;
    void *mem_buffer;
    bool no_alloc;
};

struct ggml_context *ggml_init(struct ggml_init_params params);
void ggml_free(struct ggml_context *ctx);
size_t ggml_tensor_overhead(void);
size_t ggml_graph_overhead_custom(size_t size, bool grads);
size_t ggml_nbytes(const struct ggml_tensor *t);
int ggml_n_dims(const struct ggml_tensor *t);
struct ggml_tensor *ggml_get_tensor(struct ggml_context *ctx, const char *name);
float *ggml_get_data_f32(const struct ggml_tensor *t);
struct ggml_tensor *ggml_new_tensor(struct ggml_context *ctx, enum ggml_type type, int n_dims, const int64_t *ne);
struct ggml_tensor *ggml_new_tensor_1d(struct ggml_context *ctx, enum ggml_type type, int64_t ne0);
struct ggml_tensor *ggml_new_tensor_2d(struct ggml_context *ctx, enum ggml_type type, int64_t ne0, int64_t ne1);
struct ggml_tensor *ggml_new_tensor_3d(struct ggml_context *ctx, enum ggml_type type, int64_t ne0, int64_t ne1, int64_t ne2);
struct ggml_tensor *ggml_set_name(struct ggml_tensor *t, const char *name);
void ggml_set_input(struct ggml_tensor *t);
void ggml_set_output(struct ggml_tensor *t);

struct ggml_tensor *ggml_mul_mat(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b);
void ggml_mul_mat_set_prec(struct ggml_tensor *a, enum ggml_prec prec);
struct ggml_tensor *ggml_mul(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b);
struct ggml_tensor *ggml_add(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b);
struct ggml_tensor *ggml_rms_norm(struct ggml_context *ctx, struct ggml_tensor *a, float eps);
struct ggml_tensor *ggml_silu(struct ggml_context *ctx, struct ggml_tensor *a);
struct ggml_tensor *ggml_cont(struct ggml_context *ctx, struct ggml_tensor *a);
struct ggml_tensor *ggml_cpy(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b);
struct ggml_tensor *ggml_transpose(struct ggml_context *ctx, struct ggml_tensor *a);
struct ggml_tensor *ggml_permute(struct ggml_context *ctx, struct ggml_tensor *a, int axis0, int axis1, int axis2, int axis3);
struct ggml_tensor *ggml_reshape_2d(struct ggml_context *ctx, struct ggml_tensor *a, int64_t ne0, int64_t ne1);
struct ggml_tensor *ggml_reshape_3d(struct ggml_context *ctx, struct ggml_tensor *a, int64_t ne0, int64_t ne1, int64_t ne2);
struct ggml_tensor *ggml_view_2d(struct ggml_context *ctx, struct ggml_tensor *a, int64_t ne0, int64_t ne1, size_t nb1, size_t offset);
struct ggml_tensor *ggml_view_3d(struct ggml_context *ctx, struct ggml_tensor *a, int64_t ne0, int64_t ne1, int64_t ne2,
                                 size_t nb1, size_t nb2, size_t offset);
struct ggml_tensor *ggml_diag_mask_inf(struct ggml_context *ctx, struct ggml_tensor *a, int n_past);
struct ggml_tensor *ggml_soft_max_ext(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *mask, float scale,
                                      float max_bias);
struct ggml_tensor *ggml_rope_ext(struct ggml_context *ctx, struct ggml_tensor *a, struct ggml_tensor *b, struct ggml_tensor *c,
                                  int n_dims, int mode, int n_ctx_orig, float freq_base, float freq_scale, float ext_factor,
                                  float attn_factor, float beta_fast, float beta_slow);
struct ggml_cgraph *ggml_new_graph(struct ggml_context *ctx);
struct ggml_cgraph *ggml_new_graph_custom(struct ggml_context *ctx, size_t size, bool grads);
void ggml_build_forward_expand(struct ggml_cgraph *graph, struct ggml_tensor *t);

#ifdef __cplusplus
}
#endif
