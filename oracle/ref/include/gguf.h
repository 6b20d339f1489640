/* Test infrastructure: GGUF declarations used by the reference's gguf-model.cpp
 * and tokenizer.cpp
 * (see ggml.h in this folder).  Implemented by oracle/ref/ggml_shim.cpp. */
#pragma once
#include "ggml.h"

#ifdef __cplusplus
extern "C" {
#endif

struct gguf_context;
struct gguf_init_params {
    bool no_alloc;
    struct ggml_context **ctx;
};

struct gguf_context *gguf_init_from_file(const char *fname, struct gguf_init_params params);
void gguf_free(struct gguf_context *ctx);
int64_t gguf_get_n_tensors(const struct gguf_context *ctx);
const char *gguf_get_tensor_name(const struct gguf_context *ctx, int64_t id);
size_t gguf_get_tensor_offset(const struct gguf_context *ctx, int64_t id);
size_t gguf_get_data_offset(const struct gguf_context *ctx);
int64_t gguf_find_tensor(const struct gguf_context *ctx, const char *name);
/* metadata readers used by the reference's tokenizer.cpp */
int64_t gguf_find_key(const struct gguf_context *ctx, const char *key);
uint32_t gguf_get_val_u32(const struct gguf_context *ctx, int64_t key_id);
size_t gguf_get_arr_n(const struct gguf_context *ctx, int64_t key_id);
const char *gguf_get_arr_str(const struct gguf_context *ctx, int64_t key_id, size_t i);

#ifdef __cplusplus
}
#endif
