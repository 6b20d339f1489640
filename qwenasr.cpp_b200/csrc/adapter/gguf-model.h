// Drop-in mirror of the reference's src/gguf-model.h surface (qwenasr.cpp),
// backed by this library's own bounds-checked GGUF reader (no GGML).  Same
// type and function names, so the reference's tools compile against it.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>
#include <vector>

// GGML tensor type codes as stored in GGUF files (gguf-model.h:14 uses the type).
enum ggml_type : int { GGML_TYPE_F32 = 0, GGML_TYPE_F16 = 1, GGML_TYPE_BF16 = 30, GGML_TYPE_COUNT = 64 };

namespace qkv {
class GgufFile;
}

struct QwenAsrGgufTensorView {   // gguf-model.h:12-19
    std::string name;
    ggml_type type = GGML_TYPE_COUNT;
    std::vector<int64_t> ne;
    size_t nbytes = 0;
    size_t offset = 0;
    const void *data = nullptr;
};

struct QwenAsrGgufModel {        // gguf-model.h:21-33 (GGML context pointers replaced by the reader)
    std::string path;
    qkv::GgufFile *file = nullptr;
    const uint8_t *mapping = nullptr;
    size_t file_size = 0;
    size_t data_offset = 0;
};

bool qwenasr_gguf_model_open(const char *path, QwenAsrGgufModel *model, std::string *error);
void qwenasr_gguf_model_close(QwenAsrGgufModel *model);
int64_t qwenasr_gguf_model_tensor_count(const QwenAsrGgufModel &model);
bool qwenasr_gguf_model_tensor_by_index(const QwenAsrGgufModel &model, int64_t index, QwenAsrGgufTensorView *out,
                                        std::string *error);
bool qwenasr_gguf_model_tensor_by_name(const QwenAsrGgufModel &model, const char *name, QwenAsrGgufTensorView *out,
                                       std::string *error);
