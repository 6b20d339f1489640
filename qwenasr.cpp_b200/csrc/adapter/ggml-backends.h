// Mirror of the device selector of the reference (src/ggml-backends.h:13-34).
// This library runs on a B200 only: Cpu is rejected (no CPU fallback), Auto
// and Gpu select CUDA device QWENASR_B200_DEVICE (default 0).
#pragma once

#include <string>

enum class QwenAsrGgmlDevice { Auto, Cpu, Gpu };

QwenAsrGgmlDevice qwenasr_ggml_device_auto();
QwenAsrGgmlDevice qwenasr_ggml_device_cpu();
QwenAsrGgmlDevice qwenasr_ggml_device_gpu();
bool qwenasr_ggml_device_from_string(const std::string &value, QwenAsrGgmlDevice *out, std::string *error);
const char *qwenasr_ggml_device_name(QwenAsrGgmlDevice device);
