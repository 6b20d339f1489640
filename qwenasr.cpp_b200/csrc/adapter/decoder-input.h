// Mirror of the decoder-input type the path consumes (reference
// src/decoder-input.h:11-17): prompt rows with audio rows already spliced in.
#pragma once

#include <cstdint>
#include <vector>

struct QwenAsrDecoderInputOutput {
    int tokens = 0;
    int hidden = 0;
    int audio_tokens = 0;
    std::vector<int32_t> input_ids;
    std::vector<float> values;   // [token, hidden]
};
