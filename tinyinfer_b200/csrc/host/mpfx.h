// MPFX0001 model files: the reference's weight format
// (miniprefix/src/model/model.cpp:20-56, written by miniprefix/tools/
// prepare_model.py:34-50), little-endian:
//   "MPFX0001" | int32 layers, hidden, intermediate, heads, kv_heads, vocabulary,
//   context, eos | float32 rms_epsilon, rope_theta | uint32 tied | uint32 count |
//   count x (uint32 name length, name, uint32 rank, int32 dims[rank], uint64 bytes,
//            float32 data[bytes / 4])
// Tensors are the Llama names with 2-D linears stored [in][out]. The reader
// applies the reference loader's checks in its order and with its messages, but
// streams: each tensor goes to the caller's sink as soon as it is read and
// checked, so a model is never held twice in host memory.
#pragma once
#include <cstddef>
#include <functional>
#include <string>

#include "types.h"

namespace miniprefix_b200 {

struct MpfxTensor {
    const std::string& name;
    const float* data;
    std::size_t elements;
};

// Reads and validates only the header (through the tied flag) and the config.
ModelConfig read_mpfx_config(const std::string& path);

// Reads and validates the whole file, calling `sink` once per tensor in file
// order. Throws std::runtime_error / std::invalid_argument with the reference
// loader's messages; tensors already passed to the sink stay passed.
ModelConfig read_mpfx(const std::string& path, const std::function<void(const MpfxTensor&)>& sink);

}  // namespace miniprefix_b200
