// Re-quantization of a loaded GGUF model's weight tensors (the reference's
// `rfdetr-cli quantize`, examples/cli/main.cpp:344-641).
#pragma once

#include <cstdint>
#include <string>

#include "gguf.hpp"

namespace rfb {

// Tensor rule of the reference converter / quantizer
// (scripts/convert_rfdetr_to_gguf.py:463-498, examples/cli/main.cpp:344-363):
// 2-D `.weight` tensors with both dims >= 64 whose rows are a multiple of 32
// are quantized; embeddings, biases, norms, conv kernels stay as stored.
bool should_quantize(const GgufTensor& t);

// The type a quantizable tensor gets when `type` is requested: K-quants need
// rows that are a multiple of 256 and fall back to Q8_0 otherwise
// (examples/cli/main.cpp:466-515).
uint32_t quant_type_for(uint32_t type, const GgufTensor& t);

// Re-quantize, on GPU `device`, every quantizable tensor of `f` stored as
// F32 / F16 / BF16 to quant_type_for(type, t) (1 F16, 8 Q8_0, 12 Q4_K,
// 13 Q5_K, 14 Q6_K), rewriting f's tensor table and data section.  Tensors
// already in a quantized format keep their bytes.  Returns 0 or a negative
// rfdetr_status (-1 bad type, -4 out of memory, -6 unreadable tensor, -8
// device error).
int requantize_model(GgufFile* f, uint32_t type, int device, std::string* err);

}  // namespace rfb
