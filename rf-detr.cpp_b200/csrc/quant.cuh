// GGUF block quantizers on the GPU (see quant.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace rfb {

// Elements and bytes per block of the GGUF types the quantizers produce:
// 1 F16, 8 Q8_0, 12 Q4_K, 13 Q5_K, 14 Q6_K.  False for other types.
bool quant_block_shape(uint32_t type, int* elems, int* bytes);

// Quantize n f32 values (device memory, n a multiple of the block size) into
// n / elems blocks of `type` at d_out.
cudaError_t quantize_device(uint32_t type, const float* d_src, int64_t n, uint8_t* d_out, cudaStream_t st);

}  // namespace rfb
