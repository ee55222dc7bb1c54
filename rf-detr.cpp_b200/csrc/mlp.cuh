// Fused transformer MLP on the tcgen05 tensor cores:
//   x += ls * (GELU(h . W1^T + b1) . W2^T + b2)
// with the hidden activations (rows x F) kept on chip.  See mlp.cu.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace rfb {

struct MlpArgs {
    const __half* h = nullptr;   // [M][D] f16 input rows (LayerNorm output), pitch ldh
    int ldh = 0;
    const __half* w1 = nullptr;  // [F][D] f16 (pitch ldw1)
    int ldw1 = 0;
    const float* b1 = nullptr;   // [F]
    const __half* w2 = nullptr;  // [D][F] f16 (pitch ldw2)
    int ldw2 = 0;
    const float* b2 = nullptr;   // [D]
    const float* ls = nullptr;   // [D] layer scale (nullptr = 1)
    float* x = nullptr;          // [M][D] f32 residual stream, updated in place (pitch ldx)
    int ldx = 0;
    int M = 0, D = 0, F = 0;
    int* err = nullptr;          // device error word
};

// Shapes the kernel implements: D a multiple of 128 up to 384, F a multiple of 128.
bool mlp_supported(int D, int F);

cudaError_t mlp_fused(const MlpArgs& a, cudaStream_t stream);

}  // namespace rfb
