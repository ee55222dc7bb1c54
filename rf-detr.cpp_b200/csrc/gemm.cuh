// tcgen05 GEMM with fused epilogues: C = epilogue(A[M,K] . B[N,K]^T).
// A (activations) and B (weights) are f16, K-contiguous; accumulation is f32
// in TMEM.  See gemm.cu for the kernel design.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace rfb {

enum GemmEpi : int {
    EPI_F16 = 0,    // out16 = act(acc + bias)
    EPI_F32 = 1,    // out32 = act(acc + bias)
    EPI_RESID = 2,  // out32 += colscale * act(acc + bias)        (layer-scale + residual)
    EPI_PATCH = 3,  // patch embed: windowed row remap, + bias + windowed pos-embed -> out32
    EPI_LN = 4,     // full-row LayerNorm(colscale * (acc + bias) [+ resid]) * g + b, act -> out32 / out16
                    // (BN == N = 128, 256 or 384)
};

enum GemmAct : int { ACT_NONE = 0, ACT_GELU = 1, ACT_RELU = 2, ACT_SILU = 3 };

struct GemmArgs {
    // operands (row-major, K contiguous); lda/ldb in elements
    const __half* A = nullptr;
    int lda = 0;
    const __half* B = nullptr;
    int ldb = 0;
    int M = 0, N = 0, K = 0;
    // batching: batch b uses A rows [b*a_batch_rows, ...), B rows [b*b_batch_rows, ...)
    int batches = 1;
    int a_batch_rows = 0, b_batch_rows = 0;
    long long out_batch_stride = 0;  // elements
    // kb_per > 0 (split-K): batch b covers k-blocks [b*kb_per, (b+1)*kb_per) of the same A and B rows
    // (a_batch_rows = b_batch_rows = 0) and writes its partial sums to its own output slice
    int kb_per = 0;
    // EPI_LN with few row blocks: scratch for split-K partial sums (f32); when given and large enough
    // the GEMM runs as split-K f32 partials plus an in-order reduction that applies the epilogue
    float* split_ws = nullptr;
    size_t split_ws_bytes = 0;
    // epilogue
    int epi = EPI_F16;
    int act = ACT_NONE;
    const float* bias = nullptr;
    const float* colscale = nullptr;
    const float* ln_g = nullptr;
    const float* ln_b = nullptr;
    float ln_eps = 1e-5f;
    const float* resid = nullptr;
    int ldr = 0;
    float* out32 = nullptr;
    int ld32 = 0;
    __half* out16 = nullptr;
    int ld16 = 0;
    // EPI_PATCH: rows are (image, window, patch-in-window) without CLS rows
    int patch_tp = 0;      // patches per window
    int patch_t = 0;       // tokens per window (patches + CLS)
    int patch_rows = 0;    // patch rows per image
    int patch_ntok = 0;    // tokens per image
    const float* posw = nullptr;  // [ntok][N] windowed pos-embed
    // Implicit-GEMM 3x3 convolution (stride 1, zero padding 1): when conv_src is
    // set, A is not read from memory as a matrix; row (b, y, x), column
    // (tap, c) of A is conv_src[b][y + tap/3 - 1][x + tap%3 - 1][c] (zero
    // outside the map), loaded by 4-D TMA boxes straight from the channels-last
    // map [b][conv_h][conv_w] with pixel pitch conv_lds.  M = b * conv_h *
    // conv_w, K = 9 * conv_c (conv_c a multiple of 64), B = weights [N][3][3][c].
    const __half* conv_src = nullptr;
    int conv_lds = 0, conv_h = 0, conv_w = 0, conv_c = 0;
    int conv_r = 0;        // set by the launcher: image rows per 128-row tile
    int* err = nullptr;    // device error word
    int tma_out = 0;       // set by the launcher: outputs written through TMA stores
    int patch_vec = 0;     // set by the launcher: EPI_PATCH rows written as 16-byte chunks
};

// Launch on `stream`.  Picks the tile width from N (and requires BN == N for
// EPI_LN).  Returns cudaSuccess or a launch / argument error.
cudaError_t gemm(const GemmArgs& a, cudaStream_t stream);

// Number of SMs used for the persistent grid (set once per device).
void gemm_set_num_sms(int n);

}  // namespace rfb
