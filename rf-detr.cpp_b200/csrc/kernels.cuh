// Launchers of the non-GEMM kernels of the RF-DETR forward.  All take an
// explicit stream and return the launch status.  Layouts are token-major
// (rows of channels) unless stated otherwise.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "resize_legacy.hpp"

namespace rfb {

// Fused attention: O = softmax(scale * Q K^T) V per (group, head).  Q/K/V rows
// of group g start at row g*seq_len; head h uses columns [h*hd, (h+1)*hd).
cudaError_t attention(const __half* q, const __half* k, const __half* v, int ldq, int ldk, int ldv, __half* o,
                      int ldo, int seq_len, int groups, int heads, int head_dim, float scale, cudaStream_t st);

// Same computation on the tcgen05 tensor cores (head_dim 64 only): S and O in
// TMEM, P staged in shared memory.  `err` (may be null) receives the device
// error word on a bounded-wait timeout.
cudaError_t attention_tc(const __half* q, const __half* k, const __half* v, int ldq, int ldk, int ldv, __half* o,
                         int ldo, int seq_len, int groups, int heads, float scale, int* err, cudaStream_t st);

// Patch im2col in windowed order: planar [B][3][S][S] -> A [B*NW*Tp][Kpad] f16,
// K ordered (channel, ky, kx), zero padded to Kpad.
cudaError_t patch_im2col(const float* img, int B, int S, int p, int nw, int Kpad, __half* A, cudaStream_t st);

// The legacy preprocess resize (rfdetr.preprocess.resize_mode = legacy_stb):
// uint8 HWC [B][h][w][3] -> uint8 HWC [B][oh][ow][3] with the taps `t` of that
// size pair (resize_legacy.hpp).
cudaError_t resize_legacy_rgb(const uint8_t* src, int B, int w, int h, const LegacyTapsDev& t, int ow, int oh,
                              uint8_t* dst, cudaStream_t st);

// Preprocess fused with the patch im2col: uint8 HWC [B][h][w][3] -> A as above.
cudaError_t patch_from_rgb(const uint8_t* rgb, int B, int w, int h, int S, int p, int nw, int Kpad,
                           const float* mean3, const float* std3, __half* A, cudaStream_t st);

// The output x of a tapped backbone block (window order, B * nw^2 * T rows of D f32) normalised
// twice with the same row statistics (eps 1e-6): y16 = LayerNorm(x; g1, b1) row for row (the next
// block's norm1) and the backbone tap of backbone_tap (g2, b2, CLS rows dropped, grid order, column
// col0 of f16 rows of pitch ld) from one read of x.
cudaError_t layernorm_and_tap(const float* x, int B, int G, int nw, int D, const float* g1, const float* b1,
                              __half* y16, const float* g2, const float* b2, __half* taps, int ld, int col0,
                              cudaStream_t st);

// x[b][w*T] = clsrow (one CLS token per window).
cudaError_t write_cls_rows(float* x, const float* clsrow, int B, int NW, int T, int D, cudaStream_t st);

// LN(x) * g + b over rows of D (f32 in); writes y32 and/or y16 (either may
// be null; y32 may alias x).
// Split-K epilogue of a LayerNorm GEMM: x = sum over s < S of part[s] (in order) + bias, times
// colscale, plus resid; y = act(LayerNorm(x) * g + b); out32 = y, out16 = y.  Rows of
// D = 128 / 256 / 384 (act: ACT_NONE or ACT_SILU).  out32 may alias resid.
cudaError_t splitk_layernorm(const float* part, int S, long long sstride, int rows, int D, const float* bias,
                             const float* colscale, const float* resid, int ldr, const float* g, const float* b,
                             float eps, int act, float* out32, int ld32, __half* out16, int ld16,
                             cudaStream_t st);

cudaError_t layernorm(const float* x, int rows, int D, const float* g, const float* b, float eps, float* y32,
                      __half* y16, cudaStream_t st);

// Multi-scale tap: LN(x) with the backbone final norm, CLS stripped, windows
// undone; written as f16 into taps[B*G*G][ld] at column offset col0.
cudaError_t backbone_tap(const float* x, int B, int G, int nw, int D, const float* g, const float* b, __half* taps,
                         int ld, int col0, cudaStream_t st);

// 3x3 same-padding im2col, channels-last: src rows [B*H*W] with `C` channels at
// src + c (row pitch lds) -> A [B*H*W][9*C], K ordered (ky, kx, c).  Moves 8
// channels per 16-byte access: src and A 16-byte aligned, C and lds multiples
// of 8 and lds >= C, else cudaErrorInvalidValue before any launch.
cudaError_t im2col3x3(const __half* src, int lds, int B, int H, int W, int C, __half* A, cudaStream_t st);
// The source-side part of that check (what a caller can test before it has A).
bool im2col3x3_source_ok(const __half* src, int lds, int B, int H, int W, int C);

// Copy f32 rows to f16, zeroing rows whose proposal is masked (G >= 50 only).
cudaError_t mask_memory(const float* mem, int B, int G, int C, __half* out, cudaStream_t st);

// Two-stage box reparam: delta [B*N][4] + proposal grid -> bbox [B*N][4].
cudaError_t two_stage_boxes(const float* delta, int B, int G, float* bbox, cudaStream_t st);

// Per-image top-K over the per-token max class logit (descending score, ties
// by lower token index): cls [B*N][NC] -> idx [B][K].
cudaError_t topk_tokens(const float* cls, int B, int N, int NC, int K, int32_t* idx, cudaStream_t st);

// Decoder inputs: refpoints [B*NQ][4], sine embedding f16 [B*NQ][2*Dm],
// tgt f32 [B*NQ][Dm] (+ f16 copy) from the learned queries.
cudaError_t query_init(const float* bbox_all, const int32_t* idx, const float* lrn_rp, const float* feat, int B,
                       int N, int NQ, int Dm, float* refp, __half* sine, float* tgt, __half* tgt16, cudaStream_t st);

// out16 = a + b (f32 rows) ; used for tgt + query_pos.
cudaError_t add_to_f16(const float* a, const float* b, size_t n, __half* out, cudaStream_t st);

// f32 -> f16 copy.
cudaError_t to_f16(const float* a, size_t n, __half* out, cudaStream_t st);

// Deformable sampling (one level): value f16 [B*N][Dm] (heads x 16), so_aw f32
// [B*NQ][ld_soaw] with sampling offsets in columns [0, H*P*2) and attention
// logits in [H*P*2, H*P*3), refpoints [B*NQ][4] -> out f16 [B*NQ][Dm].
cudaError_t deform_sample(const __half* value, const float* so_aw, int ld_soaw, const float* refp, int B, int NQ,
                          int G, int heads, int points, int Dm, __half* out, cudaStream_t st);


// Final boxes: delta [B*NQ][4] with refpoints -> cxcywh [B*NQ][4].
cudaError_t box_reparam(const float* delta, const float* refp, int n, float* out, cudaStream_t st);

// Bilinear resize (align_corners = false) of channels-last maps
// [B][G][G][C] -> [B][T][T][C], f32.
cudaError_t resize_bilinear(const float* src, int B, int G, int T, int C, float* dst, cudaStream_t st);

// Depthwise 3x3 (zero pad) + bias, then channel LayerNorm -> f16 rows.
cudaError_t dwconv_ln(const float* x, int B, int H, int W, int C, const float* w9, const float* bias,
                      const float* g, const float* b, float eps, __half* out, cudaStream_t st);

}  // namespace rfb
