// Operator entry points of rfdetr_b200.h: thin C wrappers over the kernels.
#include "rfdetr_b200.h"

#include "common.hpp"

#include "gemm.cuh"
#include "kernels.cuh"
#include "quant.cuh"
#include "select.cuh"

extern "C" int rfdetr_b200_op_gemm(const void* A, int lda, const void* B, int ldb, int M, int N, int K, int epi,
                                   int act, const float* bias, const float* colscale, const float* ln_g,
                                   const float* ln_b, float ln_eps, const float* resid, int ldr, float* out32,
                                   int ld32, void* out16, int ld16, void* stream) {
    if (epi != rfb::EPI_F16 && epi != rfb::EPI_F32 && epi != rfb::EPI_RESID && epi != rfb::EPI_LN)
        return (int)cudaErrorInvalidValue;
    if ((epi == rfb::EPI_F16 && !out16) || ((epi == rfb::EPI_F32 || epi == rfb::EPI_RESID) && !out32))
        return (int)cudaErrorInvalidValue;
    rfb::GemmArgs a;
    a.A = static_cast<const __half*>(A);
    a.lda = lda;
    a.B = static_cast<const __half*>(B);
    a.ldb = ldb;
    a.M = M; a.N = N; a.K = K;
    a.epi = epi; a.act = act;
    a.bias = bias; a.colscale = colscale;
    a.ln_g = ln_g; a.ln_b = ln_b; a.ln_eps = ln_eps;
    a.resid = resid; a.ldr = ldr;
    a.out32 = out32; a.ld32 = ld32;
    a.out16 = static_cast<__half*>(out16); a.ld16 = ld16;
    return (int)rfb::gemm(a, static_cast<cudaStream_t>(stream));
}

extern "C" int rfdetr_b200_op_attention(const void* q, const void* k, const void* v, int ldq, int ldk, int ldv,
                                        void* o, int ldo, int seq_len, int groups, int heads, int head_dim,
                                        float scale, void* stream) {
    if (head_dim == 64)
        return (int)rfb::attention_tc(static_cast<const __half*>(q), static_cast<const __half*>(k),
                                      static_cast<const __half*>(v), ldq, ldk, ldv, static_cast<__half*>(o), ldo,
                                      seq_len, groups, heads, scale, nullptr, static_cast<cudaStream_t>(stream));
    return (int)rfb::attention(static_cast<const __half*>(q), static_cast<const __half*>(k),
                               static_cast<const __half*>(v), ldq, ldk, ldv, static_cast<__half*>(o), ldo, seq_len,
                               groups, heads, head_dim, scale, static_cast<cudaStream_t>(stream));
}

extern "C" int rfdetr_b200_op_quantize(int type, const float* d_src, long long n, void* d_out, void* stream) {
    if (!d_src || !d_out || n < 0) return (int)cudaErrorInvalidValue;
    return (int)rfb::quantize_device((uint32_t)type, d_src, (int64_t)n, static_cast<uint8_t*>(d_out),
                                     static_cast<cudaStream_t>(stream));
}

extern "C" int rfdetr_b200_op_select(const float* d_logits, const float* d_boxes, int batch, int nq, int nc,
                                     float threshold, int top_k, const uint32_t* d_class_filter, int filter_len,
                                     int img_w, int img_h, rfdetr_b200_det* d_out, int* d_counts, void* stream) {
    return (int)rfb::select_detections_device(d_logits, d_boxes, batch, nq, nc, threshold, top_k, d_class_filter,
                                              filter_len, img_w, img_h, d_out, d_counts,
                                              static_cast<cudaStream_t>(stream));
}

static int op_resize_legacy_body(const uint8_t* d_src, int batch, int w, int h, uint8_t* d_dst, int ow, int oh,
                                 void* stream) {
    if (!d_src || !d_dst || batch < 0 || w <= 0 || h <= 0 || ow <= 0 || oh <= 0) return (int)cudaErrorInvalidValue;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    // the taps are allocated and freed by the call, which therefore synchronizes the stream: a
    // stream being captured into a graph is refused before anything is enqueued
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    cudaError_t e = cudaStreamIsCapturing(st, &cap);
    if (e != cudaSuccess) return (int)e;
    if (cap != cudaStreamCaptureStatusNone) return (int)cudaErrorStreamCaptureUnsupported;
    rfb::LegacyTapsDev t;
    e = rfb::upload_legacy_taps(w, h, ow, oh, &t);
    if (e != cudaSuccess) return (int)e;
    e = rfb::resize_legacy_rgb(d_src, batch, w, h, t, ow, oh, d_dst, st);
    const cudaError_t es = cudaStreamSynchronize(st);  // the taps are freed below
    cudaFree(t.base);
    return (int)(e != cudaSuccess ? e : es);
}

extern "C" int rfdetr_b200_op_resize_legacy(const uint8_t* d_src, int batch, int w, int h, uint8_t* d_dst, int ow,
                                           int oh, void* stream) {
    // the taps are built in host vectors: an allocation failure is reported, not thrown
    return rfdetr_c_boundary([&] { return op_resize_legacy_body(d_src, batch, w, h, d_dst, ow, oh, stream); },
                             (int)cudaErrorMemoryAllocation, (int)cudaErrorUnknown);
}

extern "C" int rfdetr_b200_op_topk(const float* d_cls, int batch, int n, int nc, int k, int32_t* d_idx,
                                   void* stream) {
    return (int)rfb::topk_tokens(d_cls, batch, n, nc, k, d_idx, static_cast<cudaStream_t>(stream));
}

extern "C" size_t rfdetr_b200_mask_bits_words(int img_w, int img_h) {
    return (img_w > 0 && img_h > 0) ? rfb::mask_bits_words(img_w, img_h) : 0;
}

extern "C" int rfdetr_b200_op_mask_bits(const float* d_masks, int batch, int nq, int side,
                                        const rfdetr_b200_det* d_dets, const int* d_counts, int max_dets, int img_w,
                                        int img_h, uint32_t* d_bits, void* stream) {
    return (int)rfb::mask_bits_device(d_masks, batch, nq, side, d_dets, d_counts, max_dets, img_w, img_h, d_bits,
                                      static_cast<cudaStream_t>(stream));
}

extern "C" int rfdetr_b200_op_deform(const void* value, const float* so_aw, int ld_soaw, const float* refp, int batch,
                                     int nq, int grid, int heads, int points, int dm, void* out, void* stream) {
    return (int)rfb::deform_sample(static_cast<const __half*>(value), so_aw, ld_soaw, refp, batch, nq, grid, heads,
                                   points, dm, static_cast<__half*>(out), static_cast<cudaStream_t>(stream));
}

extern "C" size_t rfdetr_b200_op_conv3x3_workspace(int batch, int h, int w, int c) {
    if (batch <= 0 || h <= 0 || w <= 0 || c <= 0) return 0;
    return (size_t)batch * h * w * 9 * c * sizeof(__half);
}

extern "C" int rfdetr_b200_op_conv3x3(const void* src, int lds, int batch, int h, int w, int c, const void* weight,
                                      int oc, const float* ln_g, const float* ln_b, float eps, int act, float* out32,
                                      int ld32, void* out16, int ld16, void* workspace, size_t workspace_bytes,
                                      void* stream) {
    const size_t need = rfdetr_b200_op_conv3x3_workspace(batch, h, w, c);
    if (!src || !weight || !workspace || need == 0 || workspace_bytes < need) return (int)cudaErrorInvalidValue;
    if ((size_t)batch * h * w > (size_t)INT32_MAX) return (int)cudaErrorInvalidValue;
    if ((oc != 128 && oc != 256) || (act != rfb::ACT_NONE && act != rfb::ACT_SILU)) return (int)cudaErrorInvalidValue;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (c % 64 == 0 && w <= 128) {
        // implicit GEMM: the 3x3 taps are TMA-loaded straight from `src` (the workspace is not touched)
        rfb::GemmArgs a;
        a.conv_src = static_cast<const __half*>(src);
        a.conv_lds = lds; a.conv_h = h; a.conv_w = w; a.conv_c = c;
        a.B = static_cast<const __half*>(weight); a.ldb = 9 * c;
        a.M = batch * h * w; a.N = oc; a.K = 9 * c;
        a.epi = rfb::EPI_LN; a.act = act;
        a.ln_g = ln_g; a.ln_b = ln_b; a.ln_eps = eps;
        a.out32 = out32; a.ld32 = ld32;
        a.out16 = static_cast<__half*>(out16); a.ld16 = ld16;
        return (int)rfb::gemm(a, st);
    }
    __half* col = static_cast<__half*>(workspace);
    // im2col3x3 refuses a misaligned src / workspace or lds < c before launching
    cudaError_t e = rfb::im2col3x3(static_cast<const __half*>(src), lds, batch, h, w, c, col, st);
    if (e != cudaSuccess) return (int)e;
    rfb::GemmArgs a;
    a.A = col; a.lda = 9 * c;
    a.B = static_cast<const __half*>(weight); a.ldb = 9 * c;
    a.M = batch * h * w; a.N = oc; a.K = 9 * c;
    a.epi = rfb::EPI_LN; a.act = act;
    a.ln_g = ln_g; a.ln_b = ln_b; a.ln_eps = eps;
    a.out32 = out32; a.ld32 = ld32;
    a.out16 = static_cast<__half*>(out16); a.ld16 = ld16;
    return (int)rfb::gemm(a, st);
}
