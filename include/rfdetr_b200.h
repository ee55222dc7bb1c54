/* rfdetr_b200.h — additive entry points of the B200 engine.
 *
 * The reference API (rfdetr.h) is batch-1 and single-device: one image per
 * rfdetr_detect call, with the model forward at src/rfdetr_model.cpp:77
 * (rfdetr_model_forward: one preprocessed image -> ForwardOutput).  The
 * functions below are the batched / device-placed replacements of that seam;
 * they are additions, none of the reference symbols change.  Contexts created
 * here are ordinary rfdetr_context objects (rfdetr_detect, rfdetr_free and the
 * accessors all work on them).  A context owns one GPU and one CUDA stream and
 * is not re-entrant: use one context per host thread.
 */
#ifndef RFDETR_B200_H
#define RFDETR_B200_H

#include "rfdetr.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int device;       /* CUDA device ordinal (default 0) */
    int max_batch;    /* images the activation arena is sized for at init (grows on demand) */
    int weight_type;  /* 0: weights as stored; else re-quantize at load, on the GPU, every
                         quantizable weight stored as F32/F16/BF16 to this GGUF type (1 F16,
                         8 Q8_0, 12 Q4_K, 13 Q5_K, 14 Q6_K; K-quants fall back to Q8_0 for
                         rows that are not a multiple of 256), as rfdetr_b200_quantize_gguf */
} rfdetr_b200_params;

/* Replaces rfdetr_init (src/rfdetr.cpp:37-107) with an explicit device and
 * batch capacity.  `b200` may be NULL (device 0, batch 1). */
rfdetr_context* rfdetr_b200_init(const rfdetr_params* params, const rfdetr_b200_params* b200,
                                 rfdetr_status* out_status);

/* Batched rfdetr_model_forward (src/rfdetr_model.hpp:52-60) from host uint8
 * RGB images, `batch` images of width x height, HWC, contiguous.  Images are
 * resized / normalized on the GPU exactly like rfdetr_preprocess
 * (src/image_io.cpp:207-248).  Outputs (host, may be NULL):
 *   out_logits [batch][num_queries][num_classes]  (class fastest)
 *   out_boxes  [batch][num_queries][4]            normalized cx, cy, w, h
 *   out_masks  [batch][num_queries][m][m]         seg models, m = mask side */
rfdetr_status rfdetr_b200_forward_rgb(rfdetr_context* ctx, const uint8_t* rgb, int batch, int width, int height,
                                      float* out_logits, float* out_boxes, float* out_masks);

/* Pipelined form of rfdetr_b200_forward_rgb for a stream of batches: enqueues
 * the host-to-device copy of `rgb` (on a copy stream, into one of two device
 * input slots), the forward (behind that copy) and the device-to-host copies
 * of the outputs (from a device copy of them, on a third stream), and returns
 * without waiting, so the upload of the next batch and the download of the
 * previous one overlap the forward of this one.  `rgb` and the output buffers must stay
 * valid and untouched until rfdetr_b200_wait returns; page-locked host memory
 * is needed for the copies to overlap (pageable memory works, serialized).
 * Outputs as for rfdetr_b200_forward_rgb. */
rfdetr_status rfdetr_b200_submit_rgb(rfdetr_context* ctx, const uint8_t* rgb, int batch, int width, int height,
                                     float* out_logits, float* out_boxes, float* out_masks);

/* Waits for every rfdetr_b200_submit_rgb issued so far; reports device errors
 * of any of them. */
rfdetr_status rfdetr_b200_wait(rfdetr_context* ctx);

/* Waits only for the oldest rfdetr_b200_submit_rgb not yet waited for: when it
 * returns RFDETR_OK, that submission's outputs are in host memory and its
 * input and output buffers may be reused, while later submissions keep
 * running (a streaming loop: submit batch i+1, wait_oldest, read batch i).
 * Returns RFDETR_OK at once when nothing is outstanding.  Device errors are
 * reported by rfdetr_b200_wait. */
rfdetr_status rfdetr_b200_wait_oldest(rfdetr_context* ctx);

/* Same, from already-preprocessed planar input [batch][3][S][S] (S = image
 * size), i.e. exactly the `input` argument of rfdetr_model_forward. */
rfdetr_status rfdetr_b200_forward_planar(rfdetr_context* ctx, const float* planar, int batch,
                                         float* out_logits, float* out_boxes, float* out_masks);

/* Device-resident path: `d_rgb` is a DEVICE pointer (on the context's GPU) to
 * batch x height x width x 3 uint8.  Enqueues preprocess + forward on the
 * context stream and returns without waiting; outputs stay on the device
 * (rfdetr_b200_device_outputs).  rfdetr_b200_sync waits and reports device
 * errors. */
rfdetr_status rfdetr_b200_enqueue_device(rfdetr_context* ctx, const uint8_t* d_rgb, int batch, int width,
                                         int height);
rfdetr_status rfdetr_b200_sync(rfdetr_context* ctx);
/* Device pointers of the last forward's outputs (layouts as above). */
rfdetr_status rfdetr_b200_device_outputs(rfdetr_context* ctx, const float** d_logits, const float** d_boxes,
                                         const float** d_masks);

/* One selected detection as the device post-process writes it (32 bytes). */
typedef struct rfdetr_b200_det {
    int32_t query;     /* decoder query it came from */
    int32_t class_id;
    float   score;     /* sigmoid of the winning class logit */
    float   x1, y1, x2, y2;  /* pixel box in the original image, clamped to it */
    float   pad;
} rfdetr_b200_det;

/* Batched rfdetr_detect: n images (any sizes) -> per-image detection arrays.
 * out_dets[i] / out_counts[i] follow rfdetr_detect's ownership rules
 * (free each with rfdetr_detections_free).  On an error every out_dets[i] is
 * NULL and every out_counts[i] 0: nothing is left to free. */
rfdetr_status rfdetr_b200_detect_batch(rfdetr_context* ctx, const rfdetr_image* const* imgs, size_t n,
                                       const rfdetr_detect_params* params, rfdetr_detection** out_dets,
                                       size_t* out_counts);

int   rfdetr_b200_device(const rfdetr_context* ctx);
int   rfdetr_b200_mask_side(const rfdetr_context* ctx);         /* 0 for detection models */
int   rfdetr_b200_kernels_per_forward(const rfdetr_context* ctx);
void* rfdetr_b200_stream(const rfdetr_context* ctx);              /* the context's cudaStream_t */

/* Copy a named intermediate of the last forward to host as f32 (parity
 * tests; names follow the reference's trace checkpoints, src/trace.cpp).
 * Returns the element count, or -1 (unknown name / capacity too small). */
long long rfdetr_b200_trace(rfdetr_context* ctx, const char* name, int batch, float* out, size_t cap);

/* Per-launch timing of the forward pass.  rfdetr_b200_profile_enable(ctx, 1)
 * makes subsequent forwards record a CUDA event after every kernel launch;
 * after the forward has completed, rfdetr_b200_profile_read fills up to `cap`
 * entries (launch name, NUL-terminated, at names + i*name_len; duration in
 * ms) and returns the number of launches of that forward. */
void rfdetr_b200_profile_enable(rfdetr_context* ctx, int on);
int  rfdetr_b200_profile_read(rfdetr_context* ctx, char* names, int name_len, float* ms, int cap);

/* Host-only inspection of a GGUF file (no GPU needed), for loaders and tests:
 * parses, validates the tensor inventory (src/model_loader.cpp:212-750) and
 * checks that the engine implements the configuration. */
typedef struct {
    uint32_t image_size, patch_size, num_queries, num_classes;
    uint32_t dim, depth, num_windows, dec_layers;
    int      has_segmentation_head;
    size_t   n_tensors;
    char     variant[32];
    int32_t  legacy_resize;  /* 1: images not at the model size take the legacy stb resize
                                (rfdetr.preprocess.resize_mode legacy_stb, or absent as in files
                                converted before the key existed); 0: the 1.9 bilinear path */
} rfdetr_b200_model_info;
rfdetr_status rfdetr_b200_inspect(const char* model_path, rfdetr_b200_model_info* out);

/* Host dequantizer of one GGUF tensor payload (ggml type id -> f32). Returns 0
 * on success, -1 for an unsupported type. */
int rfdetr_b200_dequantize(uint32_t ggml_type, const void* src, long long n, float* dst);

/* ---- operator entry points (device pointers, asynchronous on `stream`) ----
 * The engine's building blocks, exposed so callers can reuse them and so each
 * kernel can be checked on its own.  `stream` is a cudaStream_t (NULL = the
 * legacy default stream).  Return 0 on success, otherwise a cudaError_t code.
 *
 * GEMM: out = epilogue(A[M][K] . B[N][K]^T + bias) with f16 A / B (K
 * contiguous, lda/ldb multiples of 8) and f32 accumulation on the tcgen05
 * tensor cores.  epi: 0 f16 out, 1 f32 out, 2 f32 out += colscale * value,
 * 4 full-row LayerNorm of x = colscale * value + resid (N = 128, 256 or 384;
 * colscale and resid optional) -> f32 and/or f16, 5 residual update fused
 * with the LayerNorm that follows it: out32 = resid + colscale * value (out32
 * may alias resid) and out16 = LayerNorm(out32) (N = 128, 256 or 384, act 0).
 * value = acc + bias.  act: 0 none, 1 GELU (erf), 2 ReLU, 3 SiLU. */
int rfdetr_b200_op_gemm(const void* A, int lda, const void* B, int ldb, int M, int N, int K, int epi, int act,
                        const float* bias, const float* colscale, const float* ln_g, const float* ln_b,
                        float ln_eps, const float* resid, int ldr, float* out32, int ld32, void* out16, int ld16,
                        void* stream);

/* Fused attention O = softmax(scale * Q K^T) V, f16 in / out, head_dim 32 or
 * 64; rows of group g start at g * seq_len; head h uses columns
 * [h*head_dim, (h+1)*head_dim) of each operand. */
int rfdetr_b200_op_attention(const void* q, const void* k, const void* v, int ldq, int ldk, int ldv, void* o,
                             int ldo, int seq_len, int groups, int heads, int head_dim, float scale, void* stream);

/* The reference's `rfdetr-cli quantize` (examples/cli/main.cpp:387-640):
 * write a copy of the GGUF at in_path to out_path with every quantizable
 * weight (2-D `.weight` tensors with both dims >= 64 and rows a multiple of
 * 32, embeddings excluded) that is stored as F32 / F16 / BF16 re-quantized to
 * `type` (1 F16, 8 Q8_0, 12 Q4_K, 13 Q5_K, 14 Q6_K; K-quants fall back to
 * Q8_0 for rows that are not a multiple of 256).  The block quantizers run on
 * CUDA device `device`; metadata and every other tensor are copied unchanged. */
rfdetr_status rfdetr_b200_quantize_gguf(const char* in_path, const char* out_path, int type, int device);

/* The block quantizers behind rfdetr_b200_quantize_gguf: n f32 values
 * (device memory, n a multiple of the block size: 1 F16, 32 Q8_0, 256 Q4_K /
 * Q5_K / Q6_K) -> GGUF blocks of `type` at d_out (device memory). */
int rfdetr_b200_op_quantize(int type, const float* d_src, long long n, void* d_out, void* stream);

/* Post-processing on the device (src/postprocess.cpp:43-181): for each image
 * b of a batch, the sigmoid-argmax over the nc classes of each of the nq
 * queries (d_logits f32 [batch][nq][nc], d_boxes f32 [batch][nq][4] cxcywh in
 * [0,1]), score > threshold, class filter (d_class_filter: filter_len class
 * ids, or NULL), descending score (ties: lower query first), at most top_k
 * (0 = all), boxes to clamped pixel xyxy of an img_w x img_h image.  Writes
 * d_out[b][0 .. d_counts[b]).  nq <= 1024.  All pointers are device memory. */
int rfdetr_b200_op_select(const float* d_logits, const float* d_boxes, int batch, int nq, int nc, float threshold,
                          int top_k, const uint32_t* d_class_filter, int filter_len, int img_w, int img_h,
                          rfdetr_b200_det* d_out, int* d_counts, void* stream);

/* The legacy preprocess resize (src/image_io.cpp:249-275: models whose
 * rfdetr.preprocess.resize_mode is legacy_stb or absent resize images that are
 * not at the model size with stb_image_resize2's stbir_resize_uint8_linear):
 * d_src uint8 HWC [batch][h][w][3] -> d_dst uint8 HWC [batch][oh][ow][3],
 * Catmull-Rom for a growing axis, Mitchell for a shrinking one, a copy for an
 * axis that keeps its size, clamped edges.  Outputs equal the library's except
 * for a byte differing by one where a value lies within float rounding of a
 * half.  Device pointers.  The call allocates and frees its taps, so it
 * synchronizes `stream` before returning (the host waits for the stream's
 * earlier work too); a stream being captured into a CUDA graph is refused
 * with cudaErrorStreamCaptureUnsupported before anything is enqueued. */
int rfdetr_b200_op_resize_legacy(const uint8_t* d_src, int batch, int w, int h, uint8_t* d_dst, int ow, int oh,
                                 void* stream);

/* Two-stage query selection (src/rfdetr_model.cpp:39-62, top_k_by_max_class):
 * for each image b, the k of its n tokens with the largest maximum class logit
 * (d_cls f32 [batch][n][nc]), in descending order of that maximum (ties: lower
 * token first; the reference's partial_sort leaves tie order unspecified) ->
 * d_idx int32 [batch][k].  1 <= n <= 4096, 0 <= k <= n.  Device pointers. */
int rfdetr_b200_op_topk(const float* d_cls, int batch, int n, int nc, int k, int32_t* d_idx, void* stream);

/* 32-bit words of one bit-packed img_w x img_h mask (rows padded to 32 pixels). */
size_t rfdetr_b200_mask_bits_words(int img_w, int img_h);

/* Segmentation masks of the selected detections (d_dets / d_counts from
 * rfdetr_b200_op_select): the query's side x side mask logits (d_masks f32
 * [batch][nq][side][side]) upsampled bilinearly (half-pixel centres, clamped
 * edges) to img_w x img_h and thresholded at sigmoid > 0.5; bit j of word
 * (y, w) of d_bits[b][i] is pixel (32 w + j, y).  d_bits holds batch x
 * max_dets masks of rfdetr_b200_mask_bits_words words; detections i >=
 * d_counts[b] are left untouched. */
int rfdetr_b200_op_mask_bits(const float* d_masks, int batch, int nq, int side, const rfdetr_b200_det* d_dets,
                             const int* d_counts, int max_dets, int img_w, int img_h, uint32_t* d_bits, void* stream);

/* Deformable sampling of one level (value f16 [B*G*G][Dm], so_aw f32
 * [B*NQ][ld] = offsets (heads*points*2) then attention logits
 * (heads*points), refpoints f32 [B*NQ][4]) -> out f16 [B*NQ][Dm]. */
int rfdetr_b200_op_deform(const void* value, const float* so_aw, int ld_soaw, const float* refp, int batch, int nq,
                          int grid, int heads, int points, int dm, void* out, void* stream);

/* 3x3 convolution, stride 1, zero padding 1, no bias, over channels-last f16
 * maps (`src` rows = batch*h*w pixels, `c` channels at pitch `lds`), followed
 * by a LayerNorm over the `oc` output channels (oc = 128 or 256) and an
 * optional activation (0 none, 3 SiLU): the projector's ConvX block
 * (src/projector.cpp:46-59).  weight is f16 [oc][3][3][c].  When c is a
 * multiple of 64 and w <= 128 the convolution runs as an implicit GEMM (the
 * shifted taps are TMA-loaded from `src`, zero outside the map) with the
 * LayerNorm fused into the tcgen05 GEMM epilogue and the workspace is not
 * used; otherwise as an im2col into `workspace` followed by that GEMM.  The
 * workspace must hold rfdetr_b200_op_conv3x3_workspace(batch, h, w, c) bytes
 * of device memory either way.  src (and, on the im2col path, the workspace)
 * must be 16-byte aligned with c and lds multiples of 8 and lds >= c;
 * otherwise cudaErrorInvalidValue is returned before any launch. */
size_t rfdetr_b200_op_conv3x3_workspace(int batch, int h, int w, int c);
int rfdetr_b200_op_conv3x3(const void* src, int lds, int batch, int h, int w, int c, const void* weight, int oc,
                           const float* ln_g, const float* ln_b, float eps, int act, float* out32, int ld32,
                           void* out16, int ld16, void* workspace, size_t workspace_bytes, void* stream);

/* rfdetr_b200_op_conv3x3 without the workspace argument, for callers that
 * cannot call cudaMalloc (a latency-critical serving loop that cannot absorb
 * cudaMalloc's device-wide synchronization, a host whose memory is owned by
 * another framework's caching allocator, a plugin that only receives device
 * pointers).  No counterpart in the reference.  It allocates nothing: the
 * im2col scratch is a fixed array of 8 Mi f16 values (16 MiB) in the library's
 * device memory, present on every GPU that loads the library until exit, so
 * batch*h*w*9*c must not exceed 8388608 (larger sizes are rejected with an
 * error message and cudaErrorInvalidValue).  The first call on a device looks
 * up the array's device address (cudaGetSymbolAddress) — make that first call
 * before any stream capture.  All calls on a device share the array: calls
 * whose work overlaps on the GPU race; calls in one stream are safe.  The
 * caller still passes inputs and outputs; arguments as rfdetr_b200_op_conv3x3
 * (it always takes the im2col path: src 16-byte aligned, c and lds multiples
 * of 8, lds >= c, else cudaErrorInvalidValue before any launch). */
int rfdetr_b200_op_conv3x3_noalloc(const void* src, int lds, int batch, int h, int w, int c, const void* weight,
                                   int oc, const float* ln_g, const float* ln_b, float eps, int act, float* out32,
                                   int ld32, void* out16, int ld16, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* RFDETR_B200_H */
