/* CPU oracle for the RF-DETR forward pass — TEST INFRASTRUCTURE ONLY.
 *
 * A plain C++ restatement of the reference engine's algorithm
 * (localai-org/rf-detr.cpp, src/dinov2.cpp, src/projector.cpp,
 * src/two_stage.cpp, src/decoder.cpp, src/transformer_ops.cpp, src/heads.cpp,
 * src/segmentation.cpp, src/rfdetr_model.cpp, src/model_loader.cpp:117-208,
 * src/image_io.cpp:184-281, src/postprocess.cpp).  It is the checker that the
 * CUDA engine is compared against; only the test-suite, the smoke check and
 * the CPU-baseline leg of the benchmark may load it.  The product library
 * never links or calls it.
 *
 * The reference itself cannot be compiled here (its ggml submodule is not
 * vendored), so this restatement is pinned op-by-op against PyTorch in the
 * test-suite instead.
 */
#ifndef RFDETR_ORACLE_H
#define RFDETR_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int image_size, patch_size, num_queries, num_classes;
    int dim, depth, heads, ffn_dim, num_windows, pos_train;
    int n_global; int global_idx[16];
    int n_taps;   int tap_stage[8];       /* out_feature_indices (1-based stages) */
    int proj_out, proj_bneck, proj_nb;
    int dec_layers, dec_dim, dec_ffn, sa_heads, ca_heads, ca_points;
    int has_seg, mask_ratio;
    /* 0: f32 activations x dequantized weights.
     * 1: ggml-like: activations entering a weight matmul are rounded the way
     *    ggml's CPU vec-dot rounds them for that weight type (F16 -> f16,
     *    Q8_0 -> Q8_0 blocks, Q4_K -> Q8_K blocks). */
    int act_round;
    int n_threads;                          /* 0 = OpenMP default */
} OracleConfig;

/* Weight types (GGUF file types after dequantization to f32). */
enum { ORACLE_F32 = 0, ORACLE_F16 = 1, ORACLE_Q8_0 = 2, ORACLE_Q4_K = 3 };

typedef struct {
    const char*  name;
    const float* data;    /* dequantized, numpy/torch element order */
    int64_t      n;
    int          type;    /* ORACLE_* of the file tensor */
} OracleTensor;

/* Named-intermediate sink, mirroring the reference's trace publish()
 * (src/trace.cpp:10-20).  Layouts are token-major [tokens][channels]. */
typedef void (*oracle_publish_cb)(const char* name, const float* data, int64_t n, void* user);

/* src/image_io.cpp:184-248 (bilinear, no antialias, double coordinates):
 * uint8 HWC -> float planar [3][th][tw], normalized. */
void oracle_preprocess(const uint8_t* rgb, int w, int h, int tw, int th,
                       const float mean[3], const float std_[3], float* out);

/* Full forward for one image.  input: planar [3][S][S].
 * out_logits [NQ][NC], out_boxes [NQ][4] (cx, cy, w, h), out_topk [NQ]
 * (selected token indices, may be NULL), out_masks [NQ][Hm][Wm] (seg only,
 * may be NULL).  force_topk (may be NULL) replaces the top-K selection with
 * the given token indices, so the decoder can be compared on identical
 * queries when near-tied scores order differently.  Returns 0 on success, negative on a missing tensor or bad
 * configuration. */
int oracle_forward(const OracleConfig* cfg, const OracleTensor* tensors, int n_tensors,
                   const float* input, const int32_t* force_topk,
                   float* out_logits, float* out_boxes,
                   int32_t* out_topk, float* out_masks,
                   oracle_publish_cb publish, void* user);

/* src/model_loader.cpp:117-208: antialiased bicubic (A=-0.5) resample of a
 * [src*src][dim] patch grid to [dst*dst][dim]. */
void oracle_bicubic_resample(const float* src, int src_side, int dim, float* dst, int dst_side);

/* src/postprocess.cpp:43-113 selection: returns the number of detections and
 * fills out_query/out_class/out_score/out_xyxy (capacity num_queries). */
int oracle_select(const float* logits, const float* boxes, int nq, int nc,
                  float threshold, int top_k, int img_w, int img_h,
                  const uint32_t* class_filter, int filter_len,
                  int32_t* out_query, int32_t* out_class, float* out_score, float* out_xyxy);

/* src/postprocess.cpp:132-181: bilinear upsample + sigmoid threshold. */
void oracle_mask_upsample(const float* src, int sw, int sh, int dw, int dh, float thr, uint8_t* out);

#ifdef __cplusplus
}
#endif

#endif
