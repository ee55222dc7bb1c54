/* rfdetr.h — public C API of the B200 RF-DETR engine.
 *
 * Drop-in for the reference library's public header
 * (localai-org/rf-detr.cpp include/rfdetr.h): every type, enum value and
 * function below keeps the reference's name, signature, ownership and error
 * behaviour, so code written against librfdetr links against this build
 * unchanged.  Inference runs on an NVIDIA B200 (sm_100a); see rfdetr_b200.h
 * for the additive batch / device entry points.
 */
#ifndef RFDETR_H
#define RFDETR_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes; 0 = success (reference include/rfdetr.h:12-23). */
typedef enum {
    RFDETR_OK                  =  0,
    RFDETR_ERR_INVALID_ARG     = -1,
    RFDETR_ERR_FILE_NOT_FOUND  = -2,
    RFDETR_ERR_IO              = -3,
    RFDETR_ERR_OUT_OF_MEMORY   = -4,
    RFDETR_ERR_DECODE          = -5,
    RFDETR_ERR_MODEL_FORMAT    = -6,   /* GGUF parse / variant detection */
    RFDETR_ERR_MODEL_LOAD      = -7,   /* tensor inventory (e.g. missing tensors) */
    RFDETR_ERR_INFERENCE       = -8,   /* forward pass failed (CUDA error, device error word) */
    RFDETR_ERR_NOT_IMPLEMENTED = -99
} rfdetr_status;

/* Replaces include/rfdetr.h:25 (rfdetr_status_str). */
const char* rfdetr_status_str(rfdetr_status s);

typedef enum {
    RFDETR_LOG_DEBUG = 0,
    RFDETR_LOG_INFO  = 1,
    RFDETR_LOG_WARN  = 2,
    RFDETR_LOG_ERROR = 3
} rfdetr_log_level;

typedef void (*rfdetr_log_cb)(rfdetr_log_level lvl, const char* msg, void* user_data);
/* Process-global; replaces include/rfdetr.h:35-36. */
void rfdetr_set_log_callback(rfdetr_log_cb cb, void* user_data);

typedef struct rfdetr_context rfdetr_context;
typedef struct rfdetr_image   rfdetr_image;

/* One detection (include/rfdetr.h:42-61).  `class_name` is borrowed from the
 * context.  `mask` (segmentation models only) is a row-major 0/255 bitmap at
 * the original image size, owned by the array and released by
 * rfdetr_detections_free. */
typedef struct {
    uint32_t       class_id;
    const char*    class_name;
    float          score;
    float          x1, y1, x2, y2;   /* pixels on the original image */
    const uint8_t* mask;
    int            mask_width;
    int            mask_height;
} rfdetr_detection;

/* include/rfdetr.h:63-73.  n_threads sizes the host-side worker pool used for
 * pre/post-processing (0 or negative = hardware concurrency); the forward
 * pass itself runs on the GPU. */
typedef struct {
    const char*   model_path;
    int           n_threads;
    rfdetr_log_cb log_cb;
    void*         log_user_data;
} rfdetr_params;

/* include/rfdetr.h:75-80 */
typedef struct {
    float           threshold;          /* default 0.5 */
    uint32_t        top_k;              /* default 300 */
    const uint32_t* class_filter;       /* optional allowlist */
    size_t          class_filter_len;
} rfdetr_detect_params;

/* include/rfdetr.h:82-84: load a GGUF model onto GPU 0 (or RFDETR_DEVICE). */
rfdetr_context* rfdetr_init(const rfdetr_params* params, rfdetr_status* out_status);
void            rfdetr_free(rfdetr_context* ctx);

/* include/rfdetr.h:86-91 */
const char* rfdetr_context_variant(const rfdetr_context* ctx);
uint32_t    rfdetr_context_image_size(const rfdetr_context* ctx);
uint32_t    rfdetr_context_num_queries(const rfdetr_context* ctx);
uint32_t    rfdetr_context_num_classes(const rfdetr_context* ctx);
size_t      rfdetr_context_n_tensors(const rfdetr_context* ctx);

/* include/rfdetr.h:93-95: PNG (zlib), binary PPM, and JPEG (nvJPEG, needs a
 * GPU) are decoded. */
rfdetr_image* rfdetr_image_load_file(const char* path, rfdetr_status* out_status);
rfdetr_image* rfdetr_image_load_buffer(const uint8_t* bytes, size_t len, rfdetr_status* out_status);

/* include/rfdetr.h:97-109: copies `rgb` (HWC, width*height*3 bytes). */
rfdetr_image* rfdetr_image_from_rgb_buffer(const uint8_t* rgb, int width, int height,
                                           rfdetr_status* out_status);

void           rfdetr_image_free(rfdetr_image* img);
int            rfdetr_image_width(const rfdetr_image* img);
int            rfdetr_image_height(const rfdetr_image* img);
const uint8_t* rfdetr_image_rgb_data(const rfdetr_image* img);

/* include/rfdetr.h:125-141: in-place annotation. */
void rfdetr_visualize_draw_box(rfdetr_image* img, rfdetr_detection det, int thickness);
void rfdetr_visualize_overlay_mask(rfdetr_image* img, rfdetr_detection det, float alpha);

/* include/rfdetr.h:143-148: one image end to end (preprocess, forward on the
 * GPU, select, masks). */
rfdetr_status rfdetr_detect(rfdetr_context* ctx,
                            const rfdetr_image* img,
                            const rfdetr_detect_params* params,
                            rfdetr_detection** out_detections,
                            size_t* out_n);
void rfdetr_detections_free(rfdetr_detection* detections, size_t n);

/* include/rfdetr.h:150-153: annotated PNG. */
rfdetr_status rfdetr_render(const rfdetr_image* img,
                            const rfdetr_detection* detections, size_t n,
                            const char* out_path);

#ifdef __cplusplus
}
#endif

#endif /* RFDETR_H */
