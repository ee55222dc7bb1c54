/* rfdetr_capi.h — flat handle-based C API (the surface LocalAI binds with
 * dlopen/purego).  Same eleven symbols, signatures and return conventions as
 * the reference (localai-org/rf-detr.cpp include/rfdetr_capi.h:14-76):
 * 0 = ok, negative = error, every detect call clears the previous batch, and
 * string / PNG accessors use two-call sizing. */
#ifndef RFDETR_CAPI_H
#define RFDETR_CAPI_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef uintptr_t rfdetr_handle_t;

/* include/rfdetr_capi.h:14-15 */
int rfdetr_capi_load(const char* model_path, int n_threads, rfdetr_handle_t* out_handle);
int rfdetr_capi_unload(rfdetr_handle_t handle);

/* include/rfdetr_capi.h:17-28: JSON envelope, freed with rfdetr_capi_free_string. */
int rfdetr_capi_detect_path(rfdetr_handle_t handle, const char* image_path,
                            float threshold, uint32_t top_k, char** out_json);
int rfdetr_capi_detect_buffer(rfdetr_handle_t handle, const uint8_t* bytes, size_t len,
                              float threshold, uint32_t top_k, char** out_json);
void rfdetr_capi_free_string(char* s);

/* include/rfdetr_capi.h:39-76: accessors over the last detect call. */
int   rfdetr_capi_get_n_detections(rfdetr_handle_t handle);
int   rfdetr_capi_get_detection_class_id(rfdetr_handle_t handle, int i);
int   rfdetr_capi_get_detection_box(rfdetr_handle_t handle, int i, float out_xyxy[4]);
float rfdetr_capi_get_detection_score(rfdetr_handle_t handle, int i);
int   rfdetr_capi_get_detection_class_name(rfdetr_handle_t handle, int i, char* buf, int buf_size);
int   rfdetr_capi_get_detection_mask_png(rfdetr_handle_t handle, int i, unsigned char* buf, int buf_size);

#ifdef __cplusplus
}
#endif

#endif /* RFDETR_CAPI_H */
