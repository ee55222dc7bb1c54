#pragma once

#include "rfdetr.h"

#include <cstddef>
#include <cstdint>

namespace rfb {

// One image: logits [nq][nc], boxes [nq][4] (normalized cxcywh), optional
// mask logits [nq][mask_h][mask_w].  Result array is calloc'd (masks too) and
// released with rfdetr_detections_free.  class_name is left NULL.
void select_detections(const float* logits, const float* boxes, const float* masks, int mask_w, int mask_h,
                       size_t nq, size_t nc, float threshold, uint32_t top_k, const uint32_t* filter,
                       size_t filter_len, int img_w, int img_h, rfdetr_detection** out, size_t* out_n);

}  // namespace rfb
