// Ownership of detection results (src/postprocess.cpp:115-124 of the
// reference): the detection array and each segmentation mask are heap blocks
// released together by rfdetr_detections_free.  The selection itself
// (sigmoid-argmax, threshold, sort, top_k, boxes, mask upsampling) runs on the
// GPU in select.cu; capi.cpp builds the arrays from its results.
#include "postprocess.hpp"

#include <cstdlib>

extern "C" void rfdetr_detections_free(rfdetr_detection* dets, size_t n) {
    if (!dets) return;
    for (size_t i = 0; i < n; ++i)
        if (dets[i].mask) std::free(const_cast<uint8_t*>(dets[i].mask));
    std::free(dets);
}
