// Post-processing on the GPU: detection selection and bit-packed mask
// upsampling (see select.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "rfdetr_b200.h"

namespace rfb {

using DetRecord = rfdetr_b200_det;
static_assert(sizeof(DetRecord) == 32, "device record layout");

// Per image b: out[b][0 .. counts[b]) = the selected detections in output
// order (img_w x img_h is the original image size of every image of the batch).
cudaError_t select_detections_device(const float* logits, const float* boxes, int B, int NQ, int NC,
                                     float threshold, int top_k, const uint32_t* filter, int filter_len, int img_w,
                                     int img_h, DetRecord* out, int* counts, cudaStream_t st);

// 32-bit words of one bit-packed img_w x img_h mask (rows padded to 32 pixels).
size_t mask_bits_words(int img_w, int img_h);

// bits[b][i] (i < counts[b] <= max_dets): the upsampled, thresholded mask of
// detection i of image b; bit j of word (y, w) is pixel (x = 32 w + j, y).
cudaError_t mask_bits_device(const float* masks, int B, int NQ, int side, const DetRecord* dets, const int* counts,
                             int max_dets, int img_w, int img_h, uint32_t* bits, cudaStream_t st);

}  // namespace rfb
