// Resampling taps of the reference's legacy preprocess resize (the
// `legacy_stb` value of rfdetr.preprocess.resize_mode; src/image_io.cpp:249-275
// of the reference, which calls stb_image_resize2 v2.18's
// stbir_resize_uint8_linear on 8-bit RGB with its default filters and clamped
// edges).  The taps of one axis are computed on the host; the GPU kernel
// (kernels.cu, resize_legacy_rgb) applies both axes.
#pragma once

#include <cuda_runtime.h>

#include <vector>

namespace rfb {

// Output pixel o of one axis reads input pixels [first[o], first[o] + count[o])
// with weights coef[o * width + k], k < count[o].
struct ResizeTaps {
    int in = 0, out = 0, width = 0;
    std::vector<int> first, count;
    std::vector<float> coef;
};

ResizeTaps legacy_resize_taps(int in_size, int out_size);

// Both axes' taps of a w x h -> ow x oh resize in device memory (one
// allocation at `base`, released with cudaFree).
struct LegacyTapsDev {
    void* base = nullptr;
    const int* xf = nullptr;
    const int* xn = nullptr;
    const float* xc = nullptr;
    int xw = 0;
    const int* yf = nullptr;
    const int* yn = nullptr;
    const float* yc = nullptr;
    int yw = 0;
};

// Computes the taps and copies them to the current device (synchronously).
cudaError_t upload_legacy_taps(int w, int h, int ow, int oh, LegacyTapsDev* out);

}  // namespace rfb
