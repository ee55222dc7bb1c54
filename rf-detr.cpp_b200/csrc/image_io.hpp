// rfdetr_image and the host image helpers shared by the API sources.
#pragma once

#include "rfdetr.h"

#include <cstdint>
#include <vector>

struct rfdetr_image {
    int width = 0;
    int height = 0;
    std::vector<uint8_t> rgb;  // HWC, row-major, 8-bit RGB
};

// PNG-encode an 8-bit image with 1 (gray) or 3 (RGB) channels.
bool rfdetr_encode_png(const uint8_t* data, int width, int height, int channels, std::vector<uint8_t>& out);
