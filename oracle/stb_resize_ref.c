/* Test infrastructure only (never linked into the engine): the reference's
 * legacy preprocess resize, src/image_io.cpp:249-275, which calls
 * stb_image_resize2 v2.18 (third_party/stb/stb_image_resize.h of the
 * reference) as stbir_resize_uint8_linear(..., STBIR_RGB).  This wrapper is
 * compiled against that header where it lies in the reference tree, into
 * oracle/_ref/, and generates the golden vectors of the engine's legacy_stb
 * resize (tests/golden/make_stb_resize_golden.py). */
#define STB_IMAGE_RESIZE_IMPLEMENTATION
#define STBIR__HEADER_FILENAME "stb_image_resize.h" /* the reference vendors v2 under this name */
#include "stb_image_resize.h"

int stb_resize_rgb(const unsigned char* in, int w, int h, unsigned char* out, int ow, int oh) {
    return stbir_resize_uint8_linear(in, w, h, 0, out, ow, oh, 0, STBIR_RGB) != 0;
}
