/* The reference's image decoder, stb_image (third_party/stb/stb_image.h of the
 * reference tree, public domain), built by `make -C oracle ref` into
 * oracle/_ref/libstbimage.so: the checker of the library's image decoding
 * (tests/test_image_decode_golden.py, tests/golden/gen_jpeg_golden.py).  The
 * call is the reference's (src/image_io.cpp:30: stbi_load_from_memory forcing
 * three channels).  Test infrastructure only. */
#define STB_IMAGE_IMPLEMENTATION
#define STBI_NO_STDIO
#include "stb_image.h"

unsigned char* ref_stbi_load_rgb(const unsigned char* data, int n, int* w, int* h) {
    int comp = 0;
    return stbi_load_from_memory(data, n, w, h, &comp, 3);
}

void ref_stbi_free(unsigned char* p) { stbi_image_free(p); }
