// stb_image (public domain, vendored by the reference as third_party/stb/stb_image.h) compiled
// into the library from the reference tree at build time (`make REF_STB=<tree>/third_party/stb`),
// not copied here.  The reference decodes every input image with it, so a JPEG passed to
// rfdetr_image_load_buffer / rfdetr_capi_detect_buffer enters the network with exactly the
// reference's pixels (integer IDCT, chroma upsampling and colour conversion included).  The
// library's functions stay internal to this file (STB_IMAGE_STATIC).  Built without the tree,
// the stubs below report stb as absent and JPEG falls back to nvJPEG (not byte-identical).
#include "stb_decode.hpp"

#if defined(RFB_STB_DIR) && __has_include("stb_image.h")
#pragma GCC diagnostic push
#pragma GCC diagnostic ignored "-Wunused-function"
#pragma GCC diagnostic ignored "-Wmissing-field-initializers"
#pragma GCC diagnostic ignored "-Wsign-compare"
#pragma GCC diagnostic ignored "-Wimplicit-fallthrough"
#define STB_IMAGE_STATIC
#define STB_IMAGE_IMPLEMENTATION
#define STBI_NO_STDIO
#include "stb_image.h"
#pragma GCC diagnostic pop

bool rfb_stb_available() { return true; }

unsigned char* rfb_stb_decode_rgb(const unsigned char* data, int n, int* w, int* h) {
    int comp = 0;
    return stbi_load_from_memory(data, n, w, h, &comp, 3);
}

void rfb_stb_free(unsigned char* p) { stbi_image_free(p); }

const char* rfb_stb_reason() { return stbi_failure_reason(); }
#else
bool rfb_stb_available() { return false; }
unsigned char* rfb_stb_decode_rgb(const unsigned char*, int, int*, int*) { return nullptr; }
void rfb_stb_free(unsigned char*) {}
const char* rfb_stb_reason() { return "stb_image not built in"; }
#endif
