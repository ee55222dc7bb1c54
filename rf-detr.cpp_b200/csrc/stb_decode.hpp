// Image decoding with stb_image, the decoder the reference links
// (src/image_io.cpp:26-35: stbi_load_from_memory forcing three channels).
#pragma once

// True when the library was built with stb_image (from the reference tree, REF_STB).
bool rfb_stb_available();
// 8-bit RGB pixels (w * h * 3, row-major) of any image stb_image reads, or null; free with
// rfb_stb_free.  n must be positive and at most INT_MAX.
unsigned char* rfb_stb_decode_rgb(const unsigned char* data, int n, int* w, int* h);
void rfb_stb_free(unsigned char* p);
// Why the last decode on this thread failed.
const char* rfb_stb_reason();
