// Image I/O for the public API: rfdetr_image objects, decoding and PNG encoding
// (grayscale masks for the flat C API, RGB for rfdetr_render).  Behaviour of the
// reference's src/image_io.cpp at the API level: images are 8-bit RGB, HWC.
// Decoding: PNG (non-interlaced, via zlib) and binary PPM here (lossless, so the
// same pixels as any decoder); JPEG and every other format through stb_image, the
// decoder the reference links (stb_decode.cc), so the pixels are the reference's
// byte for byte; nvJPEG only when the library was built without stb_image.
#include "image_io.hpp"

#include "common.hpp"
#include "stb_decode.hpp"

#include <nvjpeg.h>
#include <zlib.h>

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>
#include <stdexcept>

namespace {

uint32_t be32(const uint8_t* p) { return ((uint32_t)p[0] << 24) | ((uint32_t)p[1] << 16) | ((uint32_t)p[2] << 8) | p[3]; }

// ---- PNG decode (non-interlaced; 1/2/4/8/16-bit gray, RGB, palette, +alpha)
bool decode_png(const uint8_t* d, size_t n, int* w, int* h, std::vector<uint8_t>& rgb) {
    static const uint8_t sig[8] = {0x89, 'P', 'N', 'G', 0x0D, 0x0A, 0x1A, 0x0A};
    if (n < 8 || std::memcmp(d, sig, 8) != 0) return false;
    size_t pos = 8;
    uint32_t W = 0, H = 0;
    int depth = 0, ctype = 0, interlace = 0;
    std::vector<uint8_t> idat, pal;
    bool have_ihdr = false;
    while (pos + 12 <= n) {
        const uint32_t len = be32(d + pos);
        const uint8_t* type = d + pos + 4;
        const uint8_t* body = d + pos + 8;
        if (len > n - pos - 12) return false;
        if (!std::memcmp(type, "IHDR", 4)) {
            if (len < 13) return false;
            W = be32(body);
            H = be32(body + 4);
            depth = body[8];
            ctype = body[9];
            interlace = body[12];
            have_ihdr = true;
        } else if (!std::memcmp(type, "PLTE", 4)) {
            pal.assign(body, body + len);
        } else if (!std::memcmp(type, "IDAT", 4)) {
            idat.insert(idat.end(), body, body + len);
        } else if (!std::memcmp(type, "IEND", 4)) {
            break;
        }
        pos += 12 + len;
    }
    if (!have_ihdr || W == 0 || H == 0 || W > 65535 || H > 65535 || interlace != 0) return false;
    int chans;
    switch (ctype) {
        case 0: chans = 1; break;
        case 2: chans = 3; break;
        case 3: chans = 1; break;
        case 4: chans = 2; break;
        case 6: chans = 4; break;
        default: return false;
    }
    // the bit depths the PNG specification allows for each colour type: the
    // sub-byte unpacking below relies on depth dividing 8
    bool depth_ok = false;
    switch (ctype) {
        case 0: depth_ok = depth == 1 || depth == 2 || depth == 4 || depth == 8 || depth == 16; break;
        case 3: depth_ok = depth == 1 || depth == 2 || depth == 4 || depth == 8; break;
        default: depth_ok = depth == 8 || depth == 16; break;
    }
    if (!depth_ok) return false;
    const size_t bpp_bits = (size_t)chans * depth;
    const size_t stride = (W * bpp_bits + 7) / 8;
    const size_t bpp = (bpp_bits + 7) / 8;
    // deflate expands its input at most 1032:1, so an image larger than that
    // bound of the IDAT bytes is corrupt: rejected before its buffers exist
    if ((stride + 1) * H > idat.size() * 1032 + 1024) return false;
    std::vector<uint8_t> raw((stride + 1) * H);
    uLongf rawlen = (uLongf)raw.size();
    if (uncompress(raw.data(), &rawlen, idat.data(), (uLong)idat.size()) != Z_OK || rawlen != raw.size()) return false;
    std::vector<uint8_t> img(stride * H), prev(stride, 0);
    for (uint32_t y = 0; y < H; ++y) {
        const uint8_t f = raw[y * (stride + 1)];
        const uint8_t* src = &raw[y * (stride + 1) + 1];
        uint8_t* cur = &img[y * stride];
        for (size_t x = 0; x < stride; ++x) {
            const int a = x >= bpp ? cur[x - bpp] : 0, b = prev[x], c = x >= bpp ? prev[x - bpp] : 0;
            int v = src[x];
            switch (f) {
                case 0: break;
                case 1: v += a; break;
                case 2: v += b; break;
                case 3: v += (a + b) / 2; break;
                case 4: {
                    const int p = a + b - c, pa = std::abs(p - a), pb = std::abs(p - b), pc = std::abs(p - c);
                    v += (pa <= pb && pa <= pc) ? a : (pb <= pc ? b : c);
                    break;
                }
                default: return false;
            }
            cur[x] = (uint8_t)v;
        }
        std::memcpy(prev.data(), cur, stride);
    }
    rgb.resize((size_t)W * H * 3);
    for (uint32_t y = 0; y < H; ++y) {
        const uint8_t* row = &img[y * stride];
        for (uint32_t x = 0; x < W; ++x) {
            uint8_t px[4] = {0, 0, 0, 255};
            if (depth < 8) {
                const int per = 8 / depth;
                const int v = (row[x / per] >> ((per - 1 - (x % per)) * depth)) & ((1 << depth) - 1);
                if (ctype == 3) {
                    if ((size_t)v * 3 + 2 >= pal.size()) return false;
                    px[0] = pal[v * 3]; px[1] = pal[v * 3 + 1]; px[2] = pal[v * 3 + 2];
                } else {
                    const uint8_t g = (uint8_t)(v * 255 / ((1 << depth) - 1));
                    px[0] = px[1] = px[2] = g;
                }
            } else {
                const int bps = depth / 8;
                uint8_t s[4];
                for (int c = 0; c < chans; ++c) s[c] = row[(x * chans + c) * bps];  // high byte for 16-bit
                if (ctype == 3) {
                    if ((size_t)s[0] * 3 + 2 >= pal.size()) return false;
                    px[0] = pal[s[0] * 3]; px[1] = pal[s[0] * 3 + 1]; px[2] = pal[s[0] * 3 + 2];
                } else if (chans <= 2) {
                    px[0] = px[1] = px[2] = s[0];
                } else {
                    px[0] = s[0]; px[1] = s[1]; px[2] = s[2];
                }
            }
            uint8_t* o = &rgb[((size_t)y * W + x) * 3];
            o[0] = px[0]; o[1] = px[1]; o[2] = px[2];
        }
    }
    *w = (int)W;
    *h = (int)H;
    return true;
}

// ---- binary PPM (P6, maxval 255)
bool decode_ppm(const uint8_t* d, size_t n, int* w, int* h, std::vector<uint8_t>& rgb) {
    if (n < 2 || d[0] != 'P' || d[1] != '6') return false;
    size_t pos = 2;
    long vals[3];
    for (int k = 0; k < 3; ++k) {
        while (pos < n) {
            if (d[pos] == '#') { while (pos < n && d[pos] != '\n') ++pos; }
            else if (d[pos] == ' ' || d[pos] == '\n' || d[pos] == '\r' || d[pos] == '\t') ++pos;
            else break;
        }
        long v = 0;
        bool any = false;
        while (pos < n && d[pos] >= '0' && d[pos] <= '9') { v = v * 10 + (d[pos] - '0'); ++pos; any = true; if (v > 1 << 20) return false; }
        if (!any) return false;
        vals[k] = v;
    }
    ++pos;
    if (vals[2] != 255 || vals[0] <= 0 || vals[1] <= 0) return false;
    const size_t need = (size_t)vals[0] * vals[1] * 3;
    if (pos + need > n) return false;
    rgb.assign(d + pos, d + pos + need);
    *w = (int)vals[0];
    *h = (int)vals[1];
    return true;
}

// ---- stb_image (JPEG, interlaced PNG, BMP, GIF, TGA, PSD, HDR, PIC): the reference's decoder
bool decode_stb(const uint8_t* d, size_t n, int* w, int* h, std::vector<uint8_t>& rgb) {
    if (!rfb_stb_available() || n > (size_t)INT32_MAX) return false;
    int W = 0, H = 0;
    unsigned char* px = rfb_stb_decode_rgb(d, (int)n, &W, &H);
    if (!px) return false;
    struct Free {
        unsigned char* p;
        ~Free() { rfb_stb_free(p); }
    } guard{px};
    rgb.assign(px, px + (size_t)W * (size_t)H * 3);  // std::bad_alloc is handled by the caller
    *w = W;
    *h = H;
    return true;
}

// ---- JPEG via nvJPEG (device decode, copied back to host): only without stb_image; its IDCT and
// chroma upsampling are not stb's, so the pixels can differ from the reference's by a few levels
bool decode_jpeg_nvjpeg(const uint8_t* d, size_t n, int* w, int* h, std::vector<uint8_t>& rgb) {
    if (rfb_stb_available()) return false;
    if (n < 3 || d[0] != 0xFF || d[1] != 0xD8) return false;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        rfdetr_logf(RFDETR_LOG_ERROR, "image decode: JPEG decoding needs a CUDA device (nvJPEG)");
        return false;
    }
    nvjpegHandle_t hd = nullptr;
    nvjpegJpegState_t js = nullptr;
    if (nvjpegCreateSimple(&hd) != NVJPEG_STATUS_SUCCESS) return false;
    bool ok = false;
    unsigned char* dev = nullptr;
    if (nvjpegJpegStateCreate(hd, &js) == NVJPEG_STATUS_SUCCESS) {
        int nc = 0;
        nvjpegChromaSubsampling_t ss;
        int ws[NVJPEG_MAX_COMPONENT], hs[NVJPEG_MAX_COMPONENT];
        if (nvjpegGetImageInfo(hd, d, n, &nc, &ss, ws, hs) == NVJPEG_STATUS_SUCCESS && ws[0] > 0 && hs[0] > 0) {
            const int W = ws[0], H = hs[0];
            if (cudaMalloc(&dev, (size_t)W * H * 3) == cudaSuccess) {
                nvjpegImage_t out;
                std::memset(&out, 0, sizeof(out));
                out.channel[0] = dev;
                out.pitch[0] = (unsigned)W * 3;
                if (nvjpegDecode(hd, js, d, n, NVJPEG_OUTPUT_RGBI, &out, nullptr) == NVJPEG_STATUS_SUCCESS &&
                    cudaDeviceSynchronize() == cudaSuccess) {
                    rgb.resize((size_t)W * H * 3);
                    ok = cudaMemcpy(rgb.data(), dev, rgb.size(), cudaMemcpyDeviceToHost) == cudaSuccess;
                    *w = W;
                    *h = H;
                }
                cudaFree(dev);
            }
        }
        nvjpegJpegStateDestroy(js);
    }
    nvjpegDestroy(hd);
    return ok;
}

void put_be32(std::vector<uint8_t>& o, uint32_t v) {
    o.push_back((uint8_t)(v >> 24)); o.push_back((uint8_t)(v >> 16)); o.push_back((uint8_t)(v >> 8)); o.push_back((uint8_t)v);
}
void chunk(std::vector<uint8_t>& o, const char* type, const uint8_t* body, size_t len) {
    put_be32(o, (uint32_t)len);
    const size_t start = o.size();
    o.insert(o.end(), type, type + 4);
    o.insert(o.end(), body, body + len);
    const uLong crc = crc32(0L, o.data() + start, (uInt)(len + 4));
    put_be32(o, (uint32_t)crc);
}

}  // namespace

bool rfdetr_encode_png(const uint8_t* data, int width, int height, int channels, std::vector<uint8_t>& out) {
    if (!data || width <= 0 || height <= 0 || (channels != 1 && channels != 3)) return false;
    const size_t stride = (size_t)width * channels;
    std::vector<uint8_t> raw((stride + 1) * height);
    for (int y = 0; y < height; ++y) {
        raw[y * (stride + 1)] = 0;
        std::memcpy(&raw[y * (stride + 1) + 1], data + y * stride, stride);
    }
    uLongf cap = compressBound((uLong)raw.size());
    std::vector<uint8_t> z(cap);
    if (compress2(z.data(), &cap, raw.data(), (uLong)raw.size(), 6) != Z_OK) return false;
    out.clear();
    static const uint8_t sig[8] = {0x89, 'P', 'N', 'G', 0x0D, 0x0A, 0x1A, 0x0A};
    out.insert(out.end(), sig, sig + 8);
    uint8_t ihdr[13];
    const uint32_t W = (uint32_t)width, H = (uint32_t)height;
    ihdr[0] = (uint8_t)(W >> 24); ihdr[1] = (uint8_t)(W >> 16); ihdr[2] = (uint8_t)(W >> 8); ihdr[3] = (uint8_t)W;
    ihdr[4] = (uint8_t)(H >> 24); ihdr[5] = (uint8_t)(H >> 16); ihdr[6] = (uint8_t)(H >> 8); ihdr[7] = (uint8_t)H;
    ihdr[8] = 8;
    ihdr[9] = channels == 1 ? 0 : 2;
    ihdr[10] = ihdr[11] = ihdr[12] = 0;
    chunk(out, "IHDR", ihdr, 13);
    chunk(out, "IDAT", z.data(), cap);
    chunk(out, "IEND", nullptr, 0);
    return true;
}

extern "C" rfdetr_image* rfdetr_image_load_buffer(const uint8_t* bytes, size_t len, rfdetr_status* st) {
    auto set = [&](rfdetr_status s) { if (st) *st = s; };
    if (!bytes || len == 0) { set(RFDETR_ERR_INVALID_ARG); return nullptr; }
    auto* img = new (std::nothrow) rfdetr_image();
    if (!img) { set(RFDETR_ERR_OUT_OF_MEMORY); return nullptr; }
    int w = 0, h = 0;
    bool ok = false;
    try {
        ok = decode_png(bytes, len, &w, &h, img->rgb) || decode_ppm(bytes, len, &w, &h, img->rgb) ||
             decode_stb(bytes, len, &w, &h, img->rgb) || decode_jpeg_nvjpeg(bytes, len, &w, &h, img->rgb);
    } catch (const std::bad_alloc&) {
        delete img;
        set(RFDETR_ERR_OUT_OF_MEMORY);
        return nullptr;
    }
    if (!ok) {
        rfdetr_logf(RFDETR_LOG_ERROR, "rfdetr_image_load_buffer: unsupported or corrupt image (%zu bytes): %s", len,
                    rfb_stb_reason());
        delete img;
        set(RFDETR_ERR_DECODE);
        return nullptr;
    }
    img->width = w;
    img->height = h;
    set(RFDETR_OK);
    return img;
}

static rfdetr_image* rfdetr_image_load_file_body(const char* path, rfdetr_status* st) {
    auto set = [&](rfdetr_status s) { if (st) *st = s; };
    if (!path) { set(RFDETR_ERR_INVALID_ARG); return nullptr; }
    FILE* f = std::fopen(path, "rb");
    if (!f) { set(RFDETR_ERR_FILE_NOT_FOUND); return nullptr; }
    std::vector<uint8_t> buf;
    if (std::fseek(f, 0, SEEK_END) == 0) {
        const long n = std::ftell(f);
        if (n > 0 && std::fseek(f, 0, SEEK_SET) == 0) {
            buf.resize((size_t)n);
            if (std::fread(buf.data(), 1, buf.size(), f) != buf.size()) buf.clear();
        }
    }
    std::fclose(f);
    if (buf.empty()) { set(RFDETR_ERR_IO); return nullptr; }
    return rfdetr_image_load_buffer(buf.data(), buf.size(), st);
}

extern "C" rfdetr_image* rfdetr_image_load_file(const char* path, rfdetr_status* st) {
    return rfdetr_c_boundary_ptr<rfdetr_image>([&] { return rfdetr_image_load_file_body(path, st); },
                                               st, RFDETR_ERR_IO);
}

extern "C" rfdetr_image* rfdetr_image_from_rgb_buffer(const uint8_t* rgb, int width, int height, rfdetr_status* st) {
    auto set = [&](rfdetr_status s) { if (st) *st = s; };
    if (!rgb || width <= 0 || height <= 0) { set(RFDETR_ERR_INVALID_ARG); return nullptr; }
    // more bytes than a buffer can hold: not a real image (checked before rgb + bytes is formed,
    // which would itself be undefined for such a size)
    const size_t bytes = (size_t)width * (size_t)height * 3;
    if (bytes > (size_t)PTRDIFF_MAX / 2) { set(RFDETR_ERR_INVALID_ARG); return nullptr; }
    auto* img = new (std::nothrow) rfdetr_image();
    if (!img) { set(RFDETR_ERR_OUT_OF_MEMORY); return nullptr; }
    try {
        img->rgb.assign(rgb, rgb + bytes);
    } catch (const std::bad_alloc&) {
        delete img;
        set(RFDETR_ERR_OUT_OF_MEMORY);
        return nullptr;
    } catch (const std::length_error&) {
        delete img;
        set(RFDETR_ERR_INVALID_ARG);
        return nullptr;
    }
    img->width = width;
    img->height = height;
    set(RFDETR_OK);
    return img;
}

extern "C" void rfdetr_image_free(rfdetr_image* img) { delete img; }
extern "C" int rfdetr_image_width(const rfdetr_image* img) { return img ? img->width : 0; }
extern "C" int rfdetr_image_height(const rfdetr_image* img) { return img ? img->height : 0; }
extern "C" const uint8_t* rfdetr_image_rgb_data(const rfdetr_image* img) {
    return (img && !img->rgb.empty()) ? img->rgb.data() : nullptr;
}
