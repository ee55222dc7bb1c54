// In-place annotation and PNG rendering for the public API
// (reference: src/visualize.cpp, rfdetr.h:111-153).  Boxes are drawn in a
// deterministic per-class colour from a 20-entry palette with a minimum
// stroke of 3 px; a filled label bar sits above the box (inside the top edge
// when the box touches the image top).  Label glyphs are not rasterized.
#include "rfdetr.h"

#include "common.hpp"
#include "image_io.hpp"

#include <algorithm>
#include <cmath>
#include <cstdio>

namespace {

const uint8_t kPalette[20][3] = {
    {230, 25, 75}, {60, 180, 75}, {255, 225, 25}, {0, 130, 200}, {245, 130, 48}, {145, 30, 180}, {70, 240, 240},
    {240, 50, 230}, {210, 245, 60}, {250, 190, 212}, {0, 128, 128}, {220, 190, 255}, {170, 110, 40},
    {255, 250, 200}, {128, 0, 0}, {170, 255, 195}, {128, 128, 0}, {255, 215, 180}, {0, 0, 128}, {128, 128, 128}};

void fill(rfdetr_image* img, int x0, int y0, int x1, int y1, const uint8_t* c) {
    x0 = std::max(x0, 0);
    y0 = std::max(y0, 0);
    x1 = std::min(x1, img->width);
    y1 = std::min(y1, img->height);
    for (int y = y0; y < y1; ++y)
        for (int x = x0; x < x1; ++x) {
            uint8_t* p = &img->rgb[((size_t)y * img->width + x) * 3];
            p[0] = c[0]; p[1] = c[1]; p[2] = c[2];
        }
}

// Pixel coordinate of a caller's box edge: NaN draws at 0 and values are held
// to +-1e6, so the conversion and the edge arithmetic below cannot overflow.
int coord(float v) { return std::isnan(v) ? 0 : (int)std::clamp(v, -1.0e6f, 1.0e6f); }

}  // namespace

extern "C" void rfdetr_visualize_draw_box(rfdetr_image* img, rfdetr_detection det, int thickness) {
    if (!img || img->rgb.empty()) return;
    const uint8_t* c = kPalette[det.class_id % 20];
    const int x0 = coord(det.x1), y0 = coord(det.y1), x1 = coord(det.x2), y1 = coord(det.y2);
    int t = std::max(thickness, 3);
    t = std::min(t, std::max(1, std::min(x1 - x0, y1 - y0) / 2));
    fill(img, x0, y0, x1, y0 + t, c);
    fill(img, x0, y1 - t, x1, y1, c);
    fill(img, x0, y0, x0 + t, y1, c);
    fill(img, x1 - t, y0, x1, y1, c);
    const int bar = 12;
    const int by0 = y0 - bar >= 0 ? y0 - bar : y0;
    fill(img, x0, by0, std::min(x1, x0 + 8 * 16), by0 + bar, c);
}

extern "C" void rfdetr_visualize_overlay_mask(rfdetr_image* img, rfdetr_detection det, float alpha) {
    if (!img || !det.mask || det.mask_width != img->width || det.mask_height != img->height) return;
    alpha = std::clamp(alpha, 0.f, 1.f);
    const uint8_t* c = kPalette[det.class_id % 20];
    for (size_t i = 0; i < (size_t)img->width * img->height; ++i) {
        if (!det.mask[i]) continue;
        uint8_t* p = &img->rgb[i * 3];
        for (int k = 0; k < 3; ++k) p[k] = (uint8_t)(p[k] * (1.f - alpha) + c[k] * alpha + 0.5f);
    }
}

static rfdetr_status rfdetr_render_body(const rfdetr_image* img, const rfdetr_detection* dets, size_t n,
                                        const char* out_path) {
    if (!img || !out_path || img->rgb.empty() || (n && !dets)) return RFDETR_ERR_INVALID_ARG;
    rfdetr_image copy = *img;
    for (size_t i = 0; i < n; ++i) rfdetr_visualize_overlay_mask(&copy, dets[i], 0.45f);
    for (size_t i = 0; i < n; ++i) rfdetr_visualize_draw_box(&copy, dets[i], 3);
    std::vector<uint8_t> png;
    if (!rfdetr_encode_png(copy.rgb.data(), copy.width, copy.height, 3, png)) return RFDETR_ERR_IO;
    FILE* f = std::fopen(out_path, "wb");
    if (!f) return RFDETR_ERR_IO;
    const bool ok = std::fwrite(png.data(), 1, png.size(), f) == png.size();
    std::fclose(f);
    return ok ? RFDETR_OK : RFDETR_ERR_IO;
}

extern "C" rfdetr_status rfdetr_render(const rfdetr_image* img, const rfdetr_detection* dets, size_t n,
                                       const char* out_path) {
    return rfdetr_c_boundary([&] { return rfdetr_render_body(img, dets, n, out_path); },
                             RFDETR_ERR_OUT_OF_MEMORY, RFDETR_ERR_IO);
}
