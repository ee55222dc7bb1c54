/* CPU oracle, host-side pre- and post-processing — TEST INFRASTRUCTURE ONLY.
 * Restates the reference's src/image_io.cpp:184-248 (rfdetr_preprocess, 1.9
 * bilinear path) and src/postprocess.cpp:10-181 (selection, mask upsampling).
 * This file is compiled without floating-point contraction (-ffp-contract=off),
 * as the reference builds its own sources (no -march, so no FMA): with it the
 * results equal the reference's bit for bit (tests/test_host_ref_golden.py). */
#include "oracle.h"

#include <algorithm>
#include <cmath>
#include <vector>

/* ---- preprocess: src/image_io.cpp:184-248 -------------------------------- */

extern "C" void oracle_preprocess(const uint8_t* rgb, int w, int h, int tw, int th,
                                  const float mean[3], const float std_[3], float* out) {
    const double sx = (double)w / (double)tw, sy = (double)h / (double)th;
    for (int yy = 0; yy < th; ++yy) {
        const double fy = ((double)yy + 0.5) * sy - 0.5;
        const int y0r = (int)std::floor(fy);
        const int y0 = std::clamp(y0r, 0, h - 1), y1 = std::clamp(y0r + 1, 0, h - 1);
        const float wy = (float)(fy - (double)y0r);
        for (int xx = 0; xx < tw; ++xx) {
            const double fx = ((double)xx + 0.5) * sx - 0.5;
            const int x0r = (int)std::floor(fx);
            const int x0 = std::clamp(x0r, 0, w - 1), x1 = std::clamp(x0r + 1, 0, w - 1);
            const float wx = (float)(fx - (double)x0r);
            for (int ch = 0; ch < 3; ++ch) {
                const float p00 = (float)rgb[((size_t)y0 * w + x0) * 3 + ch];
                const float p01 = (float)rgb[((size_t)y0 * w + x1) * 3 + ch];
                const float p10 = (float)rgb[((size_t)y1 * w + x0) * 3 + ch];
                const float p11 = (float)rgb[((size_t)y1 * w + x1) * 3 + ch];
                const float top = p00 + (p01 - p00) * wx;
                const float bot = p10 + (p11 - p10) * wx;
                float v = (top + (bot - top) * wy) / 255.0f;
                v = (v - mean[ch]) / std_[ch];
                out[(size_t)ch * th * tw + (size_t)yy * tw + xx] = v;
            }
        }
    }
}

/* ---- postprocess: src/postprocess.cpp:10-113, 132-181 -------------------- */

namespace {
inline float sigmoid_stable(float x) {
    if (x >= 0.f) { const float z = std::exp(-x); return 1.f / (1.f + z); }
    const float z = std::exp(x);
    return z / (1.f + z);
}
}  // namespace

extern "C" int oracle_select(const float* logits, const float* boxes, int nq, int nc,
                             float threshold, int top_k, int img_w, int img_h,
                             const uint32_t* class_filter, int filter_len,
                             int32_t* out_query, int32_t* out_class, float* out_score, float* out_xyxy) {
    struct Cand { int q, c; float s; };
    std::vector<Cand> cands;
    for (int q = 0; q < nq; ++q) {
        int bc = 0; float bs = -1.f;
        for (int ci = 0; ci < nc; ++ci) {
            const float s = sigmoid_stable(logits[(size_t)q * nc + ci]);
            if (s > bs) { bs = s; bc = ci; }
        }
        if (bs <= threshold) continue;
        // class filter (src/postprocess.cpp:43-113): keep only listed classes
        if (class_filter && filter_len > 0) {
            bool allowed = false;
            for (int i = 0; i < filter_len; ++i) allowed |= class_filter[i] == (uint32_t)bc;
            if (!allowed) continue;
        }
        cands.push_back({q, bc, bs});
    }
    std::stable_sort(cands.begin(), cands.end(), [](const Cand& a, const Cand& b) { return a.s > b.s; });
    if (top_k > 0 && (int)cands.size() > top_k) cands.resize(top_k);
    for (size_t i = 0; i < cands.size(); ++i) {
        out_query[i] = cands[i].q;
        out_class[i] = cands[i].c;
        out_score[i] = cands[i].s;
        const float* b = boxes + (size_t)cands[i].q * 4;
        const float cx = b[0], cy = b[1], w = b[2], h = b[3];
        out_xyxy[i * 4 + 0] = std::clamp((cx - 0.5f * w) * (float)img_w, 0.f, (float)img_w);
        out_xyxy[i * 4 + 1] = std::clamp((cy - 0.5f * h) * (float)img_h, 0.f, (float)img_h);
        out_xyxy[i * 4 + 2] = std::clamp((cx + 0.5f * w) * (float)img_w, 0.f, (float)img_w);
        out_xyxy[i * 4 + 3] = std::clamp((cy + 0.5f * h) * (float)img_h, 0.f, (float)img_h);
    }
    return (int)cands.size();
}

extern "C" void oracle_mask_upsample(const float* src, int sw, int sh, int dw, int dh, float thr, uint8_t* out) {
    const float sfx = (float)sw / (float)dw, sfy = (float)sh / (float)dh;
    for (int dy = 0; dy < dh; ++dy) {
        const float y = ((float)dy + 0.5f) * sfy - 0.5f;
        int y0 = (int)std::floor(y), y1 = y0 + 1;
        y0 = std::clamp(y0, 0, sh - 1); y1 = std::clamp(y1, 0, sh - 1);
        const float fy = std::clamp(y - (float)y0, 0.f, 1.f);
        for (int dx = 0; dx < dw; ++dx) {
            const float x = ((float)dx + 0.5f) * sfx - 0.5f;
            int x0 = (int)std::floor(x), x1 = x0 + 1;
            x0 = std::clamp(x0, 0, sw - 1); x1 = std::clamp(x1, 0, sw - 1);
            const float fx = std::clamp(x - (float)x0, 0.f, 1.f);
            const float a = src[(size_t)y0 * sw + x0], b = src[(size_t)y0 * sw + x1];
            const float c = src[(size_t)y1 * sw + x0], d = src[(size_t)y1 * sw + x1];
            const float v = a * (1 - fx) * (1 - fy) + b * fx * (1 - fy) + c * (1 - fx) * fy + d * fx * fy;
            out[(size_t)dy * dw + dx] = sigmoid_stable(v) > thr ? 255 : 0;
        }
    }
}
