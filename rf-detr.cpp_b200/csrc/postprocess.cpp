// Host post-processing of one image's forward output into rfdetr_detection
// records: sigmoid-argmax over classes, threshold, descending sort, top_k,
// cxcywh -> clamped pixel xyxy, and (segmentation) bilinear mask upsample to
// the original image size with a sigmoid > 0.5 threshold.  Same rules as the
// reference's src/postprocess.cpp:10-276.
#include "postprocess.hpp"

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <new>
#include <vector>

namespace {

inline float sigmoid(float x) {
    if (x >= 0.f) {
        const float z = std::exp(-x);
        return 1.f / (1.f + z);
    }
    const float z = std::exp(x);
    return z / (1.f + z);
}

void to_xyxy(const float* b, int w, int h, float* o) {
    const float cx = b[0], cy = b[1], bw = b[2], bh = b[3];
    o[0] = std::clamp((cx - 0.5f * bw) * (float)w, 0.f, (float)w);
    o[1] = std::clamp((cy - 0.5f * bh) * (float)h, 0.f, (float)h);
    o[2] = std::clamp((cx + 0.5f * bw) * (float)w, 0.f, (float)w);
    o[3] = std::clamp((cy + 0.5f * bh) * (float)h, 0.f, (float)h);
}

uint8_t* upsample_mask(const float* src, int sw, int sh, int dw, int dh, float thr) {
    auto* out = static_cast<uint8_t*>(std::calloc((size_t)dw * dh, 1));
    if (!out) return nullptr;
    const float fx = (float)sw / (float)dw, fy = (float)sh / (float)dh;
    std::vector<int> x0(dw), x1(dw);
    std::vector<float> ax(dw);
    for (int x = 0; x < dw; ++x) {
        const float sx = ((float)x + 0.5f) * fx - 0.5f;
        int a = (int)std::floor(sx), b = a + 1;
        a = std::clamp(a, 0, sw - 1);
        b = std::clamp(b, 0, sw - 1);
        x0[x] = a;
        x1[x] = b;
        ax[x] = std::clamp(sx - (float)a, 0.f, 1.f);
    }
    for (int y = 0; y < dh; ++y) {
        const float sy = ((float)y + 0.5f) * fy - 0.5f;
        int a = (int)std::floor(sy), b = a + 1;
        a = std::clamp(a, 0, sh - 1);
        b = std::clamp(b, 0, sh - 1);
        const float ay = std::clamp(sy - (float)a, 0.f, 1.f);
        const float* r0 = src + (size_t)a * sw;
        const float* r1 = src + (size_t)b * sw;
        uint8_t* o = out + (size_t)y * dw;
        for (int x = 0; x < dw; ++x) {
            const float fxv = ax[x];
            const float v = r0[x0[x]] * (1 - fxv) * (1 - ay) + r0[x1[x]] * fxv * (1 - ay) + r1[x0[x]] * (1 - fxv) * ay +
                            r1[x1[x]] * fxv * ay;
            o[x] = sigmoid(v) > thr ? 255 : 0;
        }
    }
    return out;
}

}  // namespace

namespace rfb {

void select_detections(const float* logits, const float* boxes, const float* masks, int mask_w, int mask_h,
                       size_t nq, size_t nc, float threshold, uint32_t top_k, const uint32_t* filter,
                       size_t filter_len, int img_w, int img_h, rfdetr_detection** out, size_t* out_n) {
    *out = nullptr;
    *out_n = 0;
    if (!logits || !boxes || nq == 0 || nc == 0) return;
    struct Cand { uint32_t q, c; float s; };
    try {
        std::vector<Cand> cands;
        cands.reserve(nq);
        for (size_t q = 0; q < nq; ++q) {
            const float* r = logits + q * nc;
            uint32_t bc = 0;
            float bs = -1.f;
            for (size_t c = 0; c < nc; ++c) {
                const float s = sigmoid(r[c]);
                if (s > bs) { bs = s; bc = (uint32_t)c; }
            }
            if (bs <= threshold) continue;
            if (filter && filter_len) {
                bool allowed = false;
                for (size_t i = 0; i < filter_len; ++i) allowed |= filter[i] == bc;
                if (!allowed) continue;
            }
            cands.push_back({(uint32_t)q, bc, bs});
        }
        std::stable_sort(cands.begin(), cands.end(), [](const Cand& a, const Cand& b) { return a.s > b.s; });
        if (top_k > 0 && cands.size() > top_k) cands.resize(top_k);
        if (cands.empty()) return;
        auto* d = static_cast<rfdetr_detection*>(std::calloc(cands.size(), sizeof(rfdetr_detection)));
        if (!d) return;
        for (size_t i = 0; i < cands.size(); ++i) {
            d[i].class_id = cands[i].c;
            d[i].score = cands[i].s;
            float xy[4];
            to_xyxy(boxes + (size_t)cands[i].q * 4, img_w, img_h, xy);
            d[i].x1 = xy[0]; d[i].y1 = xy[1]; d[i].x2 = xy[2]; d[i].y2 = xy[3];
            if (masks && mask_w > 0 && mask_h > 0) {
                uint8_t* m = upsample_mask(masks + (size_t)cands[i].q * mask_w * mask_h, mask_w, mask_h, img_w,
                                           img_h, 0.5f);
                d[i].mask = m;
                d[i].mask_width = m ? img_w : 0;
                d[i].mask_height = m ? img_h : 0;
            }
        }
        *out = d;
        *out_n = cands.size();
    } catch (const std::bad_alloc&) {
        *out = nullptr;
        *out_n = 0;
    }
}

}  // namespace rfb

extern "C" void rfdetr_detections_free(rfdetr_detection* dets, size_t n) {
    if (!dets) return;
    for (size_t i = 0; i < n; ++i)
        if (dets[i].mask) std::free(const_cast<uint8_t*>(dets[i].mask));
    std::free(dets);
}
