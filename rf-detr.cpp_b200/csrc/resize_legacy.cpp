// Taps of the legacy preprocess resize, restated from the published algorithm
// of stb_image_resize2 v2.18 for a whole-image resize (no sub-region, pixel
// shift 0), one axis at a time:
//  * scale = out / in (double, then float), inv_scale = float(1 / scale);
//  * an axis that keeps its size is a copy (point sampling); a growing axis
//    uses Catmull-Rom (support 2 output pixels), a shrinking axis Mitchell
//    (support 2 / scale input pixels, weights times scale);
//  * raw weights: growing - output pixel o gathers the input pixels whose
//    centres lie within the filter radius of its centre mapped to the input;
//    shrinking - every input pixel, including a margin of width / 2 outside
//    the image, spreads weights onto the output pixels within its radius;
//    magnitudes below 2^-120 count as zero and leading zero weights are dropped;
//  * when scale is a rational num / den (to 2^-24) with num below the output
//    size, only the first num output pixels are computed and the others repeat
//    them shifted by den input pixels;
//  * each pixel's weights are divided by their sum (in double) unless that is
//    exactly 1;
//  * clamped edges: weights of pixels past the right edge are added to the
//    last pixel's (right edge first), then those of pixels left of the left
//    edge to the first pixel's, in the library's order; trailing zero weights
//    are trimmed.
// The float operations are those of the library in the same order, so the
// taps match it; the kernel's sums may differ from the library's SIMD order in
// the last bit, which moves an output byte by one only when a value lies within
// rounding of a half.
#include "resize_legacy.hpp"

#include <cmath>
#include <cstdint>
#include <cstring>

namespace rfb {

namespace {

const float kTiny = (float)1 / (1 << 20) / (1 << 20) / (1 << 20) / (1 << 20) / (1 << 20) / (1 << 20);

// Catmull-Rom (B = 0, C = 1/2) and Mitchell-Netravali (B = C = 1/3) cubics, support 2.
float cubic(bool catmull_rom, float x) {
    if (x < 0.0f) x = -x;
    if (catmull_rom) {
        if (x < 1.0f) return 1.0f - x * x * (2.5f - 1.5f * x);
        if (x < 2.0f) return 2.0f - x * (4.0f + x * (0.5f * x - 2.5f));
        return 0.0f;
    }
    if (x < 1.0f) return (16.0f + x * x * (21.0f * x - 36.0f)) / 18.0f;
    if (x < 2.0f) return (32.0f + x * (-60.0f + x * (36.0f - 7.0f * x))) / 18.0f;
    return 0.0f;
}

// num / den approximating f by continued-fraction convergents of f * 2^25 / 2^25,
// stopping when the error is below 2^-24 or the limited term (den when
// limit_den, else num) reaches `limit`, then falling back to the full-range
// estimate; true when the result is within 2^-24 of f.
bool rational(double f, uint32_t limit, bool limit_den, uint32_t* num, uint32_t* den) {
    uint64_t top = (uint64_t)(f * (double)(1 << 25)), bot = 1 << 25;
    uint64_t n_prev = 0, d_prev = 1, n_est = 1, d_est = 0;
    const double tol = 1.0 / (double)(1 << 24);
    for (;;) {
        if ((limit_den ? d_est : n_est) >= limit) break;
        if (d_est) {
            const double err = std::fabs((double)n_est / (double)d_est - f);
            if (err < tol) {
                *num = (uint32_t)n_est;
                *den = (uint32_t)d_est;
                return true;
            }
        }
        if (bot == 0) break;
        const uint64_t q = top / bot, r = top % bot;
        top = bot;
        bot = r;
        uint64_t t = q * d_est + d_prev;
        d_prev = d_est;
        d_est = t;
        t = q * n_est + n_prev;
        n_prev = n_est;
        n_est = t;
    }
    if (limit_den) {
        n_est = (uint64_t)(f * (double)limit + 0.5);
        d_est = limit;
    } else {
        n_est = limit;
        d_est = (uint64_t)((double)limit / f + 0.5);
    }
    *num = (uint32_t)n_est;
    *den = (uint32_t)d_est;
    const double err = d_est ? std::fabs((double)(uint32_t)n_est / (double)(uint32_t)d_est - f) : 1.0;
    return err < tol;
}

// Add weight w of input pixel p to the tap list [n0, n1] of one output pixel
// (c[k] belongs to pixel n0 + k): accumulated when p is inside the list,
// otherwise the list grows to reach p if it stays within `width` taps (the
// weight is dropped when it would not).
void add_tap(int& n0, int& n1, float* c, int p, float w, int width) {
    if (n1 < n0) {
        n0 = n1 = p;
        c[0] = w;
    } else if (p <= n1) {
        if (p >= n0) {
            c[p - n0] += w;
        } else if (n1 - p + 1 <= width) {
            const int o = n0 - p;
            for (int j = n1 - n0; j >= 0; --j) c[j + o] = c[j];
            for (int j = 1; j < o; ++j) c[j] = 0.0f;
            c[0] = w;
            n0 = p;
        }
    } else if (p - n0 + 1 <= width) {
        const int e = p - n0;
        for (int j = n1 - n0 + 1; j < e; ++j) c[j] = 0.0f;
        c[e] = w;
        n1 = p;
    }
}

}  // namespace

ResizeTaps legacy_resize_taps(int in, int out) {
    ResizeTaps t;
    t.in = in;
    t.out = out;
    t.first.assign((size_t)out, 0);
    t.count.assign((size_t)out, 0);
    if (in <= 0 || out <= 0) return t;
    if (in == out) {
        t.width = 1;
        t.coef.assign((size_t)out, 1.0f);
        for (int o = 0; o < out; ++o) {
            t.first[o] = o;
            t.count[o] = 1;
        }
        return t;
    }
    const double scale_d = (double)out / (double)in;
    const float scale = (float)scale_d, inv_scale = (float)(1.0 / scale_d);
    const bool up = scale >= 1.0f - kTiny;
    const float support = 2.0f;
    const int width = up ? (int)std::ceil(support * 2.0f) : (int)std::ceil(support * 2.0f / scale);
    uint32_t num = 0, den = 0;
    const bool rat = rational(scale_d, scale_d <= 1.0 ? (uint32_t)out : (uint32_t)in, scale_d >= 1.0, &num, &den);
    const bool poly = rat && num < (uint32_t)out;
    const int computed = poly ? (int)num : out;

    std::vector<int> n0((size_t)out, 0), n1((size_t)out, -1);
    std::vector<float> c((size_t)out * width, 0.0f);
    if (up) {
        const float radius = support * scale;  // in output pixels
        for (int o = 0; o < computed; ++o) {
            const float oc = (float)o + 0.5f;
            const float ic = oc * inv_scale;
            int first = (int)std::floor((oc - radius) * inv_scale + 0.5f);
            int last = (int)std::floor((oc + radius) * inv_scale - 0.5f);
            if (last < first) last = first;
            if (last - first + 1 > width) last = first + width - 1;
            float* cc = &c[(size_t)o * width];
            int nonzero = -1;
            for (int i = 0; i <= last - first; ++i) {
                const float w = cubic(true, ic - ((float)(i + first) + 0.5f));
                if (w < kTiny && w > -kTiny) {
                    if (i == 0) {  // leading zero: the list starts one pixel later
                        ++first;
                        --i;
                        continue;
                    }
                    cc[i] = 0.0f;
                } else {
                    nonzero = i;
                    cc[i] = w;
                }
            }
            n0[o] = first;
            n1[o] = first + nonzero;
        }
    } else {
        const float radius = support * inv_scale;  // in input pixels
        const int margin = width / 2;
        int seen = -1;  // highest output pixel given a first weight so far
        for (int p = -margin; p < in + margin; ++p) {
            const float pc = (float)p + 0.5f;
            const float oc_of_in = pc * scale;
            int ofirst = (int)std::floor((pc - radius) * scale + 0.5f);
            int olast = (int)std::floor((pc + radius) * scale - 0.5f);
            if (ofirst < 0) ofirst = 0;
            if (olast >= out) olast = out - 1;
            if (ofirst > olast) continue;
            if (poly) {
                if (ofirst == (int)num) break;
                if (olast >= (int)num) olast = (int)num - 1;
            }
            for (int o = ofirst; o <= olast; ++o) {
                float w = cubic(false, ((float)o + 0.5f) - oc_of_in) * scale;
                if (w < kTiny && w > -kTiny) w = 0.0f;
                float* cc = &c[(size_t)o * width];
                if (o > seen) {
                    seen = o;
                    n0[o] = n1[o] = p;
                    cc[0] = w;
                } else {
                    if (cc[0] == 0.0f) n0[o] = p;  // a zero first weight is dropped
                    n1[o] = p;
                    if (p - n0[o] < width) cc[p - n0[o]] = w;
                }
            }
        }
    }
    for (int o = 0; o < computed; ++o) {
        float* cc = &c[(size_t)o * width];
        double total = 0.0;
        for (int k = 0; k <= n1[o] - n0[o]; ++k) total += (double)cc[k];
        if (total < kTiny && total > -kTiny) {
            n1[o] = n0[o];
            cc[0] = 0.0f;
        } else if (total != 1.0) {
            const double s = 1.0 / total;
            for (int k = 0; k <= n1[o] - n0[o]; ++k) cc[k] = (float)((double)cc[k] * s);
        }
    }
    for (int o = computed; o < out; ++o) {
        n0[o] = n0[o - computed] + (int)den;
        n1[o] = n1[o - computed] + (int)den;
        std::memcpy(&c[(size_t)o * width], &c[(size_t)(o - computed) * width], sizeof(float) * width);
    }
    const int last_in = in - 1;
    for (int o = 0; o < out; ++o) {
        float* cc = &c[(size_t)o * width];
        int& a = n0[o];
        int& b = n1[o];
        if (b > last_in) {  // right edge: onto the last pixel, in pixel order
            const int start = a, end = b;
            b = last_in;
            for (int i = in; i <= end; ++i) add_tap(a, b, cc, last_in, cc[i - start], width);
        }
        if (a < 0) {  // left edge: pixels -1 .. a+1 onto the first pixel, then pixel a
            for (int i = -1; i > a; --i) add_tap(a, b, cc, 0, cc[i - a], width);
            const int save_n0 = a;
            const float save_w = cc[0];
            a = 0;
            for (int i = 0; i <= b; ++i) cc[i] = cc[i - save_n0];
            add_tap(a, b, cc, 0, save_w, width);
        }
        int n = 0;
        if (a <= b) {
            n = b - a + 1;
            while (n && cc[n - 1] == 0.0f) --n;
            for (int k = n; k < width; ++k) cc[k] = 0.0f;
        }
        if (a < 0 || a + n - 1 > last_in) n = 0;  // never reads outside the image
        t.first[o] = a;
        t.count[o] = n;
    }
    t.width = width;
    t.coef = std::move(c);
    return t;
}

cudaError_t upload_legacy_taps(int w, int h, int ow, int oh, LegacyTapsDev* out) {
    *out = LegacyTapsDev{};
    if (w <= 0 || h <= 0 || ow <= 0 || oh <= 0) return cudaErrorInvalidValue;
    const ResizeTaps tx = legacy_resize_taps(w, ow), ty = legacy_resize_taps(h, oh);
    // [xf | xn | yf | yn] ints, then [xc | yc] floats
    std::vector<int32_t> ints;
    ints.insert(ints.end(), tx.first.begin(), tx.first.end());
    ints.insert(ints.end(), tx.count.begin(), tx.count.end());
    ints.insert(ints.end(), ty.first.begin(), ty.first.end());
    ints.insert(ints.end(), ty.count.begin(), ty.count.end());
    const size_t ib = ints.size() * 4, xb = tx.coef.size() * 4, yb = ty.coef.size() * 4;
    void* base = nullptr;
    cudaError_t e = cudaMalloc(&base, ib + xb + yb);
    if (e != cudaSuccess) return e;
    char* p = static_cast<char*>(base);
    if ((e = cudaMemcpy(p, ints.data(), ib, cudaMemcpyHostToDevice)) != cudaSuccess ||
        (e = cudaMemcpy(p + ib, tx.coef.data(), xb, cudaMemcpyHostToDevice)) != cudaSuccess ||
        (e = cudaMemcpy(p + ib + xb, ty.coef.data(), yb, cudaMemcpyHostToDevice)) != cudaSuccess) {
        cudaFree(base);
        return e;
    }
    const int* ip = reinterpret_cast<const int*>(p);
    out->base = base;
    out->xf = ip;
    out->xn = ip + ow;
    out->yf = ip + 2 * ow;
    out->yn = ip + 2 * ow + oh;
    out->xc = reinterpret_cast<const float*>(p + ib);
    out->xw = tx.width;
    out->yc = reinterpret_cast<const float*>(p + ib + xb);
    out->yw = ty.width;
    return cudaSuccess;
}

}  // namespace rfb
