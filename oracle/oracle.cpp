/* CPU oracle for the RF-DETR forward pass — TEST INFRASTRUCTURE ONLY.
 * See oracle.h for the contract.  Every function cites the reference
 * (localai-org/rf-detr.cpp) lines it restates.  Internal layout is
 * token-major: a (C, T) ggml tensor of the reference is stored here as
 * T rows of C floats, which is the same memory order. */
#include "oracle.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <numeric>
#include <string>
#include <unordered_map>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

using Vec = std::vector<float>;

struct W {
    const float* p = nullptr;
    int64_t n = 0;
    int type = ORACLE_F32;
};

struct Ctx {
    const OracleConfig* cfg;
    std::unordered_map<std::string, W> w;
    oracle_publish_cb pub;
    void* user;
    bool missing = false;

    const W& get(const std::string& name) {
        static W empty;
        auto it = w.find(name);
        if (it == w.end()) {
            std::fprintf(stderr, "oracle: missing tensor '%s'\n", name.c_str());
            missing = true;
            return empty;
        }
        return it->second;
    }
    void publish(const std::string& name, const Vec& v) {
        if (pub) pub(name.c_str(), v.data(), (int64_t)v.size(), user);
    }
};

/* ---- activation rounding (mode 1) ---------------------------------------- */

inline float to_f16_and_back(float x) { return (float)(_Float16)x; }

void round_row(float* x, int K, int wtype) {
    if (wtype == ORACLE_F16) {
        for (int k = 0; k < K; ++k) x[k] = to_f16_and_back(x[k]);
    } else if (wtype == ORACLE_Q8_0) {
        /* ggml quantize_row_q8_0: 32-element blocks, d = amax/127 stored f16. */
        for (int b = 0; b + 32 <= K; b += 32) {
            float amax = 0.f;
            for (int j = 0; j < 32; ++j) amax = std::max(amax, std::fabs(x[b + j]));
            const float d = amax / 127.f;
            const float id = d != 0.f ? 1.f / d : 0.f;
            const float dh = to_f16_and_back(d);
            for (int j = 0; j < 32; ++j) x[b + j] = dh * std::nearbyint(x[b + j] * id);
        }
    } else if (wtype == ORACLE_Q4_K) {
        /* ggml quantize_row_q8_K_ref: 256-element blocks, signed max. */
        for (int b = 0; b + 256 <= K; b += 256) {
            float amax = 0.f, mx = 0.f;
            for (int j = 0; j < 256; ++j) {
                const float ax = std::fabs(x[b + j]);
                if (ax > amax) { amax = ax; mx = x[b + j]; }
            }
            if (amax == 0.f) { for (int j = 0; j < 256; ++j) x[b + j] = 0.f; continue; }
            const float iscale = -127.f / mx;
            const float d = 1.f / iscale;
            for (int j = 0; j < 256; ++j) {
                int v = (int)std::nearbyint(iscale * x[b + j]);
                v = std::min(127, v);
                x[b + j] = d * (float)v;
            }
        }
    }
}

/* ---- dense linear: Y[m][n] = sum_k X[m][k] W[n][k] + b[n] ---------------- */

void linear(Ctx& c, const float* X, int M, int K, const W& Wt, const float* bias, int N, float* Y) {
    const float* Wp = Wt.p;
    const bool rnd = c.cfg->act_round && Wt.type != ORACLE_F32;
    Vec Xr;
    if (rnd) {
        Xr.assign(X, X + (size_t)M * K);
        #pragma omp parallel for schedule(static)
        for (int m = 0; m < M; ++m) round_row(Xr.data() + (size_t)m * K, K, Wt.type);
        X = Xr.data();
    }
    const int MB = 4, NB = 4;
    #pragma omp parallel for schedule(dynamic, 4) collapse(2)
    for (int m0 = 0; m0 < M; m0 += MB) {
        for (int n0 = 0; n0 < N; n0 += NB) {
            const int mc = std::min(MB, M - m0), nc = std::min(NB, N - n0);
            if (mc == MB && nc == NB) {
                const float* x0 = X + (size_t)(m0 + 0) * K; const float* x1 = X + (size_t)(m0 + 1) * K;
                const float* x2 = X + (size_t)(m0 + 2) * K; const float* x3 = X + (size_t)(m0 + 3) * K;
                const float* w0 = Wp + (size_t)(n0 + 0) * K; const float* w1 = Wp + (size_t)(n0 + 1) * K;
                const float* w2 = Wp + (size_t)(n0 + 2) * K; const float* w3 = Wp + (size_t)(n0 + 3) * K;
                float a00 = 0, a01 = 0, a02 = 0, a03 = 0, a10 = 0, a11 = 0, a12 = 0, a13 = 0;
                float a20 = 0, a21 = 0, a22 = 0, a23 = 0, a30 = 0, a31 = 0, a32 = 0, a33 = 0;
                #pragma omp simd reduction(+:a00,a01,a02,a03,a10,a11,a12,a13,a20,a21,a22,a23,a30,a31,a32,a33)
                for (int k = 0; k < K; ++k) {
                    const float v0 = x0[k], v1 = x1[k], v2 = x2[k], v3 = x3[k];
                    const float u0 = w0[k], u1 = w1[k], u2 = w2[k], u3 = w3[k];
                    a00 += v0 * u0; a01 += v0 * u1; a02 += v0 * u2; a03 += v0 * u3;
                    a10 += v1 * u0; a11 += v1 * u1; a12 += v1 * u2; a13 += v1 * u3;
                    a20 += v2 * u0; a21 += v2 * u1; a22 += v2 * u2; a23 += v2 * u3;
                    a30 += v3 * u0; a31 += v3 * u1; a32 += v3 * u2; a33 += v3 * u3;
                }
                float acc[4][4] = {{a00, a01, a02, a03}, {a10, a11, a12, a13},
                                   {a20, a21, a22, a23}, {a30, a31, a32, a33}};
                for (int i = 0; i < 4; ++i)
                    for (int j = 0; j < 4; ++j)
                        Y[(size_t)(m0 + i) * N + n0 + j] = acc[i][j] + (bias ? bias[n0 + j] : 0.f);
            } else {
                for (int i = 0; i < mc; ++i) {
                    for (int j = 0; j < nc; ++j) {
                        const float* xr = X + (size_t)(m0 + i) * K;
                        const float* wr = Wp + (size_t)(n0 + j) * K;
                        float a = 0.f;
                        #pragma omp simd reduction(+:a)
                        for (int k = 0; k < K; ++k) a += xr[k] * wr[k];
                        Y[(size_t)(m0 + i) * N + n0 + j] = a + (bias ? bias[n0 + j] : 0.f);
                    }
                }
            }
        }
    }
}

Vec linear_v(Ctx& c, const Vec& X, int M, int K, const std::string& prefix, int N) {
    const W& Wt = c.get(prefix + ".weight");
    const W& B = c.get(prefix + ".bias");
    Vec Y((size_t)M * N);
    if (c.missing) return Y;
    linear(c, X.data(), M, K, Wt, B.p, N, Y.data());
    return Y;
}

/* ggml_norm (mean/variance accumulated in double) then * w + b. */
void layer_norm_rows(float* X, int M, int C, const float* g, const float* b, float eps) {
    #pragma omp parallel for schedule(static)
    for (int m = 0; m < M; ++m) {
        float* x = X + (size_t)m * C;
        double s = 0.0;
        for (int i = 0; i < C; ++i) s += x[i];
        const float mean = (float)(s / C);
        double s2 = 0.0;
        for (int i = 0; i < C; ++i) { const float v = x[i] - mean; x[i] = v; s2 += (double)(v * v); }
        const float var = (float)(s2 / C);
        const float sc = 1.0f / std::sqrt(var + eps);
        for (int i = 0; i < C; ++i) x[i] = x[i] * sc * g[i] + b[i];
    }
}

void layer_norm_named(Ctx& c, Vec& X, int M, int C, const std::string& prefix, float eps) {
    const W& g = c.get(prefix + ".weight");
    const W& b = c.get(prefix + ".bias");
    if (c.missing) return;
    layer_norm_rows(X.data(), M, C, g.p, b.p, eps);
}

inline float gelu_erf(float x) { return 0.5f * x * (1.0f + std::erf(x * 0.70710678118654752440f)); }
inline float silu(float x) { return x / (1.0f + std::exp(-x)); }

/* Softmax over a row (ggml_soft_max: f32 max, double sum, scale by 1/sum). */
void softmax_row(float* x, int n) {
    float mx = -INFINITY;
    for (int i = 0; i < n; ++i) mx = std::max(mx, x[i]);
    double s = 0.0;
    for (int i = 0; i < n; ++i) { const float e = std::exp(x[i] - mx); x[i] = e; s += e; }
    const float inv = (float)(1.0 / s);
    for (int i = 0; i < n; ++i) x[i] *= inv;
}

/* Multi-head attention over groups of T tokens.  q/k/v are [G*T][D] with
 * heads packed (h*hd + d).  If prescale, q is multiplied by 1/sqrt(hd)
 * before the dot product (src/dinov2.cpp:67-72); otherwise the logits are
 * scaled (src/decoder.cpp:88-90). */
void mha(const float* q, const float* k, const float* v, float* out, int G, int T, int D, int H,
         bool prescale) {
    const int hd = D / H;
    const float scale = 1.0f / std::sqrt((float)hd);
    #pragma omp parallel
    {
        Vec logits(T), qv(hd);
        #pragma omp for collapse(3) schedule(dynamic, 8)
        for (int g = 0; g < G; ++g) {
            for (int h = 0; h < H; ++h) {
                for (int i = 0; i < T; ++i) {
                    const float* qi = q + ((size_t)g * T + i) * D + h * hd;
                    for (int d = 0; d < hd; ++d) qv[d] = prescale ? qi[d] * scale : qi[d];
                    for (int j = 0; j < T; ++j) {
                        const float* kj = k + ((size_t)g * T + j) * D + h * hd;
                        float a = 0.f;
                        #pragma omp simd reduction(+:a)
                        for (int d = 0; d < hd; ++d) a += kj[d] * qv[d];
                        logits[j] = prescale ? a : a * scale;
                    }
                    softmax_row(logits.data(), T);
                    float* o = out + ((size_t)g * T + i) * D + h * hd;
                    for (int d = 0; d < hd; ++d) o[d] = 0.f;
                    for (int j = 0; j < T; ++j) {
                        const float* vj = v + ((size_t)g * T + j) * D + h * hd;
                        const float p = logits[j];
                        #pragma omp simd
                        for (int d = 0; d < hd; ++d) o[d] += p * vj[d];
                    }
                }
            }
        }
    }
}

/* ---- bicubic pos-embed resample: src/model_loader.cpp:117-208 ----------- */

void bicubic_resample(const float* src, int src_side, int dim, float* dst, int dst_side) {
    constexpr float A = -0.5f;
    auto kern = [](float x) -> float {
        const float ax = std::fabs(x);
        if (ax < 1.0f) return ((A + 2.0f) * ax - (A + 3.0f)) * ax * ax + 1.0f;
        if (ax < 2.0f) return ((A * ax - 5.0f * A) * ax + 8.0f * A) * ax - 4.0f * A;
        return 0.0f;
    };
    const float scale = (float)src_side / (float)dst_side;
    const float invscale = scale >= 1.0f ? 1.0f / scale : 1.0f;
    const float support = scale >= 1.0f ? 2.0f * scale : 2.0f;
    const int max_taps = (int)std::ceil(support) * 2 + 1;
    std::vector<float> wt((size_t)dst_side * max_taps, 0.f);
    std::vector<int> ix((size_t)dst_side * max_taps, 0), cnt(dst_side, 0);
    for (int o = 0; o < dst_side; ++o) {
        const float center = scale * ((float)o + 0.5f);
        const int xmin = std::max((int)(center - support + 0.5f), 0);
        const int xmax = std::min((int)(center + support + 0.5f), src_side);
        const int n = std::min(std::max(xmax - xmin, 0), max_taps);
        float total = 0.f;
        for (int j = 0; j < n; ++j) {
            const float w = kern(((float)j + (float)xmin - center + 0.5f) * invscale);
            wt[(size_t)o * max_taps + j] = w;
            ix[(size_t)o * max_taps + j] = xmin + j;
            total += w;
        }
        if (total != 0.f)
            for (int j = 0; j < n; ++j) wt[(size_t)o * max_taps + j] /= total;
        cnt[o] = n;
    }
    for (int oy = 0; oy < dst_side; ++oy) {
        for (int ox = 0; ox < dst_side; ++ox) {
            float* d = dst + ((size_t)oy * dst_side + ox) * dim;
            for (int i = 0; i < dim; ++i) d[i] = 0.f;
            for (int ky = 0; ky < cnt[oy]; ++ky) {
                const float wy = wt[(size_t)oy * max_taps + ky];
                if (wy == 0.f) continue;
                const int sy = ix[(size_t)oy * max_taps + ky];
                for (int kx = 0; kx < cnt[ox]; ++kx) {
                    const float wx = wt[(size_t)ox * max_taps + kx];
                    if (wx == 0.f) continue;
                    const int sx = ix[(size_t)ox * max_taps + kx];
                    const float w = wx * wy;
                    const float* s = src + ((size_t)sy * src_side + sx) * dim;
                    for (int i = 0; i < dim; ++i) d[i] += w * s[i];
                }
            }
        }
    }
}

/* ---- 2-D convolution in token-major layout ------------------------------- *
 * X: [H*W][IC], weight torch (OC, IC, k, k), stride 1, pad k/2, no bias.     */
Vec conv2d_same(Ctx& c, const Vec& X, int H, int Wd, int IC, const W& Wt, int OC, int k) {
    const int M = H * Wd;
    if (k == 1) {
        Vec Y((size_t)M * OC);
        linear(c, X.data(), M, IC, Wt, nullptr, OC, Y.data());
        return Y;
    }
    /* im2col with K ordered (ic, ky, kx) to match the torch weight layout. */
    const int K = IC * k * k, p = k / 2;
    Vec col((size_t)M * K, 0.f);
    #pragma omp parallel for schedule(static)
    for (int y = 0; y < H; ++y) {
        for (int x = 0; x < Wd; ++x) {
            float* r = col.data() + ((size_t)y * Wd + x) * K;
            for (int ic = 0; ic < IC; ++ic)
                for (int ky = 0; ky < k; ++ky)
                    for (int kx = 0; kx < k; ++kx) {
                        const int sy = y + ky - p, sx = x + kx - p;
                        r[(ic * k + ky) * k + kx] =
                            (sy < 0 || sy >= H || sx < 0 || sx >= Wd) ? 0.f : X[((size_t)sy * Wd + sx) * IC + ic];
                    }
        }
    }
    Vec Y((size_t)M * OC);
    linear(c, col.data(), M, K, Wt, nullptr, OC, Y.data());
    return Y;
}

/* ConvX = conv (no bias) -> channel LN (1e-6) -> SiLU (src/projector.cpp:46-59). */
Vec convx(Ctx& c, const Vec& X, int H, int Wd, int IC, const std::string& prefix, int OC, int k) {
    const W& Wt = c.get(prefix + ".conv.weight");
    if (c.missing) return Vec();
    Vec Y = conv2d_same(c, X, H, Wd, IC, Wt, OC, k);
    layer_norm_named(c, Y, H * Wd, OC, prefix + ".norm", 1e-6f);
    for (auto& v : Y) v = silu(v);
    return Y;
}

/* ---- backbone: src/dinov2.cpp:314-556 ------------------------------------ */

struct BackboneOut { std::vector<Vec> taps; };

BackboneOut backbone(Ctx& c, const float* img) {
    const OracleConfig& k = *c.cfg;
    const int D = k.dim, S = k.image_size, p = k.patch_size, G = S / p, nw = k.num_windows;
    const int ws = G / nw, Tp = ws * ws, T = Tp + 1, NW = nw * nw, Ntok = NW * T;
    BackboneOut out;
    out.taps.resize(k.n_taps);

    /* Patch embed (conv k = s = patch) -> tokens t = gy*G + gx. */
    const W& pw = c.get("backbone.patch_embed.weight");
    const W& pb = c.get("backbone.patch_embed.bias");
    const W& cls = c.get("backbone.cls_token");
    const W& pe = c.get("backbone.pos_embed");
    if (c.missing) return out;
    const int K = 3 * p * p;
    Vec col((size_t)G * G * K);
    for (int gy = 0; gy < G; ++gy)
        for (int gx = 0; gx < G; ++gx) {
            float* r = col.data() + ((size_t)gy * G + gx) * K;
            for (int ch = 0; ch < 3; ++ch)
                for (int ky = 0; ky < p; ++ky)
                    for (int kx = 0; kx < p; ++kx)
                        r[(ch * p + ky) * p + kx] = img[((size_t)ch * S + gy * p + ky) * S + gx * p + kx];
        }
    Vec emb((size_t)G * G * D);
    linear(c, col.data(), G * G, K, pw, pb.p, D, emb.data());

    /* Bicubic pos-embed for the inference grid (CLS row copied). */
    const int ts = k.pos_train;
    Vec pos((size_t)(G * G + 1) * D);
    std::memcpy(pos.data(), pe.p, sizeof(float) * D);
    if (ts == G) std::memcpy(pos.data() + D, pe.p + D, sizeof(float) * (size_t)G * G * D);
    else bicubic_resample(pe.p + D, ts, D, pos.data() + D, G);

    /* Window partition + CLS per window + pos add (src/dinov2.cpp:146-201,268-301,390-408). */
    Vec x((size_t)Ntok * D);
    for (int wy = 0; wy < nw; ++wy)
        for (int wx = 0; wx < nw; ++wx) {
            const int win = wy * nw + wx;
            float* r0 = x.data() + (size_t)win * T * D;
            for (int d = 0; d < D; ++d) r0[d] = cls.p[d] + pos[d];
            for (int iy = 0; iy < ws; ++iy)
                for (int ix = 0; ix < ws; ++ix) {
                    const int gy = wy * ws + iy, gx = wx * ws + ix, t = gy * G + gx;
                    float* r = x.data() + ((size_t)win * T + 1 + iy * ws + ix) * D;
                    for (int d = 0; d < D; ++d) r[d] = emb[(size_t)t * D + d] + pos[(size_t)(1 + t) * D + d];
                }
        }
    c.publish("backbone.patch_embed.output", x);

    for (int i = 0; i < k.depth; ++i) {
        const std::string b = "backbone.blocks." + std::to_string(i) + ".";
        bool windowed = true;
        for (int j = 0; j < k.n_global; ++j) if (k.global_idx[j] == i) windowed = false;

        Vec h = x;
        layer_norm_named(c, h, Ntok, D, b + "norm1", 1e-6f);
        Vec q = linear_v(c, h, Ntok, D, b + "attn.q", D);
        Vec kk = linear_v(c, h, Ntok, D, b + "attn.k", D);
        Vec v = linear_v(c, h, Ntok, D, b + "attn.v", D);
        if (c.missing) return out;
        Vec a((size_t)Ntok * D);
        if (windowed) mha(q.data(), kk.data(), v.data(), a.data(), NW, T, D, k.heads, true);
        else mha(q.data(), kk.data(), v.data(), a.data(), 1, Ntok, D, k.heads, true);
        Vec o = linear_v(c, a, Ntok, D, b + "attn.proj", D);
        const W& ls1 = c.get(b + "layer_scale1");
        const W& ls2 = c.get(b + "layer_scale2");
        if (c.missing) return out;
        for (size_t t = 0; t < (size_t)Ntok; ++t)
            for (int d = 0; d < D; ++d) x[t * D + d] += o[t * D + d] * ls1.p[d];
        Vec y = x;
        layer_norm_named(c, y, Ntok, D, b + "norm2", 1e-6f);
        Vec f1 = linear_v(c, y, Ntok, D, b + "mlp.fc1", k.ffn_dim);
        for (auto& e : f1) e = gelu_erf(e);
        Vec f2 = linear_v(c, f1, Ntok, k.ffn_dim, b + "mlp.fc2", D);
        if (c.missing) return out;
        for (size_t t = 0; t < (size_t)Ntok; ++t)
            for (int d = 0; d < D; ++d) x[t * D + d] += f2[t * D + d] * ls2.p[d];
        c.publish("backbone.block." + std::to_string(i) + ".output", x);

        int level = -1;
        for (int j = 0; j < k.n_taps; ++j) if (k.tap_stage[j] == i + 1) level = j;
        if (level >= 0) {
            Vec n = x;
            layer_norm_named(c, n, Ntok, D, "backbone.norm", 1e-6f);
            /* strip CLS, un-window -> [G*G][D] row-major (gy, gx) */
            Vec sp((size_t)G * G * D);
            for (int wy = 0; wy < nw; ++wy)
                for (int wx = 0; wx < nw; ++wx)
                    for (int iy = 0; iy < ws; ++iy)
                        for (int ix = 0; ix < ws; ++ix) {
                            const int win = wy * nw + wx, gy = wy * ws + iy, gx = wx * ws + ix;
                            std::memcpy(sp.data() + ((size_t)gy * G + gx) * D,
                                        n.data() + ((size_t)win * T + 1 + iy * ws + ix) * D, sizeof(float) * D);
                        }
            c.publish("backbone.multiscale.level" + std::to_string(level), sp);
            out.taps[level] = std::move(sp);
        }
    }
    return out;
}

/* ---- projector: src/projector.cpp:85-189 (token-major [G*G][C]) ---------- */

Vec projector(Ctx& c, const BackboneOut& bb) {
    const OracleConfig& k = *c.cfg;
    const int G = k.image_size / k.patch_size, D = k.dim, L = k.n_taps, C = k.proj_out, cb = C / 2;
    const int M = G * G;
    Vec x((size_t)M * L * D);
    for (int m = 0; m < M; ++m)
        for (int l = 0; l < L; ++l)
            std::memcpy(x.data() + ((size_t)m * L + l) * D, bb.taps[l].data() + (size_t)m * D, sizeof(float) * D);
    Vec h = convx(c, x, G, G, L * D, "projector.cv1", C, 1);
    if (c.missing) return Vec();
    c.publish("projector.cv1.output", h);
    std::vector<Vec> parts;
    Vec y0((size_t)M * cb), y1((size_t)M * cb);
    for (int m = 0; m < M; ++m) {
        std::memcpy(y0.data() + (size_t)m * cb, h.data() + (size_t)m * C, sizeof(float) * cb);
        std::memcpy(y1.data() + (size_t)m * cb, h.data() + (size_t)m * C + cb, sizeof(float) * cb);
    }
    parts.push_back(y0);
    parts.push_back(y1);
    Vec cur = y1;
    for (int j = 0; j < k.proj_nb; ++j) {
        const std::string p = "projector.bottleneck." + std::to_string(j) + ".";
        cur = convx(c, cur, G, G, cb, p + "cv1", cb, 3);
        if (c.missing) return Vec();
        cur = convx(c, cur, G, G, cb, p + "cv2", cb, 3);
        if (c.missing) return Vec();
        c.publish("projector.bottleneck." + std::to_string(j) + ".output", cur);
        parts.push_back(cur);
    }
    const int CC = (int)parts.size() * cb;
    Vec cat((size_t)M * CC);
    for (int m = 0; m < M; ++m)
        for (size_t pi = 0; pi < parts.size(); ++pi)
            std::memcpy(cat.data() + (size_t)m * CC + pi * cb, parts[pi].data() + (size_t)m * cb, sizeof(float) * cb);
    Vec o = convx(c, cat, G, G, CC, "projector.cv2", C, 1);
    if (c.missing) return Vec();
    c.publish("projector.cv2.output", o);
    layer_norm_named(c, o, M, C, "projector.final_norm", 1e-6f);
    c.publish("projector.output", o);
    return o;
}

/* src/two_stage.cpp:34-89 */
void proposal_grid(int G, float wh, float* out) {
    for (int h = 0; h < G; ++h)
        for (int w = 0; w < G; ++w) {
            float* p = out + ((size_t)h * G + w) * 4;
            p[0] = ((float)w + 0.5f) / (float)G;
            p[1] = ((float)h + 0.5f) / (float)G;
            p[2] = wh;
            p[3] = wh;
            bool valid = true;
            for (int i = 0; i < 4; ++i) if (!(p[i] > 0.01f && p[i] < 0.99f)) valid = false;
            if (!valid) p[0] = p[1] = p[2] = p[3] = 0.f;
        }
}

/* src/decoder.cpp:383-417 */
void sine_embed(const float* rp, int NQ, int d_half, float* out) {
    const float TWO_PI = 6.28318530717958647692f;
    std::vector<float> inv((size_t)d_half);
    for (int kk = 0; kk < d_half; ++kk)
        inv[kk] = std::exp(-std::log(10000.0f) * (float)((kk / 2) * 2) / (float)d_half);
    const int comp[4] = {1, 0, 2, 3};
    for (int q = 0; q < NQ; ++q)
        for (int ci = 0; ci < 4; ++ci) {
            const float v = rp[q * 4 + comp[ci]] * TWO_PI;
            float* o = out + (size_t)q * 4 * d_half + (size_t)ci * d_half;
            for (int kk = 0; kk < d_half; kk += 2) {
                const float arg = v * inv[kk];
                o[kk] = std::sin(arg);
                o[kk + 1] = std::cos(arg);
            }
        }
}

}  // namespace

extern "C" void oracle_bicubic_resample(const float* src, int src_side, int dim, float* dst, int dst_side) {
    bicubic_resample(src, src_side, dim, dst, dst_side);
}


extern "C" int oracle_forward(const OracleConfig* cfg, const OracleTensor* tensors, int n_tensors,
                              const float* input, const int32_t* force_topk, float* out_logits, float* out_boxes,
                              int32_t* out_topk, float* out_masks,
                              oracle_publish_cb publish, void* user) {
#ifdef _OPENMP
    if (cfg->n_threads > 0) omp_set_num_threads(cfg->n_threads);
#endif
    Ctx c;
    c.cfg = cfg;
    c.pub = publish;
    c.user = user;
    for (int i = 0; i < n_tensors; ++i) c.w[tensors[i].name] = W{tensors[i].data, tensors[i].n, tensors[i].type};
    const OracleConfig& k = *cfg;
    const int G = k.image_size / k.patch_size, N = G * G;
    const int Dm = k.dec_dim, NQ = k.num_queries, NC = k.num_classes;
    if (G * k.patch_size != k.image_size || G % k.num_windows) return -2;
    if (NQ > N) return -2;

    BackboneOut bb = backbone(c, input);
    if (c.missing) return -7;
    Vec proj = projector(c, bb);
    if (c.missing) return -7;

    /* ---- two-stage (src/two_stage.cpp:91-236) ---- */
    Vec prop((size_t)N * 4);
    proposal_grid(G, 0.05f, prop.data());
    Vec tok = proj;
    for (int t = 0; t < N; ++t) {
        const float valid = prop[(size_t)t * 4 + 2] > 0.f ? 1.f : 0.f;
        for (int ch = 0; ch < Dm; ++ch) tok[(size_t)t * Dm + ch] *= valid;
    }
    Vec y = linear_v(c, tok, N, Dm, "two_stage.enc_output.0", Dm);
    layer_norm_named(c, y, N, Dm, "two_stage.enc_output_norm.0", 1e-5f);
    c.publish("two_stage.enc_output_norm.output", y);
    Vec cls_all = linear_v(c, y, N, Dm, "two_stage.enc_out_class_embed.0", NC);
    Vec hb = linear_v(c, y, N, Dm, "two_stage.enc_out_bbox_embed.0.layers.0", Dm);
    for (auto& e : hb) e = std::max(e, 0.f);
    hb = linear_v(c, hb, N, Dm, "two_stage.enc_out_bbox_embed.0.layers.1", Dm);
    for (auto& e : hb) e = std::max(e, 0.f);
    Vec delta = linear_v(c, hb, N, Dm, "two_stage.enc_out_bbox_embed.0.layers.2", 4);
    if (c.missing) return -7;
    Vec bbox_all((size_t)N * 4);
    for (int t = 0; t < N; ++t) {
        const float* d = &delta[(size_t)t * 4];
        const float* p = &prop[(size_t)t * 4];
        float* o = &bbox_all[(size_t)t * 4];
        o[0] = d[0] * p[2] + p[0];
        o[1] = d[1] * p[3] + p[1];
        o[2] = std::exp(d[2]) * p[2];
        o[3] = std::exp(d[3]) * p[3];
    }
    c.publish("two_stage.cls_all", cls_all);
    c.publish("two_stage.bbox_all", bbox_all);

    /* ---- top-K by per-token max class score (src/rfdetr_model.cpp:39-62).
     * partial_sort leaves the order of equal scores unspecified; ties are
     * broken here by the lower token index. */
    Vec mx(N);
    for (int t = 0; t < N; ++t) {
        const float* r = &cls_all[(size_t)t * NC];
        float m = r[0];
        for (int ci = 1; ci < NC; ++ci) if (r[ci] > m) m = r[ci];
        mx[t] = m;
    }
    std::vector<int> idx(N);
    std::iota(idx.begin(), idx.end(), 0);
    std::partial_sort(idx.begin(), idx.begin() + NQ, idx.end(), [&](int a, int b) {
        if (mx[a] != mx[b]) return mx[a] > mx[b];
        return a < b;
    });
    if (force_topk)
        for (int q = 0; q < NQ; ++q) {
            if (force_topk[q] < 0 || force_topk[q] >= N) return -1;
            idx[q] = force_topk[q];
        }
    if (out_topk) for (int q = 0; q < NQ; ++q) out_topk[q] = idx[q];

    /* ---- decoder inputs (src/rfdetr_model.cpp:233-271) ---- */
    const W& lrn = c.get("decoder.queries.refpoints");
    const W& feat = c.get("decoder.queries.feat");
    if (c.missing) return -7;
    Vec rp((size_t)NQ * 4);
    for (int q = 0; q < NQ; ++q) {
        const float* box = &bbox_all[(size_t)idx[q] * 4];
        const float* l = lrn.p + (size_t)q * 4;
        float* d = &rp[(size_t)q * 4];
        d[0] = l[0] * box[2] + box[0];
        d[1] = l[1] * box[3] + box[1];
        d[2] = std::exp(l[2]) * box[2];
        d[3] = std::exp(l[3]) * box[3];
    }
    c.publish("decoder.refpoints", rp);
    Vec sine((size_t)NQ * 2 * Dm);
    sine_embed(rp.data(), NQ, Dm / 2, sine.data());
    Vec qpos = linear_v(c, sine, NQ, 2 * Dm, "decoder.ref_point_head.layers.0", Dm);
    for (auto& e : qpos) e = std::max(e, 0.f);
    qpos = linear_v(c, qpos, NQ, Dm, "decoder.ref_point_head.layers.1", Dm);
    if (c.missing) return -7;
    c.publish("decoder.query_pos", qpos);

    Vec tgt(feat.p, feat.p + (size_t)NQ * Dm);
    const int nh = k.ca_heads, np_ = k.ca_points, chd = Dm / nh;
    std::vector<Vec> per_layer;
    for (int li = 0; li < k.dec_layers; ++li) {
        const std::string b = "decoder.layers." + std::to_string(li) + ".";
        const std::string pb = "decoder.layer." + std::to_string(li) + ".";
        /* self-attention (src/decoder.cpp:44-101, 340-349) */
        Vec qk_in(tgt.size());
        for (size_t i = 0; i < tgt.size(); ++i) qk_in[i] = tgt[i] + qpos[i];
        const W& ipw = c.get(b + "self_attn.in_proj.weight");
        const W& ipb = c.get(b + "self_attn.in_proj.bias");
        if (c.missing) return -7;
        Vec q((size_t)NQ * Dm), kk((size_t)NQ * Dm), v((size_t)NQ * Dm);
        W wq{ipw.p, (int64_t)Dm * Dm, ipw.type}, wk{ipw.p + (size_t)Dm * Dm, (int64_t)Dm * Dm, ipw.type},
            wv{ipw.p + (size_t)2 * Dm * Dm, (int64_t)Dm * Dm, ipw.type};
        linear(c, qk_in.data(), NQ, Dm, wq, ipb.p, Dm, q.data());
        linear(c, qk_in.data(), NQ, Dm, wk, ipb.p + Dm, Dm, kk.data());
        linear(c, tgt.data(), NQ, Dm, wv, ipb.p + 2 * Dm, Dm, v.data());
        Vec att((size_t)NQ * Dm);
        mha(q.data(), kk.data(), v.data(), att.data(), 1, NQ, Dm, k.sa_heads, false);
        Vec sa = linear_v(c, att, NQ, Dm, b + "self_attn.out_proj", Dm);
        if (c.missing) return -7;
        c.publish(pb + "self_attn.output", sa);
        Vec x(tgt.size());
        for (size_t i = 0; i < x.size(); ++i) x[i] = tgt[i] + sa[i];
        layer_norm_named(c, x, NQ, Dm, b + "norm1", 1e-5f);
        c.publish(pb + "norm1.output", x);

        /* deformable cross-attention (src/decoder.cpp:127-291) */
        Vec caq(x.size());
        for (size_t i = 0; i < x.size(); ++i) caq[i] = x[i] + qpos[i];
        Vec so = linear_v(c, caq, NQ, Dm, b + "cross_attn.sampling_offsets", nh * np_ * 2);
        Vec aw = linear_v(c, caq, NQ, Dm, b + "cross_attn.attention_weights", nh * np_);
        Vec val = linear_v(c, proj, N, Dm, b + "cross_attn.value_proj", Dm);
        if (c.missing) return -7;
        for (int qq = 0; qq < NQ; ++qq)
            for (int hh = 0; hh < nh; ++hh) softmax_row(&aw[(size_t)qq * nh * np_ + hh * np_], np_);
        Vec samp((size_t)NQ * Dm, 0.f);
        const float offs_scale = 0.5f / (float)np_;
        #pragma omp parallel for schedule(static)
        for (int qq = 0; qq < NQ; ++qq) {
            const float* r = &rp[(size_t)qq * 4];
            for (int hh = 0; hh < nh; ++hh)
                for (int pp = 0; pp < np_; ++pp) {
                    const float* o = &so[(size_t)qq * nh * np_ * 2 + (hh * np_ + pp) * 2];
                    const float sxl = (o[0] * offs_scale) * r[2] + r[0];
                    const float syl = (o[1] * offs_scale) * r[3] + r[1];
                    const float wa = aw[(size_t)qq * nh * np_ + hh * np_ + pp];
                    const float ix = sxl * (float)G - 0.5f, iy = syl * (float)G - 0.5f;
                    const int ix0 = (int)std::floor(ix), iy0 = (int)std::floor(iy);
                    const int ix1 = ix0 + 1, iy1 = iy0 + 1;
                    const float wx1 = ix - (float)ix0, wy1 = iy - (float)iy0;
                    const float wx0 = 1.f - wx1, wy0 = 1.f - wy1;
                    auto tokf = [&](int xi, int yi) { return (xi < 0 || xi >= G || yi < 0 || yi >= G) ? -1 : yi * G + xi; };
                    const int t00 = tokf(ix0, iy0), t10 = tokf(ix1, iy0), t01 = tokf(ix0, iy1), t11 = tokf(ix1, iy1);
                    for (int d = 0; d < chd; ++d) {
                        const int ch = hh * chd + d;
                        float s = 0.f;
                        if (t00 >= 0) s += wx0 * wy0 * val[(size_t)t00 * Dm + ch];
                        if (t10 >= 0) s += wx1 * wy0 * val[(size_t)t10 * Dm + ch];
                        if (t01 >= 0) s += wx0 * wy1 * val[(size_t)t01 * Dm + ch];
                        if (t11 >= 0) s += wx1 * wy1 * val[(size_t)t11 * Dm + ch];
                        samp[(size_t)qq * Dm + ch] += wa * s;
                    }
                }
        }
        Vec ca = linear_v(c, samp, NQ, Dm, b + "cross_attn.output_proj", Dm);
        if (c.missing) return -7;
        c.publish(pb + "cross_attn.output", ca);
        for (size_t i = 0; i < x.size(); ++i) x[i] += ca[i];
        layer_norm_named(c, x, NQ, Dm, b + "norm2", 1e-5f);
        c.publish(pb + "norm2.output", x);

        Vec f = linear_v(c, x, NQ, Dm, b + "linear1", k.dec_ffn);
        for (auto& e : f) e = std::max(e, 0.f);
        Vec f2 = linear_v(c, f, NQ, k.dec_ffn, b + "linear2", Dm);
        if (c.missing) return -7;
        for (size_t i = 0; i < x.size(); ++i) x[i] += f2[i];
        layer_norm_named(c, x, NQ, Dm, b + "norm3", 1e-5f);
        c.publish(pb + "output", x);
        tgt = x;
        if (k.has_seg) {
            Vec xn = x;
            layer_norm_named(c, xn, NQ, Dm, "decoder.norm", 1e-5f);
            per_layer.push_back(xn);
        }
    }
    Vec dec = tgt;
    layer_norm_named(c, dec, NQ, Dm, "decoder.norm", 1e-5f);
    c.publish("decoder.norm.output", dec);

    /* ---- heads (src/heads.cpp:31-56) + reparam (src/rfdetr_model.cpp:438-448) ---- */
    Vec logits = linear_v(c, dec, NQ, Dm, "heads.class_embed", NC);
    Vec hh = linear_v(c, dec, NQ, Dm, "heads.bbox_embed.layers.0", Dm);
    for (auto& e : hh) e = std::max(e, 0.f);
    hh = linear_v(c, hh, NQ, Dm, "heads.bbox_embed.layers.1", Dm);
    for (auto& e : hh) e = std::max(e, 0.f);
    Vec bd = linear_v(c, hh, NQ, Dm, "heads.bbox_embed.layers.2", 4);
    if (c.missing) return -7;
    c.publish("heads.class_logits", logits);
    c.publish("heads.bbox_pred", bd);
    std::memcpy(out_logits, logits.data(), sizeof(float) * (size_t)NQ * NC);
    for (int q = 0; q < NQ; ++q) {
        const float* d = &bd[(size_t)q * 4];
        const float* r = &rp[(size_t)q * 4];
        float* o = out_boxes + (size_t)q * 4;
        o[0] = d[0] * r[2] + r[0];
        o[1] = d[1] * r[3] + r[1];
        o[2] = std::exp(d[2]) * r[2];
        o[3] = std::exp(d[3]) * r[3];
    }

    /* ---- segmentation head (src/segmentation.cpp:170-309) ---- */
    if (k.has_seg) {
        const int Ht = k.image_size / k.mask_ratio, Wt = Ht, HW = Ht * Wt;
        /* bilinear resize, align_corners=False, in ggml_interpolate's form */
        Vec sp((size_t)HW * Dm);
        const float sf = (float)Wt / (float)G;
        for (int yy = 0; yy < Ht; ++yy) {
            const float fy = ((float)yy + 0.5f) / sf - 0.5f;
            int y0 = (int)std::floor(fy), y1 = y0 + 1;
            y0 = std::clamp(y0, 0, G - 1); y1 = std::clamp(y1, 0, G - 1);
            const float dy = std::clamp(fy - (float)y0, 0.f, 1.f);
            for (int xx = 0; xx < Wt; ++xx) {
                const float fx = ((float)xx + 0.5f) / sf - 0.5f;
                int x0 = (int)std::floor(fx), x1 = x0 + 1;
                x0 = std::clamp(x0, 0, G - 1); x1 = std::clamp(x1, 0, G - 1);
                const float dx = std::clamp(fx - (float)x0, 0.f, 1.f);
                for (int ch = 0; ch < Dm; ++ch) {
                    const float a = proj[((size_t)y0 * G + x0) * Dm + ch], bq = proj[((size_t)y0 * G + x1) * Dm + ch];
                    const float cq = proj[((size_t)y1 * G + x0) * Dm + ch], dq = proj[((size_t)y1 * G + x1) * Dm + ch];
                    sp[((size_t)yy * Wt + xx) * Dm + ch] =
                        a * (1 - dx) * (1 - dy) + bq * dx * (1 - dy) + cq * (1 - dx) * dy + dq * dx * dy;
                }
            }
        }
        c.publish("seg.spatial_features.resized", sp);
        const W& sfw = c.get("segmentation_head.spatial_features_proj.weight");
        const W& sfb = c.get("segmentation_head.spatial_features_proj.bias");
        const W& sbias = c.get("segmentation_head.bias");
        if (c.missing) return -7;
        Vec masks;
        for (int bi = 0; bi < k.dec_layers; ++bi) {
            const std::string b = "segmentation_head.blocks." + std::to_string(bi) + ".";
            const W& dw = c.get(b + "dwconv.weight");
            const W& db = c.get(b + "dwconv.bias");
            if (c.missing) return -7;
            Vec y2((size_t)HW * Dm);
            #pragma omp parallel for schedule(static)
            for (int yy = 0; yy < Ht; ++yy)
                for (int xx = 0; xx < Wt; ++xx)
                    for (int ch = 0; ch < Dm; ++ch) {
                        float s = 0.f;
                        for (int ky = 0; ky < 3; ++ky)
                            for (int kx = 0; kx < 3; ++kx) {
                                const int sy = yy + ky - 1, sx = xx + kx - 1;
                                if (sy < 0 || sy >= Ht || sx < 0 || sx >= Wt) continue;
                                s += dw.p[(size_t)ch * 9 + ky * 3 + kx] * sp[((size_t)sy * Wt + sx) * Dm + ch];
                            }
                        y2[((size_t)yy * Wt + xx) * Dm + ch] = s + db.p[ch];
                    }
            layer_norm_named(c, y2, HW, Dm, b + "norm", 1e-6f);
            Vec lin = linear_v(c, y2, HW, Dm, b + "pwconv1", Dm);
            if (c.missing) return -7;
            for (size_t i = 0; i < sp.size(); ++i) sp[i] = gelu_erf(lin[i]) + sp[i];
            c.publish("seg.block." + std::to_string(bi) + ".spatial_out", sp);
            if (bi != k.dec_layers - 1) continue;  /* only the last mask is consumed */
            Vec spp((size_t)HW * Dm);
            linear(c, sp.data(), HW, Dm, sfw, sfb.p, Dm, spp.data());
            Vec qf = per_layer[bi];
            Vec qn = qf;
            layer_norm_named(c, qn, NQ, Dm, "segmentation_head.query_features_block.norm_in", 1e-6f);
            Vec l0 = linear_v(c, qn, NQ, Dm, "segmentation_head.query_features_block.layers.0", 4 * Dm);
            for (auto& e : l0) e = gelu_erf(e);
            Vec l2 = linear_v(c, l0, NQ, 4 * Dm, "segmentation_head.query_features_block.layers.2", Dm);
            if (c.missing) return -7;
            for (size_t i = 0; i < qf.size(); ++i) l2[i] += qf[i];
            Vec qp = linear_v(c, l2, NQ, Dm, "segmentation_head.query_features_proj", Dm);
            if (c.missing) return -7;
            c.publish("seg.block." + std::to_string(bi) + ".qf_proj", qp);
            /* mask[q][pix] = sum_c spp[pix][c] * qp[q][c] + bias */
            masks.assign((size_t)NQ * HW, 0.f);
            /* both operands are activations: never rounded (F32 "weight") */
            W spw{spp.data(), (int64_t)spp.size(), ORACLE_F32};
            linear(c, qp.data(), NQ, Dm, spw, nullptr, HW, masks.data());
            for (auto& e : masks) e += sbias.p[0];
        }
        c.publish("seg.masks.final", masks);
        if (out_masks) std::memcpy(out_masks, masks.data(), sizeof(float) * masks.size());
    }
    return 0;
}
