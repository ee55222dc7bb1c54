// Memory-bound kernels around the GEMMs: preprocessing, patch/conv im2col,
// LayerNorm, backbone taps, two-stage box reparam, top-K selection, decoder
// query setup, deformable sampling, segmentation resize / depthwise conv.
// Each follows the arithmetic of the reference function cited beside it
// (paths within localai-org/rf-detr.cpp).
#include "kernels.cuh"

#include <cuda_fp16.h>
#include <stdint.h>

namespace rfb {

namespace {

inline unsigned cdiv(size_t a, size_t b) { return (unsigned)((a + b - 1) / b); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffff, v, o));
    return v;
}

// x / d for 0 <= x < 2^21 through a float reciprocal: (x + 1/2) * (1/d) lies at
// least 1/(2d) from the next integer, and the float error of that product is
// below (x/d) * 2^-22 < 1/(2d) in that range, so truncation gives the quotient.
__device__ __forceinline__ int div_small(int x, float inv_d) {
    return __float2int_rz(__fmul_rn((float)x + 0.5f, inv_d));
}

// ---- legacy preprocess resize: src/image_io.cpp:249-275 (taps: resize_legacy.cpp)
// One thread per output pixel: for each vertical tap, the horizontal weighted
// sum of the row's taps, then the weighted sum of those rows, in tap order with
// a rounding after every multiply and every add (as the library's float
// passes, horizontal first); the 0..255 result rounds half up and saturates.
__global__ void k_resize_legacy(const uint8_t* __restrict__ src, int B, int w, int h, const int* __restrict__ xf,
                                const int* __restrict__ xn, const float* __restrict__ xc, int xw,
                                const int* __restrict__ yf, const int* __restrict__ yn,
                                const float* __restrict__ yc, int yw, int ow, int oh, uint8_t* __restrict__ dst) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)B * oh * ow) return;
    const int ox = (int)(i % ow);
    const size_t r = i / ow;
    const int oy = (int)(r % oh), b = (int)(r / oh);
    const uint8_t* img = src + (size_t)b * h * w * 3;
    const int x0 = xf[ox], nx = xn[ox], y0 = yf[oy], ny = yn[oy];
    const float* cx = xc + (size_t)ox * xw;
    const float* cy = yc + (size_t)oy * yw;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f;
    for (int j = 0; j < ny; ++j) {
        const uint8_t* row = img + ((size_t)(y0 + j) * w + x0) * 3;
        float h0 = 0.f, h1 = 0.f, h2 = 0.f;
        for (int k = 0; k < nx; ++k) {
            const float c = cx[k];
            h0 = __fadd_rn(h0, __fmul_rn(c, (float)row[3 * k]));
            h1 = __fadd_rn(h1, __fmul_rn(c, (float)row[3 * k + 1]));
            h2 = __fadd_rn(h2, __fmul_rn(c, (float)row[3 * k + 2]));
        }
        const float c = cy[j];
        a0 = __fadd_rn(a0, __fmul_rn(c, h0));
        a1 = __fadd_rn(a1, __fmul_rn(c, h1));
        a2 = __fadd_rn(a2, __fmul_rn(c, h2));
    }
    uint8_t* o = dst + i * 3;
    const float a[3] = {a0, a1, a2};
#pragma unroll
    for (int ch = 0; ch < 3; ++ch) o[ch] = (uint8_t)min(max(__float2int_rz(__fadd_rn(a[ch], 0.5f)), 0), 255);
}

// ---- patch im2col in windowed order: src/dinov2.cpp:339-408 -----------------
__global__ void k_patch_im2col(const float* __restrict__ img, int B, int S, int p, int nw, int Kpad,
                               __half* __restrict__ A) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int G = S / p, ws = G / nw, Tp = ws * ws;
    const size_t rows = (size_t)B * nw * nw * Tp;
    if (i >= rows * Kpad) return;
    const size_t row = i / Kpad;
    const int k = (int)(i - row * Kpad);
    float v = 0.f;
    if (k < 3 * p * p) {
        const int b = (int)(row / ((size_t)nw * nw * Tp));
        const int rr = (int)(row - (size_t)b * nw * nw * Tp);
        const int win = rr / Tp, t = rr - win * Tp;
        const int gy = (win / nw) * ws + t / ws, gx = (win % nw) * ws + t % ws;
        const int c = k / (p * p), ky = (k / p) % p, kx = k % p;
        v = img[((size_t)b * 3 + c) * S * S + (size_t)(gy * p + ky) * S + gx * p + kx];
    }
    A[i] = __float2half_rn(v);
}

// Preprocess (src/image_io.cpp:207-248) fused into the patch im2col: each
// im2col element is one normalized model-resolution pixel, sampled straight
// from the uint8 source with the same double-precision source coordinates.
// One warp per im2col row (grid-strided); lane l writes the 16-byte chunks
// l, l + 32, l + 64 (8 consecutive elements each).  Element k of a row is
// (channel, kernel row, kernel column) = (k / p^2, k / p mod p, k mod p);
// elements past 3 p^2 are the zero K padding.  Without resizing, every element
// is (u / 255 - mean_c) / std_c of a source byte u: a per-block table of those
// 768 floats (the same float expression) replaces the two divisions.
// Identity-size patch extraction, CTA per (image, patch row): the patch row's p image rows are
// one contiguous block of p * S * 3 bytes, loaded with 16-byte loads into shared memory; the CTA
// then writes the G patches of that row (A rows in window order) as 16-byte chunks of 8 f16, each
// value lut[c][byte] through the same table as k_patch_from_rgb (identical values).
// smem: table [3][256] f32, per-k source offset (byte offset within a patch | channel << 24),
// the strip.
__global__ void __launch_bounds__(256) k_patch_strip(const uint8_t* __restrict__ rgb, int S, int p, int nw, int Kpad,
                                                     float m0, float m1, float m2, float s0, float s1, float s2,
                                                     __half* __restrict__ A) {
    extern __shared__ uint4 strip_smem[];
    float* lut = reinterpret_cast<float*>(strip_smem);
    int* koff = reinterpret_cast<int*>(lut + 3 * 256);
    uint8_t* strip = reinterpret_cast<uint8_t*>(koff + ((Kpad + 3) & ~3));
    const int G = S / p, gy = blockIdx.x, b = blockIdx.y;
    const int row_bytes = S * 3, strip_bytes = p * row_bytes;
    const uint4* src = reinterpret_cast<const uint4*>(rgb + ((size_t)b * S + (size_t)gy * p) * row_bytes);
    uint4* dst = reinterpret_cast<uint4*>(strip);
    for (int i = threadIdx.x; i < strip_bytes / 16; i += blockDim.x) dst[i] = __ldg(src + i);
    for (int t = threadIdx.x; t < 3 * 256; t += blockDim.x) {
        const int cc = t >> 8;
        const float mean = cc == 0 ? m0 : (cc == 1 ? m1 : m2), sd = cc == 0 ? s0 : (cc == 1 ? s1 : s2);
        lut[t] = ((float)(t & 255) / 255.0f - mean) / sd;
    }
    const int pp = p * p, kreal = 3 * pp;
    for (int k = threadIdx.x; k < Kpad; k += blockDim.x) {
        if (k < kreal) {
            const int c = k / pp, ky = (k - c * pp) / p, kx = k - c * pp - ky * p;
            koff[k] = (ky * row_bytes + kx * 3 + c) | (c << 24);
        } else {
            koff[k] = -1;
        }
    }
    __syncthreads();
    const int ws = G / nw, Tp = ws * ws, NT = nw * nw * Tp;
    const int wy = gy / ws, ty = gy - wy * ws;
    const int chunks = Kpad / 8;
    // consecutive threads take consecutive patches of one chunk: the offset-table reads are broadcasts
    for (int i = threadIdx.x; i < G * chunks; i += blockDim.x) {
        const int ch = i / G, gx = i - ch * G;
        const int wx = gx / ws, tx = gx - wx * ws;
        const size_t row = (size_t)b * NT + (size_t)(wy * nw + wx) * Tp + ty * ws + tx;
        const uint8_t* patch = strip + gx * p * 3;
        uint32_t out[4];
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
            const int o0 = koff[ch * 8 + e], o1 = koff[ch * 8 + e + 1];
            const float v0 = o0 < 0 ? 0.f : lut[((o0 >> 24) << 8) + patch[o0 & 0xFFFFFF]];
            const float v1 = o1 < 0 ? 0.f : lut[((o1 >> 24) << 8) + patch[o1 & 0xFFFFFF]];
            const __half2 hv = __floats2half2_rn(v0, v1);
            out[e >> 1] = *reinterpret_cast<const uint32_t*>(&hv);
        }
        reinterpret_cast<uint4*>(A + row * Kpad)[ch] = make_uint4(out[0], out[1], out[2], out[3]);
    }
}

__global__ void __launch_bounds__(256) k_patch_from_rgb(const uint8_t* __restrict__ rgb, int B, int w, int h, int S,
                                                        int p, int nw, int Kpad, float m0, float m1, float m2,
                                                        float s0, float s1, float s2, __half* __restrict__ A) {
    __shared__ float lut[3 * 256];
    const bool identity = w == S && h == S;
    if (identity) {
        for (int t = threadIdx.x; t < 3 * 256; t += blockDim.x) {
            const int cc = t >> 8;
            const float mean = cc == 0 ? m0 : (cc == 1 ? m1 : m2), sd = cc == 0 ? s0 : (cc == 1 ? s1 : s2);
            lut[t] = ((float)(t & 255) / 255.0f - mean) / sd;
        }
        __syncthreads();
    }
    const int G = S / p, ws = G / nw, Tp = ws * ws, NT = nw * nw * Tp;
    const int chunks = Kpad / 8, kreal = 3 * p * p;
    const int rows = B * NT;  // < 2^21 (checked by the host)
    const float inv_nt = 1.0f / (float)NT, inv_tp = 1.0f / (float)Tp, inv_ws = 1.0f / (float)ws;
    const float inv_nw = 1.0f / (float)nw, inv_pp = 1.0f / (float)(p * p), inv_p = 1.0f / (float)p;
    const double scx = (double)w / (double)S, scy = (double)h / (double)S;
    const int lane = threadIdx.x & 31;
    const int wstride = gridDim.x * (blockDim.x >> 5);
    for (int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < rows; row += wstride) {
        const int b = div_small(row, inv_nt);
        const int rr = row - b * NT;
        const int win = div_small(rr, inv_tp), t = rr - win * Tp;
        const int wy = div_small(win, inv_nw), ty = div_small(t, inv_ws);
        const int gy = wy * ws + ty, gx = (win - wy * nw) * ws + (t - ty * ws);
        const uint8_t* img = rgb + (size_t)b * h * w * 3;
        __half* arow = A + (size_t)row * Kpad;
        for (int ch = lane; ch < chunks; ch += 32) {
            const int k0 = ch * 8;
            int c = div_small(k0, inv_pp);
            int ky = div_small(k0 - c * p * p, inv_p);
            int kx = k0 - c * p * p - ky * p;
            uint32_t out[4];
#pragma unroll
            for (int e = 0; e < 8; e += 2) {
                float v2[2];
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                    float v = 0.f;
                    if (k0 + e + u < kreal) {
                        const int yy = gy * p + ky, xx = gx * p + kx;
                        if (identity) {
                            // identity resize: source coordinate == destination, interpolation weights 0
                            v = lut[(c << 8) + img[((size_t)yy * w + xx) * 3 + c]];
                        } else {
                            const float mean = c == 0 ? m0 : (c == 1 ? m1 : m2);
                            const float sd = c == 0 ? s0 : (c == 1 ? s1 : s2);
                            const double fy = ((double)yy + 0.5) * scy - 0.5;
                            const int y0r = (int)floor(fy);
                            const int y0 = min(max(y0r, 0), h - 1), y1 = min(max(y0r + 1, 0), h - 1);
                            const float wy_ = (float)(fy - (double)y0r);
                            const double fx = ((double)xx + 0.5) * scx - 0.5;
                            const int x0r = (int)floor(fx);
                            const int x0 = min(max(x0r, 0), w - 1), x1 = min(max(x0r + 1, 0), w - 1);
                            const float wx = (float)(fx - (double)x0r);
                            const float p00 = (float)img[((size_t)y0 * w + x0) * 3 + c];
                            const float p01 = (float)img[((size_t)y0 * w + x1) * 3 + c];
                            const float p10 = (float)img[((size_t)y1 * w + x0) * 3 + c];
                            const float p11 = (float)img[((size_t)y1 * w + x1) * 3 + c];
                            const float top = p00 + (p01 - p00) * wx;
                            const float bot = p10 + (p11 - p10) * wx;
                            v = ((top + (bot - top) * wy_) / 255.0f - mean) / sd;
                        }
                    }
                    v2[u] = v;
                    if (++kx == p) {
                        kx = 0;
                        if (++ky == p) {
                            ky = 0;
                            ++c;
                        }
                    }
                }
                __half2 hv = __floats2half2_rn(v2[0], v2[1]);
                out[e >> 1] = *reinterpret_cast<uint32_t*>(&hv);
            }
            *reinterpret_cast<uint4*>(arow + k0) = make_uint4(out[0], out[1], out[2], out[3]);
        }
    }
}

__global__ void k_cls_rows(float* __restrict__ x, const float* __restrict__ clsrow, int B, int NW, int T, int D) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)B * NW * D) return;
    const int d = (int)(i % D);
    const size_t bw = i / D;
    x[bw * T * D + d] = clsrow[d];
}

// ---- LayerNorm (ggml_norm then * g + b); warp per row, in-place safe -------
template <int VPL>
__global__ void k_layernorm(const float* x, int rows, int D, const float* __restrict__ g,
                            const float* __restrict__ b, float eps, float* y32, __half* __restrict__ y16) {
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (row >= rows) return;
    const float* xr = x + (size_t)row * D;
    float v[VPL];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const int c = lane + 32 * i;
        v[i] = c < D ? xr[c] : 0.f;
        s += v[i];
    }
    const float mean = warp_sum(s) / (float)D;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const int c = lane + 32 * i;
        const float d = c < D ? v[i] - mean : 0.f;
        q += d * d;
    }
    const float rstd = 1.0f / sqrtf(warp_sum(q) / (float)D + eps);
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
        const int c = lane + 32 * i;
        if (c < D) {
            const float o = (v[i] - mean) * rstd * g[c] + b[c];
            if (y32) y32[(size_t)row * D + c] = o;
            if (y16) y16[(size_t)row * D + c] = __float2half_rn(o);
        }
    }
}

// Same, 16-byte vectors: lane owns columns 4*(lane + 32*i) .. +3, D = 128*NV.
// Grid-stride over rows (one warp per row at a time); the next row's loads are
// issued before the current row's reductions so each warp keeps two rows of
// loads in flight.
// TAP = false: row r of the output normalises row r of x (contiguous
// outputs).  TAP = true, the backbone tap: output r is grid pixel (b, gy, gx)
// in row-major order, read from its windowed token (window-major, a CLS row
// first in each window) and written at column col0 of an f16 row of pitch ld.
struct TapMap {
    int G = 0, nw = 1, ld = 0, col0 = 0;
    float inv_gg = 0.f, inv_g = 0.f, inv_ws = 0.f;  // 1 / G^2, 1 / G, 1 / (G / nw)
    __device__ __forceinline__ size_t src_row(int r) const {
        const int GG = G * G, ws = G / nw, T = ws * ws + 1;
        const int b = div_small(r, inv_gg), pix = r - b * GG;
        const int gy = div_small(pix, inv_g), gx = pix - gy * G;
        const int wy = div_small(gy, inv_ws), wx = div_small(gx, inv_ws);
        const int win = wy * nw + wx;
        return (size_t)b * nw * nw * T + win * T + 1 + (gy - wy * ws) * ws + (gx - wx * ws);
    }
};

template <int NV, bool TAP = false>
__global__ void __launch_bounds__(256) k_layernorm_v4(const float* x, int rows, const float* __restrict__ g,
                                                     const float* __restrict__ b, float eps, float* y32,
                                                     __half* __restrict__ y16, TapMap tm) {
    constexpr int D = 128 * NV;
    const int lane = threadIdx.x & 31;
    const size_t ld16 = TAP ? (size_t)tm.ld : (size_t)D;
    const int col0 = TAP ? tm.col0 : 0;
    const int stride = gridDim.x * (blockDim.x >> 5);
    int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= rows) return;
    float4 gg[NV], bb[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        gg[i] = *reinterpret_cast<const float4*>(g + 4 * (lane + 32 * i));
        bb[i] = *reinterpret_cast<const float4*>(b + 4 * (lane + 32 * i));
    }
    float4 v[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i)
        v[i] = reinterpret_cast<const float4*>(x + (TAP ? tm.src_row(row) : (size_t)row) * D)[lane + 32 * i];
    for (; row < rows; row += stride) {
        const int nxt = row + stride;
        float4 vn[NV];
        if (nxt < rows) {
            const float4* xn = reinterpret_cast<const float4*>(x + (TAP ? tm.src_row(nxt) : (size_t)nxt) * D);
#pragma unroll
            for (int i = 0; i < NV; ++i) vn[i] = xn[lane + 32 * i];
        }
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < NV; ++i) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
        const float mean = warp_sum(s) / (float)D;
        float q = 0.f;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const float a = v[i].x - mean, bq = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
            q += (a * a + bq * bq) + (c * c + d * d);
        }
        const float rstd = 1.0f / sqrtf(warp_sum(q) / (float)D + eps);
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const int c0 = 4 * (lane + 32 * i);
            float4 o;
            o.x = (v[i].x - mean) * rstd * gg[i].x + bb[i].x;
            o.y = (v[i].y - mean) * rstd * gg[i].y + bb[i].y;
            o.z = (v[i].z - mean) * rstd * gg[i].z + bb[i].z;
            o.w = (v[i].w - mean) * rstd * gg[i].w + bb[i].w;
            if (y32) *reinterpret_cast<float4*>(y32 + (size_t)row * D + c0) = o;
            if (y16) {
                __half2 h0 = __floats2half2_rn(o.x, o.y), h1 = __floats2half2_rn(o.z, o.w);
                uint2 u;
                u.x = *reinterpret_cast<uint32_t*>(&h0);
                u.y = *reinterpret_cast<uint32_t*>(&h1);
                *reinterpret_cast<uint2*>(y16 + (size_t)row * ld16 + col0 + c0) = u;
            }
        }
        if (nxt < rows) {
#pragma unroll
            for (int i = 0; i < NV; ++i) v[i] = vn[i];
        }
    }
}

// A tapped block's output read once for two LayerNorms with the same statistics (eps 1e-6 both):
// the next block's norm1 (src/dinov2.cpp:17-23, y16 row r = x row r, window order) and the
// backbone tap (src/dinov2.cpp:490-537: the final norm, CLS rows dropped, written at grid pixel
// (b, gy, gx), column col0 of an f16 row of pitch ld).  The arithmetic is k_layernorm_v4's, so
// both outputs equal those of the two separate launches bit for bit.
struct DualTapMap {
    int G = 0, nw = 1, ld = 0, col0 = 0;
    float inv_bt = 0.f, inv_t = 0.f, inv_ws = 0.f, inv_nw = 0.f;  // 1 / (nw^2 T), 1 / T, 1 / ws, 1 / nw
    // grid row of window-order token row r, or -1 for a CLS row
    __device__ __forceinline__ long long dst_row(int r) const {
        const int ws = G / nw, T = ws * ws + 1, BT = nw * nw * T;
        const int b = div_small(r, inv_bt), rr = r - b * BT;
        const int win = div_small(rr, inv_t), t = rr - win * T;
        if (t == 0) return -1;
        const int py = div_small(t - 1, inv_ws), px = (t - 1) - py * ws;
        const int wy = div_small(win, inv_nw), wx = win - wy * nw;
        return ((long long)b * G + wy * ws + py) * G + wx * ws + px;
    }
};

template <int NV>
__global__ void __launch_bounds__(256) k_layernorm_dual(const float* x, int rows, const float* __restrict__ g1,
                                                       const float* __restrict__ b1, __half* __restrict__ y16,
                                                       const float* __restrict__ g2, const float* __restrict__ b2,
                                                       __half* __restrict__ taps, DualTapMap tm) {
    constexpr int D = 128 * NV;
    constexpr float eps = 1e-6f;
    const int lane = threadIdx.x & 31;
    const int stride = gridDim.x * (blockDim.x >> 5);
    int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= rows) return;
    float4 ga[NV], ba[NV], gt[NV], bt[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        ga[i] = *reinterpret_cast<const float4*>(g1 + 4 * (lane + 32 * i));
        ba[i] = *reinterpret_cast<const float4*>(b1 + 4 * (lane + 32 * i));
        gt[i] = *reinterpret_cast<const float4*>(g2 + 4 * (lane + 32 * i));
        bt[i] = *reinterpret_cast<const float4*>(b2 + 4 * (lane + 32 * i));
    }
    float4 v[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) v[i] = reinterpret_cast<const float4*>(x + (size_t)row * D)[lane + 32 * i];
    for (; row < rows; row += stride) {
        const int nxt = row + stride;
        float4 vn[NV];
        if (nxt < rows) {
            const float4* xn = reinterpret_cast<const float4*>(x + (size_t)nxt * D);
#pragma unroll
            for (int i = 0; i < NV; ++i) vn[i] = xn[lane + 32 * i];
        }
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < NV; ++i) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
        const float mean = warp_sum(s) / (float)D;
        float q = 0.f;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const float a = v[i].x - mean, bq = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
            q += (a * a + bq * bq) + (c * c + d * d);
        }
        const float rstd = 1.0f / sqrtf(warp_sum(q) / (float)D + eps);
        const long long trow = tm.dst_row(row);
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const int c0 = 4 * (lane + 32 * i);
            float4 o;
            o.x = (v[i].x - mean) * rstd * ga[i].x + ba[i].x;
            o.y = (v[i].y - mean) * rstd * ga[i].y + ba[i].y;
            o.z = (v[i].z - mean) * rstd * ga[i].z + ba[i].z;
            o.w = (v[i].w - mean) * rstd * ga[i].w + ba[i].w;
            __half2 h0 = __floats2half2_rn(o.x, o.y), h1 = __floats2half2_rn(o.z, o.w);
            uint2 u;
            u.x = *reinterpret_cast<uint32_t*>(&h0);
            u.y = *reinterpret_cast<uint32_t*>(&h1);
            *reinterpret_cast<uint2*>(y16 + (size_t)row * D + c0) = u;
            if (trow >= 0) {
                o.x = (v[i].x - mean) * rstd * gt[i].x + bt[i].x;
                o.y = (v[i].y - mean) * rstd * gt[i].y + bt[i].y;
                o.z = (v[i].z - mean) * rstd * gt[i].z + bt[i].z;
                o.w = (v[i].w - mean) * rstd * gt[i].w + bt[i].w;
                h0 = __floats2half2_rn(o.x, o.y);
                h1 = __floats2half2_rn(o.z, o.w);
                u.x = *reinterpret_cast<uint32_t*>(&h0);
                u.y = *reinterpret_cast<uint32_t*>(&h1);
                *reinterpret_cast<uint2*>(taps + trow * tm.ld + tm.col0 + c0) = u;
            }
        }
        if (nxt < rows) {
#pragma unroll
            for (int i = 0; i < NV; ++i) v[i] = vn[i];
        }
    }
}

// ---- backbone tap: src/dinov2.cpp:490-537 -----------------------------------
__global__ void k_tap(const float* __restrict__ x, int B, int G, int nw, int D, const float* __restrict__ g,
                      const float* __restrict__ bb, __half* __restrict__ taps, int ld, int col0) {
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);  // output pixel (b, gy, gx)
    const int lane = threadIdx.x & 31;
    if (row >= B * G * G) return;
    const int b = row / (G * G), pix = row - b * G * G;
    const int gy = pix / G, gx = pix - gy * G;
    const int ws = G / nw, T = ws * ws + 1;
    const int win = (gy / ws) * nw + gx / ws;
    const int tok = win * T + 1 + (gy % ws) * ws + gx % ws;
    const float* xr = x + ((size_t)b * nw * nw * T + tok) * D;
    float v[12];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 12; ++i) {
        const int c = lane + 32 * i;
        v[i] = c < D ? xr[c] : 0.f;
        s += v[i];
    }
    const float mean = warp_sum(s) / (float)D;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < 12; ++i) {
        const int c = lane + 32 * i;
        const float d = c < D ? v[i] - mean : 0.f;
        q += d * d;
    }
    const float rstd = 1.0f / sqrtf(warp_sum(q) / (float)D + 1e-6f);
    __half* o = taps + (size_t)row * ld + col0;
#pragma unroll
    for (int i = 0; i < 12; ++i) {
        const int c = lane + 32 * i;
        if (c < D) o[c] = __float2half_rn((v[i] - mean) * rstd * g[c] + bb[c]);
    }
}

// ---- 3x3 im2col (channels-last, 16-byte chunks) -----------------------------
__global__ void k_im2col3x3(const __half* __restrict__ src, int lds, int B, int H, int W, int C,
                            __half* __restrict__ A) {
    const int chunks = C / 8;
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const size_t total = (size_t)B * H * W * 9 * chunks;
    if (i >= total) return;
    const int ch = (int)(i % chunks);
    const int tap = (int)((i / chunks) % 9);
    const size_t row = i / ((size_t)9 * chunks);
    const int b = (int)(row / ((size_t)H * W));
    const int pix = (int)(row - (size_t)b * H * W);
    const int y = pix / W + tap / 3 - 1, x = pix % W + tap % 3 - 1;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (y >= 0 && y < H && x >= 0 && x < W)
        v = *reinterpret_cast<const uint4*>(src + ((size_t)b * H * W + (size_t)y * W + x) * lds + ch * 8);
    *reinterpret_cast<uint4*>(A + row * (size_t)(9 * C) + tap * C + ch * 8) = v;
}

// proposal of token (gy, gx) on a G x G grid, zeroed outside (0.01, 0.99):
// src/two_stage.cpp:69-88
__device__ __forceinline__ void proposal(int gy, int gx, int G, float (&p)[4]) {
    const float fg = (float)G;
    p[0] = ((float)gx + 0.5f) / fg;
    p[1] = ((float)gy + 0.5f) / fg;
    p[2] = 0.05f;
    p[3] = 0.05f;
    bool valid = true;
#pragma unroll
    for (int c = 0; c < 4; ++c)
        if (!(p[c] > 0.01f && p[c] < 0.99f)) valid = false;
    if (!valid) p[0] = p[1] = p[2] = p[3] = 0.f;
}

__global__ void k_mask_memory(const float* __restrict__ mem, int B, int G, int C, __half* __restrict__ out) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)B * G * G * C) return;
    const int tok = (int)((i / C) % ((size_t)G * G));
    float p[4];
    proposal(tok / G, tok % G, G, p);
    out[i] = __float2half_rn(p[2] > 0.f ? mem[i] : 0.f);
}

// src/two_stage.cpp:203-234
__global__ void k_two_stage_boxes(const float* __restrict__ delta, int B, int G, float* __restrict__ bbox) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= B * G * G) return;
    const int tok = i % (G * G);
    float p[4];
    proposal(tok / G, tok % G, G, p);
    const float* d = delta + (size_t)i * 4;
    float* o = bbox + (size_t)i * 4;
    o[0] = d[0] * p[2] + p[0];
    o[1] = d[1] * p[3] + p[1];
    o[2] = expf(d[2]) * p[2];
    o[3] = expf(d[3]) * p[3];
}

// ---- top-K: src/rfdetr_model.cpp:39-62 --------------------------------------
constexpr int kTopkMax = 4096;

__device__ __forceinline__ uint32_t float_order(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// One 1024-thread CTA per image.  Key of token t: (~order(max_c cls[t][c]) << 32) | t, so that
// ascending keys are descending maxima with ties to the lower token, as the output wants.
//  1. class maxima (the work is issue-bound on the CTA's one SM, so instructions are what count):
//     a warp takes 8 tokens per step, issues their 24 class loads before any reduction, and
//     reduces the 8 per-lane maxima with a transposed butterfly (9 shuffles for the 8 tokens);
//  2. K < N: radix select of the K-th smallest key over 8-bit digits (the 4 score bytes, then
//     the 2 low index bytes; N <= 4096 keeps index bits 16-31 zero) with warp-aggregated
//     shared-memory histograms, and compaction of the K keys <= it to keys[0, K);
//  3. bitonic sort of those K keys (padded to a power of two) instead of all N.
// Keys are unique, so the result is the first K of the full (score desc, index asc) order.
__global__ void __launch_bounds__(1024) k_topk(const float* __restrict__ cls, int N, int NC, int K,
                                                int32_t* __restrict__ idx) {
    __shared__ unsigned long long keys[kTopkMax];
    __shared__ unsigned hist[256];
    __shared__ int s_digit, s_want, s_count;
    const int b = blockIdx.x;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
    if (NC <= 96) {
        constexpr int U = 8;
        const bool h16 = lane & 16, h8 = lane & 8, h4 = lane & 4;
        const int mine = (h16 ? 4 : 0) + (h8 ? 2 : 0) + (h4 ? 1 : 0);  // token of this lane after the butterfly
        for (int t0 = warp * U; t0 < N; t0 += nwarps * U) {
            float v[U][3];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const float* r = cls + ((size_t)b * N + min(t0 + u, N - 1)) * NC;
#pragma unroll
                for (int j = 0; j < 3; ++j) v[u][j] = lane + 32 * j < NC ? __ldg(r + lane + 32 * j) : -INFINITY;
            }
            float a[U];
#pragma unroll
            for (int u = 0; u < U; ++u) a[u] = fmaxf(fmaxf(v[u][0], v[u][1]), v[u][2]);
            // each exchange halves the tokens a lane holds: the lane keeps one half and receives
            // its partner's values of that half
            float a4[4], a2[2];
#pragma unroll
            for (int i = 0; i < 4; ++i)
                a4[i] = fmaxf(h16 ? a[i + 4] : a[i], __shfl_xor_sync(0xffffffffu, h16 ? a[i] : a[i + 4], 16));
#pragma unroll
            for (int i = 0; i < 2; ++i)
                a2[i] = fmaxf(h8 ? a4[i + 2] : a4[i], __shfl_xor_sync(0xffffffffu, h8 ? a4[i] : a4[i + 2], 8));
            float m = fmaxf(h4 ? a2[1] : a2[0], __shfl_xor_sync(0xffffffffu, h4 ? a2[0] : a2[1], 4));
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
            m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
            const int t = t0 + mine;
            if ((lane & 3) == 0 && t < N) keys[t] = ((unsigned long long)(~float_order(m)) << 32) | (unsigned)t;
        }
    } else {
        for (int t = warp; t < N; t += nwarps) {
            const float* r = cls + ((size_t)b * N + t) * NC;
            float m = -INFINITY;
            for (int c = lane; c < NC; c += 32) m = fmaxf(m, r[c]);
            m = warp_max(m);
            if (lane == 0) keys[t] = ((unsigned long long)(~float_order(m)) << 32) | (unsigned)t;
        }
    }
    __syncthreads();
    int P = 1;
    if (K < N) {
        const int jn = (N + blockDim.x - 1) / blockDim.x;  // keys per thread, <= 4
        unsigned long long prefix = 0, mask = 0;
        int want = K;  // rank of the wanted key among the keys that match prefix under mask
#pragma unroll 1
        for (int pass = 0; pass < 6; ++pass) {
            const int sh = pass < 4 ? 56 - 8 * pass : 8 * (5 - pass);  // 56, 48, 40, 32, 8, 0
            if (threadIdx.x < 256) hist[threadIdx.x] = 0;
            __syncthreads();
            for (int j = 0; j < jn; ++j) {
                const int t = threadIdx.x + j * blockDim.x;
                const unsigned long long key = t < N ? keys[t] : ~0ull;
                const bool cand = t < N && (key & mask) == prefix;
                const unsigned d = cand ? (unsigned)(key >> sh) & 255u : 256u;
                const unsigned peers = __match_any_sync(0xffffffffu, d);
                if (cand && lane == __ffs(peers) - 1) atomicAdd(&hist[d], (unsigned)__popc(peers));
            }
            __syncthreads();
            if (warp == 0) {
                unsigned c[8], sum = 0;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    c[i] = hist[lane * 8 + i];
                    sum += c[i];
                }
                unsigned incl = sum;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const unsigned n = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= o) incl += n;
                }
                const unsigned excl = incl - sum;
                if (excl < (unsigned)want && (unsigned)want <= incl) {  // exactly one lane
                    unsigned w = (unsigned)want - excl;
                    int i = 0;
                    for (; i < 7 && w > c[i]; ++i) w -= c[i];
                    s_digit = lane * 8 + i;
                    s_want = (int)w;
                }
            }
            __syncthreads();
            prefix |= (unsigned long long)s_digit << sh;
            mask |= 255ull << sh;
            want = s_want;
        }
        // prefix is now the K-th smallest key: keys <= prefix move to keys[0, K) (any order)
        unsigned long long snap[kTopkMax / 1024];
#pragma unroll
        for (int j = 0; j < kTopkMax / 1024; ++j) {
            const int t = threadIdx.x + j * blockDim.x;
            snap[j] = j < jn && t < N ? keys[t] : ~0ull;
        }
        if (threadIdx.x == 0) s_count = 0;
        __syncthreads();
#pragma unroll
        for (int j = 0; j < kTopkMax / 1024; ++j) {
            if (j < jn) {
                const bool sel = snap[j] <= prefix;
                const unsigned bal = __ballot_sync(0xffffffffu, sel);
                int base = 0;
                if (lane == 0 && bal) base = atomicAdd(&s_count, __popc(bal));
                base = __shfl_sync(0xffffffffu, base, 0);
                if (sel) keys[base + __popc(bal & ((1u << lane) - 1u))] = snap[j];
            }
        }
        while (P < K) P <<= 1;
    } else {
        while (P < N) P <<= 1;
    }
    for (int t = min(K, N) + threadIdx.x; t < P; t += blockDim.x) keys[t] = ~0ull;  // padding sorts last
    __syncthreads();
    // bitonic sort ascending (smaller key = higher score, then lower index)
    if (P >= 64 && P <= 2 * (int)blockDim.x) {
        // thread t < P/2 owns keys 2t and 2t+1: the stages whose partner distance j is at most 32
        // run in registers (j = 1 inside the thread, 2..32 by warp shuffles, partner thread t ^ j/2);
        // only the wider ones go through shared memory
        const int t = threadIdx.x;
        const bool act = t < P / 2;
        unsigned long long k0 = act ? keys[2 * t] : 0ull, k1 = act ? keys[2 * t + 1] : 0ull;
        for (int k = 2; k <= P; k <<= 1) {
            int j = k >> 1;
            if (j >= 64) {
                __syncthreads();
                if (act) {
                    keys[2 * t] = k0;
                    keys[2 * t + 1] = k1;
                }
                __syncthreads();
                for (; j >= 64; j >>= 1) {
                    for (int i = threadIdx.x; i < P; i += blockDim.x) {
                        const int ixj = i ^ j;
                        if (ixj > i) {
                            const unsigned long long a = keys[i], c = keys[ixj];
                            const bool up = (i & k) == 0;
                            if ((a > c) == up) {
                                keys[i] = c;
                                keys[ixj] = a;
                            }
                        }
                    }
                    __syncthreads();
                }
                if (act) {
                    k0 = keys[2 * t];
                    k1 = keys[2 * t + 1];
                }
            }
            if (act) {
                const bool up = ((2 * t) & k) == 0;  // the same for both keys (k >= 2)
                for (; j >= 2; j >>= 1) {
                    const int d = j >> 1;                       // partner thread t ^ d, same slot
                    const bool lower = ((2 * t) & j) == 0;      // this thread holds the lower index
                    const unsigned long long p0 = __shfl_xor_sync(0xffffffffu, k0, d);
                    const unsigned long long p1 = __shfl_xor_sync(0xffffffffu, k1, d);
                    const bool keep_min = lower == up;
                    k0 = keep_min ? (k0 < p0 ? k0 : p0) : (k0 > p0 ? k0 : p0);
                    k1 = keep_min ? (k1 < p1 ? k1 : p1) : (k1 > p1 ? k1 : p1);
                }
                if ((k0 > k1) == up) {
                    const unsigned long long tmp = k0;
                    k0 = k1;
                    k1 = tmp;
                }
            }
        }
        __syncthreads();
        if (act) {
            keys[2 * t] = k0;
            keys[2 * t + 1] = k1;
        }
        __syncthreads();
    } else {
    for (int k = 2; k <= P; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < P; i += blockDim.x) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const unsigned long long a = keys[i], c = keys[ixj];
                    const bool up = (i & k) == 0;
                    if ((a > c) == up) {
                        keys[i] = c;
                        keys[ixj] = a;
                    }
                }
            }
            __syncthreads();
        }
    }
    }
    for (int q = threadIdx.x; q < K; q += blockDim.x) idx[(size_t)b * K + q] = (int32_t)(keys[q] & 0xffffffffu);
}

// ---- decoder inputs: src/rfdetr_model.cpp:233-271, src/decoder.cpp:383-417 ---
__global__ void k_query_init(const float* __restrict__ bbox_all, const int32_t* __restrict__ idx,
                             const float* __restrict__ lrn, const float* __restrict__ feat, int N, int NQ, int Dm,
                             float* __restrict__ refp, __half* __restrict__ sine, float* __restrict__ tgt,
                             __half* __restrict__ tgt16) {
    const int bq = blockIdx.x;  // b*NQ + q
    const int b = bq / NQ, q = bq - b * NQ;
    const int t = idx[bq];
    const float* box = bbox_all + ((size_t)b * N + t) * 4;
    const float* l = lrn + (size_t)q * 4;
    float rp[4];
    rp[0] = l[0] * box[2] + box[0];
    rp[1] = l[1] * box[3] + box[1];
    rp[2] = expf(l[2]) * box[2];
    rp[3] = expf(l[3]) * box[3];
    if (threadIdx.x < 4) refp[(size_t)bq * 4 + threadIdx.x] = rp[threadIdx.x];
    const int half = Dm / 2;
    const int comp[4] = {1, 0, 2, 3};
    for (int j = threadIdx.x; j < 2 * Dm; j += blockDim.x) {
        const int c = j / half, kk = j - c * half;
        const float v = rp[comp[c]] * 6.28318530717958647692f;
        const float inv = expf(-logf(10000.0f) * (float)((kk / 2) * 2) / (float)half);
        const float arg = v * inv;
        sine[(size_t)bq * 2 * Dm + j] = __float2half_rn((kk & 1) ? cosf(arg) : sinf(arg));
    }
    for (int d = threadIdx.x; d < Dm; d += blockDim.x) {
        const float f = feat[(size_t)q * Dm + d];
        tgt[(size_t)bq * Dm + d] = f;
        tgt16[(size_t)bq * Dm + d] = __float2half_rn(f);
    }
}

// The same for Dm = 256, warp per query: the 64 frequencies 10000^(-2k/128) computed once per CTA
// (the expression above), lane per 8 consecutive (sin, cos) pairs (two 16-byte stores), 16-byte
// copies of the query features.  Same values as k_query_init.
__global__ void __launch_bounds__(256) k_query_init256(const float* __restrict__ bbox_all,
                                                       const int32_t* __restrict__ idx,
                                                       const float* __restrict__ lrn,
                                                       const float* __restrict__ feat, int N, int NQ, int rows,
                                                       float* __restrict__ refp, __half* __restrict__ sine,
                                                       float* __restrict__ tgt, __half* __restrict__ tgt16) {
    constexpr int Dm = 256, half = Dm / 2;
    __shared__ float inv[half / 2];
    if (threadIdx.x < half / 2)
        inv[threadIdx.x] = expf(-logf(10000.0f) * (float)(2 * threadIdx.x) / (float)half);
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int bq = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (bq >= rows) return;
    const int b = bq / NQ, q = bq - b * NQ;
    const int t = idx[bq];
    const float* box = bbox_all + ((size_t)b * N + t) * 4;
    const float* l = lrn + (size_t)q * 4;
    float rp[4];
    rp[0] = l[0] * box[2] + box[0];
    rp[1] = l[1] * box[3] + box[1];
    rp[2] = expf(l[2]) * box[2];
    rp[3] = expf(l[3]) * box[3];
    if (lane < 4) refp[(size_t)bq * 4 + lane] = rp[lane];
    // pairs 8 lane .. 8 lane + 7: component c = lane / 8 (64 pairs each), in [y, x, w, h] order
    const int comp[4] = {1, 0, 2, 3};
    const int c = lane >> 3, kp0 = (lane & 7) * 8;
    const float v = rp[comp[c]] * 6.28318530717958647692f;
    uint32_t h[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float arg = v * inv[kp0 + i];
        const __half2 sc = __floats2half2_rn(sinf(arg), cosf(arg));
        h[i] = *reinterpret_cast<const uint32_t*>(&sc);
    }
    uint4* so = reinterpret_cast<uint4*>(sine + (size_t)bq * 2 * Dm + c * half + 2 * kp0);
    so[0] = make_uint4(h[0], h[1], h[2], h[3]);
    so[1] = make_uint4(h[4], h[5], h[6], h[7]);
    const float4* f = reinterpret_cast<const float4*>(feat + (size_t)q * Dm) + 2 * lane;
    const float4 f0 = f[0], f1 = f[1];
    float4* to = reinterpret_cast<float4*>(tgt + (size_t)bq * Dm) + 2 * lane;
    to[0] = f0;
    to[1] = f1;
    const __half2 a0 = __floats2half2_rn(f0.x, f0.y), a1 = __floats2half2_rn(f0.z, f0.w);
    const __half2 a2 = __floats2half2_rn(f1.x, f1.y), a3 = __floats2half2_rn(f1.z, f1.w);
    reinterpret_cast<uint4*>(tgt16 + (size_t)bq * Dm)[lane] =
        make_uint4(*reinterpret_cast<const uint32_t*>(&a0), *reinterpret_cast<const uint32_t*>(&a1),
                   *reinterpret_cast<const uint32_t*>(&a2), *reinterpret_cast<const uint32_t*>(&a3));
}

__global__ void k_add_to_f16(const float* __restrict__ a, const float* __restrict__ b, size_t n,
                             __half* __restrict__ out) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = __float2half_rn(a[i] + b[i]);
}

// Four values per thread (16-byte loads, 8-byte stores) when n % 4 == 0 and the pointers allow.
__global__ void k_add_to_f16_v4(const float4* __restrict__ a, const float4* __restrict__ b, unsigned n4,
                                uint2* __restrict__ out) {
    const unsigned i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n4) return;
    const float4 x = a[i], y = b[i];
    __half2 h0 = __floats2half2_rn(x.x + y.x, x.y + y.y), h1 = __floats2half2_rn(x.z + y.z, x.w + y.w);
    out[i] = make_uint2(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1));
}

__global__ void k_to_f16(const float* __restrict__ a, size_t n, __half* __restrict__ out) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) out[i] = __float2half_rn(a[i]);
}

// 8 values per thread: two 16-byte loads, one 16-byte store (grid-strided)
__global__ void k_to_f16_v8(const float4* __restrict__ a, size_t n8, uint4* __restrict__ out) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (size_t)gridDim.x * blockDim.x) {
        const float4 u = a[2 * i], v = a[2 * i + 1];
        const __half2 h0 = __floats2half2_rn(u.x, u.y), h1 = __floats2half2_rn(u.z, u.w);
        const __half2 h2 = __floats2half2_rn(v.x, v.y), h3 = __floats2half2_rn(v.z, v.w);
        out[i] = make_uint4(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1),
                            *reinterpret_cast<const uint32_t*>(&h2), *reinterpret_cast<const uint32_t*>(&h3));
    }
}

// ---- deformable sampling: src/decoder.cpp:127-207, 236-285 ------------------
// One warp per query; each lane owns 8 consecutive channels (16 bytes of f16
// value per corner), 2 lanes per 16-channel head.  `row` holds the query's
// sampling offsets (H*P*2) then attention logits (H*P); vb is its image's value map.
// PP > 0: the point count as a compile-time constant, so the loads of every (point, corner) of the
// lane's 8 channels are issued before any of them is used (one memory latency per query instead of
// one per corner); PP == 0: any count P at run time.  Same arithmetic either way (an out-of-map
// corner contributes nothing).
template <int PP>
__device__ __forceinline__ void deform_query(const __half* __restrict__ vb, const float* row, const float* rp,
                                             int G, int H, int P_rt, int Dm, int lane, __half* __restrict__ orow) {
    const int P = PP > 0 ? PP : P_rt;
    const int hd = Dm / H;
    const float r0 = rp[0], r1 = rp[1], r2 = rp[2], r3 = rp[3];
    const float off_scale = 0.5f / (float)P;
    for (int c = lane; c < Dm / 8; c += 32) {
        const int h = (c * 8) / hd;
        // softmax over the P attention logits of head h (ggml_soft_max)
        float mx = -INFINITY;
        for (int p = 0; p < P; ++p) mx = fmaxf(mx, row[H * P * 2 + h * P + p]);
        float sum = 0.f;
        for (int p = 0; p < P; ++p) sum += expf(row[H * P * 2 + h * P + p] - mx);
        const float inv = 1.0f / sum;
        float acc[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = 0.f;
        constexpr int NP = PP > 0 ? PP : 1;  // points whose corners are loaded together
        for (int p0 = 0; p0 < P; p0 += NP) {
            uint4 u[NP][4];
            float wc[NP][4], wa[NP];
#pragma unroll
            for (int k = 0; k < NP; ++k) {
                const int p = p0 + k;
                wa[k] = expf(row[H * P * 2 + h * P + p] - mx) * inv;
                const float sx = (row[(h * P + p) * 2 + 0] * off_scale) * r2 + r0;
                const float sy = (row[(h * P + p) * 2 + 1] * off_scale) * r3 + r1;
                const float ix = sx * (float)G - 0.5f, iy = sy * (float)G - 0.5f;
                const int ix0 = (int)floorf(ix), iy0 = (int)floorf(iy);
                const float wx1 = ix - (float)ix0, wy1 = iy - (float)iy0;
                const float wx0 = 1.f - wx1, wy0 = 1.f - wy1;
#pragma unroll
                for (int corner = 0; corner < 4; ++corner) {
                    const int xi = ix0 + (corner & 1), yi = iy0 + (corner >> 1);
                    const bool in = xi >= 0 && xi < G && yi >= 0 && yi < G;
                    wc[k][corner] = ((corner & 1) ? wx1 : wx0) * ((corner >> 1) ? wy1 : wy0);
                    u[k][corner] = in ? __ldg(reinterpret_cast<const uint4*>(vb + ((size_t)yi * G + xi) * Dm + c * 8))
                                      : make_uint4(0u, 0u, 0u, 0u);
                }
            }
#pragma unroll
            for (int k = 0; k < NP; ++k) {
                float s[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) s[e] = 0.f;
#pragma unroll
                for (int corner = 0; corner < 4; ++corner) {
                    const __half2* h2 = reinterpret_cast<const __half2*>(&u[k][corner]);
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float2 f = __half22float2(h2[e]);
                        s[2 * e] += wc[k][corner] * f.x;
                        s[2 * e + 1] += wc[k][corner] * f.y;
                    }
                }
#pragma unroll
                for (int e = 0; e < 8; ++e) acc[e] += wa[k] * s[e];
            }
        }
        uint4 o;
        __half2* oh = reinterpret_cast<__half2*>(&o);
#pragma unroll
        for (int e = 0; e < 4; ++e) oh[e] = __floats2half2_rn(acc[2 * e], acc[2 * e + 1]);
        *reinterpret_cast<uint4*>(orow + c * 8) = o;
    }
}

// so_aw rows precomputed (f32 [B*NQ][ld_soaw]).
__global__ void k_deform(const __half* __restrict__ value, const float* __restrict__ so_aw, int ld_soaw,
                         const float* __restrict__ refp, int B, int NQ, int G, int H, int P, int Dm,
                         __half* __restrict__ out) {
    const int bq = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (bq >= B * NQ) return;
    const int b = bq / NQ;
    if (P == 2)  // the converter's variants: loads of both points issued together
        deform_query<2>(value + (size_t)b * G * G * Dm, so_aw + (size_t)bq * ld_soaw, refp + (size_t)bq * 4, G, H, P,
                        Dm, lane, out + (size_t)bq * Dm);
    else
        deform_query<0>(value + (size_t)b * G * G * Dm, so_aw + (size_t)bq * ld_soaw, refp + (size_t)bq * 4, G, H, P,
                        Dm, lane, out + (size_t)bq * Dm);
}

// src/rfdetr_model.cpp:438-448
__global__ void k_box_reparam(const float* __restrict__ d, const float* __restrict__ r, int n, float* __restrict__ o) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float* dd = d + (size_t)i * 4;
    const float* rr = r + (size_t)i * 4;
    float* oo = o + (size_t)i * 4;
    oo[0] = dd[0] * rr[2] + rr[0];
    oo[1] = dd[1] * rr[3] + rr[1];
    oo[2] = expf(dd[2]) * rr[2];
    oo[3] = expf(dd[3]) * rr[3];
}

// ---- segmentation: src/segmentation.cpp:187-199 (ggml_interpolate bilinear) --
__global__ void k_resize_bilinear(const float* __restrict__ src, int B, int G, int T, int C, float* __restrict__ dst) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)B * T * T * C) return;
    const int c = (int)(i % C);
    const size_t pix = i / C;
    const int b = (int)(pix / ((size_t)T * T));
    const int r = (int)(pix - (size_t)b * T * T);
    const int yy = r / T, xx = r - (r / T) * T;
    const float sf = (float)T / (float)G;
    const float fy = ((float)yy + 0.5f) / sf - 0.5f;
    int y0 = (int)floorf(fy), y1 = y0 + 1;
    y0 = min(max(y0, 0), G - 1);
    y1 = min(max(y1, 0), G - 1);
    const float dy = fminf(fmaxf(fy - (float)y0, 0.f), 1.f);
    const float fx = ((float)xx + 0.5f) / sf - 0.5f;
    int x0 = (int)floorf(fx), x1 = x0 + 1;
    x0 = min(max(x0, 0), G - 1);
    x1 = min(max(x1, 0), G - 1);
    const float dx = fminf(fmaxf(fx - (float)x0, 0.f), 1.f);
    const float* s = src + (size_t)b * G * G * C + c;
    const float a = s[((size_t)y0 * G + x0) * C], bb = s[((size_t)y0 * G + x1) * C];
    const float cc = s[((size_t)y1 * G + x0) * C], d = s[((size_t)y1 * G + x1) * C];
    dst[i] = a * (1 - dx) * (1 - dy) + bb * dx * (1 - dy) + cc * (1 - dx) * dy + d * dx * dy;
}

// Bilinear resize (align_corners = False, clamped edges), 4 channels per thread with 16-byte loads and
// stores and 32-bit index arithmetic; the same per-element arithmetic as k_resize_bilinear.
__global__ void k_resize_bilinear4(const float* __restrict__ src, int B, int G, int T, int C, float* __restrict__ dst) {
    const int C4 = C >> 2;
    const unsigned n = (unsigned)B * T * T * C4;
    const float sf = (float)T / (float)G;
    for (unsigned i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const unsigned c4 = i % (unsigned)C4;
        const unsigned pix = i / (unsigned)C4;
        const unsigned b = pix / (unsigned)(T * T);
        const unsigned r = pix - b * (unsigned)(T * T);
        const int yy = (int)(r / (unsigned)T), xx = (int)(r - (r / (unsigned)T) * (unsigned)T);
        const float fy = ((float)yy + 0.5f) / sf - 0.5f;
        int y0 = (int)floorf(fy), y1 = y0 + 1;
        y0 = min(max(y0, 0), G - 1);
        y1 = min(max(y1, 0), G - 1);
        const float dy = fminf(fmaxf(fy - (float)y0, 0.f), 1.f);
        const float fx = ((float)xx + 0.5f) / sf - 0.5f;
        int x0 = (int)floorf(fx), x1 = x0 + 1;
        x0 = min(max(x0, 0), G - 1);
        x1 = min(max(x1, 0), G - 1);
        const float dx = fminf(fmaxf(fx - (float)x0, 0.f), 1.f);
        const float4* s = reinterpret_cast<const float4*>(src + (size_t)b * G * G * C) + c4;
        const float4 a = s[((size_t)y0 * G + x0) * C4], bq = s[((size_t)y0 * G + x1) * C4];
        const float4 cq = s[((size_t)y1 * G + x0) * C4], d = s[((size_t)y1 * G + x1) * C4];
        float4 o;
        o.x = a.x * (1 - dx) * (1 - dy) + bq.x * dx * (1 - dy) + cq.x * (1 - dx) * dy + d.x * dx * dy;
        o.y = a.y * (1 - dx) * (1 - dy) + bq.y * dx * (1 - dy) + cq.y * (1 - dx) * dy + d.y * dx * dy;
        o.z = a.z * (1 - dx) * (1 - dy) + bq.z * dx * (1 - dy) + cq.z * (1 - dx) * dy + d.z * dx * dy;
        o.w = a.w * (1 - dx) * (1 - dy) + bq.w * dx * (1 - dy) + cq.w * (1 - dx) * dy + d.w * dx * dy;
        reinterpret_cast<float4*>(dst)[i] = o;
    }
}

// Depthwise 3x3 + bias + channel LN of 256-channel maps (src/segmentation.cpp:68-92), bandwidth-shaped:
// warp per pixel (warps of a CTA on consecutive pixels, so neighbours are L1 hits), lane per 8
// consecutive channels (two 16-byte loads per tap, one 16-byte f16 store), the taps' weights
// transposed tap-major into shared memory once per CTA, the loads of all nine taps issued before
// their sums (an out-of-map tap reads an in-map pixel and adds it with weight 0): one memory
// latency per pixel.  Per channel the same sequence of multiply-adds as k_dwconv_ln; the LayerNorm
// sums run in another order.
__global__ void __launch_bounds__(256, 2) k_dwconv_ln256(const float* __restrict__ x, int B, int H, int W,
                                                         const float* __restrict__ w9,
                                                         const float* __restrict__ bias,
                                                         const float* __restrict__ g,
                                                         const float* __restrict__ bb, float eps,
                                                         __half* __restrict__ out) {
    constexpr int C = 256;
    __shared__ __align__(16) float sw[9 * C];  // [tap][channel]
    __shared__ __align__(16) float sp[3 * C];  // bias, gamma, beta
    for (int i = threadIdx.x; i < 9 * C; i += blockDim.x) {
        const int k = i / C, c = i - k * C;
        sw[i] = w9[c * 9 + k];
    }
    for (int i = threadIdx.x; i < C; i += blockDim.x) {
        sp[i] = bias[i];
        sp[C + i] = g[i];
        sp[2 * C + i] = bb[i];
    }
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int c0 = lane * 8;
    const int npix = B * H * W;
    for (int pix = blockIdx.x * (blockDim.x >> 5) + warp; pix < npix; pix += gridDim.x * (blockDim.x >> 5)) {
        const int b = pix / (H * W), r = pix - b * (H * W);
        const int y = r / W, xq = r - y * W;
        float4 u[9][2];
        float wm[9];
#pragma unroll
        for (int k = 0; k < 9; ++k) {
            const int sy = y + k / 3 - 1, sx = xq + k % 3 - 1;
            const bool in = sy >= 0 && sy < H && sx >= 0 && sx < W;
            const float4* src =
                reinterpret_cast<const float4*>(x + ((size_t)(b * H + (in ? sy : y)) * W + (in ? sx : xq)) * C + c0);
            u[k][0] = src[0];
            u[k][1] = src[1];
            wm[k] = in ? 1.f : 0.f;
        }
        float acc[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = 0.f;
#pragma unroll
        for (int k = 0; k < 9; ++k) {
            const float4 w0 = *reinterpret_cast<const float4*>(sw + k * C + c0);
            const float4 w1 = *reinterpret_cast<const float4*>(sw + k * C + c0 + 4);
            acc[0] += (w0.x * wm[k]) * u[k][0].x;
            acc[1] += (w0.y * wm[k]) * u[k][0].y;
            acc[2] += (w0.z * wm[k]) * u[k][0].z;
            acc[3] += (w0.w * wm[k]) * u[k][0].w;
            acc[4] += (w1.x * wm[k]) * u[k][1].x;
            acc[5] += (w1.y * wm[k]) * u[k][1].y;
            acc[6] += (w1.z * wm[k]) * u[k][1].z;
            acc[7] += (w1.w * wm[k]) * u[k][1].w;
        }
        float s = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            acc[e] += sp[c0 + e];
            s += acc[e];
        }
        const float mean = warp_sum(s) / (float)C;
        float q = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const float d = acc[e] - mean;
            q += d * d;
        }
        const float rstd = 1.0f / sqrtf(warp_sum(q) / (float)C + eps);
        uint32_t h[4];
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
            const __half2 hv = __floats2half2_rn((acc[e] - mean) * rstd * sp[C + c0 + e] + sp[2 * C + c0 + e],
                                                 (acc[e + 1] - mean) * rstd * sp[C + c0 + e + 1] + sp[2 * C + c0 + e + 1]);
            h[e / 2] = *reinterpret_cast<const uint32_t*>(&hv);
        }
        *reinterpret_cast<uint4*>(out + (size_t)pix * C + c0) = make_uint4(h[0], h[1], h[2], h[3]);
    }
}

// depthwise 3x3 + bias + channel LN (src/segmentation.cpp:68-92); warp per pixel
__global__ void k_dwconv_ln(const float* __restrict__ x, int B, int H, int W, int C, const float* __restrict__ w9,
                            const float* __restrict__ bias, const float* __restrict__ g, const float* __restrict__ bb,
                            float eps, __half* __restrict__ out) {
    const int pix = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (pix >= B * H * W) return;
    const int b = pix / (H * W), r = pix - b * H * W;
    const int y = r / W, xq = r - (r / W) * W;
    float v[8];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int c = lane + 32 * i;
        float acc = 0.f;
        if (c < C) {
#pragma unroll
            for (int ky = 0; ky < 3; ++ky)
#pragma unroll
                for (int kx = 0; kx < 3; ++kx) {
                    const int sy = y + ky - 1, sx = xq + kx - 1;
                    if (sy < 0 || sy >= H || sx < 0 || sx >= W) continue;
                    acc += w9[c * 9 + ky * 3 + kx] * x[(((size_t)b * H + sy) * W + sx) * C + c];
                }
            acc += bias[c];
        }
        v[i] = acc;
        s += c < C ? acc : 0.f;
    }
    const float mean = warp_sum(s) / (float)C;
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int c = lane + 32 * i;
        const float d = c < C ? v[i] - mean : 0.f;
        q += d * d;
    }
    const float rstd = 1.0f / sqrtf(warp_sum(q) / (float)C + eps);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int c = lane + 32 * i;
        if (c < C) out[(size_t)pix * C + c] = __float2half_rn((v[i] - mean) * rstd * g[c] + bb[c]);
    }
}

}  // namespace

cudaError_t patch_im2col(const float* img, int B, int S, int p, int nw, int Kpad, __half* A, cudaStream_t st) {
    const int G = S / p, Tp = (G / nw) * (G / nw);
    const size_t n = (size_t)B * nw * nw * Tp * Kpad;
    k_patch_im2col<<<cdiv(n, 256), 256, 0, st>>>(img, B, S, p, nw, Kpad, A);
    return cudaGetLastError();
}

cudaError_t patch_from_rgb(const uint8_t* rgb, int B, int w, int h, int S, int p, int nw, int Kpad,
                           const float* mean3, const float* std3, __half* A, cudaStream_t st) {
    const int G = S / p, Tp = (G / nw) * (G / nw);
    const size_t rows = (size_t)B * nw * nw * Tp;
    if (Kpad % 8 || Kpad < 3 * p * p || ((uintptr_t)A & 15)) return cudaErrorInvalidValue;  // 16-byte stores
    if (rows >= (1u << 21)) return cudaErrorInvalidValue;
    // identity size with 16-byte aligned strips: CTA per (image, patch row)
    const size_t strip_smem = 3 * 256 * 4 + (size_t)((Kpad + 3) & ~3) * 4 + (size_t)p * S * 3;
    if (w == S && h == S && S % p == 0 && ((size_t)p * S * 3) % 16 == 0 && !((uintptr_t)rgb & 15) &&
        strip_smem <= 48 * 1024 && B <= 65535) {
        k_patch_strip<<<dim3(S / p, B), 256, strip_smem, st>>>(rgb, S, p, nw, Kpad, mean3[0], mean3[1], mean3[2],
                                                               std3[0], std3[1], std3[2], A);
        return cudaGetLastError();
    }
    const unsigned blocks = cdiv(rows, 8) < 148u * 8u ? cdiv(rows, 8) : 148u * 8u;  // warp per row, grid-strided
    k_patch_from_rgb<<<blocks, 256, 0, st>>>(rgb, B, w, h, S, p, nw, Kpad, mean3[0], mean3[1], mean3[2],
                                                   std3[0], std3[1], std3[2], A);
    return cudaGetLastError();
}

cudaError_t write_cls_rows(float* x, const float* clsrow, int B, int NW, int T, int D, cudaStream_t st) {
    const size_t n = (size_t)B * NW * D;
    k_cls_rows<<<cdiv(n, 256), 256, 0, st>>>(x, clsrow, B, NW, T, D);
    return cudaGetLastError();
}

// Split-K epilogue (see splitk_layernorm): warp per row, grid-strided, lane owns columns
// 4 * (lane + 32 i) .. + 3.
template <int NV>
__global__ void __launch_bounds__(256) k_splitk_ln(const float* __restrict__ part, int S, long long sstride, int rows,
                                                  const float* __restrict__ bias, const float* __restrict__ colscale,
                                                  const float* resid, int ldr, const float* __restrict__ g,
                                                  const float* __restrict__ bb, float eps, int silu,
                                                  float* out32, int ld32, __half* __restrict__ out16, int ld16) {
    constexpr int D = 128 * NV;
    const int lane = threadIdx.x & 31;
    const int stride = gridDim.x * (blockDim.x >> 5);
    for (int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < rows; row += stride) {
        float4 v[NV];
#pragma unroll
        for (int i = 0; i < NV; ++i) v[i] = reinterpret_cast<const float4*>(part + (size_t)row * D)[lane + 32 * i];
        for (int sp = 1; sp < S; ++sp) {
            const float4* q = reinterpret_cast<const float4*>(part + sp * sstride + (size_t)row * D);
#pragma unroll
            for (int i = 0; i < NV; ++i) {
                const float4 u = q[lane + 32 * i];
                v[i].x += u.x; v[i].y += u.y; v[i].z += u.z; v[i].w += u.w;
            }
        }
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const int c0 = 4 * (lane + 32 * i);
            if (bias) {
                const float4 u = *reinterpret_cast<const float4*>(bias + c0);
                v[i].x += u.x; v[i].y += u.y; v[i].z += u.z; v[i].w += u.w;
            }
            if (colscale) {
                const float4 u = *reinterpret_cast<const float4*>(colscale + c0);
                v[i].x *= u.x; v[i].y *= u.y; v[i].z *= u.z; v[i].w *= u.w;
            }
            if (resid) {
                const float4 u = *reinterpret_cast<const float4*>(resid + (size_t)row * ldr + c0);
                v[i].x += u.x; v[i].y += u.y; v[i].z += u.z; v[i].w += u.w;
            }
            s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
        }
        const float mean = warp_sum(s) / (float)D;
        float q = 0.f;
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const float a = v[i].x - mean, b2 = v[i].y - mean, c = v[i].z - mean, d = v[i].w - mean;
            q += (a * a + b2 * b2) + (c * c + d * d);
        }
        const float rstd = 1.0f / sqrtf(warp_sum(q) / (float)D + eps);
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const int c0 = 4 * (lane + 32 * i);
            const float4 gg = *reinterpret_cast<const float4*>(g + c0);
            const float4 be = *reinterpret_cast<const float4*>(bb + c0);
            float4 y;
            y.x = (v[i].x - mean) * rstd * gg.x + be.x;
            y.y = (v[i].y - mean) * rstd * gg.y + be.y;
            y.z = (v[i].z - mean) * rstd * gg.z + be.z;
            y.w = (v[i].w - mean) * rstd * gg.w + be.w;
            if (silu) {
                y.x = __fdividef(y.x, 1.0f + __expf(-y.x));
                y.y = __fdividef(y.y, 1.0f + __expf(-y.y));
                y.z = __fdividef(y.z, 1.0f + __expf(-y.z));
                y.w = __fdividef(y.w, 1.0f + __expf(-y.w));
            }
            if (out32) *reinterpret_cast<float4*>(out32 + (size_t)row * ld32 + c0) = y;
            if (out16) {
                __half2 h0 = __floats2half2_rn(y.x, y.y), h1 = __floats2half2_rn(y.z, y.w);
                *reinterpret_cast<uint2*>(out16 + (size_t)row * ld16 + c0) =
                    make_uint2(*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1));
            }
        }
    }
}

cudaError_t splitk_layernorm(const float* part, int S, long long sstride, int rows, int D, const float* bias,
                             const float* colscale, const float* resid, int ldr, const float* g, const float* b,
                             float eps, int act, float* out32, int ld32, __half* out16, int ld16,
                             cudaStream_t st) {
    if (S < 1 || rows <= 0 || (act != 0 && act != 3) || !g || !b) return cudaErrorInvalidValue;
    const unsigned blocks = cdiv(rows, 8) < 148u * 6u ? cdiv(rows, 8) : 148u * 6u;
    const int silu = act == 3;
    if (D == 384)
        k_splitk_ln<3><<<blocks, 256, 0, st>>>(part, S, sstride, rows, bias, colscale, resid, ldr, g, b, eps, silu,
                                               out32, ld32, out16, ld16);
    else if (D == 256)
        k_splitk_ln<2><<<blocks, 256, 0, st>>>(part, S, sstride, rows, bias, colscale, resid, ldr, g, b, eps, silu,
                                               out32, ld32, out16, ld16);
    else if (D == 128)
        k_splitk_ln<1><<<blocks, 256, 0, st>>>(part, S, sstride, rows, bias, colscale, resid, ldr, g, b, eps, silu,
                                               out32, ld32, out16, ld16);
    else
        return cudaErrorInvalidValue;
    return cudaGetLastError();
}

cudaError_t layernorm(const float* x, int rows, int D, const float* g, const float* b, float eps, float* y32,
                      __half* y16, cudaStream_t st) {
    if (D > 512) return cudaErrorInvalidValue;
    const unsigned blocks = cdiv(rows, 8);
    const bool vec = (D % 128 == 0) && !(((uintptr_t)x | (uintptr_t)y32 | (uintptr_t)y16) & 15);
    // the vector kernel is grid-strided: a few resident blocks per SM
    const unsigned vblocks = blocks < (unsigned)(148 * 6) ? blocks : (unsigned)(148 * 6);
    if (vec && D == 384) k_layernorm_v4<3><<<vblocks, 256, 0, st>>>(x, rows, g, b, eps, y32, y16, TapMap{});
    else if (vec && D == 256) k_layernorm_v4<2><<<vblocks, 256, 0, st>>>(x, rows, g, b, eps, y32, y16, TapMap{});
    else if (D <= 256) k_layernorm<8><<<blocks, 256, 0, st>>>(x, rows, D, g, b, eps, y32, y16);
    else k_layernorm<16><<<blocks, 256, 0, st>>>(x, rows, D, g, b, eps, y32, y16);
    return cudaGetLastError();
}

cudaError_t backbone_tap(const float* x, int B, int G, int nw, int D, const float* g, const float* b, __half* taps,
                         int ld, int col0, cudaStream_t st) {
    if (D > 384) return cudaErrorInvalidValue;
    const int rows = B * G * G;
    if ((D == 384 || D == 256) && rows < (1 << 21) && ld % 4 == 0 && col0 % 4 == 0 && !(((uintptr_t)x | (uintptr_t)taps) & 15) &&
        !(((uintptr_t)g | (uintptr_t)b) & 15)) {
        // vectorised, grid-strided LayerNorm over the gathered rows (8-byte f16 stores)
        TapMap tm;
        tm.G = G; tm.nw = nw; tm.ld = ld; tm.col0 = col0;
        tm.inv_gg = 1.0f / (float)(G * G);
        tm.inv_g = 1.0f / (float)G;
        tm.inv_ws = 1.0f / (float)(G / nw);
        const unsigned blocks = cdiv(rows, 8) < (unsigned)(148 * 6) ? cdiv(rows, 8) : (unsigned)(148 * 6);
        if (D == 384) k_layernorm_v4<3, true><<<blocks, 256, 0, st>>>(x, rows, g, b, 1e-6f, nullptr, taps, tm);
        else k_layernorm_v4<2, true><<<blocks, 256, 0, st>>>(x, rows, g, b, 1e-6f, nullptr, taps, tm);
        return cudaGetLastError();
    }
    k_tap<<<cdiv((size_t)rows, 8), 256, 0, st>>>(x, B, G, nw, D, g, b, taps, ld, col0);
    return cudaGetLastError();
}

cudaError_t layernorm_and_tap(const float* x, int B, int G, int nw, int D, const float* g1, const float* b1,
                              __half* y16, const float* g2, const float* b2, __half* taps, int ld, int col0,
                              cudaStream_t st) {
    const int ws = G / nw, T = ws * ws + 1;
    const long long rows = (long long)B * nw * nw * T;
    const bool fused = (D == 384 || D == 256) && rows < (1 << 21) && ld % 4 == 0 && col0 % 4 == 0 &&
                       !(((uintptr_t)x | (uintptr_t)y16 | (uintptr_t)taps) & 15) &&
                       !(((uintptr_t)g1 | (uintptr_t)b1 | (uintptr_t)g2 | (uintptr_t)b2) & 15);
    if (!fused) {
        const cudaError_t e = layernorm(x, (int)rows, D, g1, b1, 1e-6f, nullptr, y16, st);
        if (e != cudaSuccess) return e;
        return backbone_tap(x, B, G, nw, D, g2, b2, taps, ld, col0, st);
    }
    DualTapMap tm;
    tm.G = G; tm.nw = nw; tm.ld = ld; tm.col0 = col0;
    tm.inv_bt = 1.0f / (float)(nw * nw * T);
    tm.inv_t = 1.0f / (float)T;
    tm.inv_ws = 1.0f / (float)ws;
    tm.inv_nw = 1.0f / (float)nw;
    const unsigned blocks = cdiv((size_t)rows, 8) < (unsigned)(148 * 6) ? cdiv((size_t)rows, 8) : (unsigned)(148 * 6);
    if (D == 384) k_layernorm_dual<3><<<blocks, 256, 0, st>>>(x, (int)rows, g1, b1, y16, g2, b2, taps, tm);
    else k_layernorm_dual<2><<<blocks, 256, 0, st>>>(x, (int)rows, g1, b1, y16, g2, b2, taps, tm);
    return cudaGetLastError();
}

bool im2col3x3_source_ok(const __half* src, int lds, int B, int H, int W, int C) {
    return src && B > 0 && H > 0 && W > 0 && C > 0 && C % 8 == 0 && lds % 8 == 0 && lds >= C &&
           !((uintptr_t)src & 15);
}

cudaError_t im2col3x3(const __half* src, int lds, int B, int H, int W, int C, __half* A, cudaStream_t st) {
    // 16-byte loads of 8 channels at (pixel * lds + 8 * chunk) and 16-byte stores into A
    if (!im2col3x3_source_ok(src, lds, B, H, W, C) || !A || ((uintptr_t)A & 15)) return cudaErrorInvalidValue;
    const size_t n = (size_t)B * H * W * 9 * (C / 8);
    k_im2col3x3<<<cdiv(n, 256), 256, 0, st>>>(src, lds, B, H, W, C, A);
    return cudaGetLastError();
}

cudaError_t mask_memory(const float* mem, int B, int G, int C, __half* out, cudaStream_t st) {
    const size_t n = (size_t)B * G * G * C;
    k_mask_memory<<<cdiv(n, 256), 256, 0, st>>>(mem, B, G, C, out);
    return cudaGetLastError();
}

cudaError_t resize_legacy_rgb(const uint8_t* src, int B, int w, int h, const LegacyTapsDev& t, int ow, int oh,
                              uint8_t* dst, cudaStream_t st) {
    if (!src || !dst || !t.base || B < 0 || w <= 0 || h <= 0 || ow <= 0 || oh <= 0) return cudaErrorInvalidValue;
    if (B == 0) return cudaSuccess;
    const size_t n = (size_t)B * ow * oh;
    k_resize_legacy<<<cdiv(n, 256), 256, 0, st>>>(src, B, w, h, t.xf, t.xn, t.xc, t.xw, t.yf, t.yn, t.yc, t.yw, ow,
                                                  oh, dst);
    return cudaGetLastError();
}

cudaError_t two_stage_boxes(const float* delta, int B, int G, float* bbox, cudaStream_t st) {
    k_two_stage_boxes<<<cdiv((size_t)B * G * G, 256), 256, 0, st>>>(delta, B, G, bbox);
    return cudaGetLastError();
}

cudaError_t topk_tokens(const float* cls, int B, int N, int NC, int K, int32_t* idx, cudaStream_t st) {
    if (!cls || !idx || B < 0 || N <= 0 || N > kTopkMax || NC <= 0 || K < 0 || K > N) return cudaErrorInvalidValue;
    if (B == 0 || K == 0) return cudaSuccess;
    k_topk<<<B, 1024, 0, st>>>(cls, N, NC, K, idx);
    return cudaGetLastError();
}

cudaError_t query_init(const float* bbox_all, const int32_t* idx, const float* lrn_rp, const float* feat, int B,
                       int N, int NQ, int Dm, float* refp, __half* sine, float* tgt, __half* tgt16, cudaStream_t st) {
    auto al = [](const void* q) { return !((uintptr_t)q & 15); };
    if (Dm == 256 && al(feat) && al(sine) && al(tgt) && al(tgt16)) {
        const int rows = B * NQ;
        if (rows > 0) k_query_init256<<<cdiv((size_t)rows, 8), 256, 0, st>>>(bbox_all, idx, lrn_rp, feat, N, NQ, rows,
                                                                          refp, sine, tgt, tgt16);
        return cudaGetLastError();
    }
    k_query_init<<<B * NQ, 256, 0, st>>>(bbox_all, idx, lrn_rp, feat, N, NQ, Dm, refp, sine, tgt, tgt16);
    return cudaGetLastError();
}

cudaError_t add_to_f16(const float* a, const float* b, size_t n, __half* out, cudaStream_t st) {
    if (n % 4 == 0 && n / 4 < (1ull << 31) && !(((uintptr_t)a | (uintptr_t)b) & 15) && !((uintptr_t)out & 7)) {
        const size_t n4 = n / 4;
        k_add_to_f16_v4<<<cdiv(n4, 256), 256, 0, st>>>(reinterpret_cast<const float4*>(a),
                                                        reinterpret_cast<const float4*>(b), (unsigned)n4,
                                                        reinterpret_cast<uint2*>(out));
        return cudaGetLastError();
    }
    k_add_to_f16<<<cdiv(n, 256), 256, 0, st>>>(a, b, n, out);
    return cudaGetLastError();
}

cudaError_t to_f16(const float* a, size_t n, __half* out, cudaStream_t st) {
    if (n % 8 == 0 && !((uintptr_t)a & 15) && !((uintptr_t)out & 15)) {
        const size_t n8 = n / 8;
        const unsigned blocks = cdiv(n8, 256) < 148u * 16u ? cdiv(n8, 256) : 148u * 16u;
        if (n8) k_to_f16_v8<<<blocks, 256, 0, st>>>(reinterpret_cast<const float4*>(a), n8, reinterpret_cast<uint4*>(out));
        return cudaGetLastError();
    }
    k_to_f16<<<cdiv(n, 256), 256, 0, st>>>(a, n, out);
    return cudaGetLastError();
}

cudaError_t deform_sample(const __half* value, const float* so_aw, int ld_soaw, const float* refp, int B, int NQ,
                          int G, int heads, int points, int Dm, __half* out, cudaStream_t st) {
    if (Dm % 8 || (Dm / heads) % 8) return cudaErrorInvalidValue;
    k_deform<<<cdiv((size_t)B * NQ, 4), 128, 0, st>>>(value, so_aw, ld_soaw, refp, B, NQ, G, heads, points, Dm, out);
    return cudaGetLastError();
}

cudaError_t box_reparam(const float* delta, const float* refp, int n, float* out, cudaStream_t st) {
    k_box_reparam<<<cdiv(n, 256), 256, 0, st>>>(delta, refp, n, out);
    return cudaGetLastError();
}

cudaError_t resize_bilinear(const float* src, int B, int G, int T, int C, float* dst, cudaStream_t st) {
    const size_t n = (size_t)B * T * T * C;
    if (C % 4 == 0 && n / 4 < (1ull << 32) && !((uintptr_t)src & 15) && !((uintptr_t)dst & 15)) {
        const unsigned blocks = cdiv(n / 4, 256) < 148u * 16u ? cdiv(n / 4, 256) : 148u * 16u;
        if (n) k_resize_bilinear4<<<blocks, 256, 0, st>>>(src, B, G, T, C, dst);
        return cudaGetLastError();
    }
    k_resize_bilinear<<<cdiv(n, 256), 256, 0, st>>>(src, B, G, T, C, dst);
    return cudaGetLastError();
}

cudaError_t dwconv_ln(const float* x, int B, int H, int W, int C, const float* w9, const float* bias,
                      const float* g, const float* b, float eps, __half* out, cudaStream_t st) {
    if (C > 256) return cudaErrorInvalidValue;
    const size_t npix = (size_t)B * H * W;
    if (C == 256 && npix < (1u << 30) && !((uintptr_t)x & 15) && !((uintptr_t)out & 15)) {
        const unsigned blocks = cdiv(npix, 8) < 148u * 8u ? cdiv(npix, 8) : 148u * 8u;
        if (npix) k_dwconv_ln256<<<blocks, 256, 0, st>>>(x, B, H, W, w9, bias, g, b, eps, out);
        return cudaGetLastError();
    }
    k_dwconv_ln<<<cdiv(npix, 8), 256, 0, st>>>(x, B, H, W, C, w9, bias, g, b, eps, out);
    return cudaGetLastError();
}

}  // namespace rfb
