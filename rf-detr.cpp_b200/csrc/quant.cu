// GGUF block quantizers on the GPU: re-quantization of a model's weight
// tensors (the reference's `rfdetr-cli quantize`, examples/cli/main.cpp:387-640,
// which calls ggml_quantize_chunk) at load time or into a new file.
//
// One thread quantizes one block.  Every floating-point step is written with
// explicit round-to-nearest intrinsics (no fused multiply-add contraction) in
// the order of the scalar reference algorithms, so the bytes equal those of
// the float32 host restatements (gguf-py's Q8_0; the ggml K-quant reference
// quantizers quantize_row_q4_K_ref / _q5_K_ref / _q6_K_ref as restated here,
// without an importance matrix):
//   Q8_0  32 values: d = max|x| / 127, q = round-half-away(x * (1/d))      34 B
//   Q4_K  256 values, 8 sub-blocks of 32 with 6-bit scale and min found by
//         the weighted least-squares search make_qkx2 (nmax 15, rmin -1,
//         rdelta 0.1, 20 steps), 4-bit values                              144 B
//   Q5_K  as Q4_K with 5-bit values (nmax 31, rmin -0.5, rdelta 0.1, 15 steps) 176 B
//   Q6_K  16 sub-blocks of 16, signed 6-bit values, 8-bit sub-block scales
//         from the rmse search make_qx_quants (nmax 32, weights x^2)       210 B
#include "quant.cuh"

#include <cuda_fp16.h>

#include <cstring>

namespace rfb {

namespace {

__device__ __forceinline__ float fm(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fa(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fs(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fd(float a, float b) { return __fdiv_rn(a, b); }
__device__ __forceinline__ int nearest(float v) { return __float2int_rn(v); }  // half to even (rint)

// Every f16 field of these formats is 2-byte aligned (F16 elements; the block
// scales at offset 0 / 2 of Q8_0, Q4_K and Q5_K blocks and at offset 208 of
// 210-byte Q6_K blocks): one 16-bit store.
__device__ __forceinline__ void put_f16(uint8_t* p, float v) {
    *reinterpret_cast<__half*>(p) = __float2half_rn(v);
}
__device__ __forceinline__ float f16_round(float v) { return __half2float(__float2half_rn(v)); }

// ---- Q8_0 -------------------------------------------------------------------
__global__ void k_q8_0(const float* __restrict__ x, int64_t nblk, uint8_t* __restrict__ out) {
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nblk) return;
    const float* v = x + b * 32;
    float amax = 0.f;
    for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(v[i]));
    const float d = fd(amax, 127.f);
    const float id = d == 0.f ? 0.f : fd(1.f, d);
    uint8_t* o = out + b * 34;
    put_f16(o, d);
    for (int i = 0; i < 32; ++i) o[2 + i] = (uint8_t)(int8_t)(int)roundf(fm(v[i], id));
}

// ---- K-quant helpers ----------------------------------------------------------
// make_qkx2: 6-bit-able scale and min of one sub-block of n values (weighted).
__device__ void make_qkx2(const float* x, const float* w, int n, int nmax, float rmin, float rdelta, int nstep,
                          uint8_t* L, float* scale_out, float* min_out) {
    float mn = x[0], mx = x[0];
    for (int i = 1; i < n; ++i) {
        mn = fminf(mn, x[i]);
        mx = fmaxf(mx, x[i]);
    }
    float sum_w = w[0];
    float sum_x = fm(sum_w, x[0]);
    for (int i = 1; i < n; ++i) {
        sum_w = fa(sum_w, w[i]);
        sum_x = fa(sum_x, fm(w[i], x[i]));
    }
    mn = fminf(mn, 0.f);
    if (mx == mn) {
        for (int i = 0; i < n; ++i) L[i] = 0;
        *scale_out = 0.f;
        *min_out = -mn;
        return;
    }
    const float rng = fs(mx, mn);
    float iscale = fd((float)nmax, rng);
    float scale = fd(1.f, iscale);
    float best = 0.f;
    for (int i = 0; i < n; ++i) {
        int l = nearest(fm(iscale, fs(x[i], mn)));
        l = l < 0 ? 0 : (l > nmax ? nmax : l);
        L[i] = (uint8_t)l;
        const float diff = fs(fa(fm(scale, (float)l), mn), x[i]);
        best = fa(best, fm(w[i], fm(diff, diff)));
    }
    float the_min = mn;
    uint8_t La[32];
    for (int st = 0; st <= nstep; ++st) {
        const float isc = fd(fa(fa(rmin, fm(rdelta, (float)st)), (float)nmax), rng);
        float sl = 0.f, sl2 = 0.f, sxl = 0.f;
        for (int i = 0; i < n; ++i) {
            int l = nearest(fm(isc, fs(x[i], mn)));
            l = l < 0 ? 0 : (l > nmax ? nmax : l);
            La[i] = (uint8_t)l;
            const float wl = fm(w[i], (float)l);
            sl = fa(sl, wl);
            sl2 = fa(sl2, fm(wl, (float)l));
            sxl = fa(sxl, fm(wl, x[i]));
        }
        const float D = fs(fm(sum_w, sl2), fm(sl, sl));
        if (!(D > 0.f)) continue;
        float this_scale = fd(fs(fm(sum_w, sxl), fm(sum_x, sl)), D);
        float this_min = fd(fs(fm(sl2, sum_x), fm(sl, sxl)), D);
        if (this_min > 0.f) {
            this_scale = fd(sxl, sl2 == 0.f ? 1.f : sl2);
            this_min = 0.f;
        }
        float mad = 0.f;
        for (int i = 0; i < n; ++i) {
            const float d2 = fs(fa(fm(this_scale, (float)La[i]), this_min), x[i]);
            mad = fa(mad, fm(w[i], fm(d2, d2)));
        }
        if (mad < best) {
            for (int i = 0; i < n; ++i) L[i] = La[i];
            best = mad;
            scale = this_scale;
            the_min = this_min;
        }
    }
    *scale_out = scale;
    *min_out = -the_min;
}

// Shared by Q4_K and Q5_K: the 8 sub-block scales/mins of a 256-value block,
// packed as 12 bytes of 6-bit fields, with the f16 super-block scale and min.
__device__ void k4_scales(const float* scales, const float* mins, uint8_t* sc, float* d_out, float* dmin_out,
                          uint8_t* o_d) {
    float max_scale = 0.f, max_min = 0.f;
    for (int j = 0; j < 8; ++j) {
        if (scales[j] > max_scale) max_scale = scales[j];
        if (mins[j] > max_min) max_min = mins[j];
    }
    const float inv_scale = max_scale > 0.f ? fd(63.f, max_scale) : 0.f;
    const float inv_min = max_min > 0.f ? fd(63.f, max_min) : 0.f;
    uint8_t ls[8], lm[8];
    for (int j = 0; j < 8; ++j) {
        int a = nearest(fm(inv_scale, scales[j]));
        int b = nearest(fm(inv_min, mins[j]));
        ls[j] = (uint8_t)(a < 63 ? a : 63);  // the minimum first, then the byte (values >= 0 in practice)
        lm[j] = (uint8_t)(b < 63 ? b : 63);
    }
    for (int j = 0; j < 12; ++j) sc[j] = 0;
    for (int j = 0; j < 8; ++j) {
        if (j < 4) {
            sc[j] = ls[j];
            sc[j + 4] = lm[j];
        } else {
            sc[j + 4] = (uint8_t)((ls[j] & 0xF) | ((lm[j] & 0xF) << 4));
            sc[j - 4] |= (uint8_t)((ls[j] >> 4) << 6);
            sc[j] |= (uint8_t)((lm[j] >> 4) << 6);
        }
    }
    put_f16(o_d, fd(max_scale, 63.f));
    put_f16(o_d + 2, fd(max_min, 63.f));
    *d_out = f16_round(fd(max_scale, 63.f));
    *dmin_out = f16_round(fd(max_min, 63.f));
}

__device__ __forceinline__ void scale_min(const uint8_t* sc, int j, int* s, int* m) {
    if (j < 4) {
        *s = sc[j] & 63;
        *m = sc[j + 4] & 63;
    } else {
        *s = (sc[j + 4] & 0xF) | ((sc[j - 4] >> 6) << 4);
        *m = (sc[j + 4] >> 4) | ((sc[j] >> 6) << 4);
    }
}

// Q4_K (nbits 4) and Q5_K (nbits 5): one thread per 256-value block.
template <int NBITS>
__global__ void k_qk(const float* __restrict__ x, int64_t nblk, uint8_t* __restrict__ out) {
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nblk) return;
    constexpr int NMAX = (1 << NBITS) - 1;
    constexpr int BYTES = NBITS == 4 ? 144 : 176;
    const float* v = x + b * 256;
    uint8_t L[256];
    float scales[8], mins[8];
    for (int j = 0; j < 8; ++j) {
        const float* xs = v + 32 * j;
        float sum_x2 = 0.f;
        for (int i = 0; i < 32; ++i) sum_x2 = fa(sum_x2, fm(xs[i], xs[i]));
        const float av = __fsqrt_rn(fd(sum_x2, 32.f));
        float w[32];
        for (int i = 0; i < 32; ++i) w[i] = fa(av, fabsf(xs[i]));
        make_qkx2(xs, w, 32, NMAX, NBITS == 4 ? -1.f : -0.5f, 0.1f, NBITS == 4 ? 20 : 15, L + 32 * j, &scales[j],
                  &mins[j]);
    }
    uint8_t* o = out + b * BYTES;
    uint8_t* sc = o + 4;
    float d, dmin;
    k4_scales(scales, mins, sc, &d, &dmin, o);
    for (int j = 0; j < 8; ++j) {
        int s, m;
        scale_min(sc, j, &s, &m);
        const float dj = fm(d, (float)s);
        const float dmj = fm(dmin, (float)m);
        for (int i = 0; i < 32; ++i) {
            int l = 0;
            if (dj != 0.f) {
                l = nearest(fd(fa(v[32 * j + i], dmj), dj));
                l = l < 0 ? 0 : (l > NMAX ? NMAX : l);
            }
            L[32 * j + i] = (uint8_t)l;
        }
    }
    if (NBITS == 4) {
        uint8_t* qs = o + 16;
        for (int t = 0; t < 4; ++t)
            for (int l = 0; l < 32; ++l) qs[32 * t + l] = (uint8_t)(L[64 * t + l] | (L[64 * t + 32 + l] << 4));
    } else {
        uint8_t* qh = o + 16;
        uint8_t* ql = o + 48;
        for (int j = 0; j < 32; ++j) qh[j] = 0;
        uint8_t m1 = 1, m2 = 2;
        for (int n = 0; n < 256; n += 64) {
            for (int j = 0; j < 32; ++j) {
                int l1 = L[n + j];
                if (l1 > 15) {
                    l1 -= 16;
                    qh[j] |= m1;
                }
                int l2 = L[n + j + 32];
                if (l2 > 15) {
                    l2 -= 16;
                    qh[j] |= m2;
                }
                ql[n / 2 + j] = (uint8_t)(l1 | (l2 << 4));
            }
            m1 <<= 2;
            m2 <<= 2;
        }
    }
}

// make_qx_quants with rmse_type 1 (weights x^2): signed levels in [-nmax, nmax-1].
__device__ float make_qx(const float* x, int n, int nmax, int8_t* L) {
    float mx = 0.f, amax = 0.f;
    for (int i = 0; i < n; ++i) {
        const float ax = fabsf(x[i]);
        if (ax > amax) {
            amax = ax;
            mx = x[i];
        }
    }
    if (amax < 1e-15f) {
        for (int i = 0; i < n; ++i) L[i] = 0;
        return 0.f;
    }
    float iscale = fd(-(float)nmax, mx);
    float sumlx = 0.f, suml2 = 0.f;
    for (int i = 0; i < n; ++i) {
        int l = nearest(fm(iscale, x[i]));
        l = l < -nmax ? -nmax : (l > nmax - 1 ? nmax - 1 : l);
        L[i] = (int8_t)(l + nmax);
        const float w = fm(x[i], x[i]);
        sumlx = fa(sumlx, fm(fm(w, x[i]), (float)l));
        suml2 = fa(suml2, fm(fm(w, (float)l), (float)l));
    }
    float scale = suml2 != 0.f ? fd(sumlx, suml2) : 0.f;
    float best = fm(scale, sumlx);
    for (int is = -9; is <= 9; ++is) {
        if (is == 0) continue;
        iscale = fd(-fa((float)nmax, fm(0.1f, (float)is)), mx);
        sumlx = suml2 = 0.f;
        for (int i = 0; i < n; ++i) {
            int l = nearest(fm(iscale, x[i]));
            l = l < -nmax ? -nmax : (l > nmax - 1 ? nmax - 1 : l);
            const float w = fm(x[i], x[i]);
            sumlx = fa(sumlx, fm(fm(w, x[i]), (float)l));
            suml2 = fa(suml2, fm(fm(w, (float)l), (float)l));
        }
        if (suml2 > 0.f && fm(sumlx, sumlx) > fm(best, suml2)) {
            for (int i = 0; i < n; ++i) {
                int l = nearest(fm(iscale, x[i]));
                l = l < -nmax ? -nmax : (l > nmax - 1 ? nmax - 1 : l);
                L[i] = (int8_t)(l + nmax);
            }
            scale = fd(sumlx, suml2);
            best = fm(scale, sumlx);
        }
    }
    return scale;
}

__global__ void k_q6_K(const float* __restrict__ x, int64_t nblk, uint8_t* __restrict__ out) {
    const int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nblk) return;
    const float* v = x + b * 256;
    int8_t L[256];
    float scales[16];
    float max_scale = 0.f, max_abs = 0.f;
    for (int ib = 0; ib < 16; ++ib) {
        const float s = make_qx(v + 16 * ib, 16, 32, L + 16 * ib);
        scales[ib] = s;
        const float a = fabsf(s);
        if (a > max_abs) {
            max_abs = a;
            max_scale = s;
        }
    }
    uint8_t* o = out + b * 210;
    uint8_t* ql = o;
    uint8_t* qh = o + 128;
    int8_t* sc = reinterpret_cast<int8_t*>(o + 192);
    if (max_abs == 0.f) {
        for (int i = 0; i < 210; ++i) o[i] = 0;
        return;
    }
    const float iscale = fd(-128.f, max_scale);
    put_f16(o + 208, fd(1.f, iscale));
    const float d = f16_round(fd(1.f, iscale));
    for (int ib = 0; ib < 16; ++ib) {
        const int q = nearest(fm(iscale, scales[ib]));
        sc[ib] = (int8_t)(q < 127 ? q : 127);
    }
    for (int j = 0; j < 16; ++j) {
        const float dj = fm(d, (float)sc[j]);
        if (dj == 0.f) continue;
        for (int i = 0; i < 16; ++i) {
            int l = nearest(fd(v[16 * j + i], dj));
            l = l < -32 ? -32 : (l > 31 ? 31 : l);
            L[16 * j + i] = (int8_t)(l + 32);
        }
    }
    for (int j = 0; j < 256; j += 128) {
        for (int l = 0; l < 32; ++l) {
            const uint8_t q1 = (uint8_t)(L[j + l] & 0xF), q2 = (uint8_t)(L[j + l + 32] & 0xF);
            const uint8_t q3 = (uint8_t)(L[j + l + 64] & 0xF), q4 = (uint8_t)(L[j + l + 96] & 0xF);
            ql[j / 2 + l] = (uint8_t)(q1 | (q3 << 4));
            ql[j / 2 + l + 32] = (uint8_t)(q2 | (q4 << 4));
            qh[j / 4 + l] = (uint8_t)(((uint8_t)L[j + l] >> 4) | (((uint8_t)L[j + l + 32] >> 4) << 2) |
                                      (((uint8_t)L[j + l + 64] >> 4) << 4) | (((uint8_t)L[j + l + 96] >> 4) << 6));
        }
    }
}

__global__ void k_f16(const float* __restrict__ x, int64_t n, uint8_t* __restrict__ out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) put_f16(out + 2 * i, x[i]);
}

}  // namespace

bool quant_block_shape(uint32_t type, int* elems, int* bytes) {
    switch (type) {
        case 1: *elems = 1; *bytes = 2; return true;      // F16
        case 8: *elems = 32; *bytes = 34; return true;    // Q8_0
        case 12: *elems = 256; *bytes = 144; return true; // Q4_K
        case 13: *elems = 256; *bytes = 176; return true; // Q5_K
        case 14: *elems = 256; *bytes = 210; return true; // Q6_K
        default: return false;
    }
}

cudaError_t quantize_device(uint32_t type, const float* d_src, int64_t n, uint8_t* d_out, cudaStream_t st) {
    int be, bb;
    if (!quant_block_shape(type, &be, &bb) || n < 0 || n % be) return cudaErrorInvalidValue;
    const int64_t nblk = n / be;
    if (nblk == 0) return cudaSuccess;
    const int threads = type == 1 ? 256 : 64;
    const unsigned grid = (unsigned)((nblk + threads - 1) / threads);
    switch (type) {
        case 1: k_f16<<<grid, threads, 0, st>>>(d_src, nblk, d_out); break;
        case 8: k_q8_0<<<grid, threads, 0, st>>>(d_src, nblk, d_out); break;
        case 12: k_qk<4><<<grid, threads, 0, st>>>(d_src, nblk, d_out); break;
        case 13: k_qk<5><<<grid, threads, 0, st>>>(d_src, nblk, d_out); break;
        case 14: k_q6_K<<<grid, threads, 0, st>>>(d_src, nblk, d_out); break;
    }
    return cudaGetLastError();
}

}  // namespace rfb
