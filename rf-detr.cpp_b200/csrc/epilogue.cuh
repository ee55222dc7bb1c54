// Epilogue arithmetic shared by the tcgen05 GEMM and the fused MLP kernel:
// activations (erf-GELU as a packed-f32 polynomial, ReLU, SiLU), f16
// packing, 128-byte-swizzled staging addresses, warp-uniform per-column
// constant loads and row stores.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "gemm.cuh"
#include "sm100.cuh"

namespace rfb {
namespace {

// erf-GELU, 0.5 v (1 + erf(v / sqrt 2)), written as
//   GELU(v) = max(v, 0) - a e^{-a^2/2} R(a),  a = min(|v|, 6),
//   R(a) = 0.5 erfcx(a / sqrt 2)
// (erfcx = the scaled complementary error function).  -R is a polynomial,
// a near-minimax fit on [0, 6] weighted by a e^{-a^2/2}: weighted least
// squares on 200001 points against scipy.special.erfcx, refined by Lawson's
// iteratively reweighted least squares (C. L. Lawson, 1961), 60 iterations.
// Evaluated in float32 with exp2, the absolute error of GELU for
// every input is <= 1.1e-7 with degree 10, <= 7.9e-7 with degree 8 and
// <= 2.9e-6 with degree 7 (f16 spacing is 9.8e-7 at 0.002 and 2.4e-4 at 0.5);
// the clamp at 6 adds < 7e-9.  One exp2 and (degree + 1) FMAs per value, no
// divide: the packed pair form below runs the polynomial on the f32x2 FMA
// path (two values per instruction).  The epilogue of a GEMM with a GELU is
// bound by these FMAs, so RFB_GELU_DEGREE trades them against accuracy.
// Build with -DRFB_GELU_ERFF=1 to use erff instead.
#ifndef RFB_GELU_ERFF
#define RFB_GELU_ERFF 0
#endif
#ifndef RFB_GELU_DEGREE
#define RFB_GELU_DEGREE 8
#endif
#if RFB_GELU_DEGREE == 10
static __constant__ float kGeluNegR[11] = {
    -9.078557923e-07f, 2.187343125e-05f, -2.361505467e-04f, 1.531139482e-03f, -6.791573483e-03f,
    2.246006206e-02f, -5.929261073e-02f, 1.313898265e-01f, -2.495388836e-01f, 3.988756537e-01f,
    -4.999966621e-01f};
#elif RFB_GELU_DEGREE == 8
static __constant__ float kGeluNegR[9] = {
    -2.124682942e-05f, 3.925739147e-04f, -3.196175443e-03f, 1.543588843e-02f, -5.079322681e-02f,
    1.252110153e-01f, -2.470255792e-01f, 3.983812630e-01f, -4.999636412e-01f};
#elif RFB_GELU_DEGREE == 7
static __constant__ float kGeluNegR[8] = {
    9.495724225e-05f, -1.505025313e-03f, 1.039928570e-02f, -4.231634364e-02f, 1.171148866e-01f,
    -2.428599894e-01f, 3.973712325e-01f, -4.998818636e-01f};
#else
#error "RFB_GELU_DEGREE must be 10, 8 or 7"
#endif
constexpr int kGeluTerms = RFB_GELU_DEGREE + 1;
constexpr float kGeluClamp = 6.0f;
constexpr float kNegHalfLog2e = -0.72134752044448170368f;  // -0.5 / ln 2

__device__ __forceinline__ float ex2_approx(float x) {
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}

__device__ __forceinline__ float gelu_erf(float v) {
#if RFB_GELU_ERFF
    return 0.5f * v * (1.0f + erff(v * 0.70710678118654752440f));
#else
    const float a = fminf(fabsf(v), kGeluClamp);
    const float e = ex2_approx((a * kNegHalfLog2e) * a);
    float p = kGeluNegR[0];
#pragma unroll
    for (int k = 1; k < kGeluTerms; ++k) p = fmaf(p, a, kGeluNegR[k]);
    return fmaf(a * e, p, fmaxf(v, 0.0f));
#endif
}

// Two values at once; the same arithmetic as gelu_erf, bit for bit.
__device__ __forceinline__ float2 gelu_erf2(float2 v) {
#if RFB_GELU_ERFF
    return make_float2(gelu_erf(v.x), gelu_erf(v.y));
#else
    const float2 a = make_float2(fminf(fabsf(v.x), kGeluClamp), fminf(fabsf(v.y), kGeluClamp));
    const float2 s = __fmul2_rn(__fmul2_rn(a, make_float2(kNegHalfLog2e, kNegHalfLog2e)), a);
    const float2 e = make_float2(ex2_approx(s.x), ex2_approx(s.y));
    float2 p = make_float2(kGeluNegR[0], kGeluNegR[0]);
#pragma unroll
    for (int k = 1; k < kGeluTerms; ++k) p = __ffma2_rn(p, a, make_float2(kGeluNegR[k], kGeluNegR[k]));
    return __ffma2_rn(__fmul2_rn(a, e), p, make_float2(fmaxf(v.x, 0.0f), fmaxf(v.y, 0.0f)));
#endif
}

template <int ACT>
__device__ __forceinline__ float act_fn(float v) {
    if constexpr (ACT == ACT_GELU) return gelu_erf(v);
    else if constexpr (ACT == ACT_RELU) return fmaxf(v, 0.0f);
    else if constexpr (ACT == ACT_SILU) return __fdividef(v, 1.0f + __expf(-v));  // 0 for v < -88
    else return v;
}

template <int ACT>
__device__ __forceinline__ float2 act2(float2 v) {
    if constexpr (ACT == ACT_GELU) return gelu_erf2(v);
    else if constexpr (ACT == ACT_NONE) return v;
    else return make_float2(act_fn<ACT>(v.x), act_fn<ACT>(v.y));
}

// Store 32 consecutive values of one row (columns n0..n0+31, masked by N).
__device__ __forceinline__ void store_row_f32(float* dst, const float* v, int n0, int N) {
    if (n0 + 32 <= N && (((uintptr_t)dst) & 15) == 0) {
        float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
        for (int j = 0; j < 8; ++j) d4[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
            if (n0 + j < N) dst[j] = v[j];
    }
}

__device__ __forceinline__ void store_row_f16(__half* dst, const float* v, int n0, int N) {
    if (n0 + 32 <= N && (((uintptr_t)dst) & 15) == 0) {
        uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            __half2 h0 = __floats2half2_rn(v[8 * j + 0], v[8 * j + 1]);
            __half2 h1 = __floats2half2_rn(v[8 * j + 2], v[8 * j + 3]);
            __half2 h2 = __floats2half2_rn(v[8 * j + 4], v[8 * j + 5]);
            __half2 h3 = __floats2half2_rn(v[8 * j + 6], v[8 * j + 7]);
            uint4 u;
            u.x = *reinterpret_cast<uint32_t*>(&h0);
            u.y = *reinterpret_cast<uint32_t*>(&h1);
            u.z = *reinterpret_cast<uint32_t*>(&h2);
            u.w = *reinterpret_cast<uint32_t*>(&h3);
            d4[j] = u;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
            if (n0 + j < N) dst[j] = __float2half_rn(v[j]);
    }
}

// Value of lane j's register (static j after unrolling).
__device__ __forceinline__ float bcast(float x, int j) { return __shfl_sync(0xffffffffu, x, j); }

// Swizzled (128-byte pattern) staging of one 32-row x 128-byte box: thread
// `lane` owns row `lane`; 16-byte chunk j lands at chunk (j ^ (lane & 7)).
__device__ __forceinline__ uint32_t swz(uint32_t base, int lane, int j) {
    return base + lane * 128 + ((j ^ (lane & 7)) << 4);
}

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

// `4 * NV` consecutive per-column constants starting at column n0, the same
// for every lane of the warp (one output row per lane): 16-byte broadcast
// loads when `vec`, else guarded scalar loads (columns >= N read `dflt`).
template <int NV>
__device__ __forceinline__ void load_cols(float (&d)[4 * NV], const float* src, int n0, int N, bool vec,
                                          float dflt) {
    if (vec) {
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const float4 u = __ldg(reinterpret_cast<const float4*>(src + n0) + i);
            d[4 * i] = u.x; d[4 * i + 1] = u.y; d[4 * i + 2] = u.z; d[4 * i + 3] = u.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 4 * NV; ++i) d[i] = (src && n0 + i < N) ? src[n0 + i] : dflt;
    }
}

__device__ __forceinline__ bool aligned16(const void* q) { return (((uintptr_t)q) & 15) == 0; }


}  // namespace
}  // namespace rfb
