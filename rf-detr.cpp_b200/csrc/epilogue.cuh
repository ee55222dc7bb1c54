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

// erf-GELU, 0.5 v (1 + erf(v / sqrt 2)) = v Phi(v), written as
//   GELU(v) = max(v, 0) - a 2^L(a),  a = min(|v|, 6),  L(a) = log2 Phi(-a)
// (v Phi(v) is v - a Phi(-a) for v = a >= 0 and -a Phi(-a) for v = -a; Phi is the
// standard normal CDF).  L, the Gaussian factor included, is a degree-6 polynomial:
// a near-minimax fit on [0, 6], weighted so that the error of a 2^L stays below a
// quarter of the f16 spacing of a Phi(-a) where that is a normal f16 (and 1e-7
// absolute below), by least squares on 400001 points against scipy.special.log_ndtr
// refined with Lawson's iteratively reweighted least squares (C. L. Lawson, 1961).
// Evaluated in float32 with one exp2, |GELU error| <= 3.2e-7 for every input, and
// 99.93 % of the outputs in the f16 normal range round to the correctly rounded f16;
// the clamp at 6 adds < 6e-9.  Six FMAs, one exp2 and one FMA per value, no divide:
// the packed pair form below runs them on the f32x2 FMA path (two values per
// instruction).  Build with -DRFB_GELU_ERFF=1 to use erff instead.
#ifndef RFB_GELU_ERFF
#define RFB_GELU_ERFF 0
#endif
static __constant__ float kGeluL[7] = {3.525229477e-05f,  -7.827336667e-04f, 8.099309169e-03f, -5.338359997e-02f,
                                       -4.588511288e-01f, -1.151151538e+00f, -1.000000477e+00f};
constexpr int kGeluTerms = 7;
constexpr float kGeluClamp = 6.0f;

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
    float p = kGeluL[0];
#pragma unroll
    for (int k = 1; k < kGeluTerms; ++k) p = fmaf(p, a, kGeluL[k]);
    return fmaf(-a, ex2_approx(p), fmaxf(v, 0.0f));
#endif
}

// Two values at once; the same arithmetic as gelu_erf, bit for bit.
__device__ __forceinline__ float2 gelu_erf2(float2 v) {
#if RFB_GELU_ERFF
    return make_float2(gelu_erf(v.x), gelu_erf(v.y));
#else
    const float2 a = make_float2(fminf(fabsf(v.x), kGeluClamp), fminf(fabsf(v.y), kGeluClamp));
    float2 p = make_float2(kGeluL[0], kGeluL[0]);
#pragma unroll
    for (int k = 1; k < kGeluTerms; ++k) p = __ffma2_rn(p, a, make_float2(kGeluL[k], kGeluL[k]));
    const float2 e = make_float2(ex2_approx(p.x), ex2_approx(p.y));
    return __ffma2_rn(make_float2(-a.x, -a.y), e, make_float2(fmaxf(v.x, 0.0f), fmaxf(v.y, 0.0f)));
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

// The same for a 32-row x 64-byte box (64-byte swizzle: address bits 4-5 XOR bits 7-8): row
// `lane` starts at byte lane * 64 and its 16-byte chunk j lands at chunk (j ^ ((lane >> 1) & 3)).
__device__ __forceinline__ uint32_t swz64(uint32_t base, int lane, int j) {
    return base + lane * 64 + ((j ^ ((lane >> 1) & 3)) << 4);
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
