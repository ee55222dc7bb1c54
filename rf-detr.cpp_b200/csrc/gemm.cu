// Persistent, warp-specialized tcgen05 GEMM for sm_100a.
//
//   warp 0      TMA producer (one lane): A and B K-tiles -> smem ring
//   warp 1      TMEM allocator; one lane issues tcgen05.mma (M=128, N=BN, K=16)
//   warps 2..9  epilogue: tcgen05.ld accumulator rows, fused epilogue, TMA store
//               (two warps per TMEM lane quadrant, each owning half the columns)
//
// The accumulator is double-buffered in TMEM (2 x BN columns) so the epilogue
// of tile i overlaps the mainloop of tile i+1.  Tiles are assigned round-robin
// over a grid of one CTA per SM, N-fastest so that CTAs running together share
// the same A rows through L2 (A = activations, much larger than B = weights).
// Every mbarrier wait is bounded; on timeout the CTA records an error word and
// unwinds (no trap, no endless spin).
#include "gemm.cuh"
#include "sm100.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cstdio>
#include <cstring>
#include <atomic>
#include <mutex>

namespace rfb {

namespace {

constexpr int BM = 128;
constexpr int BK = 64;

template <int BN>
struct Cfg {
    static constexpr int STAGES = BN >= 192 ? 4 : (BN == 128 ? 6 : 8);
    static constexpr int A_BYTES = BM * BK * 2;
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int TMEM_COLS = BN == 192 ? 512 : 2 * BN;  // power of two >= 2 * BN
    static constexpr int OUT_STAGE = 8 * 4096;  // per epilogue warp: one 32-row x 128-byte box
    static constexpr int SMEM = STAGES * STAGE_BYTES + OUT_STAGE + 1024 /*align*/ + 256 /*barriers*/;
};

// erf-GELU, 0.5 v (1 + erf(v / sqrt 2)).
#ifndef RFB_GELU_AS
#define RFB_GELU_AS 1
#endif
__device__ __forceinline__ float rcp_approx(float x) {
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
}
__device__ __forceinline__ float gelu_erf(float v) {
#if RFB_GELU_AS
    // erf from Abramowitz & Stegun, Handbook of Mathematical Functions,
    // eq. 7.1.26 (Hastings' rational approximation):
    // erf(z) = 1 - t (a1 + t (a2 + t (a3 + t (a4 + t a5)))) e^{-z^2},
    // t = 1 / (1 + p z), z >= 0, |error| <= 1.5e-7.
    const float z = fabsf(v) * 0.70710678118654752440f;
    const float t = rcp_approx(fmaf(0.3275911f, z, 1.0f));
    const float poly = t * fmaf(t, fmaf(t, fmaf(t, fmaf(t, 1.061405429f, -1.453152027f), 1.421413741f),
                                        -0.284496736f), 0.254829592f);
    const float erf_abs = fmaf(-poly, __expf(-z * z), 1.0f);
    const float erf_v = __int_as_float(__float_as_int(erf_abs) | (__float_as_int(v) & 0x80000000));
    return 0.5f * v * (1.0f + erf_v);
#else
    return 0.5f * v * (1.0f + erff(v * 0.70710678118654752440f));
#endif
}

template <int ACT>
__device__ __forceinline__ float act_fn(float v) {
    if constexpr (ACT == ACT_GELU) return gelu_erf(v);
    else if constexpr (ACT == ACT_RELU) return fmaxf(v, 0.0f);
    else if constexpr (ACT == ACT_SILU) return v / (1.0f + expf(-v));
    else return v;
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

constexpr int kThreads = 320;     // 10 warps
constexpr int kEpiThreads = 256;  // warps 2..9

template <int BN, int EPI, int ACT>
__global__ void __launch_bounds__(kThreads, 1)
k_gemm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
       const __grid_constant__ CUtensorMap tmO16, const __grid_constant__ CUtensorMap tmO32, const GemmArgs p) {
    using C = Cfg<BN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + C::STAGES * C::A_BYTES;
    uint8_t* out_stage = smem + C::STAGES * C::STAGE_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(out_stage + C::OUT_STAGE);
    uint64_t* empty = full + C::STAGES;
    uint64_t* tfull = empty + C::STAGES;
    uint64_t* tempty = tfull + 2;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tempty + 2);
    volatile int* cta_abort = reinterpret_cast<volatile int*>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int m_tiles = (p.M + BM - 1) / BM;
    const int n_tiles = (p.N + BN - 1) / BN;
    const int tiles_per_batch = m_tiles * n_tiles;
    const int num_tiles = tiles_per_batch * p.batches;
    const int num_kb = (p.K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            mbar_init(&tfull[a], 1);
            mbar_init(&tempty[a], kEpiThreads);
        }
        *cta_abort = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
    }
    if (warp == 1) tmem_alloc(tmem_holder, C::TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;

    if (warp == 0) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
                const int b = tile / tiles_per_batch;
                const int r = tile - b * tiles_per_batch;
                const int mt = r / n_tiles, nt = r - mt * n_tiles;
                const int arow = b * p.a_batch_rows + mt * BM;
                const int brow = b * p.b_batch_rows + nt * BN;
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait(&empty[stage], phase ^ 1, cta_abort, p.err)) goto done;
                    mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
                    tma_load_2d(&tmA, &full[stage], sA + stage * C::A_BYTES, kb * BK, arow);
                    tma_load_2d(&tmB, &full[stage], sB + stage * C::B_BYTES, kb * BK, brow);
                    if (++stage == C::STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t IDESC = idesc_f16_f32(BM, BN);
            int stage = 0;
            uint32_t phase = 0;
            int local = 0;
            for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
                const int acc = local & 1;
                const uint32_t acc_phase = (local >> 1) & 1;
                if (!mbar_wait(&tempty[acc], acc_phase ^ 1, cta_abort, p.err)) goto done;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!mbar_wait(&full[stage], phase, cta_abort, p.err)) goto done;
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sA + stage * C::A_BYTES);
                    const uint32_t b0 = smem_u32(sB + stage * C::B_BYTES);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
                        umma_f16(d_tmem, sw128_kmajor_desc(a0 + kk * 32), sw128_kmajor_desc(b0 + kk * 32), IDESC,
                                 (kb | kk) != 0);
                    }
                    umma_commit(&empty[stage]);
                    if (++stage == C::STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                umma_commit(&tfull[acc]);
            }
        }
    } else {
        // ---------------- epilogue warps ----------------
        const int e = warp - 2;            // 0..7
        const int quad = warp & 3;         // TMEM lanes [32*quad, 32*quad + 32)
        const int half = e >> 2;           // which half of the tile's columns
        const int row_in_tile = quad * 32 + lane;
        // staging: [quad][half] boxes of 4 KB; the LN path uses both halves of its quad
        uint8_t* wptr = out_stage + quad * 8192 + half * 4096;
        const uint32_t wbuf = smem_u32(wptr);
        constexpr bool kSplit = (EPI != EPI_LN) && (BN >= 128);
        constexpr int kHalf0 = ((BN / 2 + 63) / 64) * 64;  // first half: whole 64-column chunks
        const bool active = kSplit || half == 0;
        const int col_begin = kSplit ? half * kHalf0 : 0;
        const int col_end = kSplit ? (half ? BN : kHalf0) : BN;
        int local = 0;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
            const int b = tile / tiles_per_batch;
            const int r = tile - b * tiles_per_batch;
            const int mt = r / n_tiles, nt = r - mt * n_tiles;
            const int acc = local & 1;
            const uint32_t acc_phase = (local >> 1) & 1;
            if (!mbar_wait(&tfull[acc], acc_phase, cta_abort, p.err)) goto done;
            tc_fence_after();
            const int m = mt * BM + row_in_tile;
            const int m0w = mt * BM + quad * 32;
            const bool row_ok = m < p.M;
            const uint32_t tbase = tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN;
            const long long boff = (long long)b * p.out_batch_stride;
            uint32_t raw[32];
            float v[32];

            if (!active) {
                // idle warp of the LN / narrow-tile paths
            } else if constexpr (EPI == EPI_LN) {
                // BN == N: this thread owns the whole output row.
                const float* rrow = (p.resid && row_ok) ? p.resid + (size_t)m * p.ldr : nullptr;
                float sum = 0.f;
                for (int c0 = 0; c0 < BN; c0 += 32) {
                    tmem_ld32(tbase + c0, raw);
                    const float bl = p.bias ? p.bias[c0 + lane] : 0.f;
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        float x = __uint_as_float(raw[j]) + bcast(bl, j);
                        if (rrow) x += rrow[c0 + j];
                        sum += x;
                    }
                }
                const float mean = sum / (float)BN;
                float sq = 0.f;
                for (int c0 = 0; c0 < BN; c0 += 32) {
                    tmem_ld32(tbase + c0, raw);
                    const float bl = p.bias ? p.bias[c0 + lane] : 0.f;
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        float x = __uint_as_float(raw[j]) + bcast(bl, j);
                        if (rrow) x += rrow[c0 + j];
                        const float d = x - mean;
                        sq += d * d;
                    }
                }
                const float rstd = 1.0f / sqrtf(sq / (float)BN + p.ln_eps);
                for (int c0 = 0; c0 < BN; c0 += 32) {
                    tmem_ld32(tbase + c0, raw);
                    const float bl = p.bias ? p.bias[c0 + lane] : 0.f;
                    const float gl = p.ln_g[c0 + lane], bbl = p.ln_b[c0 + lane];
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        float x = __uint_as_float(raw[j]) + bcast(bl, j);
                        if (rrow) x += rrow[c0 + j];
                        x = (x - mean) * rstd * bcast(gl, j) + bcast(bbl, j);
                        v[j] = act_fn<ACT>(x);
                    }
                    if (p.tma_out) {
                        // f32 box [32 rows][32 cols] at wbuf, f16 box [32 rows][64 cols] at wbuf + 4096
                        const int hf = (c0 >> 5) & 1;
                        if (lane == 0) bulk_wait_read<0>();
                        __syncwarp();
                        if (p.out32) {
#pragma unroll
                            for (int j = 0; j < 8; ++j)
                                st_shared_v4(swz(wbuf, lane, j), __float_as_uint(v[4 * j]), __float_as_uint(v[4 * j + 1]),
                                             __float_as_uint(v[4 * j + 2]), __float_as_uint(v[4 * j + 3]));
                        }
                        if (p.out16) {
#pragma unroll
                            for (int j = 0; j < 4; ++j)
                                st_shared_v4(swz(wbuf + 4096, lane, j + 4 * hf), pack_half2(v[8 * j], v[8 * j + 1]),
                                             pack_half2(v[8 * j + 2], v[8 * j + 3]), pack_half2(v[8 * j + 4], v[8 * j + 5]),
                                             pack_half2(v[8 * j + 6], v[8 * j + 7]));
                        }
                        fence_async_smem();
                        __syncwarp();
                        if (lane == 0) {
                            if (p.out32) tma_store_3d(&tmO32, wptr, c0, m0w, b);
                            if (p.out16 && (hf == 1 || c0 + 32 >= BN))
                                tma_store_3d(&tmO16, wptr + 4096, c0 & ~63, m0w, b);
                            bulk_commit();
                        }
                    } else if (row_ok) {
                        if (p.out32) store_row_f32(p.out32 + boff + (size_t)m * p.ld32 + c0, v, c0, p.N);
                        if (p.out16) store_row_f16(p.out16 + boff + (size_t)m * p.ld16 + c0, v, c0, p.N);
                    }
                }
            } else if (EPI != EPI_PATCH && p.tma_out) {
                if constexpr (EPI == EPI_F16) {
                    // 64-column chunks: one 128-byte f16 box row per thread
                    for (int c0 = col_begin; c0 < col_end; c0 += 64) {
                        uint32_t raw2[32];
                        tmem_ld32(tbase + c0, raw);
                        tmem_ld32(tbase + c0 + 32, raw2);
                        const int n0 = nt * BN + c0;
                        const float b0 = (p.bias && n0 + lane < p.N) ? p.bias[n0 + lane] : 0.f;
                        const float b1 = (p.bias && n0 + 32 + lane < p.N) ? p.bias[n0 + 32 + lane] : 0.f;
                        tmem_wait_ld();
                        if (lane == 0) bulk_wait_read<0>();
                        __syncwarp();
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            float w8[8];
#pragma unroll
                            for (int q = 0; q < 8; ++q) {
                                const int jj = 8 * j + q;
                                const float rv = __uint_as_float(jj < 32 ? raw[jj] : raw2[jj - 32]);
                                w8[q] = act_fn<ACT>(rv + (jj < 32 ? bcast(b0, jj) : bcast(b1, jj - 32)));
                            }
                            st_shared_v4(swz(wbuf, lane, j), pack_half2(w8[0], w8[1]), pack_half2(w8[2], w8[3]),
                                         pack_half2(w8[4], w8[5]), pack_half2(w8[6], w8[7]));
                        }
                        fence_async_smem();
                        __syncwarp();
                        if (lane == 0) {
                            if (n0 < p.N) tma_store_3d(&tmO16, wptr, n0, m0w, b);
                            bulk_commit();
                        }
                    }
                } else {
                    // f32 (store or residual reduce-add): 32-column chunks
                    for (int c0 = col_begin; c0 < col_end; c0 += 32) {
                        tmem_ld32(tbase + c0, raw);
                        const int n0 = nt * BN + c0;
                        const bool nok = n0 + lane < p.N;
                        const float bl = (p.bias && nok) ? p.bias[n0 + lane] : 0.f;
                        const float sl = (EPI == EPI_RESID && p.colscale) ? (nok ? p.colscale[n0 + lane] : 0.f) : 1.f;
                        tmem_wait_ld();
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            float x = act_fn<ACT>(__uint_as_float(raw[j]) + bcast(bl, j));
                            if (EPI == EPI_RESID) x *= bcast(sl, j);
                            v[j] = x;
                        }
                        if (lane == 0) bulk_wait_read<0>();
                        __syncwarp();
#pragma unroll
                        for (int j = 0; j < 8; ++j)
                            st_shared_v4(swz(wbuf, lane, j), __float_as_uint(v[4 * j]), __float_as_uint(v[4 * j + 1]),
                                         __float_as_uint(v[4 * j + 2]), __float_as_uint(v[4 * j + 3]));
                        fence_async_smem();
                        __syncwarp();
                        if (lane == 0) {
                            if (n0 < p.N) {
                                if (EPI == EPI_RESID) tma_reduce_add_3d(&tmO32, wptr, n0, m0w, b);
                                else tma_store_3d(&tmO32, wptr, n0, m0w, b);
                            }
                            bulk_commit();
                        }
                    }
                }
            } else {
                // direct stores (PATCH remap, or outputs a TMA map cannot describe)
                for (int c0 = col_begin; c0 < col_end; c0 += 32) {
                    tmem_ld32(tbase + c0, raw);
                    const int n0 = nt * BN + c0;
                    const bool nok = n0 + lane < p.N;
                    const float bl = (p.bias && nok) ? p.bias[n0 + lane] : 0.f;
                    const float sl = (EPI == EPI_RESID && p.colscale && nok) ? p.colscale[n0 + lane] : 1.f;
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] = act_fn<ACT>(__uint_as_float(raw[j]) + bcast(bl, j));
                    if constexpr (EPI == EPI_RESID) {
#pragma unroll
                        for (int j = 0; j < 32; ++j) v[j] *= bcast(sl, j);
                    }
                    if (!row_ok || n0 >= p.N) continue;
                    if constexpr (EPI == EPI_F16) {
                        store_row_f16(p.out16 + boff + (size_t)m * p.ld16 + n0, v, n0, p.N);
                    } else if constexpr (EPI == EPI_F32) {
                        store_row_f32(p.out32 + boff + (size_t)m * p.ld32 + n0, v, n0, p.N);
                    } else if constexpr (EPI == EPI_RESID) {
                        float* dst = p.out32 + boff + (size_t)m * p.ld32 + n0;
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (n0 + j < p.N) v[j] += dst[j];
                        store_row_f32(dst, v, n0, p.N);
                    } else if constexpr (EPI == EPI_PATCH) {
                        const int img = m / p.patch_rows;
                        const int rr = m - img * p.patch_rows;
                        const int win = rr / p.patch_tp;
                        const int tok = win * p.patch_t + 1 + (rr - win * p.patch_tp);
                        const float* pos = p.posw + (size_t)tok * p.N + n0;
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (n0 + j < p.N) v[j] += pos[j];
                        store_row_f32(p.out32 + ((size_t)img * p.patch_ntok + tok) * p.ld32 + n0, v, n0, p.N);
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&tempty[acc]);
        }
        if (lane == 0) bulk_wait<0>();
    }
done:
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::TMEM_COLS);
    }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;
int g_num_sms = 148;

bool load_encode() {
    std::call_once(g_encode_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    return g_encode != nullptr;
}

bool make_map(CUtensorMap* map, const void* base, int cols, long long rows, int ld, int box_rows) {
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

// 3-D output map (cols, rows, batch) with a 128-byte swizzled box of 32 rows.
bool make_out_map(CUtensorMap* map, const void* base, bool f16, int cols, int rows, int batches, int ld,
                  long long batch_stride) {
    const int esz = f16 ? 2 : 4;
    if (!base || ((uintptr_t)base & 15) || ((size_t)ld * esz) % 16) return false;
    if (batches > 1 && ((size_t)batch_stride * esz) % 16) return false;
    cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)batches};
    cuuint64_t strides[2] = {(cuuint64_t)ld * esz,
                             (cuuint64_t)(batches > 1 ? batch_stride : (long long)ld * rows) * esz};
    cuuint32_t box[3] = {(cuuint32_t)(128 / esz), 32, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    return g_encode(map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3,
                    const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, int EPI, int ACT>
cudaError_t launch(const GemmArgs& a_in, cudaStream_t st) {
    GemmArgs a = a_in;
    static std::atomic<uint64_t> attr_set{0};  // per (BN, EPI) instantiation, one bit per device
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = 1ull << (dev & 63);
    if (!(attr_set.load() & bit)) {
        e = cudaFuncSetAttribute(k_gemm<BN, EPI, ACT>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<BN>::SMEM);
        if (e != cudaSuccess) return e;
        attr_set.fetch_or(bit);
    }
    CUtensorMap ta, tb;
    const long long a_rows = (long long)a.a_batch_rows * (a.batches - 1) + a.M;
    const long long b_rows = (long long)a.b_batch_rows * (a.batches - 1) + a.N;
    if (!make_map(&ta, a.A, a.K, a_rows, a.lda, BM)) return cudaErrorInvalidValue;
    if (!make_map(&tb, a.B, a.K, b_rows, a.ldb, BN)) return cudaErrorInvalidValue;
    CUtensorMap to16, to32;
    std::memset(&to16, 0, sizeof(to16));
    std::memset(&to32, 0, sizeof(to32));
    bool tma = EPI != EPI_PATCH;
    if (tma && a.out16) tma = make_out_map(&to16, a.out16, true, a.N, a.M, a.batches, a.ld16, a.out_batch_stride);
    if (tma && a.out32) tma = make_out_map(&to32, a.out32, false, a.N, a.M, a.batches, a.ld32, a.out_batch_stride);
    a.tma_out = tma ? 1 : 0;
    const int tiles = ((a.M + BM - 1) / BM) * ((a.N + BN - 1) / BN) * a.batches;
    const int grid = tiles < g_num_sms ? tiles : g_num_sms;
    k_gemm<BN, EPI, ACT><<<grid, kThreads, Cfg<BN>::SMEM, st>>>(ta, tb, to16, to32, a);
    return cudaGetLastError();
}

template <int EPI, int ACT>
cudaError_t dispatch_bn(const GemmArgs& a, int bn, cudaStream_t st) {
    switch (bn) {
        case 256: return launch<256, EPI, ACT>(a, st);
        case 192: return launch<192, EPI, ACT>(a, st);
        case 128: return launch<128, EPI, ACT>(a, st);
        default: return launch<64, EPI, ACT>(a, st);
    }
}

}  // namespace

void gemm_set_num_sms(int n) { g_num_sms = n > 0 ? n : 148; }

cudaError_t gemm(const GemmArgs& a, cudaStream_t stream) {
    if (!load_encode()) return cudaErrorNotSupported;
    if (a.M <= 0 || a.N <= 0 || a.K <= 0 || a.batches <= 0) return cudaErrorInvalidValue;
    // TMA: 16-byte aligned base and row pitch
    if ((a.lda % 8) || (a.ldb % 8) || (((uintptr_t)a.A) & 15) || (((uintptr_t)a.B) & 15)) return cudaErrorInvalidValue;
    int bn;
    if (a.epi == EPI_LN) {
        if (a.N != 128 && a.N != 256) return cudaErrorInvalidValue;
        if (!a.ln_g || !a.ln_b) return cudaErrorInvalidValue;
        bn = a.N;
    } else if (a.N % 256 == 0) {
        bn = 256;
    } else if (a.N % 192 == 0) {
        bn = 192;  // N = 384 / 1152: two or six 192-wide tiles instead of 128-wide ones
    } else if (a.N > 64) {
        bn = 128;
    } else {
        bn = 64;
    }
    // instantiated (epilogue, activation) pairs
    switch (a.epi) {
        case EPI_F16:
            if (a.act == ACT_NONE) return dispatch_bn<EPI_F16, ACT_NONE>(a, bn, stream);
            if (a.act == ACT_GELU) return dispatch_bn<EPI_F16, ACT_GELU>(a, bn, stream);
            if (a.act == ACT_RELU) return dispatch_bn<EPI_F16, ACT_RELU>(a, bn, stream);
            return cudaErrorInvalidValue;
        case EPI_F32:
            if (a.act == ACT_NONE) return dispatch_bn<EPI_F32, ACT_NONE>(a, bn, stream);
            if (a.act == ACT_GELU) return dispatch_bn<EPI_F32, ACT_GELU>(a, bn, stream);
            if (a.act == ACT_RELU) return dispatch_bn<EPI_F32, ACT_RELU>(a, bn, stream);
            return cudaErrorInvalidValue;
        case EPI_RESID:
            if (a.act == ACT_NONE) return dispatch_bn<EPI_RESID, ACT_NONE>(a, bn, stream);
            if (a.act == ACT_GELU) return dispatch_bn<EPI_RESID, ACT_GELU>(a, bn, stream);
            return cudaErrorInvalidValue;
        case EPI_PATCH:
            if (a.act == ACT_NONE) return dispatch_bn<EPI_PATCH, ACT_NONE>(a, bn, stream);
            return cudaErrorInvalidValue;
        case EPI_LN:
            if (a.act == ACT_NONE) return bn == 256 ? launch<256, EPI_LN, ACT_NONE>(a, stream) : launch<128, EPI_LN, ACT_NONE>(a, stream);
            if (a.act == ACT_SILU) return bn == 256 ? launch<256, EPI_LN, ACT_SILU>(a, stream) : launch<128, EPI_LN, ACT_SILU>(a, stream);
            return cudaErrorInvalidValue;
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace rfb
