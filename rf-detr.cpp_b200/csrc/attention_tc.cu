// Fused multi-head attention on the 5th-generation tensor cores (head_dim 64):
// the windowed and global blocks of the DINOv2 backbone.  Sequences longer than
// 128 tokens (the global blocks) run k_attn_tc128 (128-key blocks, P kept in
// TMEM; described above that kernel); the windows run the 64-key kernels below.
//
// One CTA = 128 query rows of one (group, head); keys in blocks of 64.
//   warp 0      TMA: Q once, then K/V blocks into a 4-slot ring (3-D tensor
//               maps (column, token, group): rows past the sequence end load
//               as zeros)
//   warp 1      TMEM allocation; one lane issues tcgen05.mma:
//                 S = Q K^T            (M=128, N=64,  K=64)  -> TMEM cols [0, 64)
//                 O += P V             (M=128, N=64,  K=64)  -> TMEM cols [64, 128)
//               S of block j+1 is issued as soon as the softmax has read S_j.
//   warps 2..5  one thread per query row: read S_j from TMEM, online softmax in
//               f32 (exp2 domain); the reference max is only raised (and O in
//               TMEM rescaled) when a row's max grows by more than 2^8, so P
//               stays <= 256 and the rescale is rare (the result is the same
//               softmax: numerator and denominator share the reference);
//               write P_j (f16) into 128B-swizzled shared memory as the A
//               operand of the P V product; at the end O / l -> f16 -> TMA store
//               (3-D map clips rows past the sequence end).
// V is consumed in its natural [key][dim] layout as an MN-major B operand.
// Every mbarrier wait is bounded (see sm100.cuh).
#include "kernels.cuh"
#include "sm100.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdlib>
#include <cstring>
#include <mutex>

namespace rfb {

namespace {

constexpr int AQ = 128;                 // query rows per CTA
constexpr int AK = 64;                  // keys per block
constexpr int HD = 64;                  // head dim
constexpr int Q_BYTES = AQ * HD * 2;    // 16 KB
constexpr int KV_BYTES = AK * HD * 2;   // 8 KB
constexpr int P_BYTES = AQ * AK * 2;    // 16 KB
constexpr float kRescaleLog2 = 8.0f;    // lazy rescale threshold (log2 units)
constexpr int TMEM_COLS = 128;          // S: [0,64), O: [64,128)

// NS = K/V ring slots (prefetch depth).  Sequences of at most two key blocks
// (windows of up to 128 tokens, e.g. the 101-token windows of a 40 x 40
// grid) use two slots, which keeps a CTA at 64 KB of shared memory and lets
// three run per SM; longer ones use four (96 KB, two per SM).
// Longest sequence that takes the two-slot, three-CTAs-per-SM variant.
#ifndef RFB_ATTN_SHORT_KEYS
#define RFB_ATTN_SHORT_KEYS (2 * AK)
#endif

#ifndef RFB_ATTN_FMA_EXP
#define RFB_ATTN_FMA_EXP 3
#endif

template <int NS>
struct AttnCfg {
    static constexpr int SMEM_TILES = Q_BYTES + 2 * NS * KV_BYTES + P_BYTES;
    static constexpr int SMEM = SMEM_TILES + 1024 + 256;
    static constexpr int MIN_CTAS = NS == 2 ? 3 : 2;
};

// max of three floats in one instruction (sm_100): the row max takes one per two scores
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float r;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
    return r;
}

__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 2^x on the FMA pipe, two values at a time, for the share of the softmax
// exponentials that the MUFU (ex2) cannot take without becoming the bound:
// n = rint(x) (the 1.5 * 2^23 shift), f = x - n in [-1/2, 1/2], 2^f from a
// degree-4 near-minimax polynomial (relative error <= 2.7e-6 in float32; a
// relative-error-weighted least-squares fit on [-1/2, 1/2] refined by Lawson's
// iteratively reweighted least squares), then n added to the exponent field.  x is clamped at -125 (2^-125 is 0 once P is rounded to f16).
constexpr float kExpShift = 12582912.0f;  // 1.5 * 2^23
__device__ __forceinline__ float2 exp2_fma2(float2 x) {
    x = make_float2(fmaxf(x.x, -125.0f), fmaxf(x.y, -125.0f));
    const float2 r = __fadd2_rn(x, make_float2(kExpShift, kExpShift));
    const float2 n = __fadd2_rn(r, make_float2(-kExpShift, -kExpShift));
    const float2 f = __ffma2_rn(n, make_float2(-1.0f, -1.0f), x);
    float2 p = __ffma2_rn(make_float2(9.570021182e-03f, 9.570021182e-03f), f,
                          make_float2(5.591763183e-02f, 5.591763183e-02f));
    p = __ffma2_rn(p, f, make_float2(2.402474433e-01f, 2.402474433e-01f));
    p = __ffma2_rn(p, f, make_float2(6.931218505e-01f, 6.931218505e-01f));
    p = __ffma2_rn(p, f, make_float2(9.999992847e-01f, 9.999992847e-01f));
    // low mantissa bits of r hold n; shifted by 23 they land in the exponent field
    return make_float2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(r.x) << 23)),
                       __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(r.y) << 23)));
}

__device__ __forceinline__ uint32_t swz(uint32_t base, int row, int j) {
    return base + row * 128 + ((j ^ (row & 7)) << 4);
}

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
}

template <int NS>
__global__ void __launch_bounds__(192, AttnCfg<NS>::MIN_CTAS)
k_attn_tc(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
          const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO, int L, float sl2,
          int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem;
    uint8_t* sK = sQ + Q_BYTES;            // NS slots
    uint8_t* sV = sK + NS * KV_BYTES;      // NS slots
    uint8_t* sP = sV + NS * KV_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + AttnCfg<NS>::SMEM_TILES);
    uint64_t* q_full = bars + 0;
    uint64_t* kv_full = bars + 1;        // [NS]
    uint64_t* kv_empty = bars + 1 + NS;  // [NS]
    uint64_t* s_full = bars + 1 + 2 * NS;
    uint64_t* s_free = s_full + 1;
    uint64_t* p_full = s_full + 2;
    uint64_t* pv_done = s_full + 3;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(s_full + 4);
    volatile int* cta_abort = reinterpret_cast<volatile int*>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q0 = blockIdx.x * AQ;
    const int head = blockIdx.y;
    const int g = blockIdx.z;
    const int nb = (L + AK - 1) / AK;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int i = 0; i < NS; ++i) {
            mbar_init(&kv_full[i], 1);
            mbar_init(&kv_empty[i], 1);
        }
        mbar_init(s_full, 1);
        mbar_init(s_free, 128);
        mbar_init(p_full, 128);
        mbar_init(pv_done, 1);
        *cta_abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_holder, TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    const uint32_t tS = tmem, tO = tmem + AK;

    if (warp == 0) {
        if (lane == 0) {
            prefetch_tmap(&tmQ);
            prefetch_tmap(&tmK);
            prefetch_tmap(&tmV);
            mbar_arrive_expect_tx(q_full, Q_BYTES);
            tma_load_3d(&tmQ, q_full, sQ, head * HD, q0, g);
            for (int j = 0; j < nb; ++j) {
                const int slot = j % NS;
                if (!mbar_wait(&kv_empty[slot], ((j / NS) & 1) ^ 1, cta_abort, err)) break;
                mbar_arrive_expect_tx(&kv_full[slot], 2 * KV_BYTES);
                tma_load_3d(&tmK, &kv_full[slot], sK + slot * KV_BYTES, head * HD, j * AK, g);
                tma_load_3d(&tmV, &kv_full[slot], sV + slot * KV_BYTES, head * HD, j * AK, g);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t IDESC_S = idesc_f16_f32(AQ, AK);
            constexpr uint32_t IDESC_PV = idesc_f16_f32(AQ, HD) | (1u << 16);  // B (V) MN-major
            const uint32_t q_s = smem_u32(sQ), p_s = smem_u32(sP);
            bool ok = mbar_wait(q_full, 0, cta_abort, err) && mbar_wait(&kv_full[0], 0, cta_abort, err);
            if (ok) {
                tc_fence_after();
                const uint32_t k_s = smem_u32(sK);
#pragma unroll
                for (int kk = 0; kk < HD / 16; ++kk)
                    umma_f16(tS, sw128_kmajor_desc(q_s + kk * 32), sw128_kmajor_desc(k_s + kk * 32), IDESC_S, kk > 0);
                umma_commit(s_full);
            }
            for (int j = 0; ok && j < nb; ++j) {
                const int slot = j % NS;
                if (j + 1 < nb) {
                    const int ns = (j + 1) % NS;
                    if (!mbar_wait(s_free, j & 1, cta_abort, err)) break;
                    if (!mbar_wait(&kv_full[ns], ((j + 1) / NS) & 1, cta_abort, err)) break;
                    tc_fence_after();
                    const uint32_t k_s = smem_u32(sK + ns * KV_BYTES);
#pragma unroll
                    for (int kk = 0; kk < HD / 16; ++kk)
                        umma_f16(tS, sw128_kmajor_desc(q_s + kk * 32), sw128_kmajor_desc(k_s + kk * 32), IDESC_S,
                                 kk > 0);
                    umma_commit(s_full);
                }
                if (!mbar_wait(p_full, j & 1, cta_abort, err)) break;
                tc_fence_after();
                const uint32_t v_s = smem_u32(sV + slot * KV_BYTES);
#pragma unroll
                for (int kk = 0; kk < AK / 16; ++kk)
                    umma_f16(tO, sw128_kmajor_desc(p_s + kk * 32), sw128_kmajor_desc(v_s + kk * 2048), IDESC_PV,
                             (j > 0 || kk > 0) ? 1u : 0u);
                umma_commit(pv_done);
                umma_commit(&kv_empty[slot]);
            }
        }
    } else {
        // ---- softmax warps: thread = query row (q0 + quad*32 + lane)
        const int quad = warp & 3;
        const int row = quad * 32 + lane;
        const uint32_t lanebase = (uint32_t)(quad * 32) << 16;
        const uint32_t p_s = smem_u32(sP);
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < nb; ++j) {
            if (!mbar_wait(s_full, j & 1, cta_abort, err)) { ok = false; break; }
            tc_fence_after();
            uint32_t r0[32], r1[32];
            tmem_ld32(tS + lanebase, r0);
            tmem_ld32(tS + lanebase + 32, r1);
            tmem_wait_ld();
            tc_fence_before();
            mbar_arrive(s_free);
            const int kbase = j * AK;
            const bool full_block = kbase + AK <= L;
            float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};  // row max of raw scores
#pragma unroll
            for (int e = 0; e < 32; ++e) {
                float x0 = __uint_as_float(r0[e]), x1 = __uint_as_float(r1[e]);
                if (!full_block) {
                    if (kbase + e >= L) x0 = -INFINITY;
                    if (kbase + 32 + e >= L) x1 = -INFINITY;
                    r0[e] = __float_as_uint(x0);
                    r1[e] = __float_as_uint(x1);
                }
                mx4[e & 3] = fmax3(mx4[e & 3], x0, x1);
            }
            // scale > 0 commutes with max; running max in log2 units
            const float m_cand = fmaxf(m, fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * sl2);
            const float m_new = m_cand > m + kRescaleLog2 ? m_cand : m;  // always taken on the first block
            const float alpha = ex2(m - m_new);  // 1 while the reference holds; 0 on the first block
            float2 rs2 = make_float2(0.f, 0.f);
            const float2 sl2v = make_float2(sl2, sl2), negm = make_float2(-m_new, -m_new);
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
                const float2 a = __ffma2_rn(make_float2(__uint_as_float(r0[e]), __uint_as_float(r0[e + 1])), sl2v, negm);
                const float2 c = __ffma2_rn(make_float2(__uint_as_float(r1[e]), __uint_as_float(r1[e + 1])), sl2v, negm);
                // long sequences: RFB_ATTN_FMA_EXP of every 8 key pairs take their exponentials on the
                // FMA pipe, the rest on the MUFU, whose pipe (shared with the f16 packing) is the
                // softmax's bound; the three-CTA short-sequence variant has no registers to spare
                const bool on_fma = NS == 4 && ((e >> 1) & 7) >= 8 - RFB_ATTN_FMA_EXP;
                const float2 pa = on_fma ? exp2_fma2(a) : make_float2(ex2(a.x), ex2(a.y));
                const float2 pc = on_fma ? exp2_fma2(c) : make_float2(ex2(c.x), ex2(c.y));
                r0[e] = __float_as_uint(pa.x);
                r0[e + 1] = __float_as_uint(pa.y);
                r1[e] = __float_as_uint(pc.x);
                r1[e + 1] = __float_as_uint(pc.y);
                rs2 = __fadd2_rn(rs2, __fadd2_rn(pa, pc));
            }
            l = l * alpha + (rs2.x + rs2.y);
            m = m_new;
            if (j > 0) {
                // previous P V done: P buffer reusable, O stable for the rescale
                if (!mbar_wait(pv_done, (j - 1) & 1, cta_abort, err)) { ok = false; break; }
                tc_fence_after();
            }
            // P (f16) row -> swizzled K-major tile [128 rows][64 keys]: 16-byte chunk cc holds keys 8cc..8cc+7
#pragma unroll
            for (int cc = 0; cc < 8; ++cc) {
                const int o = (cc & 3) * 8;
                float w[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) w[e] = __uint_as_float(cc < 4 ? r0[o + e] : r1[o + e]);
                st_shared_v4(swz(p_s, row, cc), pack_half2(w[0], w[1]), pack_half2(w[2], w[3]), pack_half2(w[4], w[5]),
                             pack_half2(w[6], w[7]));
            }
            if (j > 0) {
                if (__any_sync(0xffffffffu, alpha != 1.0f)) {
                    uint32_t o[32];
#pragma unroll
                    for (int c = 0; c < HD; c += 32) {
                        tmem_ld32(tO + lanebase + c, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int e = 0; e < 32; e += 2) {
                            const float2 y = __fmul2_rn(make_float2(__uint_as_float(o[e]), __uint_as_float(o[e + 1])),
                                                        make_float2(alpha, alpha));
                            o[e] = __float_as_uint(y.x);
                            o[e + 1] = __float_as_uint(y.y);
                        }
                        tmem_st32(tO + lanebase + c, o);
                    }
                    tmem_wait_st();
                }
            }
            fence_async_smem();
            tc_fence_before();
            mbar_arrive(p_full);
        }
        if (ok && mbar_wait(pv_done, (nb - 1) & 1, cta_abort, err)) {
            tc_fence_after();
            const float inv = 1.0f / l;
            // stage O / l as f16 in this warp's quarter of the (now idle) P buffer
            uint8_t* stage = sP + quad * 4096;
            const uint32_t st_s = smem_u32(stage);
            uint32_t o[32];
#pragma unroll
            for (int c = 0; c < HD; c += 32) {
                tmem_ld32(tO + lanebase + c, o);
                tmem_wait_ld();
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    st_shared_v4(swz(st_s, lane, (c >> 3) + q),
                                 pack_half2(__uint_as_float(o[8 * q + 0]) * inv, __uint_as_float(o[8 * q + 1]) * inv),
                                 pack_half2(__uint_as_float(o[8 * q + 2]) * inv, __uint_as_float(o[8 * q + 3]) * inv),
                                 pack_half2(__uint_as_float(o[8 * q + 4]) * inv, __uint_as_float(o[8 * q + 5]) * inv),
                                 pack_half2(__uint_as_float(o[8 * q + 6]) * inv, __uint_as_float(o[8 * q + 7]) * inv));
            }
            fence_async_smem();
            __syncwarp();
            if (lane == 0) {
                tma_store_3d(&tmO, stage, head * HD, q0 + quad * 32, g);
                bulk_commit();
                bulk_wait<0>();
            }
        }
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

// Persistent form: each CTA loops over items (query tile, head, group),
// item = blockIdx.x + k * gridDim.x, so the TMA warp loads the next item's Q
// and K/V while the current one is in softmax, and the per-CTA setup (TMEM
// allocation, barrier initialisation) is paid once.  The K/V ring and every
// barrier phase run on per-CTA counters across items; two more barriers
// order the reuse: q_free (the item's S MMAs are done; Q may be replaced) and
// o_free (the softmax warps have read O; the next item's first P V may
// overwrite it).  The P buffer doubles as the O staging box of each TMEM lane
// quadrant, so a warp waits for its previous O store to be read out before it
// writes the next item's P rows.
template <int NS>
__global__ void __launch_bounds__(192, AttnCfg<NS>::MIN_CTAS)
k_attn_tc_items(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO, int L, float sl2,
                int n_qt, int heads, int n_items, int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem;
    uint8_t* sK = sQ + Q_BYTES;            // NS slots
    uint8_t* sV = sK + NS * KV_BYTES;      // NS slots
    uint8_t* sP = sV + NS * KV_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + AttnCfg<NS>::SMEM_TILES);
    uint64_t* q_full = bars + 0;
    uint64_t* kv_full = bars + 1;        // [NS]
    uint64_t* kv_empty = bars + 1 + NS;  // [NS]
    uint64_t* s_full = bars + 1 + 2 * NS;
    uint64_t* s_free = s_full + 1;
    uint64_t* p_full = s_full + 2;
    uint64_t* pv_done = s_full + 3;
    uint64_t* q_free = s_full + 4;
    uint64_t* o_free = s_full + 5;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(s_full + 6);
    volatile int* cta_abort = reinterpret_cast<volatile int*>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nb = (L + AK - 1) / AK;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int i = 0; i < NS; ++i) {
            mbar_init(&kv_full[i], 1);
            mbar_init(&kv_empty[i], 1);
        }
        mbar_init(s_full, 1);
        mbar_init(s_free, 128);
        mbar_init(p_full, 128);
        mbar_init(pv_done, 1);
        mbar_init(q_free, 1);
        mbar_init(o_free, 128);
        *cta_abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_holder, TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    const uint32_t tS = tmem, tO = tmem + AK;

    if (warp == 0) {
        if (lane == 0) {
            prefetch_tmap(&tmQ);
            prefetch_tmap(&tmK);
            prefetch_tmap(&tmV);
            int kvj = 0, it = 0;
            for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++it) {
                const int qt = item % n_qt, hg = item / n_qt;
                const int head = hg % heads, g = hg / heads;
                if (it > 0 && !mbar_wait(q_free, (it - 1) & 1, cta_abort, err)) break;
                mbar_arrive_expect_tx(q_full, Q_BYTES);
                tma_load_3d(&tmQ, q_full, sQ, head * HD, qt * AQ, g);
                bool ok = true;
                for (int j = 0; j < nb; ++j, ++kvj) {
                    const int slot = kvj % NS;
                    if (!mbar_wait(&kv_empty[slot], ((kvj / NS) & 1) ^ 1, cta_abort, err)) { ok = false; break; }
                    mbar_arrive_expect_tx(&kv_full[slot], 2 * KV_BYTES);
                    tma_load_3d(&tmK, &kv_full[slot], sK + slot * KV_BYTES, head * HD, j * AK, g);
                    tma_load_3d(&tmV, &kv_full[slot], sV + slot * KV_BYTES, head * HD, j * AK, g);
                }
                if (!ok) break;
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t IDESC_S = idesc_f16_f32(AQ, AK);
            constexpr uint32_t IDESC_PV = idesc_f16_f32(AQ, HD) | (1u << 16);  // B (V) MN-major
            const uint32_t q_s = smem_u32(sQ), p_s = smem_u32(sP);
            int kvj = 0, sidx = 0, pidx = 0, it = 0;
            bool ok = true;
            for (int item = blockIdx.x; ok && item < n_items; item += gridDim.x, ++it) {
                // S of block j (running index sidx) once the softmax has read the previous S
                auto issue_s = [&](int kv) -> bool {
                    if (sidx > 0 && !mbar_wait(s_free, (sidx - 1) & 1, cta_abort, err)) return false;
                    if (!mbar_wait(&kv_full[kv % NS], (kv / NS) & 1, cta_abort, err)) return false;
                    tc_fence_after();
                    const uint32_t k_s = smem_u32(sK + (kv % NS) * KV_BYTES);
#pragma unroll
                    for (int kk = 0; kk < HD / 16; ++kk)
                        umma_f16(tS, sw128_kmajor_desc(q_s + kk * 32), sw128_kmajor_desc(k_s + kk * 32), IDESC_S,
                                 kk > 0);
                    umma_commit(s_full);
                    ++sidx;
                    return true;
                };
                if (!mbar_wait(q_full, it & 1, cta_abort, err) || !issue_s(kvj)) break;
                for (int j = 0; j < nb; ++j, ++kvj) {
                    if (j + 1 < nb && !issue_s(kvj + 1)) { ok = false; break; }
                    if (j + 1 == nb) umma_commit(q_free);  // every S of the item issued: Q is free once they finish
                    if (!mbar_wait(p_full, pidx & 1, cta_abort, err)) { ok = false; break; }
                    if (j == 0 && it > 0 && !mbar_wait(o_free, (it - 1) & 1, cta_abort, err)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t v_s = smem_u32(sV + (kvj % NS) * KV_BYTES);
#pragma unroll
                    for (int kk = 0; kk < AK / 16; ++kk)
                        umma_f16(tO, sw128_kmajor_desc(p_s + kk * 32), sw128_kmajor_desc(v_s + kk * 2048), IDESC_PV,
                                 (j > 0 || kk > 0) ? 1u : 0u);
                    umma_commit(pv_done);
                    umma_commit(&kv_empty[kvj % NS]);
                    ++pidx;
                }
            }
        }
    } else {
        // ---- softmax warps: thread = query row (tile row quad*32 + lane)
        const int quad = warp & 3;
        const int row = quad * 32 + lane;
        const uint32_t lanebase = (uint32_t)(quad * 32) << 16;
        const uint32_t p_s = smem_u32(sP);
        uint8_t* stage = sP + quad * 4096;  // this quadrant's rows of P, and its O staging box
        const uint32_t st_s = smem_u32(stage);
        int sidx = 0, pidx = 0, it = 0;
        bool ok = true;
        for (int item = blockIdx.x; ok && item < n_items; item += gridDim.x, ++it) {
            const int qt = item % n_qt, hg = item / n_qt;
            const int head = hg % heads, g = hg / heads;
            float m = -INFINITY, l = 0.f;
            for (int j = 0; j < nb; ++j) {
                if (!mbar_wait(s_full, sidx & 1, cta_abort, err)) { ok = false; break; }
                ++sidx;
                tc_fence_after();
                uint32_t r0[32], r1[32];
                tmem_ld32(tS + lanebase, r0);
                tmem_ld32(tS + lanebase + 32, r1);
                tmem_wait_ld();
                tc_fence_before();
                mbar_arrive(s_free);
                const int kbase = j * AK;
                const bool full_block = kbase + AK <= L;
                float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                    float x0 = __uint_as_float(r0[e]), x1 = __uint_as_float(r1[e]);
                    if (!full_block) {
                        if (kbase + e >= L) x0 = -INFINITY;
                        if (kbase + 32 + e >= L) x1 = -INFINITY;
                        r0[e] = __float_as_uint(x0);
                        r1[e] = __float_as_uint(x1);
                    }
                    mx4[e & 3] = fmax3(mx4[e & 3], x0, x1);
                }
                const float m_cand = fmaxf(m, fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * sl2);
                const float m_new = m_cand > m + kRescaleLog2 ? m_cand : m;
                const float alpha = ex2(m - m_new);
                float2 rs2 = make_float2(0.f, 0.f);
                const float2 sl2v = make_float2(sl2, sl2), negm = make_float2(-m_new, -m_new);
#pragma unroll
                for (int e = 0; e < 32; e += 2) {
                    const float2 a = __ffma2_rn(make_float2(__uint_as_float(r0[e]), __uint_as_float(r0[e + 1])), sl2v, negm);
                    const float2 c = __ffma2_rn(make_float2(__uint_as_float(r1[e]), __uint_as_float(r1[e + 1])), sl2v, negm);
                    const bool on_fma = NS == 4 && ((e >> 1) & 7) >= 8 - RFB_ATTN_FMA_EXP;
                    const float2 pa = on_fma ? exp2_fma2(a) : make_float2(ex2(a.x), ex2(a.y));
                    const float2 pc = on_fma ? exp2_fma2(c) : make_float2(ex2(c.x), ex2(c.y));
                    r0[e] = __float_as_uint(pa.x);
                    r0[e + 1] = __float_as_uint(pa.y);
                    r1[e] = __float_as_uint(pc.x);
                    r1[e + 1] = __float_as_uint(pc.y);
                    rs2 = __fadd2_rn(rs2, __fadd2_rn(pa, pc));
                }
                l = l * alpha + (rs2.x + rs2.y);
                m = m_new;
                if (j > 0) {
                    // previous P V done: P buffer reusable, O stable for the rescale
                    if (!mbar_wait(pv_done, (pidx - 1) & 1, cta_abort, err)) { ok = false; break; }
                    tc_fence_after();
                } else if (it > 0) {
                    // this quadrant's rows of P held the previous item's O box: its store has read them
                    if (lane == 0) bulk_wait_read<0>();
                    __syncwarp();
                }
#pragma unroll
                for (int cc = 0; cc < 8; ++cc) {
                    const int o = (cc & 3) * 8;
                    float w[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) w[e] = __uint_as_float(cc < 4 ? r0[o + e] : r1[o + e]);
                    st_shared_v4(swz(p_s, row, cc), pack_half2(w[0], w[1]), pack_half2(w[2], w[3]),
                                 pack_half2(w[4], w[5]), pack_half2(w[6], w[7]));
                }
                if (j > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
                    uint32_t o[32];
#pragma unroll
                    for (int c = 0; c < HD; c += 32) {
                        tmem_ld32(tO + lanebase + c, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int e = 0; e < 32; e += 2) {
                            const float2 y = __fmul2_rn(make_float2(__uint_as_float(o[e]), __uint_as_float(o[e + 1])),
                                                        make_float2(alpha, alpha));
                            o[e] = __float_as_uint(y.x);
                            o[e + 1] = __float_as_uint(y.y);
                        }
                        tmem_st32(tO + lanebase + c, o);
                    }
                    tmem_wait_st();
                }
                fence_async_smem();
                tc_fence_before();
                mbar_arrive(p_full);
                ++pidx;
            }
            if (!ok || !mbar_wait(pv_done, (pidx - 1) & 1, cta_abort, err)) { ok = false; break; }
            tc_fence_after();
            const float inv = 1.0f / l;
            uint32_t o0[32], o1[32];
            tmem_ld32(tO + lanebase, o0);
            tmem_ld32(tO + lanebase + 32, o1);
            tmem_wait_ld();
            tc_fence_before();
            mbar_arrive(o_free);  // O is in registers: the next item's first P V may overwrite it
#pragma unroll
            for (int c = 0; c < 2; ++c) {
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const uint32_t* o = c ? o1 : o0;
                    st_shared_v4(swz(st_s, lane, 4 * c + q),
                                 pack_half2(__uint_as_float(o[8 * q + 0]) * inv, __uint_as_float(o[8 * q + 1]) * inv),
                                 pack_half2(__uint_as_float(o[8 * q + 2]) * inv, __uint_as_float(o[8 * q + 3]) * inv),
                                 pack_half2(__uint_as_float(o[8 * q + 4]) * inv, __uint_as_float(o[8 * q + 5]) * inv),
                                 pack_half2(__uint_as_float(o[8 * q + 6]) * inv, __uint_as_float(o[8 * q + 7]) * inv));
                }
            }
            fence_async_smem();
            __syncwarp();
            if (lane == 0) {
                tma_store_3d(&tmO, stage, head * HD, qt * AQ + quad * 32, g);
                bulk_commit();
            }
        }
        if (lane == 0) bulk_wait<0>();
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM_COLS);
    }
}

// 128-key blocks for long sequences (the global blocks): S = Q K^T of a block is M=128 x N=128,
// and P goes back into TMEM as packed f16 (tcgen05.st), from where the P V product reads it as its
// A operand.  The per-block hand-off (S ready, S read, P ready, P V done) is paid once per 128 keys
// instead of once per 64, and without a P tile in shared memory a CTA holds Q (16 KB) and two-slot
// K and V rings of 128-key tiles (64 KB), so two CTAs still fit per SM.
//   TMEM (256 columns): S [0,128) f32, O [128,192) f32, P [192,256) f16 pairs.
//   K and V slots have their own barriers: K_j's slot is released when S_j is computed, V_j's
//   when P_j V_j is, so the next K tiles load while the softmax of the current block runs.
//   The final O / l staging box of each lane quadrant is its quarter of Q's tile (free once the
//   last S product has completed).
constexpr int AK2 = 128;                  // keys per block
constexpr int KV2_BYTES = AK2 * HD * 2;   // 16 KB
constexpr int NS2 = 2;                    // ring slots
constexpr int SMEM2_TILES = Q_BYTES + 2 * NS2 * KV2_BYTES;
constexpr int SMEM2 = SMEM2_TILES + 1024 + 256;
constexpr int TMEM2_COLS = 256;

__global__ void __launch_bounds__(192, 2)
k_attn_tc128(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
             const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO, int L, float sl2,
             int* err) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem;
    uint8_t* sK = sQ + Q_BYTES;              // NS2 slots
    uint8_t* sV = sK + NS2 * KV2_BYTES;      // NS2 slots
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SMEM2_TILES);
    uint64_t* q_full = bars + 0;
    uint64_t* k_full = bars + 1;               // [NS2]
    uint64_t* k_empty = k_full + NS2;          // [NS2]
    uint64_t* v_full = k_empty + NS2;          // [NS2]
    uint64_t* v_empty = v_full + NS2;          // [NS2]
    uint64_t* s_full = v_empty + NS2;
    uint64_t* s_free = s_full + 1;
    uint64_t* p_full = s_full + 2;
    uint64_t* pv_done = s_full + 3;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(s_full + 4);
    volatile int* cta_abort = reinterpret_cast<volatile int*>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int q0 = blockIdx.x * AQ;
    const int head = blockIdx.y;
    const int g = blockIdx.z;
    const int nb = (L + AK2 - 1) / AK2;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int i = 0; i < NS2; ++i) {
            mbar_init(&k_full[i], 1);
            mbar_init(&k_empty[i], 1);
            mbar_init(&v_full[i], 1);
            mbar_init(&v_empty[i], 1);
        }
        mbar_init(s_full, 1);
        mbar_init(s_free, 128);
        mbar_init(p_full, 128);
        mbar_init(pv_done, 1);
        *cta_abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_holder, TMEM2_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;
    const uint32_t tS = tmem, tO = tmem + AK2, tP = tmem + AK2 + HD;

    if (warp == 0) {
        if (lane == 0) {
            prefetch_tmap(&tmQ);
            prefetch_tmap(&tmK);
            prefetch_tmap(&tmV);
            mbar_arrive_expect_tx(q_full, Q_BYTES);
            tma_load_3d(&tmQ, q_full, sQ, head * HD, q0, g);
            for (int j = 0; j < nb; ++j) {
                const int slot = j % NS2;
                const uint32_t ph = ((j / NS2) & 1) ^ 1;
                if (!mbar_wait(&k_empty[slot], ph, cta_abort, err)) break;
                mbar_arrive_expect_tx(&k_full[slot], KV2_BYTES);
                tma_load_3d(&tmK, &k_full[slot], sK + slot * KV2_BYTES, head * HD, j * AK2, g);
                if (!mbar_wait(&v_empty[slot], ph, cta_abort, err)) break;
                mbar_arrive_expect_tx(&v_full[slot], KV2_BYTES);
                tma_load_3d(&tmV, &v_full[slot], sV + slot * KV2_BYTES, head * HD, j * AK2, g);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t IDESC_S = idesc_f16_f32(AQ, AK2);
            constexpr uint32_t IDESC_PV = idesc_f16_f32(AQ, HD) | (1u << 16);  // B (V) MN-major
            const uint32_t q_s = smem_u32(sQ);
            auto issue_s = [&](int j) -> bool {
                const int slot = j % NS2;
                if (!mbar_wait(&k_full[slot], (j / NS2) & 1, cta_abort, err)) return false;
                tc_fence_after();
                const uint32_t k_s = smem_u32(sK + slot * KV2_BYTES);
#pragma unroll
                for (int kk = 0; kk < HD / 16; ++kk)
                    umma_f16(tS, sw128_kmajor_desc(q_s + kk * 32), sw128_kmajor_desc(k_s + kk * 32), IDESC_S, kk > 0);
                umma_commit(s_full);
                umma_commit(&k_empty[slot]);
                return true;
            };
            bool ok = mbar_wait(q_full, 0, cta_abort, err) && issue_s(0);
            for (int j = 0; ok && j < nb; ++j) {
                const int slot = j % NS2;
                if (j + 1 < nb) {
                    if (!mbar_wait(s_free, j & 1, cta_abort, err) || !issue_s(j + 1)) break;
                }
                if (!mbar_wait(p_full, j & 1, cta_abort, err)) break;
                if (!mbar_wait(&v_full[slot], (j / NS2) & 1, cta_abort, err)) break;
                tc_fence_after();
                const uint32_t v_s = smem_u32(sV + slot * KV2_BYTES);
#pragma unroll
                for (int kk = 0; kk < AK2 / 16; ++kk)
                    umma_f16_ts(tO, tP + kk * 8, sw128_kmajor_desc(v_s + kk * 2048), IDESC_PV,
                                (j > 0 || kk > 0) ? 1u : 0u);
                umma_commit(pv_done);
                umma_commit(&v_empty[slot]);
            }
        }
    } else {
        // ---- softmax warps: thread = query row (q0 + quad*32 + lane)
        const int quad = warp & 3;
        const uint32_t lanebase = (uint32_t)(quad * 32) << 16;
        float m = -INFINITY, l = 0.f;
        bool ok = true;
        for (int j = 0; j < nb; ++j) {
            if (!mbar_wait(s_full, j & 1, cta_abort, err)) { ok = false; break; }
            tc_fence_after();
            uint32_t r[4][32];
#pragma unroll
            for (int h = 0; h < 4; ++h) tmem_ld32(tS + lanebase + 32 * h, r[h]);
            tmem_wait_ld();
            tc_fence_before();
            mbar_arrive(s_free);
            const int kbase = j * AK2;
            if (kbase + AK2 > L) {
#pragma unroll
                for (int h = 0; h < 4; ++h)
#pragma unroll
                    for (int e = 0; e < 32; ++e)
                        if (kbase + 32 * h + e >= L) r[h][e] = __float_as_uint(-INFINITY);
            }
            float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};  // row max of raw scores
#pragma unroll
            for (int h = 0; h < 4; h += 2)
#pragma unroll
                for (int e = 0; e < 32; ++e)
                    mx4[e & 3] = fmax3(mx4[e & 3], __uint_as_float(r[h][e]), __uint_as_float(r[h + 1][e]));
            // scale > 0 commutes with max; running max in log2 units
            const float m_cand = fmaxf(m, fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * sl2);
            const float m_new = m_cand > m + kRescaleLog2 ? m_cand : m;  // always taken on the first block
            const float alpha = ex2(m - m_new);  // 1 while the reference holds; 0 on the first block
            float2 rs2 = make_float2(0.f, 0.f);
            const float2 sl2v = make_float2(sl2, sl2), negm = make_float2(-m_new, -m_new);
            uint32_t p[2][32];  // P row as f16 pairs: column c holds keys 2c, 2c + 1
#pragma unroll
            for (int h = 0; h < 4; ++h) {
#pragma unroll
                for (int e = 0; e < 32; e += 2) {
                    const float2 a = __ffma2_rn(make_float2(__uint_as_float(r[h][e]), __uint_as_float(r[h][e + 1])),
                                                sl2v, negm);
                    // RFB_ATTN_FMA_EXP of every 8 key pairs take their exponentials on the FMA pipe
                    const bool on_fma = ((e >> 1) & 7) >= 8 - RFB_ATTN_FMA_EXP;
                    const float2 pa = on_fma ? exp2_fma2(a) : make_float2(ex2(a.x), ex2(a.y));
                    rs2 = __fadd2_rn(rs2, pa);
                    p[h >> 1][(h & 1) * 16 + (e >> 1)] = pack_half2(pa.x, pa.y);
                }
            }
            l = l * alpha + (rs2.x + rs2.y);
            m = m_new;
            if (j > 0) {
                // previous P V done: P columns reusable, O stable for the rescale
                if (!mbar_wait(pv_done, (j - 1) & 1, cta_abort, err)) { ok = false; break; }
                tc_fence_after();
            }
            tmem_st32(tP + lanebase, p[0]);
            tmem_st32(tP + lanebase + 32, p[1]);
            if (j > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
                uint32_t o[32];
#pragma unroll
                for (int c = 0; c < HD; c += 32) {
                    tmem_ld32(tO + lanebase + c, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 32; e += 2) {
                        const float2 y = __fmul2_rn(make_float2(__uint_as_float(o[e]), __uint_as_float(o[e + 1])),
                                                    make_float2(alpha, alpha));
                        o[e] = __float_as_uint(y.x);
                        o[e + 1] = __float_as_uint(y.y);
                    }
                    tmem_st32(tO + lanebase + c, o);
                }
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(p_full);
        }
        if (ok && mbar_wait(pv_done, (nb - 1) & 1, cta_abort, err)) {
            tc_fence_after();
            const float inv = 1.0f / l;
            // stage O / l as f16 in this warp's quarter of Q's tile (every S product has completed)
            uint8_t* stage = sQ + quad * 4096;
            const uint32_t st_s = smem_u32(stage);
            uint32_t o[32];
#pragma unroll
            for (int c = 0; c < HD; c += 32) {
                tmem_ld32(tO + lanebase + c, o);
                tmem_wait_ld();
#pragma unroll
                for (int q = 0; q < 4; ++q)
                    st_shared_v4(swz(st_s, lane, (c >> 3) + q),
                                 pack_half2(__uint_as_float(o[8 * q + 0]) * inv, __uint_as_float(o[8 * q + 1]) * inv),
                                 pack_half2(__uint_as_float(o[8 * q + 2]) * inv, __uint_as_float(o[8 * q + 3]) * inv),
                                 pack_half2(__uint_as_float(o[8 * q + 4]) * inv, __uint_as_float(o[8 * q + 5]) * inv),
                                 pack_half2(__uint_as_float(o[8 * q + 6]) * inv, __uint_as_float(o[8 * q + 7]) * inv));
            }
            fence_async_smem();
            __syncwarp();
            if (lane == 0) {
                tma_store_3d(&tmO, stage, head * HD, q0 + quad * 32, g);
                bulk_commit();
                bulk_wait<0>();
            }
        }
    }
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, TMEM2_COLS);
    }
}

PFN_cuTensorMapEncodeTiled_v12000 g_enc = nullptr;
std::once_flag g_enc_once;

bool encode_fn() {
    std::call_once(g_enc_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_enc = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    return g_enc != nullptr;
}

// (cols, seq, group) view of a [groups*seq][ld] f16 matrix; box of `rows` x 64 columns.
bool make_seq_map(CUtensorMap* m, const void* base, int cols, int seq, int groups, int ld, int rows) {
    if (((uintptr_t)base & 15) || (ld % 8)) return false;
    cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)seq, (cuuint64_t)groups};
    cuuint64_t strides[2] = {(cuuint64_t)ld * 2, (cuuint64_t)seq * ld * 2};
    cuuint32_t box[3] = {(cuuint32_t)HD, (cuuint32_t)rows, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    return g_enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                 CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

cudaError_t attention_tc(const __half* q, const __half* k, const __half* v, int ldq, int ldk, int ldv, __half* o,
                         int ldo, int seq_len, int groups, int heads, float scale, int* err, cudaStream_t st) {
    if (seq_len <= 0 || groups <= 0) return cudaSuccess;
    if (!encode_fn()) return cudaErrorNotSupported;
    static std::atomic<uint64_t> attr_set{0};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = 1ull << (dev & 63);
    if (!(attr_set.load() & bit)) {
        e = cudaFuncSetAttribute(k_attn_tc<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, AttnCfg<2>::SMEM);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(k_attn_tc<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, AttnCfg<4>::SMEM);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(k_attn_tc_items<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, AttnCfg<2>::SMEM);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(k_attn_tc_items<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, AttnCfg<4>::SMEM);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(k_attn_tc128, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM2);
        if (e != cudaSuccess) return e;
        attr_set.fetch_or(bit);
    }
    const int cols = heads * HD;
    CUtensorMap mq, mk, mv, mo;
    // long sequences: 128-key blocks with P in TMEM (RFDETR_ATTN_KB=64 keeps the 64-key kernels,
    // =128 takes the 128-key kernel for short sequences too)
    const char* kbenv = std::getenv("RFDETR_ATTN_KB");
    const int kb = kbenv ? std::atoi(kbenv) : 0;
    const bool wide_keys = kb == 128 || (seq_len > RFB_ATTN_SHORT_KEYS && kb != 64);
    if (wide_keys) {
        if (!make_seq_map(&mq, q, cols, seq_len, groups, ldq, AQ) ||
            !make_seq_map(&mk, k, cols, seq_len, groups, ldk, AK2) ||
            !make_seq_map(&mv, v, cols, seq_len, groups, ldv, AK2) ||
            !make_seq_map(&mo, o, cols, seq_len, groups, ldo, 32))
            return cudaErrorInvalidValue;
        const dim3 grid2((seq_len + AQ - 1) / AQ, heads, groups);
        k_attn_tc128<<<grid2, 192, SMEM2, st>>>(mq, mk, mv, mo, seq_len, scale * 1.4426950408889634f, err);
        return cudaGetLastError();
    }
    if (!make_seq_map(&mq, q, cols, seq_len, groups, ldq, AQ) || !make_seq_map(&mk, k, cols, seq_len, groups, ldk, AK) ||
        !make_seq_map(&mv, v, cols, seq_len, groups, ldv, AK) || !make_seq_map(&mo, o, cols, seq_len, groups, ldo, 32))
        return cudaErrorInvalidValue;
    const dim3 grid((seq_len + AQ - 1) / AQ, heads, groups);
    const float sl2 = scale * 1.4426950408889634f;
    // persistent CTAs over (tile, head, group) items: RFDETR_ATTN_ITEMS = 0 off, 1 short sequences, 2 all
    const char* ienv = std::getenv("RFDETR_ATTN_ITEMS");
    const int items_mode = ienv ? std::atoi(ienv) : 1;
    const bool short_seq = seq_len <= RFB_ATTN_SHORT_KEYS;
    if (items_mode >= 2 || (items_mode == 1 && short_seq)) {
        int sms = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
        const long long n_items = (long long)grid.x * heads * groups;
        if (n_items >= (1ll << 31)) return cudaErrorInvalidValue;
        const int per_sm = short_seq ? AttnCfg<2>::MIN_CTAS : AttnCfg<4>::MIN_CTAS;
        const int ctas = (int)(n_items < (long long)per_sm * sms ? n_items : (long long)per_sm * sms);
        if (short_seq)
            k_attn_tc_items<2><<<ctas, 192, AttnCfg<2>::SMEM, st>>>(mq, mk, mv, mo, seq_len, sl2, (int)grid.x, heads,
                                                                   (int)n_items, err);
        else
            k_attn_tc_items<4><<<ctas, 192, AttnCfg<4>::SMEM, st>>>(mq, mk, mv, mo, seq_len, sl2, (int)grid.x, heads,
                                                                   (int)n_items, err);
        return cudaGetLastError();
    }
    if (seq_len <= RFB_ATTN_SHORT_KEYS)
        k_attn_tc<2><<<grid, 192, AttnCfg<2>::SMEM, st>>>(mq, mk, mv, mo, seq_len, sl2, err);
    else
        k_attn_tc<4><<<grid, 192, AttnCfg<4>::SMEM, st>>>(mq, mk, mv, mo, seq_len, sl2, err);
    return cudaGetLastError();
}

}  // namespace rfb
