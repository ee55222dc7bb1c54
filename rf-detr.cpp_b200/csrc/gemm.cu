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
#include "kernels.cuh"
#include "epilogue.cuh"
#include "sm100.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <atomic>
#include <mutex>

namespace rfb {

namespace {

constexpr int BM = 128;
constexpr int BK = 64;


template <int BN, int EPI, bool CTA2 = false>
struct Cfg {
    // Two TMEM accumulators (epilogue of tile i overlaps the mainloop of tile
    // i+1) whenever 2 x BN columns fit in TMEM's 512; BN = 384 (full-row
    // LayerNorm of a 384-wide output) runs with one.
    static constexpr int NACC = 2 * BN <= 512 ? 2 : 1;
    // CTA2: the tile is 256 x BN over a pair of SMs; this CTA holds its 128 A
    // rows and half of the B rows, so its stages are smaller and more of them fit
    static constexpr int B_ROWS = CTA2 ? BN / 2 : BN;
    static constexpr int NEPI = 8;  // epilogue warps: two per TMEM lane quadrant
    static constexpr int THREADS = 64 + 32 * NEPI;
    // f16 outputs of the one-SM 192-wide tile stage through 32-row x 64-byte boxes (32 columns)
    // instead of 128-byte ones: the 16 KB this frees holds a fifth operand stage, and the K = 384
    // linears with this tile (the attention's qkv) are bound by the k-blocks in flight
    static constexpr bool SMALL_BOX = EPI == EPI_F16 && BN == 192 && !CTA2;
    static constexpr int BOX_BYTES = SMALL_BOX ? 2048 : 4096;  // per epilogue warp
    static constexpr int STAGES =
        CTA2 ? (BN > 256 ? 4 : (BN >= 192 ? 6 : 8))
             : (BN > 256 ? 3 : (SMALL_BOX ? 5 : (BN >= 192 ? 4 : (BN == 128 ? 6 : 8))));
    static constexpr int A_BYTES = BM * BK * 2;
    static constexpr int B_BYTES = B_ROWS * BK * 2;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int TMEM_COLS = NACC == 1 ? 512 : (BN == 192 ? 512 : 2 * BN);  // power of two
    // the tile's columns as NSPLIT slabs of one MMA each (N <= 256); a CTA loads HSLAB rows of B per
    // slab: the whole slab, or with CTA2 its half of it (the pair MMA reads both CTAs' halves)
    static constexpr int NSPLIT = BN > 256 ? 2 : 1;
    static constexpr int SLAB = BN / NSPLIT;
    static constexpr int HSLAB = B_ROWS / NSPLIT;
    static constexpr int OUT_STAGE = NEPI * BOX_BYTES;  // per epilogue warp: one 32-row box
    static constexpr int RED_BYTES = EPI == EPI_LN ? 1024 : 0;  // LN: per-row partial sums of 2 warps
    static constexpr int SMEM = STAGES * STAGE_BYTES + OUT_STAGE + 1024 /*align*/ + 256 /*barriers*/ + RED_BYTES;
    static_assert(SMEM <= 232448, "shared memory budget");
};


// CONV: A is the implicit im2col of a 3x3 convolution (GemmArgs::conv_src);
// a 128-row tile is conv_r whole image rows of one image, its rows past
// conv_r * conv_w (and past the image) are computed but not stored.
// CTA2: launched as clusters of two CTAs; each 256 x BN tile is computed by
// tcgen05.mma.cta_group::2 issued by the pair's first CTA (rank 0):
//   both producers   load their 128 A rows and BN/2 B rows; the bytes count on
//                    rank 0's full[s] (expect_tx of both halves by rank 0)
//   rank 0's MMA     commits "stage s consumed" to empty[s] and "accumulator a
//                    ready" to tfull[a] of each CTA (one commit per CTA)
//   both epilogues   arrive "TMEM buffer a free" on rank 0's tempty[a]
// Barriers that the peer arrives on are waited with cluster-scope acquire.
template <int BN, int EPI, int ACT, bool CONV = false, bool CTA2 = false>
__global__ void __launch_bounds__(Cfg<BN, EPI, CTA2>::THREADS, 1)
k_gemm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
       const __grid_constant__ CUtensorMap tmO16, const __grid_constant__ CUtensorMap tmO32, const GemmArgs p) {
    using C = Cfg<BN, EPI, CTA2>;
    constexpr int TM = CTA2 ? 2 * BM : BM;  // rows per tile
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sB = smem + C::STAGES * C::A_BYTES;
    uint8_t* out_stage = smem + C::STAGES * C::STAGE_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(out_stage + C::OUT_STAGE);
    uint64_t* empty = full + C::STAGES;
    uint64_t* tfull = empty + C::STAGES;
    uint64_t* tempty = tfull + 2;
    uint64_t* pairbar = tempty + 2;  // LN: one per TMEM lane quadrant (its two epilogue warps)
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(pairbar + 4);
    volatile int* cta_abort = reinterpret_cast<volatile int*>(tmem_holder + 1);
    float* red = reinterpret_cast<float*>(out_stage + C::OUT_STAGE + 256);  // LN: [2 halves][128 rows]

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // CONV: tiles per image (conv_r image rows each) x images
    const int conv_tpi = CONV ? (p.conv_h + p.conv_r - 1) / p.conv_r : 1;
    const int m_tiles = CONV ? conv_tpi * (p.M / (p.conv_h * p.conv_w)) : (p.M + TM - 1) / TM;
    const uint32_t rank = CTA2 ? cluster_ctarank() : 0u;
    const int tile0 = CTA2 ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
    const int tstep = CTA2 ? (int)(gridDim.x >> 1) : (int)gridDim.x;
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
            mbar_init(&tempty[a], (CTA2 ? 2 : 1) * 32 * C::NEPI);  // CTA2: both CTAs' epilogues
        }
        for (int q = 0; q < 4; ++q) mbar_init(&pairbar[q], 64);
        *cta_abort = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
    }
    if (warp == 1) {
        if constexpr (CTA2) tmem_alloc_pair(tmem_holder, C::TMEM_COLS);
        else tmem_alloc(tmem_holder, C::TMEM_COLS);
    }
    tc_fence_before();
    if constexpr (CTA2) cluster_sync();  // the peer's barriers are initialised before any remote arrive
    else __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;

    if (warp == 0) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            for (int tile = tile0; tile < num_tiles; tile += tstep) {
                const int b = tile / tiles_per_batch;
                const int r = tile - b * tiles_per_batch;
                const int mt = r / n_tiles, nt = r - mt * n_tiles;
                const int arow = b * p.a_batch_rows + mt * TM + (int)rank * BM;
                const int brow = b * p.b_batch_rows + nt * BN + (int)rank * C::HSLAB;  // + sp * SLAB
                const int cimg = CONV ? mt / conv_tpi : 0;
                const int cy0 = CONV ? (mt - cimg * conv_tpi) * p.conv_r : 0;
                const int cch = CONV ? p.conv_c / BK : 1;  // 64-channel chunks per tap
                const int kb0 = p.kb_per ? b * p.kb_per : 0;
                const int kb1 = p.kb_per ? min(num_kb, kb0 + p.kb_per) : num_kb;
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait<CTA2>(&empty[stage], phase ^ 1, cta_abort, p.err)) goto done;
                    if constexpr (CTA2) {
                        if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * C::STAGE_BYTES);  // both halves
                        const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);
                        tma_load_2d_peer_bar(&tmA, fb, sA + stage * C::A_BYTES, kb * BK, arow);
#pragma unroll
                        for (int sp = 0; sp < C::NSPLIT; ++sp)
                            tma_load_2d_peer_bar(&tmB, fb, sB + stage * C::B_BYTES + sp * C::HSLAB * 128, kb * BK,
                                                 brow + sp * C::SLAB);
                    } else if constexpr (CONV) {
                        // box (64 channels, conv_w pixels, conv_r rows) of the map shifted by the tap
                        const int tap = kb / cch, cc = kb - tap * cch;
                        mbar_arrive_expect_tx(&full[stage], C::B_BYTES + BK * 2 * p.conv_w * p.conv_r);
                        tma_load_4d(&tmA, &full[stage], sA + stage * C::A_BYTES, cc * BK, tap % 3 - 1,
                                    cy0 + tap / 3 - 1, cimg);
                    } else {
                        mbar_arrive_expect_tx(&full[stage], C::STAGE_BYTES);
                        tma_load_2d(&tmA, &full[stage], sA + stage * C::A_BYTES, kb * BK, arow);
                    }
                    if constexpr (!CTA2) {
#pragma unroll
                        for (int sp = 0; sp < C::NSPLIT; ++sp)
                            tma_load_2d(&tmB, &full[stage], sB + stage * C::B_BYTES + sp * C::HSLAB * 128, kb * BK,
                                        brow + sp * C::SLAB);
                    }
                    if (++stage == C::STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            constexpr uint32_t IDESC = idesc_f16_f32(TM, C::SLAB);
            int stage = 0;
            uint32_t phase = 0;
            int local = 0;
            for (int tile = tile0; tile < num_tiles; tile += tstep, ++local) {
                const int acc = C::NACC == 2 ? (local & 1) : 0;
                const uint32_t acc_phase = C::NACC == 2 ? ((local >> 1) & 1) : (local & 1);
                if (!mbar_wait<CTA2>(&tempty[acc], acc_phase ^ 1, cta_abort, p.err)) goto done;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                const int kb0 = p.kb_per ? (tile / tiles_per_batch) * p.kb_per : 0;
                const int kb1 = p.kb_per ? min(num_kb, kb0 + p.kb_per) : num_kb;
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait<CTA2>(&full[stage], phase, cta_abort, p.err)) goto done;
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(sA + stage * C::A_BYTES);
                    const uint32_t b0 = smem_u32(sB + stage * C::B_BYTES);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
#pragma unroll
                        for (int sp = 0; sp < C::NSPLIT; ++sp) {
                            const uint64_t ad = sw128_kmajor_desc(a0 + kk * 32);
                            const uint64_t bd = sw128_kmajor_desc(b0 + sp * C::HSLAB * 128 + kk * 32);
                            const uint32_t accum = (kb > kb0 || kk > 0) ? 1u : 0u;
                            if constexpr (CTA2) umma_f16_pair(d_tmem + sp * C::SLAB, ad, bd, IDESC, accum);
                            else umma_f16(d_tmem + sp * C::SLAB, ad, bd, IDESC, accum);
                        }
                    }
                    if constexpr (CTA2) {
                        umma_commit_pair(smem_u32(&empty[stage]));  // the stage is free in both CTAs
                        umma_commit_pair(mapa_shared(smem_u32(&empty[stage]), 1));
                    } else {
                        umma_commit(&empty[stage]);
                    }
                    if (++stage == C::STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if constexpr (CTA2) {
                    umma_commit_pair(smem_u32(&tfull[acc]));  // both CTAs' accumulator halves are ready
                    umma_commit_pair(mapa_shared(smem_u32(&tfull[acc]), 1));
                } else {
                    umma_commit(&tfull[acc]);
                }
            }
        }
    } else {
        // ---------------- epilogue warps ----------------
        const int e = warp - 2;            // 0..7
        const int quad = warp & 3;         // TMEM lanes [32*quad, 32*quad + 32)
        const int half = e >> 2;           // which half of the tile's columns
        const int row_in_tile = quad * 32 + lane;
        // staging: [quad][half] boxes of BOX_BYTES; the LN path uses both halves of its quad
        uint8_t* wptr = out_stage + (quad * 2 + half) * C::BOX_BYTES;
        const uint32_t wbuf = smem_u32(wptr);
        constexpr bool kSplit = (EPI == EPI_LN) || (BN >= 128);
        // first half: whole chunks (64 columns for f16 outputs with 128-byte boxes, else 32)
        constexpr int kChunk = (EPI == EPI_F16 && !C::SMALL_BOX) ? 64 : 32;
        constexpr int kHalf0 = ((BN / 2 + kChunk - 1) / kChunk) * kChunk;
        const bool active = kSplit || half == 0;
        const int col_begin = kSplit ? half * kHalf0 : 0;
        const int col_end = kSplit ? (half ? BN : kHalf0) : BN;
        int local = 0;
        uint32_t pair_phase = 0;
        for (int tile = tile0; tile < num_tiles; tile += tstep, ++local) {
            const int b = tile / tiles_per_batch;
            const int r = tile - b * tiles_per_batch;
            const int mt = r / n_tiles, nt = r - mt * n_tiles;
            const int acc = C::NACC == 2 ? (local & 1) : 0;
            const uint32_t acc_phase = C::NACC == 2 ? ((local >> 1) & 1) : (local & 1);
            if constexpr (EPI == EPI_LN && C::NACC == 1) {
                // One accumulator: this tile's mainloop is running now.  Pull the residual rows the
                // epilogue is about to read into L2 meanwhile (32 rows per TMEM lane quadrant).
                const int r0 = mt * BM + quad * 32;
                if (p.resid && half == 0 && lane == 0 && r0 < p.M && (p.ldr & 3) == 0 && aligned16(p.resid)) {
                    const int nr = p.M - r0 < 32 ? p.M - r0 : 32;
                    prefetch_l2_bulk(p.resid + (size_t)r0 * p.ldr, (uint32_t)nr * p.ldr * 4u);
                }
            }
            if (!__all_sync(0xffffffffu, mbar_wait<CTA2>(&tfull[acc], acc_phase, cta_abort, p.err))) goto done;
            tc_fence_after();
            int m = mt * TM + (int)rank * BM + row_in_tile;
            const int m0w = mt * TM + (int)rank * BM + quad * 32;
            bool row_ok = m < p.M;
            if constexpr (CONV) {
                const int cimg = mt / conv_tpi, cy0 = (mt - cimg * conv_tpi) * p.conv_r;
                const int ry = p.conv_h - cy0 < p.conv_r ? p.conv_h - cy0 : p.conv_r;
                row_ok = row_in_tile < ry * p.conv_w;
                m = (cimg * p.conv_h + cy0) * p.conv_w + row_in_tile;
            }
            const uint32_t tbase = tmem_base + ((uint32_t)(quad * 32) << 16) + acc * BN;
            const long long boff = (long long)b * p.out_batch_stride;
            uint32_t raw[32];
            float v[32];

            if (!active) {
                // idle warp of the LN / narrow-tile paths
            } else if constexpr (EPI == EPI_LN) {
                // BN == N: the two warps of a TMEM lane quadrant own the same 32 rows (one per lane)
                // and split the columns in halves.  Pass 1 forms x = (acc + bias) * colscale + resid,
                // writes it back over the accumulator in TMEM and sums it; passes 2 and 3 reread x
                // from TMEM (sum of squared deviations, then normalise and store).  The two warps
                // exchange per-row partial sums through `red`.
                constexpr int HC = BN / 2;
                const int cbeg = half * HC;
                const float* rrow = (p.resid && row_ok) ? p.resid + (size_t)m * p.ldr : nullptr;
                const bool rvec = rrow && (p.ldr & 3) == 0 && aligned16(p.resid);
                const bool bvec = p.bias && aligned16(p.bias);
                const bool svec = p.colscale && aligned16(p.colscale);
                const bool gvec = aligned16(p.ln_g) && aligned16(p.ln_b);
                float2 s2 = make_float2(0.f, 0.f);
                for (int c0 = cbeg; c0 < cbeg + HC; c0 += 32) {
                    tmem_ld32(tbase + c0, raw);
                    // 16-column sub-chunks keep the residual / bias / scale operands within the
                    // register budget of 10 warps (at most 168 registers per thread)
#pragma unroll
                    for (int sc = 0; sc < 32; sc += 16) {
                        float rv[16], bj[16], sj[16];
                        if (rvec) {
#pragma unroll
                            for (int j = 0; j < 4; ++j) {
                                const float4 u = *reinterpret_cast<const float4*>(rrow + c0 + sc + 4 * j);
                                rv[4 * j] = u.x; rv[4 * j + 1] = u.y; rv[4 * j + 2] = u.z; rv[4 * j + 3] = u.w;
                            }
                        } else {
#pragma unroll
                            for (int j = 0; j < 16; ++j) rv[j] = rrow ? rrow[c0 + sc + j] : 0.f;
                        }
                        load_cols<4>(bj, p.bias, c0 + sc, BN, bvec, 0.f);
                        load_cols<4>(sj, p.colscale, c0 + sc, BN, svec, 1.f);
                        if (sc == 0) tmem_wait_ld();
#pragma unroll
                        for (int j = 0; j < 16; j += 2) {
                            float2 x = __fadd2_rn(
                                make_float2(__uint_as_float(raw[sc + j]), __uint_as_float(raw[sc + j + 1])),
                                make_float2(bj[j], bj[j + 1]));
                            if (p.colscale) x = __fmul2_rn(x, make_float2(sj[j], sj[j + 1]));
                            if (rrow) x = __fadd2_rn(x, make_float2(rv[j], rv[j + 1]));
                            raw[sc + j] = __float_as_uint(x.x);
                            raw[sc + j + 1] = __float_as_uint(x.y);
                            s2 = __fadd2_rn(s2, x);
                        }
                    }
                    tmem_st32(tbase + c0, raw);
                }
                tmem_wait_st();
                red[half * 128 + row_in_tile] = s2.x + s2.y;
                if (!pair_sync(&pairbar[quad], pair_phase, cta_abort, p.err)) goto done;
                const float mean = (red[row_in_tile] + red[128 + row_in_tile]) / (float)BN;
                float2 q2 = make_float2(0.f, 0.f);
                for (int c0 = cbeg; c0 < cbeg + HC; c0 += 32) {
                    tmem_ld32(tbase + c0, raw);
                    tmem_wait_ld();
#pragma unroll
                    for (int j = 0; j < 32; j += 2) {
                        const float2 d = __fadd2_rn(make_float2(__uint_as_float(raw[j]), __uint_as_float(raw[j + 1])),
                                                    make_float2(-mean, -mean));
                        q2 = __ffma2_rn(d, d, q2);
                    }
                }
                // the partner has read this half's sum before `red` is reused
                if (!pair_sync(&pairbar[quad], pair_phase, cta_abort, p.err)) goto done;
                red[half * 128 + row_in_tile] = q2.x + q2.y;
                if (!pair_sync(&pairbar[quad], pair_phase, cta_abort, p.err)) goto done;
                const float var = (red[row_in_tile] + red[128 + row_in_tile]) / (float)BN;
                const float rstd = 1.0f / sqrtf(var + p.ln_eps);
                for (int c0 = cbeg; c0 < cbeg + HC; c0 += 64) {
                    uint32_t raw2[32];
                    tmem_ld32(tbase + c0, raw);
                    tmem_ld32(tbase + c0 + 32, raw2);
                    tmem_wait_ld();
                    const bool tma_out = p.tma_out;
                    // y = act((x - mean) * rstd * g + b), in place, 16 columns at a time
#pragma unroll
                    for (int sc = 0; sc < 64; sc += 16) {
                        float gj[16], bb[16];
                        load_cols<4>(gj, p.ln_g, c0 + sc, BN, gvec, 1.f);
                        load_cols<4>(bb, p.ln_b, c0 + sc, BN, gvec, 0.f);
#pragma unroll
                        for (int t = 0; t < 16; t += 2) {
                            const int j = sc + t;
                            const float2 x = make_float2(__uint_as_float(j < 32 ? raw[j] : raw2[j - 32]),
                                                         __uint_as_float(j < 32 ? raw[j + 1] : raw2[j - 31]));
                            const float2 d =
                                __fmul2_rn(__fadd2_rn(x, make_float2(-mean, -mean)), make_float2(rstd, rstd));
                            const float2 y = act2<ACT>(__ffma2_rn(d, make_float2(gj[t], gj[t + 1]),
                                                                  make_float2(bb[t], bb[t + 1])));
                            if (j < 32) {
                                raw[j] = __float_as_uint(y.x);
                                raw[j + 1] = __float_as_uint(y.y);
                            } else {
                                raw2[j - 32] = __float_as_uint(y.x);
                                raw2[j - 31] = __float_as_uint(y.y);
                            }
                        }
                    }
                    if (tma_out) {
                        if (p.out32) {
#pragma unroll
                            for (int hh = 0; hh < 2; ++hh) {
                                if (lane == 0) bulk_wait_read<0>();
                                __syncwarp();
#pragma unroll
                                for (int j = 0; j < 8; ++j) {
                                    const int jj = 4 * j;
                                    if (hh == 0)
                                        st_shared_v4(swz(wbuf, lane, j), raw[jj], raw[jj + 1], raw[jj + 2], raw[jj + 3]);
                                    else
                                        st_shared_v4(swz(wbuf, lane, j), raw2[jj], raw2[jj + 1], raw2[jj + 2],
                                                     raw2[jj + 3]);
                                }
                                fence_async_smem();
                                __syncwarp();
                                if (lane == 0) {
                                    tma_store_3d(&tmO32, wptr, c0 + 32 * hh, m0w, b);
                                    bulk_commit();
                                }
                            }
                        }
                        if (p.out16) {
                            if (lane == 0) bulk_wait_read<0>();
                            __syncwarp();
#pragma unroll
                            for (int j = 0; j < 8; ++j) {
                                const int jj = 8 * j;
                                uint32_t h4[4];
#pragma unroll
                                for (int q = 0; q < 4; ++q) {
                                    const int c = jj + 2 * q;
                                    h4[q] = pack_half2(__uint_as_float(c < 32 ? raw[c] : raw2[c - 32]),
                                                       __uint_as_float(c < 32 ? raw[c + 1] : raw2[c - 31]));
                                }
                                st_shared_v4(swz(wbuf, lane, j), h4[0], h4[1], h4[2], h4[3]);
                            }
                            fence_async_smem();
                            __syncwarp();
                            if (lane == 0) {
                                tma_store_3d(&tmO16, wptr, c0, m0w, b);
                                bulk_commit();
                            }
                        }
                    } else if (row_ok) {
#pragma unroll
                        for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
                            for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(hh ? raw2[j] : raw[j]);
                            if (p.out32)
                                store_row_f32(p.out32 + boff + (size_t)m * p.ld32 + c0 + 32 * hh, v, c0 + 32 * hh, p.N);
                            if (p.out16)
                                store_row_f16(p.out16 + boff + (size_t)m * p.ld16 + c0 + 32 * hh, v, c0 + 32 * hh, p.N);
                        }
                    }
                }
            } else if (EPI != EPI_PATCH && p.tma_out) {
                if constexpr (EPI == EPI_F16 && C::SMALL_BOX) {
                    // 32-column chunks: one 64-byte f16 box row per thread
                    for (int c0 = col_begin; c0 < col_end; c0 += 32) {
                        tmem_ld32(tbase + c0, raw);
                        const int n0 = nt * BN + c0;
                        float bj[32];
                        load_cols<8>(bj, p.bias, n0, p.N, p.bias && n0 + 32 <= p.N && aligned16(p.bias + n0), 0.f);
                        tmem_wait_ld();
                        uint32_t h[16];
#pragma unroll
                        for (int q = 0; q < 16; ++q) {
                            const float2 w = act2<ACT>(__fadd2_rn(
                                make_float2(__uint_as_float(raw[2 * q]), __uint_as_float(raw[2 * q + 1])),
                                make_float2(bj[2 * q], bj[2 * q + 1])));
                            h[q] = pack_half2(w.x, w.y);
                        }
                        if (lane == 0) bulk_wait_read<0>();
                        __syncwarp();
#pragma unroll
                        for (int j = 0; j < 4; ++j)
                            st_shared_v4(swz64(wbuf, lane, j), h[4 * j], h[4 * j + 1], h[4 * j + 2], h[4 * j + 3]);
                        fence_async_smem();
                        __syncwarp();
                        if (lane == 0) {
                            if (n0 < p.N) tma_store_3d(&tmO16, wptr, n0, m0w, b);
                            bulk_commit();
                        }
                    }
                } else if constexpr (EPI == EPI_F16) {
                    // 64-column chunks: one 128-byte f16 box row per thread
                    for (int c0 = col_begin; c0 < col_end; c0 += 64) {
                        uint32_t raw2[32];
                        tmem_ld32(tbase + c0, raw);
                        tmem_ld32(tbase + c0 + 32, raw2);
                        const int n0 = nt * BN + c0;
                        // The chunk's bias is the same for every lane (one row per lane): warp-uniform
                        // 16-byte loads, issued before the waits so their latency overlaps them.
                        float bj[64];
                        load_cols<16>(bj, p.bias, n0, p.N, p.bias && n0 + 64 <= p.N && aligned16(p.bias + n0), 0.f);
                        tmem_wait_ld();
                        // the whole chunk is computed before waiting for the previous bulk store
                        // to release the staging box, so that wait overlaps the arithmetic
                        uint32_t h[32];
#pragma unroll
                        for (int q = 0; q < 32; ++q) {
                            const int jj = 2 * q;
                            const float2 rv = make_float2(__uint_as_float(jj < 32 ? raw[jj] : raw2[jj - 32]),
                                                          __uint_as_float(jj < 32 ? raw[jj + 1] : raw2[jj - 31]));
                            const float2 w = act2<ACT>(__fadd2_rn(rv, make_float2(bj[jj], bj[jj + 1])));
                            h[q] = pack_half2(w.x, w.y);
                        }
                        if (lane == 0) bulk_wait_read<0>();
                        __syncwarp();
#pragma unroll
                        for (int j = 0; j < 8; ++j)
                            st_shared_v4(swz(wbuf, lane, j), h[4 * j], h[4 * j + 1], h[4 * j + 2], h[4 * j + 3]);
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
                        const bool full = n0 + 32 <= p.N;
                        const bool scaled = EPI == EPI_RESID && p.colscale;
                        // bias / layer scale are warp-uniform per column: broadcast 16-byte loads,
                        // issued before the wait so their latency overlaps it
                        float bj[32], sj[32];
                        load_cols<8>(bj, p.bias, n0, p.N, p.bias && full && aligned16(p.bias + n0), 0.f);
                        if (scaled)
                            load_cols<8>(sj, p.colscale, n0, p.N, full && aligned16(p.colscale + n0), 0.f);
                        tmem_wait_ld();
#pragma unroll
                        for (int jj = 0; jj < 32; jj += 2) {
                            float2 x = act2<ACT>(__fadd2_rn(
                                make_float2(__uint_as_float(raw[jj]), __uint_as_float(raw[jj + 1])),
                                make_float2(bj[jj], bj[jj + 1])));
                            if (scaled) x = __fmul2_rn(x, make_float2(sj[jj], sj[jj + 1]));
                            v[jj] = x.x;
                            v[jj + 1] = x.y;
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
            } else if (EPI == EPI_PATCH && p.patch_vec) {
                // window remap + position add: each 32-column chunk goes through the warp's staging box,
                // then 8 lanes write one 128-byte row (4 rows per instruction), so the remapped stores
                // and the position loads are coalesced.  A lane's eight rows are the same for every
                // chunk of the tile: their output and position rows are found once per tile, and
                // all eight position loads of a chunk are issued before the stores.
                long long orow[8];
                int prow[8];
#pragma unroll
                for (int it = 0; it < 8; ++it) {
                    const int mr = mt * BM + quad * 32 + it * 4 + (lane >> 3);
                    const int img = mr / p.patch_rows;
                    const int rr = mr - img * p.patch_rows;
                    const int win = rr / p.patch_tp;
                    const int tok = win * p.patch_t + 1 + (rr - win * p.patch_tp);
                    orow[it] = mr < p.M ? ((long long)img * p.patch_ntok + tok) * p.ld32 : -1;
                    prow[it] = tok * p.N;
                }
                for (int c0 = col_begin; c0 < col_end; c0 += 32) {
                    tmem_ld32(tbase + c0, raw);
                    const int n0 = nt * BN + c0;
                    const float bl = (p.bias && n0 + lane < p.N) ? p.bias[n0 + lane] : 0.f;
                    tmem_wait_ld();
                    __syncwarp();
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        st_shared_v4(swz(wbuf, lane, j),
                                     __float_as_uint(__uint_as_float(raw[4 * j]) + bcast(bl, 4 * j)),
                                     __float_as_uint(__uint_as_float(raw[4 * j + 1]) + bcast(bl, 4 * j + 1)),
                                     __float_as_uint(__uint_as_float(raw[4 * j + 2]) + bcast(bl, 4 * j + 2)),
                                     __float_as_uint(__uint_as_float(raw[4 * j + 3]) + bcast(bl, 4 * j + 3)));
                    __syncwarp();
                    const int ch = lane & 7;
                    const int n = n0 + 4 * ch;
                    if (n < p.N) {
                        float4 ps[8];
#pragma unroll
                        for (int it = 0; it < 8; ++it)
                            ps[it] = orow[it] >= 0 ? __ldg(reinterpret_cast<const float4*>(p.posw + prow[it] + n))
                                                   : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                        for (int it = 0; it < 8; ++it) {
                            if (orow[it] < 0) continue;
                            float4 x = ld_shared_v4f(swz(wbuf, it * 4 + (lane >> 3), ch));
                            x.x += ps[it].x; x.y += ps[it].y; x.z += ps[it].z; x.w += ps[it].w;
                            *reinterpret_cast<float4*>(p.out32 + orow[it] + n) = x;
                        }
                    }
                    __syncwarp();
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
                    if constexpr (EPI == EPI_F32) {
                        // through the warp's staging box: each store instruction then writes 32
                        // consecutive columns of one row instead of one value of 32 rows.  The
                        // quadrant's rows are consecutive (m - lane + r), the ballot marks the
                        // valid ones.
                        const unsigned okmask = __ballot_sync(0xffffffffu, row_ok);
                        __syncwarp();
#pragma unroll
                        for (int j = 0; j < 8; ++j)
                            st_shared_v4(swz(wbuf, lane, j), __float_as_uint(v[4 * j]), __float_as_uint(v[4 * j + 1]),
                                         __float_as_uint(v[4 * j + 2]), __float_as_uint(v[4 * j + 3]));
                        __syncwarp();
                        if (nok) {
                            float* col = p.out32 + boff + (long long)(m - lane) * p.ld32 + n0 + lane;
#pragma unroll 8
                            for (int r = 0; r < 32; ++r)
                                if ((okmask >> r) & 1u)
                                    col[(long long)r * p.ld32] = ld_shared_f32(swz(wbuf, r, lane >> 2) + (lane & 3) * 4);
                        }
                        __syncwarp();
                        continue;
                    }
                    if (!row_ok || n0 >= p.N) continue;
                    if constexpr (EPI == EPI_F16) {
                        store_row_f16(p.out16 + boff + (size_t)m * p.ld16 + n0, v, n0, p.N);
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
            if constexpr (CTA2) mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[acc]), 0));
            else mbar_arrive(&tempty[acc]);
        }
        if (lane == 0) bulk_wait<0>();
    }
done:
    if constexpr (CTA2) {
        cluster_sync();  // no CTA leaves while its peer may still signal its barriers
        if (warp == 1) {
            tc_fence_after();
            tmem_dealloc_pair(tmem_base, C::TMEM_COLS);
        }
    } else {
        __syncthreads();
        if (warp == 1) {
            tc_fence_after();
            tmem_dealloc(tmem_base, C::TMEM_COLS);
        }
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

// 3-D output map (cols, rows, batch) with a swizzled box of 32 rows of `row_bytes` (128 or 64) bytes.
bool make_out_map(CUtensorMap* map, const void* base, bool f16, int cols, int rows, int batches, int ld,
                  long long batch_stride, int row_bytes = 128) {
    const int esz = f16 ? 2 : 4;
    if (!base || ((uintptr_t)base & 15) || ((size_t)ld * esz) % 16) return false;
    if (batches > 1 && ((size_t)batch_stride * esz) % 16) return false;
    cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)batches};
    cuuint64_t strides[2] = {(cuuint64_t)ld * esz,
                             (cuuint64_t)(batches > 1 ? batch_stride : (long long)ld * rows) * esz};
    cuuint32_t box[3] = {(cuuint32_t)(row_bytes / esz), 32, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    return g_encode(map, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3,
                    const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    row_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_NONE,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 4-D map (channel, x, y, image) of a channels-last f16 map with pixel pitch
// `lds`, box (64 channels, w, rows, 1): the implicit im2col operand.
bool make_conv_map(CUtensorMap* map, const void* base, int c, int w, int h, int imgs, int lds, int rows) {
    if (!base || ((uintptr_t)base & 15) || (lds % 8) || c % BK || w > 256 || rows > 256 || w * rows > BM)
        return false;
    cuuint64_t dims[4] = {(cuuint64_t)c, (cuuint64_t)w, (cuuint64_t)h, (cuuint64_t)imgs};
    cuuint64_t strides[3] = {(cuuint64_t)lds * 2, (cuuint64_t)lds * 2 * w, (cuuint64_t)lds * 2 * w * h};
    cuuint32_t box[4] = {(cuuint32_t)BK, (cuuint32_t)w, (cuuint32_t)rows, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    return g_encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BN, int EPI, int ACT, bool CONV = false, bool CTA2 = false>
cudaError_t launch(const GemmArgs& a_in, cudaStream_t st) {
    using C = Cfg<BN, EPI, CTA2>;
    GemmArgs a = a_in;
    static std::atomic<uint64_t> attr_set{0};  // per (BN, EPI) instantiation, one bit per device
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = 1ull << (dev & 63);
    if (!(attr_set.load() & bit)) {
        e = cudaFuncSetAttribute(k_gemm<BN, EPI, ACT, CONV, CTA2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 C::SMEM);
        if (e != cudaSuccess) return e;
        attr_set.fetch_or(bit);
    }
    CUtensorMap ta, tb;
    const long long a_rows = (long long)a.a_batch_rows * (a.batches - 1) + a.M;
    const long long b_rows = (long long)a.b_batch_rows * (a.batches - 1) + a.N;
    if constexpr (CONV) {
        a.conv_r = BM / a.conv_w;
        // batches > 1 only as split-K partial sums of one convolution (kb_per > 0)
        if ((a.batches != 1 && !a.kb_per) || a.conv_r < 1 || a.K != 9 * a.conv_c || a.M % (a.conv_h * a.conv_w))
            return cudaErrorInvalidValue;
        if (!make_conv_map(&ta, a.conv_src, a.conv_c, a.conv_w, a.conv_h, a.M / (a.conv_h * a.conv_w), a.conv_lds,
                           a.conv_r))
            return cudaErrorInvalidValue;
    } else if (!make_map(&ta, a.A, a.K, a_rows, a.lda, BM)) {
        return cudaErrorInvalidValue;
    }
    if (!make_map(&tb, a.B, a.K, b_rows, a.ldb, C::HSLAB))
        return cudaErrorInvalidValue;
    CUtensorMap to16, to32;
    std::memset(&to16, 0, sizeof(to16));
    std::memset(&to32, 0, sizeof(to32));
    bool tma = EPI != EPI_PATCH && !CONV;  // CONV tiles hold fewer than 128 valid rows: direct stores
    if (tma && a.out16)
        tma = make_out_map(&to16, a.out16, true, a.N, a.M, a.batches, a.ld16, a.out_batch_stride, C::BOX_BYTES / 32);
    if (tma && a.out32) tma = make_out_map(&to32, a.out32, false, a.N, a.M, a.batches, a.ld32, a.out_batch_stride);
    a.tma_out = tma ? 1 : 0;
    a.patch_vec = (EPI == EPI_PATCH && a.N % 4 == 0 && a.ld32 % 4 == 0 && !((uintptr_t)a.out32 & 15) &&
                   !((uintptr_t)a.posw & 15)) ? 1 : 0;
    constexpr int TM = CTA2 ? 2 * BM : BM;
    const int m_tiles = CONV ? ((a.conv_h + a.conv_r - 1) / a.conv_r) * (a.M / (a.conv_h * a.conv_w))
                             : (a.M + TM - 1) / TM;
    const int tiles = m_tiles * ((a.N + BN - 1) / BN) * a.batches;
    if constexpr (CTA2) {
        // clusters of two CTAs, one cluster per pair of SMs (or per tile when there are fewer)
        const int pairs = g_num_sms / 2;
        const int grid = 2 * (tiles < pairs ? tiles : pairs);
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)grid);
        cfg.blockDim = dim3(C::THREADS);
        cfg.dynamicSmemBytes = C::SMEM;
        cfg.stream = st;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        e = cudaLaunchKernelEx(&cfg, k_gemm<BN, EPI, ACT, CONV, CTA2>, ta, tb, to16, to32, a);
        if (e != cudaSuccess) return e;
        return cudaGetLastError();
    }
    const int grid = tiles < g_num_sms ? tiles : g_num_sms;
    k_gemm<BN, EPI, ACT, CONV><<<grid, C::THREADS, C::SMEM, st>>>(ta, tb, to16, to32, a);
    return cudaGetLastError();
}

// Two-SM tiles (256 x BN over a cluster of two CTAs) for plain GEMMs: f16 /
// f32 / residual epilogues, BN 192, 256 or 384 (residual only), one batch.
bool use_pair(const GemmArgs& a, int bn) {
    if (a.batches != 1 || (bn != 192 && bn != 256 && bn != 384) || a.conv_src) return false;
    if (a.epi != EPI_F16 && a.epi != EPI_F32 && a.epi != EPI_RESID) return false;
    // RFDETR_GEMM_2SM=0 never, =1 always, =auto whenever there are at least two pair-tiles per pair
    // of SMs; by default only for the 384-wide residual tile (the MLP's long-K output GEMM), the
    // one shape where pairs measured faster (Base batch 32: 72.3 -> 71.0 us; the K = 384 shapes
    // are 5-15 % slower as pairs)
    const char* env = std::getenv("RFDETR_GEMM_2SM");
    if (env && env[0] == '0') return false;
    if (env && env[0] == '1') return true;
    const long long tiles = (long long)((a.M + 2 * BM - 1) / (2 * BM)) * ((a.N + bn - 1) / bn);
    if (env) return tiles >= (long long)g_num_sms;
    return bn == 384 && tiles >= (long long)g_num_sms;
}

// RFDETR_GEMM_SPLITK=0 keeps the full-row LayerNorm tiles for few row blocks.
bool splitk_enabled() {
    const char* env = std::getenv("RFDETR_GEMM_SPLITK");
    return !(env && env[0] == '0');
}

// What the split-K LayerNorm row kernel handles: rows of 128 / 256 / 384, no activation or SiLU,
// 16-byte aligned f32 rows and 8-byte aligned f16 rows.
bool splitk_ln_supported(const GemmArgs& a) {
    auto al = [](const void* q, uintptr_t m) { return !((uintptr_t)q & m); };
    return (a.N == 128 || a.N == 256 || a.N == 384) && (a.act == ACT_NONE || a.act == ACT_SILU) &&
           al(a.split_ws, 15) && al(a.bias, 15) && al(a.colscale, 15) && al(a.ln_g, 15) && al(a.ln_b, 15) &&
           (!a.resid || (al(a.resid, 15) && a.ldr % 4 == 0)) && (!a.out32 || (al(a.out32, 15) && a.ld32 % 4 == 0)) &&
           (!a.out16 || (al(a.out16, 7) && a.ld16 % 4 == 0));
}

// Residual GEMMs of N = 384 and long K (the MLP's second linear) as one
// 384-wide tile per row block; RFDETR_GEMM_BN384=0 falls back to two 192-wide tiles.
bool wide_resid() {
    const char* env = std::getenv("RFDETR_GEMM_BN384");
    return !(env && env[0] == '0');
}

template <int EPI, int ACT>
cudaError_t dispatch_bn(const GemmArgs& a, int bn, cudaStream_t st) {
    if constexpr (EPI == EPI_F16 || EPI == EPI_F32 || EPI == EPI_RESID) {
        if (use_pair(a, bn)) {
            if constexpr (EPI == EPI_RESID && ACT == ACT_NONE)
                if (bn == 384) return launch<384, EPI, ACT, false, true>(a, st);
            if constexpr (ACT == ACT_NONE || ACT == ACT_GELU)
                return bn == 256 ? launch<256, EPI, ACT, false, true>(a, st) : launch<192, EPI, ACT, false, true>(a, st);
        }
    }
    if constexpr (EPI == EPI_RESID && ACT == ACT_NONE)
        if (bn == 384) return launch<384, EPI, ACT>(a, st);
    switch (bn) {
        case 256: return launch<256, EPI, ACT>(a, st);
        case 192: return launch<192, EPI, ACT>(a, st);
        case 128: return launch<128, EPI, ACT>(a, st);
        default: return launch<64, EPI, ACT>(a, st);
    }
}

}  // namespace

void gemm_set_num_sms(int n) { g_num_sms = n > 0 ? n : 148; }


cudaError_t gemm(const GemmArgs& a_in, cudaStream_t stream) {
    if (!load_encode()) return cudaErrorNotSupported;
    GemmArgs a = a_in;
    if (a.M <= 0 || a.N <= 0 || a.K <= 0 || a.batches <= 0) return cudaErrorInvalidValue;
    // TMA: 16-byte aligned base and row pitch
    if ((a.lda % 8) || (a.ldb % 8) || (((uintptr_t)a.A) & 15) || (((uintptr_t)a.B) & 15)) return cudaErrorInvalidValue;
    if (a.conv_src) {
        // implicit-GEMM 3x3 convolution with the ConvX LayerNorm (+ SiLU) epilogue
        if (a.epi != EPI_LN || (a.N != 128 && a.N != 256) || !a.ln_g || !a.ln_b || a.conv_c % BK || a.conv_w < 1 ||
            a.conv_w > BM || a.conv_h < 1 || (a.act != ACT_NONE && a.act != ACT_SILU))
            return cudaErrorInvalidValue;
        if (a.split_ws && a.batches == 1 && splitk_enabled() && splitk_ln_supported(a)) {
            // few row-tiles (small batches): split-K f32 partial sums + in-order LayerNorm rows, as below
            const int num_kb = (a.K + BK - 1) / BK;
            const int conv_r = BM / a.conv_w;
            const long long tiles = (long long)((a.conv_h + conv_r - 1) / conv_r) * (a.M / (a.conv_h * a.conv_w));
            if (tiles * 2 <= g_num_sms && num_kb >= 2) {
                int ks = (int)(g_num_sms / tiles);
                ks = ks < num_kb ? ks : num_kb;
                const int kbp = (num_kb + ks - 1) / ks;
                ks = (num_kb + kbp - 1) / kbp;
                if (ks >= 2 && (size_t)ks * a.M * a.N * sizeof(float) <= a.split_ws_bytes) {
                    GemmArgs s = a;
                    s.epi = EPI_F32; s.act = ACT_NONE;
                    s.bias = nullptr; s.ln_g = nullptr; s.ln_b = nullptr;
                    s.out32 = a.split_ws; s.ld32 = a.N; s.out16 = nullptr; s.ld16 = 0;
                    s.batches = ks; s.a_batch_rows = 0; s.b_batch_rows = 0;
                    s.out_batch_stride = (long long)a.M * a.N;
                    s.kb_per = kbp;
                    const cudaError_t e = a.N == 256 ? launch<256, EPI_F32, ACT_NONE, true>(s, stream)
                                                     : launch<128, EPI_F32, ACT_NONE, true>(s, stream);
                    if (e != cudaSuccess) return e;
                    return splitk_layernorm(a.split_ws, ks, (long long)a.M * a.N, a.M, a.N, a.bias, nullptr, nullptr,
                                            0, a.ln_g, a.ln_b, a.ln_eps, a.act, nullptr, 0, a.out16, a.ld16, stream);
                }
            }
        }
        if (a.act == ACT_SILU)
            return a.N == 256 ? launch<256, EPI_LN, ACT_SILU, true>(a, stream) : launch<128, EPI_LN, ACT_SILU, true>(a, stream);
        return a.N == 256 ? launch<256, EPI_LN, ACT_NONE, true>(a, stream) : launch<128, EPI_LN, ACT_NONE, true>(a, stream);
    }
    int bn;
    if (a.epi == EPI_LN) {
        if (a.N != 128 && a.N != 256 && a.N != 384) return cudaErrorInvalidValue;
        if (!a.ln_g || !a.ln_b) return cudaErrorInvalidValue;
        bn = a.N;
    } else if (a.N == 384 && a.epi == EPI_RESID && a.act == ACT_NONE && a.K >= 768 && wide_resid() &&
               (long long)((a.M + BM - 1) / BM) * a.batches >= g_num_sms) {
        bn = 384;  // one full-row tile: A crosses from L2 once per row block instead of twice
    } else if (a.N % 256 == 0) {
        bn = 256;
    } else if (a.N % 192 == 0) {
        bn = 192;  // N = 384 / 1152: two or six 192-wide tiles instead of 128-wide ones
    } else if (a.N > 64) {
        bn = 128;
    } else {
        bn = 64;
    }
    if (a.epi == EPI_LN && a.split_ws && a.batches == 1 && splitk_enabled()) {
        // Few row blocks (small batches): a full-row LayerNorm tile per row block would leave most
        // SMs idle, so the K range is split: f32 partial sums per split into the scratch, then
        // one row kernel adds them in split order and applies bias, scale, residual, LayerNorm and
        // the activation (deterministic: the order of the additions is fixed).
        const int num_kb = (a.K + BK - 1) / BK;
        const long long m_tiles = (a.M + BM - 1) / BM;
        int sbn = a.N % 256 == 0 ? 256 : (a.N % 192 == 0 ? 192 : (a.N > 64 ? 128 : 64));
        for (const int w : {128, 64})
            if (m_tiles * ((a.N + sbn - 1) / sbn) < g_num_sms && w < sbn) sbn = w;
        const long long tiles = m_tiles * ((a.N + sbn - 1) / sbn);
        if (tiles * 2 <= g_num_sms && num_kb >= 2 && splitk_ln_supported(a)) {
            int ks = (int)(g_num_sms / tiles);
            ks = ks < num_kb ? ks : num_kb;
            const int kbp = (num_kb + ks - 1) / ks;
            ks = (num_kb + kbp - 1) / kbp;  // no empty split
            if (ks >= 2 && (size_t)ks * a.M * a.N * sizeof(float) <= a.split_ws_bytes) {
                GemmArgs s = a;
                s.epi = EPI_F32; s.act = ACT_NONE;
                s.bias = nullptr; s.colscale = nullptr; s.resid = nullptr;
                s.ln_g = nullptr; s.ln_b = nullptr;
                s.out32 = a.split_ws; s.ld32 = a.N; s.out16 = nullptr; s.ld16 = 0;
                s.batches = ks; s.a_batch_rows = 0; s.b_batch_rows = 0;
                s.out_batch_stride = (long long)a.M * a.N;
                s.kb_per = kbp;
                const cudaError_t e = dispatch_bn<EPI_F32, ACT_NONE>(s, sbn, stream);
                if (e != cudaSuccess) return e;
                return splitk_layernorm(a.split_ws, ks, (long long)a.M * a.N, a.M, a.N, a.bias, a.colscale, a.resid,
                                        a.ldr, a.ln_g, a.ln_b, a.ln_eps, a.act, a.out32, a.ld32, a.out16,
                                        a.ld16, stream);
            }
        }
    }
    if (a.epi != EPI_LN) {
        // few row blocks (small batches): narrower tiles until the grid covers every SM, so a
        // batch-1 forward does not run its GEMMs on a tenth of the GPU
        const long long m_tiles = (long long)((a.M + BM - 1) / BM) * a.batches;
        auto tiles = [&](int w) { return m_tiles * ((a.N + w - 1) / w); };
        for (const int w : {128, 64}) {
            if (tiles(bn) >= g_num_sms || w >= bn) continue;
            bn = w;
        }
        // tuning override: RFDETR_GEMM_BN = 128 / 192 / 256 where it divides N
        const char* env = std::getenv("RFDETR_GEMM_BN");
        const int f = env ? std::atoi(env) : 0;
        if ((f == 128 || f == 192 || f == 256) && a.N % f == 0) bn = f;
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
            if (a.act == ACT_NONE) {
                if (bn == 384) return launch<384, EPI_LN, ACT_NONE>(a, stream);
                return bn == 256 ? launch<256, EPI_LN, ACT_NONE>(a, stream) : launch<128, EPI_LN, ACT_NONE>(a, stream);
            }
            if (a.act == ACT_SILU && bn != 384)
                return bn == 256 ? launch<256, EPI_LN, ACT_SILU>(a, stream) : launch<128, EPI_LN, ACT_SILU>(a, stream);
            return cudaErrorInvalidValue;
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace rfb
