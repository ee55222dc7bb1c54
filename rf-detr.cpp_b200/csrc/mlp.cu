// Fused MLP of a DINOv2 block (src/dinov2.cpp:93-101 with the layer scale and
// residual of :483-486): x += ls * (fc2(GELU(fc1(h))) ), the 1536-wide hidden
// activations never leaving the SM.
//
// One persistent CTA per SM, 128-row tiles, the hidden dimension in chunks of
// 128 columns.  Per tile:
//   G1(c)   S  = h . W1[c]^T                 (M=128, N=128, K=D)  TMEM cols [384, 512)
//   epi(c)  P  = GELU(S + b1[c]) as f16      -> 128B-swizzled smem (A operand of G2)
//   G2(c)   O += P . W2[:, c]^T              (M=128, N=D as D/128 parts of 128, K=128)
//                                                               TMEM cols [0, D)
//   final   x += ls * (O + b2)                TMA reduce-add into the f32 stream
// Roles (320 threads):
//   warp 0      TMA: the tile's input rows h (D x 128, resident for the tile)
//               and the W1 / W2 boxes (128 x 64 f16) through a 6-stage ring in
//               exactly the order the MMAs consume them
//   warp 1      TMEM allocation; one lane issues the MMAs in the order
//               G1(0) G1(1) G2(0) G1(2) G2(1) ... G2(last): fc1 of chunk c+1
//               runs on the tensor cores while the epilogue computes GELU of c
//   warps 2..9  epilogue (two per TMEM lane quadrant, 64 columns of S each);
//               P has one buffer: GELU(c+1) overwrites it once G2(c) has read
//               it, and G1(c+2) keeps the tensor cores busy meanwhile, so the
//               32 KB saved go to a deeper weight ring (6 x 16 KB in flight)
// The final epilogue stages its f32 boxes in the P buffer the finished tile no
// longer reads.  Every mbarrier wait is bounded (sm100.cuh).
#include "mlp.cuh"

#include "epilogue.cuh"
#include "sm100.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <atomic>
#include <cstring>
#include <mutex>

namespace rfb {

namespace {

constexpr int MB = 128;                        // rows per tile
constexpr int HN = 128;                        // hidden columns per chunk
constexpr int KB = 64;                         // K of one swizzle atom / TMA box (128 bytes of f16)
constexpr int DMAX = 384;                      // widest D: TMEM holds O (DMAX) + S (HN) = 512 columns
constexpr int NST = 6;                         // weight ring stages
constexpr int ATOM = MB * KB * 2;              // 16 KB: 128 rows x 64 f16
constexpr int A_BYTES = (DMAX / KB) * ATOM;    // 96 KB resident input tile
constexpr int P_BYTES = (HN / KB) * ATOM;      // 32 KB GELU buffer
constexpr int SMEM = A_BYTES + P_BYTES + NST * ATOM + 1024 /*align*/ + 256 /*barriers*/;
constexpr int kThreadsMlp = 320;
constexpr int kEpiMlp = 256;
static_assert(SMEM <= 232448, "shared memory budget");

__global__ void __launch_bounds__(kThreadsMlp, 1)
k_mlp(const __grid_constant__ CUtensorMap tmH, const __grid_constant__ CUtensorMap tmW1,
      const __grid_constant__ CUtensorMap tmW2, const __grid_constant__ CUtensorMap tmX, const MlpArgs p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sA = smem;
    uint8_t* sP = sA + A_BYTES;      // GELU output of the current chunk
    uint8_t* sW = sP + P_BYTES;      // [NST][ATOM]
    uint64_t* w_full = reinterpret_cast<uint64_t*>(sW + NST * ATOM);  // [NST]
    uint64_t* w_empty = w_full + NST;                                  // [NST]
    uint64_t* a_full = w_empty + NST;
    uint64_t* a_empty = a_full + 1;
    uint64_t* s_full = a_full + 2;
    uint64_t* s_empty = a_full + 3;
    uint64_t* p_full = a_full + 4;
    uint64_t* p_empty = a_full + 5;
    uint64_t* o_full = a_full + 6;
    uint64_t* o_empty = a_full + 7;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(a_full + 8);
    volatile int* cta_abort = reinterpret_cast<volatile int*>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nd = p.D / KB;  // swizzle atoms of the input row (K of fc1)
    const int np = p.D / HN;  // 128-wide parts of the fc2 output (N of fc2)
    const int nc = p.F / HN;  // hidden chunks
    const int m_tiles = (p.M + MB - 1) / MB;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NST; ++s) {
            mbar_init(&w_full[s], 1);
            mbar_init(&w_empty[s], 1);
        }
        mbar_init(a_full, 1);
        mbar_init(a_empty, 1);
        mbar_init(s_full, 1);
        mbar_init(s_empty, kEpiMlp);
        mbar_init(p_full, kEpiMlp);
        mbar_init(p_empty, 1);
        mbar_init(o_full, 1);
        mbar_init(o_empty, kEpiMlp);
        *cta_abort = 0;
        fence_mbar_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmH);
        prefetch_tmap(&tmW1);
        prefetch_tmap(&tmW2);
        prefetch_tmap(&tmX);
    }
    if (warp == 1) tmem_alloc(tmem_holder, 512);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_holder;
    const uint32_t tO = tmem_base, tS = tmem_base + DMAX;

    if (warp == 0) {
        if (lane == 0) {
            int ws = 0;
            uint32_t wph = 0;
            int local = 0;
            for (int tile = blockIdx.x; tile < m_tiles; tile += gridDim.x, ++local) {
                // the tile's input rows, once the previous tile's last fc1 MMAs are done with sA
                if (!mbar_wait(a_empty, (local & 1) ^ 1, cta_abort, p.err)) goto done;
                mbar_arrive_expect_tx(a_full, nd * ATOM);
                for (int kb = 0; kb < nd; ++kb) tma_load_2d(&tmH, a_full, sA + kb * ATOM, kb * KB, tile * MB);
                // weights in MMA order: W1(0), W1(1), W2(0), W1(2), W2(1), ..., W1(nc-1), W2(nc-2), W2(nc-1)
                for (int c = 0; c <= nc; ++c) {
                    for (int j = 0; j < (c < nc ? nd : 0) + (c >= 1 ? 2 * np : 0); ++j) {
                        if (!mbar_wait(&w_empty[ws], wph ^ 1, cta_abort, p.err)) goto done;
                        mbar_arrive_expect_tx(&w_full[ws], ATOM);
                        if (c < nc && j < nd) {
                            tma_load_2d(&tmW1, &w_full[ws], sW + ws * ATOM, j * KB, c * HN);
                        } else {
                            const int q = j - (c < nc ? nd : 0);  // (kk, n) = (q / np, q % np)
                            tma_load_2d(&tmW2, &w_full[ws], sW + ws * ATOM, (c - 1) * HN + (q / np) * KB,
                                        (q % np) * HN);
                        }
                        if (++ws == NST) {
                            ws = 0;
                            wph ^= 1;
                        }
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t IDESC = idesc_f16_f32(MB, HN);
            int ws = 0;
            uint32_t wph = 0;
            uint32_t s_cnt = 0;  // fc1 chunks issued so far
            uint32_t g = 0;      // fc2 chunks issued so far (p_full / p_empty phase = g & 1)
            int local = 0;
            for (int tile = blockIdx.x; tile < m_tiles; tile += gridDim.x, ++local) {
                if (!mbar_wait(a_full, local & 1, cta_abort, p.err)) goto done;
                tc_fence_after();
                for (int c = 0; c <= nc; ++c) {
                    if (c < nc) {
                        // G1(c) into S, once the epilogue has read S of the previous chunk
                        if (!mbar_wait(s_empty, (s_cnt & 1) ^ 1, cta_abort, p.err)) goto done;
                        tc_fence_after();
                        for (int kb = 0; kb < nd; ++kb) {
                            if (!mbar_wait(&w_full[ws], wph, cta_abort, p.err)) goto done;
                            tc_fence_after();
                            const uint32_t a0 = smem_u32(sA + kb * ATOM), b0 = smem_u32(sW + ws * ATOM);
#pragma unroll
                            for (int kk = 0; kk < KB / 16; ++kk)
                                umma_f16(tS, sw128_kmajor_desc(a0 + kk * 32), sw128_kmajor_desc(b0 + kk * 32), IDESC,
                                         (kb | kk) != 0);
                            umma_commit(&w_empty[ws]);
                            if (++ws == NST) {
                                ws = 0;
                                wph ^= 1;
                            }
                        }
                        umma_commit(s_full);
                        ++s_cnt;
                        if (c == nc - 1) umma_commit(a_empty);
                    }
                    if (c >= 1) {
                        // G2(c-1) into O from the GELU output of chunk c-1
                        const int cc = c - 1;
                        if (!mbar_wait(p_full, g & 1, cta_abort, p.err)) goto done;
                        if (cc == 0 && !mbar_wait(o_empty, (local & 1) ^ 1, cta_abort, p.err)) goto done;
                        tc_fence_after();
                        for (int q = 0; q < 2 * np; ++q) {
                            const int kk = q / np, n = q - kk * np;
                            if (!mbar_wait(&w_full[ws], wph, cta_abort, p.err)) goto done;
                            tc_fence_after();
                            const uint32_t a0 = smem_u32(sP + kk * ATOM), b0 = smem_u32(sW + ws * ATOM);
#pragma unroll
                            for (int k16 = 0; k16 < KB / 16; ++k16)
                                umma_f16(tO + n * HN, sw128_kmajor_desc(a0 + k16 * 32),
                                         sw128_kmajor_desc(b0 + k16 * 32), IDESC, (cc | kk | k16) != 0);
                            umma_commit(&w_empty[ws]);
                            if (++ws == NST) {
                                ws = 0;
                                wph ^= 1;
                            }
                        }
                        umma_commit(p_empty);
                        ++g;
                        if (cc == nc - 1) umma_commit(o_full);
                    }
                }
            }
        }
    } else {
        // ---------------- epilogue warps ----------------
        const int e = warp - 2;
        const int quad = warp & 3;  // TMEM lanes [32 quad, 32 quad + 32)
        const int half = e >> 2;    // 64 columns of S; half of the columns of O
        const int row = quad * 32 + lane;
        const uint32_t lanebase = (uint32_t)(quad * 32) << 16;
        const bool b1vec = aligned16(p.b1), b2vec = aligned16(p.b2), lsvec = p.ls && aligned16(p.ls);
        uint32_t g = 0;
        int local = 0;
        for (int tile = blockIdx.x; tile < m_tiles; tile += gridDim.x, ++local) {
            for (int c = 0; c < nc; ++c, ++g) {
                const int h0 = c * HN + half * 64;  // hidden column of this warp's first S column
                float bj[64];
                load_cols<16>(bj, p.b1, h0, p.F, b1vec, 0.f);
                if (!__all_sync(0xffffffffu, mbar_wait(s_full, g & 1, cta_abort, p.err))) goto done;
                tc_fence_after();
                uint32_t r0[32], r1[32];
                tmem_ld32(tS + lanebase + half * 64, r0);
                tmem_ld32(tS + lanebase + half * 64 + 32, r1);
                tmem_wait_ld();
                tc_fence_before();
                mbar_arrive(s_empty);
                uint32_t hp[32];
#pragma unroll
                for (int j = 0; j < 64; j += 2) {
                    const float2 v = make_float2(__uint_as_float(j < 32 ? r0[j] : r1[j - 32]),
                                                 __uint_as_float(j < 32 ? r0[j + 1] : r1[j - 31]));
                    const float2 y = gelu_erf2(__fadd2_rn(v, make_float2(bj[j], bj[j + 1])));
                    hp[j >> 1] = pack_half2(y.x, y.y);
                }
                // P of the previous chunk has been read by its fc2 MMAs (issued after fc1 of this chunk,
                // so the tensor cores stay busy while this waits)
                if (!__all_sync(0xffffffffu, mbar_wait(p_empty, (g & 1) ^ 1, cta_abort, p.err))) goto done;
                // this thread's row of the 64-column atom `half` of P (K-major, 128-byte swizzle)
                const uint32_t pa = smem_u32(sP + half * ATOM);
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    st_shared_v4(swz(pa, row, j), hp[4 * j], hp[4 * j + 1], hp[4 * j + 2], hp[4 * j + 3]);
                fence_async_smem();
                mbar_arrive(p_full);
            }
            // final: x += ls * (O + b2), staged in this warp's 4 KB of the (now idle) P buffer
            if (!__all_sync(0xffffffffu, mbar_wait(o_full, local & 1, cta_abort, p.err))) goto done;
            tc_fence_after();
            {
                uint8_t* stage = sP + half * ATOM + quad * 4096;
                const uint32_t st_s = smem_u32(stage);
                const int cb = half * (p.D / 2), ce = cb + p.D / 2;
                for (int c0 = cb; c0 < ce; c0 += 32) {
                    float b2j[32], sj[32];
                    uint32_t raw[32];
                    load_cols<8>(b2j, p.b2, c0, p.D, b2vec, 0.f);
                    load_cols<8>(sj, p.ls, c0, p.D, lsvec, 1.f);
                    tmem_ld32(tO + lanebase + c0, raw);
                    tmem_wait_ld();
                    if (c0 + 32 >= ce) {
                        tc_fence_before();
                        mbar_arrive(o_empty);  // this thread's last read of O for the tile
                    }
#pragma unroll
                    for (int j = 0; j < 32; j += 2) {
                        float2 v = __fadd2_rn(make_float2(__uint_as_float(raw[j]), __uint_as_float(raw[j + 1])),
                                              make_float2(b2j[j], b2j[j + 1]));
                        if (p.ls) v = __fmul2_rn(v, make_float2(sj[j], sj[j + 1]));
                        raw[j] = __float_as_uint(v.x);
                        raw[j + 1] = __float_as_uint(v.y);
                    }
                    if (lane == 0) bulk_wait_read<0>();
                    __syncwarp();
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        st_shared_v4(swz(st_s, lane, j), raw[4 * j], raw[4 * j + 1], raw[4 * j + 2], raw[4 * j + 3]);
                    fence_async_smem();
                    __syncwarp();
                    if (lane == 0) {
                        tma_reduce_add_3d(&tmX, stage, c0, tile * MB + quad * 32, 0);
                        bulk_commit();
                    }
                }
                // the slice is this warp's part of P for the next tile: its reads must be done
                if (lane == 0) bulk_wait_read<0>();
                __syncwarp();
            }
        }
        if (lane == 0) bulk_wait<0>();
    }
done:
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, 512);
    }
}

PFN_cuTensorMapEncodeTiled_v12000 g_enc_mlp = nullptr;
std::once_flag g_enc_mlp_once;
int g_sms_mlp = 0;

bool encode_ready() {
    std::call_once(g_enc_mlp_once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_enc_mlp = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
    return g_enc_mlp != nullptr;
}

// 2-D f16 map (cols, rows) with a 64 x 128 box, 128-byte swizzle.
bool map_f16(CUtensorMap* m, const void* base, int cols, int rows, int ld) {
    if (!base || ((uintptr_t)base & 15) || (ld % 8)) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    cuuint32_t box[2] = {(cuuint32_t)KB, (cuuint32_t)MB};
    cuuint32_t estr[2] = {1, 1};
    return g_enc_mlp(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 3-D f32 map (cols, rows, 1) with a 32 x 32 box, 128-byte swizzle: the reduce-add target.
bool map_f32_out(CUtensorMap* m, float* base, int cols, int rows, int ld) {
    if (!base || ((uintptr_t)base & 15) || (ld % 4)) return false;
    cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, 1};
    cuuint64_t strides[2] = {(cuuint64_t)ld * 4, (cuuint64_t)ld * 4 * rows};
    cuuint32_t box[3] = {32, 32, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    return g_enc_mlp(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

bool mlp_supported(int D, int F) { return D > 0 && D % HN == 0 && D <= DMAX && F > 0 && F % HN == 0; }

cudaError_t mlp_fused(const MlpArgs& a, cudaStream_t st) {
    if (a.M <= 0) return cudaSuccess;
    if (!mlp_supported(a.D, a.F) || !a.b1 || !a.b2) return cudaErrorInvalidValue;
    if (!encode_ready()) return cudaErrorNotSupported;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    static std::atomic<uint64_t> attr_set{0};
    const uint64_t bit = 1ull << (dev & 63);
    if (!(attr_set.load() & bit)) {
        e = cudaFuncSetAttribute(k_mlp, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
        if (e != cudaSuccess) return e;
        attr_set.fetch_or(bit);
    }
    int sms = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    CUtensorMap mh, m1, m2, mx;
    if (!map_f16(&mh, a.h, a.D, a.M, a.ldh) || !map_f16(&m1, a.w1, a.D, a.F, a.ldw1) ||
        !map_f16(&m2, a.w2, a.F, a.D, a.ldw2) || !map_f32_out(&mx, a.x, a.D, a.M, a.ldx))
        return cudaErrorInvalidValue;
    const int tiles = (a.M + MB - 1) / MB;
    const int grid = tiles < sms ? tiles : sms;
    k_mlp<<<grid, kThreadsMlp, SMEM, st>>>(mh, m1, m2, mx, a);
    return cudaGetLastError();
}

}  // namespace rfb
