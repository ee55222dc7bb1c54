// Fused multi-head attention (flash-style, online softmax) for the windowed /
// global DINOv2 blocks (head_dim 64) and the decoder self-attention
// (head_dim 32).  One CTA = 64 query rows of one (group, head); 4 warps x 16
// rows; key/value tiles of 64 rows double-buffered through shared memory with
// cp.async (zero-filled past the sequence end).  Scores, the running max and
// the running sum stay in f32 registers; P is re-packed to f16 in registers
// as the A operand of P.V.
#include "kernels.cuh"

#include <cuda_fp16.h>
#include <stdint.h>

namespace rfb {

namespace {

constexpr int QT = 64;  // query rows per CTA
constexpr int KT = 64;  // keys per tile

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
    const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
    const int n = valid ? 16 : 0;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
    const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(p));
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(s));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
    const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(p));
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(s));
}

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
}

template <int HD>
__global__ void __launch_bounds__(128)
k_attn(const __half* __restrict__ Q, const __half* __restrict__ K, const __half* __restrict__ V, int ldq, int ldk,
       int ldv, __half* __restrict__ O, int ldo, int L, float scale_log2) {
    constexpr int LDS = HD + 8;  // padded smem row (halves): conflict-free ldmatrix
    constexpr int CH = HD / 8;   // 16-byte chunks per row
    __shared__ __align__(16) __half sQ[QT * LDS];
    __shared__ __align__(16) __half sK[2][KT * LDS];
    __shared__ __align__(16) __half sV[2][KT * LDS];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int q0 = blockIdx.x * QT;
    const int head = blockIdx.y;
    const size_t grow0 = (size_t)blockIdx.z * L;  // first row of this group
    const __half* Qg = Q + head * HD;
    const __half* Kg = K + head * HD;
    const __half* Vg = V + head * HD;

    // Q tile
    for (int c = tid; c < QT * CH; c += 128) {
        const int r = c / CH, ch = c % CH;
        const bool ok = q0 + r < L;
        cp_async16(&sQ[r * LDS + ch * 8], ok ? (const void*)(Qg + (grow0 + q0 + r) * ldq + ch * 8) : (const void*)Q, ok);
    }
    auto load_kv = [&](int buf, int k0) {
        for (int c = tid; c < KT * CH; c += 128) {
            const int r = c / CH, ch = c % CH;
            const bool ok = k0 + r < L;
            cp_async16(&sK[buf][r * LDS + ch * 8], ok ? (const void*)(Kg + (grow0 + k0 + r) * ldk + ch * 8) : (const void*)K, ok);
            cp_async16(&sV[buf][r * LDS + ch * 8], ok ? (const void*)(Vg + (grow0 + k0 + r) * ldv + ch * 8) : (const void*)V, ok);
        }
    };
    load_kv(0, 0);
    cp_commit();

    const int g = lane >> 2, t = lane & 3;
    uint32_t qa[HD / 16][4];
    float o[HD / 8][4];
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

    const int nkt = (L + KT - 1) / KT;
    for (int j = 0; j < nkt; ++j) {
        if (j + 1 < nkt) {
            load_kv((j + 1) & 1, (j + 1) * KT);
            cp_commit();
            cp_wait<1>();
        } else {
            cp_wait<0>();
        }
        __syncthreads();
        if (j == 0) {
#pragma unroll
            for (int ks = 0; ks < HD / 16; ++ks) {
                const int r = warp * 16 + (lane & 15);
                const int cc = ks * 16 + (lane >> 4) * 8;
                ldsm_x4(qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3], &sQ[r * LDS + cc]);
            }
        }
        const __half* kb = sK[j & 1];
        const __half* vb = sV[j & 1];
        // S = Q K^T : 16 x 64 per warp
        float s[KT / 8][4];
#pragma unroll
        for (int n = 0; n < KT / 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
        for (int ks = 0; ks < HD / 16; ++ks) {
#pragma unroll
            for (int np = 0; np < KT / 16; ++np) {
                const int mi = lane >> 3, rr = lane & 7;
                const int key = np * 16 + (mi >> 1) * 8 + rr;
                const int dc = ks * 16 + (mi & 1) * 8;
                uint32_t b0, b1, b2, b3;
                ldsm_x4(b0, b1, b2, b3, &kb[key * LDS + dc]);
                mma16816(s[2 * np], qa[ks], b0, b1);
                mma16816(s[2 * np + 1], qa[ks], b2, b3);
            }
        }
        // scale (log2 domain), mask, row max
        const int kbase = j * KT;
        float mx0 = m0, mx1 = m1;
#pragma unroll
        for (int n = 0; n < KT / 8; ++n) {
            const int key = kbase + n * 8 + 2 * t;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const bool valid = key + (e & 1) < L;
                s[n][e] = valid ? s[n][e] * scale_log2 : -INFINITY;
            }
            mx0 = fmaxf(mx0, fmaxf(s[n][0], s[n][1]));
            mx1 = fmaxf(mx1, fmaxf(s[n][2], s[n][3]));
        }
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffff, mx0, 1));
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffff, mx0, 2));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffff, mx1, 1));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffff, mx1, 2));
        const float c0 = exp2f(m0 - mx0), c1 = exp2f(m1 - mx1);  // m = -inf first time -> 0
        m0 = mx0;
        m1 = mx1;
        float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
        for (int n = 0; n < KT / 8; ++n) {
            s[n][0] = exp2f(s[n][0] - m0);
            s[n][1] = exp2f(s[n][1] - m0);
            s[n][2] = exp2f(s[n][2] - m1);
            s[n][3] = exp2f(s[n][3] - m1);
            rs0 += s[n][0] + s[n][1];
            rs1 += s[n][2] + s[n][3];
        }
        l0 = l0 * c0 + rs0;
        l1 = l1 * c1 + rs1;
#pragma unroll
        for (int i = 0; i < HD / 8; ++i) {
            o[i][0] *= c0;
            o[i][1] *= c0;
            o[i][2] *= c1;
            o[i][3] *= c1;
        }
        // O += P V
#pragma unroll
        for (int ks = 0; ks < KT / 16; ++ks) {
            uint32_t pa[4];
            pa[0] = pack_h2(s[2 * ks][0], s[2 * ks][1]);
            pa[1] = pack_h2(s[2 * ks][2], s[2 * ks][3]);
            pa[2] = pack_h2(s[2 * ks + 1][0], s[2 * ks + 1][1]);
            pa[3] = pack_h2(s[2 * ks + 1][2], s[2 * ks + 1][3]);
#pragma unroll
            for (int dp = 0; dp < HD / 16; ++dp) {
                const int mi = lane >> 3, rr = lane & 7;
                const int key = ks * 16 + (mi & 1) * 8 + rr;
                const int dc = dp * 16 + (mi >> 1) * 8;
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(b0, b1, b2, b3, &vb[key * LDS + dc]);
                mma16816(o[2 * dp], pa, b0, b1);
                mma16816(o[2 * dp + 1], pa, b2, b3);
            }
        }
        __syncthreads();
    }
    // finalize
    l0 += __shfl_xor_sync(0xffffffff, l0, 1);
    l0 += __shfl_xor_sync(0xffffffff, l0, 2);
    l1 += __shfl_xor_sync(0xffffffff, l1, 1);
    l1 += __shfl_xor_sync(0xffffffff, l1, 2);
    const float inv0 = 1.f / l0, inv1 = 1.f / l1;
    const int r0 = q0 + warp * 16 + g, r1 = r0 + 8;
    __half* Og = O + head * HD;
#pragma unroll
    for (int i = 0; i < HD / 8; ++i) {
        const int d = i * 8 + 2 * t;
        if (r0 < L) *reinterpret_cast<uint32_t*>(Og + (grow0 + r0) * ldo + d) = pack_h2(o[i][0] * inv0, o[i][1] * inv0);
        if (r1 < L) *reinterpret_cast<uint32_t*>(Og + (grow0 + r1) * ldo + d) = pack_h2(o[i][2] * inv1, o[i][3] * inv1);
    }
}

}  // namespace

cudaError_t attention(const __half* q, const __half* k, const __half* v, int ldq, int ldk, int ldv, __half* o,
                      int ldo, int seq_len, int groups, int heads, int head_dim, float scale, cudaStream_t st) {
    if (seq_len <= 0 || groups <= 0) return cudaSuccess;
    if ((ldq | ldk | ldv | ldo) & 7) return cudaErrorInvalidValue;
    const dim3 grid((seq_len + QT - 1) / QT, heads, groups);
    const float sl2 = scale * 1.4426950408889634f;
    if (head_dim == 64) {
        k_attn<64><<<grid, 128, 0, st>>>(q, k, v, ldq, ldk, ldv, o, ldo, seq_len, sl2);
    } else if (head_dim == 32) {
        k_attn<32><<<grid, 128, 0, st>>>(q, k, v, ldq, ldk, ldv, o, ldo, seq_len, sl2);
    } else {
        return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

}  // namespace rfb
