// Post-processing on the GPU (src/postprocess.cpp:43-181 of the reference):
// per image, the sigmoid-argmax over classes of every query, the score
// threshold and class filter, a descending sort by score (ties: lower query
// first, the order std::stable_sort gives the host version), top_k, and the
// cxcywh -> clamped pixel xyxy boxes; for segmentation models the selected
// queries' masks are upsampled (bilinear, clamped edges, half-pixel centres)
// to the original image size and thresholded at sigmoid > 0.5, one bit per
// pixel.  The host then only copies back the kept records and bit masks.
#include "select.cuh"

#include <cstdint>

namespace rfb {

namespace {

// The host rule: two branches so that neither exp overflows.
__device__ __forceinline__ float sigmoid_ref(float x) {
    if (x >= 0.f) {
        const float z = expf(-x);
        return 1.f / (1.f + z);
    }
    const float z = expf(x);
    return z / (1.f + z);
}

constexpr int kSelThreads = 1024;  // one thread per query; NQ <= 1024

__global__ void __launch_bounds__(kSelThreads)
k_select(const float* __restrict__ logits, const float* __restrict__ boxes, int NQ, int NC, float threshold,
         int top_k, const uint32_t* __restrict__ filter, int filter_len, int img_w, int img_h,
         DetRecord* __restrict__ out, int* __restrict__ counts) {
    __shared__ unsigned long long key[kSelThreads];
    __shared__ int cls[kSelThreads];
    __shared__ float score[kSelThreads];
    const int b = blockIdx.x, t = threadIdx.x;
    unsigned long long k = ~0ull;
    if (t < NQ) {
        const float* r = logits + ((size_t)b * NQ + t) * NC;
        int bc = 0;
        float bs = -1.f;
        for (int c = 0; c < NC; ++c) {
            const float s = sigmoid_ref(r[c]);
            if (s > bs) {
                bs = s;
                bc = c;
            }
        }
        bool keep = bs > threshold;
        if (keep && filter && filter_len > 0) {
            bool allowed = false;
            for (int i = 0; i < filter_len; ++i) allowed |= filter[i] == (uint32_t)bc;
            keep = allowed;
        }
        cls[t] = bc;
        score[t] = bs;
        // scores are in (0, 1]: their bit patterns order like the values
        if (keep) k = ((unsigned long long)(0xFFFFFFFFu - __float_as_uint(bs)) << 32) | (unsigned)t;
    }
    key[t] = k;
    const int kept = __syncthreads_count(k != ~0ull);
    // bitonic sort, ascending key = descending score, then ascending query
    for (int size = 2; size <= kSelThreads; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            const int partner = t ^ stride;
            if (partner > t) {
                const unsigned long long a = key[t], c = key[partner];
                const bool up = (t & size) == 0;
                if ((a > c) == up) {
                    key[t] = c;
                    key[partner] = a;
                }
            }
            __syncthreads();
        }
    }
    const int n = (top_k > 0 && kept > top_k) ? top_k : kept;
    if (t < n) {
        const int q = (int)(key[t] & 0xFFFFFFFFu);
        const float* bx = boxes + ((size_t)b * NQ + q) * 4;
        const float cx = bx[0], cy = bx[1], bw = bx[2], bh = bx[3];
        const float W = (float)img_w, H = (float)img_h;
        DetRecord d;
        d.query = q;
        d.class_id = cls[q];
        d.score = score[q];
        d.x1 = fminf(fmaxf((cx - 0.5f * bw) * W, 0.f), W);
        d.y1 = fminf(fmaxf((cy - 0.5f * bh) * H, 0.f), H);
        d.x2 = fminf(fmaxf((cx + 0.5f * bw) * W, 0.f), W);
        d.y2 = fminf(fmaxf((cy + 0.5f * bh) * H, 0.f), H);
        d.pad = 0.f;
        out[(size_t)b * NQ + t] = d;
    }
    if (t == 0) counts[b] = n;
}

// One thread = one 32-pixel word of one row of one selected mask.
__global__ void k_mask_bits(const float* __restrict__ masks, int NQ, int side, const DetRecord* __restrict__ dets,
                            const int* __restrict__ counts, int max_dets, int img_w, int img_h, int words,
                            uint32_t* __restrict__ bits) {
    const int b = blockIdx.z, i = blockIdx.y;
    if (i >= counts[b]) return;
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= img_h * words) return;
    const int y = idx / words, wx = idx - y * words;
    const DetRecord d = dets[(size_t)b * NQ + i];
    const float* src = masks + ((size_t)b * NQ + d.query) * side * side;
    const float fx = (float)side / (float)img_w, fy = (float)side / (float)img_h;
    const float sy = ((float)y + 0.5f) * fy - 0.5f;
    int ya = (int)floorf(sy), yb = ya + 1;
    ya = min(max(ya, 0), side - 1);
    yb = min(max(yb, 0), side - 1);
    const float ay = fminf(fmaxf(sy - (float)ya, 0.f), 1.f);
    const float* r0 = src + (size_t)ya * side;
    const float* r1 = src + (size_t)yb * side;
    uint32_t w = 0;
    for (int j = 0; j < 32; ++j) {
        const int x = wx * 32 + j;
        if (x >= img_w) break;
        const float sx = ((float)x + 0.5f) * fx - 0.5f;
        int xa = (int)floorf(sx), xb = xa + 1;
        xa = min(max(xa, 0), side - 1);
        xb = min(max(xb, 0), side - 1);
        const float ax = fminf(fmaxf(sx - (float)xa, 0.f), 1.f);
        const float v = r0[xa] * (1 - ax) * (1 - ay) + r0[xb] * ax * (1 - ay) + r1[xa] * (1 - ax) * ay +
                        r1[xb] * ax * ay;
        if (sigmoid_ref(v) > 0.5f) w |= 1u << j;
    }
    bits[(((size_t)b * max_dets + i) * img_h + y) * words + wx] = w;
}

}  // namespace

cudaError_t select_detections_device(const float* logits, const float* boxes, int B, int NQ, int NC,
                                     float threshold, int top_k, const uint32_t* filter, int filter_len, int img_w,
                                     int img_h, DetRecord* out, int* counts, cudaStream_t st) {
    if (B <= 0) return cudaSuccess;
    if (NQ <= 0 || NQ > kSelThreads || NC <= 0 || img_w <= 0 || img_h <= 0 || !logits || !boxes || !out || !counts)
        return cudaErrorInvalidValue;
    k_select<<<B, kSelThreads, 0, st>>>(logits, boxes, NQ, NC, threshold, top_k, filter, filter_len, img_w, img_h,
                                        out, counts);
    return cudaGetLastError();
}

size_t mask_bits_words(int img_w, int img_h) { return (size_t)img_h * ((img_w + 31) / 32); }

cudaError_t mask_bits_device(const float* masks, int B, int NQ, int side, const DetRecord* dets, const int* counts,
                             int max_dets, int img_w, int img_h, uint32_t* bits, cudaStream_t st) {
    if (B <= 0 || max_dets <= 0) return cudaSuccess;
    if (!masks || !dets || !counts || !bits || side <= 0 || img_w <= 0 || img_h <= 0 || max_dets > NQ)
        return cudaErrorInvalidValue;
    const int words = (img_w + 31) / 32;
    const long long per = (long long)img_h * words;
    const dim3 grid((unsigned)((per + 255) / 256), (unsigned)max_dets, (unsigned)B);
    k_mask_bits<<<grid, 256, 0, st>>>(masks, NQ, side, dets, counts, max_dets, img_w, img_h, words, bits);
    return cudaGetLastError();
}

}  // namespace rfb
