// ConvX (3x3 convolution + channel LayerNorm + optional SiLU) that allocates
// nothing: the im2col scratch lives in a fixed, file-scope device array.
//
// Who needs this: code that must not call cudaMalloc — e.g. a serving loop
// whose latency budget cannot absorb cudaMalloc's implicit device-wide
// synchronization, a host running under another framework's caching
// allocator with a hard memory budget that a raw cudaMalloc would bypass, or
// a plugin that only ever receives device pointers from its host and has no
// allocator of its own.  rfdetr_b200_op_conv3x3 needs a caller workspace of
// batch*h*w*9*c f16 values; this variant needs none.
//
// Limits and sharing: the array holds kMaxColElems f16 values (16 MiB) on
// every GPU that loads the library, for the life of the process.  Every call
// on a device reuses the same array, so two calls whose kernels overlap on
// the GPU (different streams, or different host threads on one device) race;
// calls in one stream are ordered and safe.  Each call's im2col writes every
// scratch element its GEMM reads (zero padding included), so stale contents
// from a previous call never leak into a result.
#include "rfdetr_b200.h"

#include "common.hpp"
#include "gemm.cuh"
#include "kernels.cuh"

#include <cuda_fp16.h>

#include <mutex>

namespace {

constexpr size_t kMaxColElems = (size_t)8 << 20;  // 8 Mi f16 values = 16 MiB
constexpr int kMaxDevices = 64;

__device__ __align__(256) __half g_col_scratch[kMaxColElems];

std::mutex g_mu;
__half* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_col_scratch on the current device.  Host code cannot use
// the symbol itself (it names a host-side shadow, not device memory); the
// address is looked up once per device with that device current.
cudaError_t scratch_address(__half** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_col_scratch);
        if (e != cudaSuccess) {
            rfdetr_logf(RFDETR_LOG_ERROR, "conv3x3 (no-alloc): cudaGetSymbolAddress failed on device %d: %s", dev,
                        cudaGetErrorString(e));
            return e;
        }
        g_scratch_ptr[dev] = static_cast<__half*>(p);
    }
    *out = g_scratch_ptr[dev];
    return cudaSuccess;
}

}  // namespace

extern "C" int rfdetr_b200_op_conv3x3_noalloc(const void* src, int lds, int batch, int h, int w, int c,
                                              const void* weight, int oc, const float* ln_g, const float* ln_b,
                                              float eps, int act, float* out32, int ld32, void* out16, int ld16,
                                              void* stream) {
    if (!src || !weight || batch <= 0 || h <= 0 || w <= 0 || c <= 0) return (int)cudaErrorInvalidValue;
    if ((oc != 128 && oc != 256) || (act != rfb::ACT_NONE && act != rfb::ACT_SILU)) return (int)cudaErrorInvalidValue;
    // the im2col reads src 16 bytes at a time: a misaligned src, or a pixel pitch shorter than the
    // channel count, is refused here, before any address lookup or launch
    if (!rfb::im2col3x3_source_ok(static_cast<const __half*>(src), lds, batch, h, w, c))
        return (int)cudaErrorInvalidValue;
    const size_t need = (size_t)batch * h * w * 9 * c;
    if (need > kMaxColElems) {
        rfdetr_logf(RFDETR_LOG_ERROR,
                    "conv3x3 (no-alloc): batch*h*w*9*c = %zu exceeds the fixed scratch of %zu f16 values "
                    "(at most %zu pixels for c = %d); use rfdetr_b200_op_conv3x3 with a workspace",
                    need, kMaxColElems, kMaxColElems / (9 * (size_t)c), c);
        return (int)cudaErrorInvalidValue;
    }
    __half* col = nullptr;
    cudaError_t e = scratch_address(&col);
    if (e != cudaSuccess) return (int)e;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    e = rfb::im2col3x3(static_cast<const __half*>(src), lds, batch, h, w, c, col, st);
    if (e != cudaSuccess) return (int)e;
    rfb::GemmArgs a;
    a.A = col; a.lda = 9 * c;
    a.B = static_cast<const __half*>(weight); a.ldb = 9 * c;
    a.M = batch * h * w; a.N = oc; a.K = 9 * c;
    a.epi = rfb::EPI_LN; a.act = act;
    a.ln_g = ln_g; a.ln_b = ln_b; a.ln_eps = eps;
    a.out32 = out32; a.ld32 = ld32;
    a.out16 = static_cast<__half*>(out16); a.ld16 = ld16;
    return (int)rfb::gemm(a, st);
}
