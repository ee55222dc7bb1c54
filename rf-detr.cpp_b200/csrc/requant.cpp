// Re-quantization of GGUF weight tensors on the GPU: load-time
// (rfdetr_b200_params.weight_type) and into a new file
// (rfdetr_b200_quantize_gguf, the reference's `rfdetr-cli quantize`).
#include "requant.hpp"

#include "common.hpp"
#include "quant.cuh"
#include "rfdetr_b200.h"

#include <cuda_runtime.h>

#include <cstring>
#include <vector>

namespace rfb {

namespace {

const char* kSkip[] = {"backbone.pos_embed", "decoder.queries.feat", "decoder.queries.refpoints"};

bool ends_with(const std::string& s, const char* suf) {
    const size_t n = std::strlen(suf);
    return s.size() >= n && s.compare(s.size() - n, n, suf) == 0;
}

struct DevBuf {
    void* p = nullptr;
    ~DevBuf() { if (p) cudaFree(p); }
};

}  // namespace

bool should_quantize(const GgufTensor& t) {
    if (!ends_with(t.name, ".weight") || t.n_dims != 2) return false;
    if (t.ne[0] < 64 || t.ne[1] < 64) return false;
    for (const char* s : kSkip)
        if (t.name == s) return false;
    return t.ne[0] % 32 == 0;
}

uint32_t quant_type_for(uint32_t type, const GgufTensor& t) {
    if ((type == GT_Q4_K || type == GT_Q5_K || type == GT_Q6_K) && t.ne[0] % 256) return GT_Q8_0;
    return type;
}

int requantize_model(GgufFile* f, uint32_t type, int device, std::string* err) {
    int be, bb;
    if (!quant_block_shape(type, &be, &bb)) {
        if (err) *err = "unsupported re-quantization type " + std::to_string(type);
        return -1;
    }
    auto converts = [&](const GgufTensor& t) {
        return should_quantize(t) && (t.type == GT_F32 || t.type == GT_F16 || t.type == GT_BF16) &&
               quant_type_for(type, t) != t.type;
    };
    // largest tensor to convert, for one pair of device buffers (none: nothing to do, no GPU needed)
    int64_t max_n = 0;
    for (const auto& t : f->tensors)
        if (converts(t)) max_n = std::max<int64_t>(max_n, t.nelements());
    if (max_n == 0) return 0;
    if (cudaSetDevice(device) != cudaSuccess) {
        cudaGetLastError();
        if (err) *err = "cannot select CUDA device " + std::to_string(device);
        return -8;
    }
    DevBuf d_src, d_dst;
    if (cudaMalloc(&d_src.p, (size_t)max_n * 4) != cudaSuccess || cudaMalloc(&d_dst.p, (size_t)max_n * 2) != cudaSuccess) {
        if (err) *err = "out of device memory for re-quantization";
        return -4;
    }
    std::vector<uint8_t> data;
    data.reserve(f->data.size());
    std::vector<float> tmp;
    std::vector<uint8_t> q;
    const uint64_t al = f->alignment ? f->alignment : 32;
    for (auto& t : f->tensors) {
        const uint8_t* src = f->data.data() + t.offset;
        const uint64_t off = (data.size() + al - 1) / al * al;
        data.resize(off);
        const bool convert = converts(t);
        const uint32_t tt = convert ? quant_type_for(type, t) : t.type;
        if (!convert) {
            data.insert(data.end(), src, src + t.nbytes);
        } else {
            const int64_t n = t.nelements();
            int e2, b2;
            quant_block_shape(tt, &e2, &b2);
            tmp.resize((size_t)n);
            if (!dequantize(t.type, src, n, tmp.data())) {
                if (err) *err = "cannot read tensor " + t.name;
                return -6;
            }
            const size_t qbytes = (size_t)(n / e2) * b2;
            q.resize(qbytes);
            if (cudaMemcpy(d_src.p, tmp.data(), (size_t)n * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
                quantize_device(tt, static_cast<const float*>(d_src.p), n, static_cast<uint8_t*>(d_dst.p), nullptr) !=
                    cudaSuccess ||
                cudaMemcpy(q.data(), d_dst.p, qbytes, cudaMemcpyDeviceToHost) != cudaSuccess) {
                cudaGetLastError();
                if (err) *err = "re-quantization of " + t.name + " failed on the device";
                return -8;
            }
            data.insert(data.end(), q.begin(), q.end());
            t.type = tt;
            t.nbytes = qbytes;
        }
        t.offset = off;
    }
    f->data.swap(data);
    return 0;
}

}  // namespace rfb

static rfdetr_status rfdetr_b200_quantize_gguf_body(const char* in_path, const char* out_path, int type, int device) {
    if (!in_path || !out_path) return RFDETR_ERR_INVALID_ARG;
    rfb::GgufFile f;
    std::string err;
    int rc = rfb::gguf_read(in_path, &f, &err);
    if (rc != 0) {
        rfdetr_logf(RFDETR_LOG_ERROR, "quantize: %s", err.c_str());
        return (rfdetr_status)rc;
    }
    rc = rfb::requantize_model(&f, (uint32_t)type, device, &err);
    if (rc != 0) {
        rfdetr_logf(RFDETR_LOG_ERROR, "quantize: %s", err.c_str());
        return (rfdetr_status)rc;
    }
    rc = rfb::gguf_write(out_path, f, &err);
    if (rc != 0) {
        rfdetr_logf(RFDETR_LOG_ERROR, "quantize: %s", err.c_str());
        return (rfdetr_status)rc;
    }
    return RFDETR_OK;
}

extern "C" rfdetr_status rfdetr_b200_quantize_gguf(const char* in_path, const char* out_path, int type, int device) {
    return rfdetr_c_boundary([&] { return rfdetr_b200_quantize_gguf_body(in_path, out_path, type, device); },
                             RFDETR_ERR_OUT_OF_MEMORY, RFDETR_ERR_IO);
}
