// Public C ABI: rfdetr.h (context lifecycle, detect, accessors),
// rfdetr_capi.h (flat handle API used by LocalAI) and rfdetr_b200.h (batched /
// device entry points).  Semantics follow the reference's src/rfdetr.cpp and
// src/rfdetr_capi.cpp: status codes, ownership, "clear the previous batch on
// every detect call", two-call sizing.
#include "rfdetr.h"
#include "rfdetr_b200.h"
#include "rfdetr_capi.h"

#include "common.hpp"
#include "engine.hpp"
#include "image_io.hpp"
#include "model.hpp"
#include "postprocess.hpp"
#include "requant.hpp"
#include "select.cuh"

#include <algorithm>
#include <atomic>
#include <deque>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <new>
#include <sstream>
#include <string>
#include <thread>
#include <vector>

struct rfdetr_context {
    std::unique_ptr<rfb::Model> model;
    std::unique_ptr<rfb::Engine> engine;
    size_t n_tensors = 0;
    int n_threads = 1;
    // pinned host staging
    uint8_t* h_in = nullptr;
    size_t h_in_cap = 0;
    float* h_out = nullptr;
    size_t h_out_cap = 0;
    // device post-process: records, counts, class filter and bit masks on the
    // device; pinned host copies of what comes back
    rfdetr_b200_det* d_dets = nullptr;
    int* d_counts = nullptr;
    uint32_t* d_filter = nullptr;
    uint32_t* d_bits = nullptr;
    size_t dets_cap = 0, counts_cap = 0, filter_cap = 0, bits_cap = 0;
    rfdetr_b200_det* h_dets = nullptr;
    int* h_counts = nullptr;
    uint32_t* h_bits = nullptr;
    size_t h_dets_cap = 0, h_counts_cap = 0, h_bits_cap = 0;
    int* h_err = nullptr;  // the forward's device error word, copied back with the detections
    size_t h_err_cap = 0;
    // pipelined submissions (rfdetr_b200_submit_rgb): two device input slots
    // filled on a copy stream; the forward runs on the engine stream behind
    // slot_ready, and slot_free marks the slot's last reader
    cudaStream_t copy_stream = nullptr;
    uint8_t* d_slot[2] = {nullptr, nullptr};
    size_t slot_cap[2] = {0, 0};
    cudaEvent_t slot_ready[2] = {nullptr, nullptr};
    cudaEvent_t slot_free[2] = {nullptr, nullptr};
    int next_slot = 0;
    // outputs of submission slot k: copied on the device into d_out[k] behind the
    // forward (out_ready), then to the caller on d2h_stream (out_free), so the
    // next forward does not wait for the PCIe transfer
    cudaStream_t d2h_stream = nullptr;
    uint8_t* d_out[2] = {nullptr, nullptr};
    size_t out_cap[2] = {0, 0};
    cudaEvent_t out_ready[2] = {nullptr, nullptr};
    cudaEvent_t out_free[2] = {nullptr, nullptr};
    // one event per outstanding submission (after its output copies), oldest first; spare events
    std::deque<cudaEvent_t> inflight;
    std::vector<cudaEvent_t> spare_events;

    ~rfdetr_context() {
        if (h_in) cudaFreeHost(h_in);
        if (h_out) cudaFreeHost(h_out);
        if (h_dets) cudaFreeHost(h_dets);
        if (h_counts) cudaFreeHost(h_counts);
        if (h_bits) cudaFreeHost(h_bits);
        if (h_err) cudaFreeHost(h_err);
        if (engine) cudaSetDevice(engine->device());
        if (copy_stream) cudaStreamSynchronize(copy_stream);
        if (engine) cudaStreamSynchronize(engine->stream());
        if (d2h_stream) cudaStreamSynchronize(d2h_stream);
        for (cudaEvent_t ev : inflight) cudaEventDestroy(ev);
        for (cudaEvent_t ev : spare_events) cudaEventDestroy(ev);
        for (int k = 0; k < 2; ++k) {
            if (d_slot[k]) cudaFree(d_slot[k]);
            if (slot_ready[k]) cudaEventDestroy(slot_ready[k]);
            if (slot_free[k]) cudaEventDestroy(slot_free[k]);
            if (d_out[k]) cudaFree(d_out[k]);
            if (out_ready[k]) cudaEventDestroy(out_ready[k]);
            if (out_free[k]) cudaEventDestroy(out_free[k]);
        }
        if (copy_stream) cudaStreamDestroy(copy_stream);
        if (d2h_stream) cudaStreamDestroy(d2h_stream);
        if (d_dets) cudaFree(d_dets);
        if (d_counts) cudaFree(d_counts);
        if (d_filter) cudaFree(d_filter);
        if (d_bits) cudaFree(d_bits);
    }
    // grow-only buffers (elements of T); false on allocation failure
    template <typename T>
    static bool grow_dev(T** p, size_t* cap, size_t n) {
        if (n <= *cap) return true;
        if (*p) cudaFree(*p);
        *p = nullptr;
        *cap = 0;
        if (cudaMalloc(reinterpret_cast<void**>(p), n * sizeof(T)) != cudaSuccess) return false;
        *cap = n;
        return true;
    }
    template <typename T>
    static bool grow_host(T** p, size_t* cap, size_t n) {
        if (n <= *cap) return true;
        if (*p) cudaFreeHost(*p);
        *p = nullptr;
        *cap = 0;
        if (cudaMallocHost(reinterpret_cast<void**>(p), n * sizeof(T)) != cudaSuccess) return false;
        *cap = n;
        return true;
    }
    bool stage_in(size_t bytes) {
        if (bytes <= h_in_cap) return true;
        if (h_in) cudaFreeHost(h_in);
        h_in = nullptr;
        h_in_cap = 0;
        if (cudaMallocHost(&h_in, bytes) != cudaSuccess) return false;
        h_in_cap = bytes;
        return true;
    }
    bool stage_out(size_t floats) {
        if (floats <= h_out_cap) return true;
        if (h_out) cudaFreeHost(h_out);
        h_out = nullptr;
        h_out_cap = 0;
        if (cudaMallocHost(&h_out, floats * 4) != cudaSuccess) return false;
        h_out_cap = floats;
        return true;
    }
};

namespace {

int resolve_threads(int n) {
    if (n > 0) return n;
    const unsigned hc = std::thread::hardware_concurrency();
    return hc ? (int)hc : 1;
}

rfdetr_context* init_impl(const rfdetr_params* params, int device, int max_batch, rfdetr_status* out_status,
                          int weight_type = 0) {
    auto set = [&](rfdetr_status s) { if (out_status) *out_status = s; };
    if (!params || !params->model_path) { set(RFDETR_ERR_INVALID_ARG); return nullptr; }
    if (params->log_cb) rfdetr_set_log_callback(params->log_cb, params->log_user_data);
    rfdetr_status st;
    std::unique_ptr<rfb::Model> m(rfb::model_load(params->model_path, &st));
    if (!m) { set(st); return nullptr; }
    st = rfb::model_validate(*m);
    if (st != RFDETR_OK) { set(st); return nullptr; }
    if (weight_type != 0) {
        std::string err;
        const int rc = rfb::requantize_model(&m->file, (uint32_t)weight_type, device, &err);
        if (rc != 0) {
            rfdetr_logf(RFDETR_LOG_ERROR, "rfdetr_init: re-quantization failed: %s", err.c_str());
            set((rfdetr_status)rc);
            return nullptr;
        }
    }
    auto eng = rfb::Engine::create(*m, device, max_batch, &st);
    if (!eng) { set(st); return nullptr; }
    auto* ctx = new (std::nothrow) rfdetr_context();
    if (!ctx) { set(RFDETR_ERR_OUT_OF_MEMORY); return nullptr; }
    ctx->n_tensors = m->file.tensors.size();
    m->file.data.clear();          // weights now live on the GPU
    m->file.data.shrink_to_fit();
    ctx->model = std::move(m);
    ctx->engine = std::move(eng);
    ctx->n_threads = resolve_threads(params->n_threads);
    const rfb::Config& c = ctx->model->cfg;
    rfdetr_logf(RFDETR_LOG_INFO, "rfdetr_init: loaded variant=%s, num_classes=%u, num_queries=%u, device=%d",
                c.variant.c_str(), c.num_classes, c.num_queries, device);
    set(RFDETR_OK);
    return ctx;
}

// Copy the last forward's outputs for `batch` images to host buffers.
// Enqueue the device-to-host copies of the outputs on the engine stream.
rfdetr_status enqueue_output_copies(rfdetr_context* ctx, int batch, float* logits, float* boxes, float* masks) {
    rfb::Engine& e = *ctx->engine;
    const rfb::Config& c = e.cfg();
    const size_t nq = c.num_queries, nc = c.num_classes;
    cudaStream_t st = e.stream();
    if (logits && RFB_CUDA_FAIL(cudaMemcpyAsync(logits, e.logits(), (size_t)batch * nq * nc * 4,
                                                cudaMemcpyDeviceToHost, st)))
        return RFDETR_ERR_INFERENCE;
    if (boxes && RFB_CUDA_FAIL(cudaMemcpyAsync(boxes, e.boxes(), (size_t)batch * nq * 4 * 4, cudaMemcpyDeviceToHost, st)))
        return RFDETR_ERR_INFERENCE;
    if (masks && c.has_seg) {
        const size_t hw = (size_t)e.mask_side() * e.mask_side();
        if (RFB_CUDA_FAIL(cudaMemcpyAsync(masks, e.masks(), (size_t)batch * nq * hw * 4, cudaMemcpyDeviceToHost, st)))
            return RFDETR_ERR_INFERENCE;
    }
    return RFDETR_OK;
}

rfdetr_status fetch_outputs(rfdetr_context* ctx, int batch, float* logits, float* boxes, float* masks) {
    rfdetr_status s = enqueue_output_copies(ctx, batch, logits, boxes, masks);
    if (s != RFDETR_OK) return s;
    return RFB_CUDA_FAIL(cudaStreamSynchronize(ctx->engine->stream())) ? RFDETR_ERR_INFERENCE : RFDETR_OK;
}

// Run the forward for `batch` same-sized RGB images already packed at h_rgb.
rfdetr_status forward_rgb_impl(rfdetr_context* ctx, const uint8_t* h_rgb, int batch, int w, int h) {
    rfb::Engine& e = *ctx->engine;
    const size_t bytes = (size_t)batch * w * h * 3;
    rfdetr_status s = e.reserve(batch);
    if (s != RFDETR_OK) return s;
    s = e.reserve_rgb(bytes);
    if (s != RFDETR_OK) return s;
    if (RFB_CUDA_FAIL(cudaMemcpyAsync(e.d_rgb(), h_rgb, bytes, cudaMemcpyHostToDevice, e.stream())))
        return RFDETR_ERR_INFERENCE;
    s = e.enqueue(batch, e.d_rgb(), w, h);
    if (s != RFDETR_OK) return s;
    return e.finish();
}

// Release the detection arrays of out_dets[0..n) and clear them (error paths:
// a failed call hands back no arrays).
void release_results(rfdetr_detection** out_dets, size_t* out_counts, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        rfdetr_detections_free(out_dets[i], out_counts[i]);
        out_dets[i] = nullptr;
        out_counts[i] = 0;
    }
}

// An image whose pixel buffer holds exactly width x height RGB triples.
bool image_ok(const rfdetr_image* img) {
    return img && img->width > 0 && img->height > 0 &&
           img->rgb.size() == (size_t)img->width * (size_t)img->height * 3;
}

// Upload n images of img_bytes each to the engine's device input buffer, back to
// back, through the pinned staging buffer in chunks: the host copy of a chunk
// overlaps the DMA of the one before it.
rfdetr_status upload_images(rfdetr_context* ctx, const rfdetr_image* const* imgs, size_t n, size_t img_bytes) {
    rfb::Engine& e = *ctx->engine;
    const size_t total = img_bytes * n;
    if (RFB_CUDA_FAIL(cudaSetDevice(e.device()))) return RFDETR_ERR_INFERENCE;
    if (!ctx->stage_in(total)) return RFDETR_ERR_OUT_OF_MEMORY;
    const rfdetr_status s = e.reserve_rgb(total);
    if (s != RFDETR_OK) return s;
    constexpr size_t kChunk = 256u << 10;
    for (size_t i = 0; i < n; ++i) {
        const uint8_t* src = imgs[i]->rgb.data();
        for (size_t off = 0; off < img_bytes; off += kChunk) {
            const size_t len = std::min(kChunk, img_bytes - off), at = i * img_bytes + off;
            std::memcpy(ctx->h_in + at, src + off, len);
            if (RFB_CUDA_FAIL(cudaMemcpyAsync(e.d_rgb() + at, ctx->h_in + at, len, cudaMemcpyHostToDevice,
                                              e.stream())))
                return RFDETR_ERR_INFERENCE;
        }
    }
    return RFDETR_OK;
}

// Host-side fault injection for the error-path tests: RFDETR_FAULT_INJECT=postprocess_alloc:N
// makes the N-th post-processing call of the process (counting from 1) throw std::bad_alloc once
// its first detection array has been handed out, as an allocation failure there would.
bool inject_postprocess_fault() {
    static std::atomic<long> calls{0};
    const char* env = std::getenv("RFDETR_FAULT_INJECT");
    if (!env || std::strncmp(env, "postprocess_alloc:", 18) != 0) return false;
    return calls.fetch_add(1) + 1 == std::atol(env + 18);
}

void attach_names(const rfdetr_context* ctx, rfdetr_detection* d, size_t n) {
    const auto& names = ctx->model->cfg.class_names;
    for (size_t i = 0; i < n; ++i)
        if (d[i].class_id < names.size()) d[i].class_name = names[d[i].class_id].c_str();
}

// 0/255 byte masks from the device's bit masks: each byte of a mask word
// becomes 8 output bytes through a 256-entry table of 8-byte patterns.
struct MaskExpand {
    uint64_t lut[256];
    MaskExpand() {
        for (int b = 0; b < 256; ++b) {
            uint64_t v = 0;
            for (int k = 0; k < 8; ++k)
                if (b >> k & 1) v |= 0xFFull << (8 * k);
            lut[b] = v;
        }
    }
    void run(const uint32_t* bits, int w, int h, uint8_t* out) const {
        const size_t wpr = (size_t)(w + 31) / 32;
        for (int y = 0; y < h; ++y) {
            const uint32_t* row = bits + y * wpr;
            uint8_t* o = out + (size_t)y * w;
            int x = 0;
            for (; x + 8 <= w; x += 8) {
                const uint64_t v = lut[(row[x >> 5] >> (x & 31)) & 0xFF];
                std::memcpy(o + x, &v, 8);
            }
            for (; x < w; ++x) o[x] = (row[x >> 5] >> (x & 31)) & 1u ? 255 : 0;
        }
    }
};
const MaskExpand g_mask_expand;

// Post-process the forward of `batch` images of w x h pixels queued last on
// the engine stream, on the device (select.cu), and build the per-image
// rfdetr_detection arrays: only the selected records and their bit masks cross
// PCIe; the 0/255 masks of the reference API are expanded from the bits on the
// host.  The forward's device error word comes back with the records, so the
// forward and the selection share one synchronization; a nonzero word fails
// the call before any array is built.
rfdetr_status postprocess_device(rfdetr_context* ctx, int batch, int w, int h, const rfdetr_detect_params* params,
                                 rfdetr_detection** out_dets, size_t* out_counts) {
    rfb::Engine& e = *ctx->engine;
    const rfb::Config& c = ctx->model->cfg;
    const int nq = (int)c.num_queries, nc = (int)c.num_classes;
    const bool seg = c.has_seg && e.masks() != nullptr;
    const int ms = e.mask_side();
    const int max_dets = params->top_k > 0 && (int)params->top_k < nq ? (int)params->top_k : nq;
    const size_t words = rfb::mask_bits_words(w, h);
    const size_t flen = params->class_filter ? params->class_filter_len : 0;
    if (RFB_CUDA_FAIL(cudaSetDevice(e.device()))) return RFDETR_ERR_INFERENCE;
    if (!rfdetr_context::grow_dev(&ctx->d_dets, &ctx->dets_cap, (size_t)batch * nq) ||
        !rfdetr_context::grow_dev(&ctx->d_counts, &ctx->counts_cap, (size_t)batch) ||
        (flen && !rfdetr_context::grow_dev(&ctx->d_filter, &ctx->filter_cap, flen)) ||
        (seg && !rfdetr_context::grow_dev(&ctx->d_bits, &ctx->bits_cap, (size_t)batch * max_dets * words)) ||
        !rfdetr_context::grow_host(&ctx->h_dets, &ctx->h_dets_cap, (size_t)batch * nq) ||
        !rfdetr_context::grow_host(&ctx->h_counts, &ctx->h_counts_cap, (size_t)batch) ||
        !rfdetr_context::grow_host(&ctx->h_err, &ctx->h_err_cap, 1))
        return RFDETR_ERR_OUT_OF_MEMORY;
    const cudaStream_t st = e.stream();
    *ctx->h_err = 0;
    if (e.enqueue_error_copy(ctx->h_err) != RFDETR_OK) return RFDETR_ERR_INFERENCE;
    if (flen && RFB_CUDA_FAIL(cudaMemcpyAsync(ctx->d_filter, params->class_filter, flen * 4, cudaMemcpyHostToDevice, st)))
        return RFDETR_ERR_INFERENCE;
    if (RFB_CUDA_FAIL(rfb::select_detections_device(e.logits(), e.boxes(), batch, nq, nc, params->threshold,
                                                    (int)params->top_k, flen ? ctx->d_filter : nullptr, (int)flen, w,
                                                    h, ctx->d_dets, ctx->d_counts, st)))
        return RFDETR_ERR_INFERENCE;
    if (seg && RFB_CUDA_FAIL(rfb::mask_bits_device(e.masks(), batch, nq, ms, ctx->d_dets, ctx->d_counts, max_dets, w,
                                                   h, ctx->d_bits, st)))
        return RFDETR_ERR_INFERENCE;
    if (RFB_CUDA_FAIL(cudaMemcpyAsync(ctx->h_counts, ctx->d_counts, (size_t)batch * sizeof(int), cudaMemcpyDeviceToHost,
                                      st)) ||
        RFB_CUDA_FAIL(cudaMemcpyAsync(ctx->h_dets, ctx->d_dets, (size_t)batch * nq * sizeof(rfdetr_b200_det),
                                      cudaMemcpyDeviceToHost, st)) ||
        RFB_CUDA_FAIL(cudaStreamSynchronize(st)))
        return RFDETR_ERR_INFERENCE;
    if (e.device_error(*ctx->h_err) != RFDETR_OK) return RFDETR_ERR_INFERENCE;
    size_t kept = 0;
    for (int b = 0; b < batch; ++b) kept += (size_t)ctx->h_counts[b];
    if (seg && kept) {
        if (!rfdetr_context::grow_host(&ctx->h_bits, &ctx->h_bits_cap, kept * words)) return RFDETR_ERR_OUT_OF_MEMORY;
        size_t off = 0;
        for (int b = 0; b < batch; ++b) {
            const size_t n = (size_t)ctx->h_counts[b] * words;
            if (n && RFB_CUDA_FAIL(cudaMemcpyAsync(ctx->h_bits + off, ctx->d_bits + (size_t)b * max_dets * words,
                                                   n * 4, cudaMemcpyDeviceToHost, st)))
                return RFDETR_ERR_INFERENCE;
            off += n;
        }
        if (RFB_CUDA_FAIL(cudaStreamSynchronize(st))) return RFDETR_ERR_INFERENCE;
    }
    // masks to expand: (destination, bits) pairs, filled while building the records.  Every
    // allocation that can throw happens before the first array is built, and each array is
    // handed to out_dets as soon as it exists, so a failure leaves nothing unowned.
    for (int b = 0; b < batch; ++b) {
        out_dets[b] = nullptr;
        out_counts[b] = 0;
    }
    std::vector<std::pair<uint8_t*, const uint32_t*>> jobs;
    if (seg) jobs.reserve(kept);
    const bool fault = inject_postprocess_fault();
    size_t off = 0;
    for (int b = 0; b < batch; ++b) {
        const int n = ctx->h_counts[b];
        if (n <= 0) continue;
        auto* d = static_cast<rfdetr_detection*>(std::calloc((size_t)n, sizeof(rfdetr_detection)));
        if (!d) {
            release_results(out_dets, out_counts, (size_t)b);
            return RFDETR_ERR_OUT_OF_MEMORY;
        }
        out_dets[b] = d;
        out_counts[b] = (size_t)n;
        for (int i = 0; i < n; ++i) {
            const rfdetr_b200_det& r = ctx->h_dets[(size_t)b * nq + i];
            d[i].class_id = (uint32_t)r.class_id;
            d[i].score = r.score;
            d[i].x1 = r.x1; d[i].y1 = r.y1; d[i].x2 = r.x2; d[i].y2 = r.y2;
            if (seg) {
                auto* m = static_cast<uint8_t*>(std::malloc((size_t)w * h));
                if (m) jobs.emplace_back(m, ctx->h_bits + off + (size_t)i * words);
                d[i].mask = m;
                d[i].mask_width = m ? w : 0;
                d[i].mask_height = m ? h : 0;
            }
        }
        off += (size_t)n * words;
        attach_names(ctx, d, (size_t)n);
        if (fault) throw std::bad_alloc();
    }
    // expand the masks, over the context's host threads when there is enough of it
    const size_t pixels = jobs.size() * (size_t)w * h;
    const int nt = (int)std::min<size_t>((size_t)ctx->n_threads, std::max<size_t>(1, pixels / (1u << 20)));
    auto work = [&](int t) {
        for (size_t j = (size_t)t; j < jobs.size(); j += (size_t)nt) g_mask_expand.run(jobs[j].second, w, h, jobs[j].first);
    };
    // workers 1 .. started-1 run on their own threads; if a thread cannot be created, the
    // shares of the workers that did not start run here (the started ones are still joined)
    std::vector<std::thread> pool;
    int started = 1;
    try {
        if (nt > 1) pool.reserve((size_t)nt - 1);
        for (int t = 1; t < nt; ++t) {
            pool.emplace_back(work, t);
            ++started;
        }
    } catch (const std::exception&) {
        rfdetr_logf(RFDETR_LOG_WARN, "mask expansion: %d of %d host threads started", started, nt);
    }
    work(0);
    for (int t = started; t < nt; ++t) work(t);
    for (auto& th : pool) th.join();
    return RFDETR_OK;
}

}  // namespace

// ============================================================================
// rfdetr.h
// ============================================================================

static rfdetr_context* rfdetr_init_body(const rfdetr_params* params, rfdetr_status* out_status) {
    int device = 0;
    if (const char* d = std::getenv("RFDETR_DEVICE")) device = std::atoi(d);
    return init_impl(params, device, 1, out_status);
}

extern "C" rfdetr_context* rfdetr_init(const rfdetr_params* params, rfdetr_status* out_status) {
    return rfdetr_c_boundary_ptr<rfdetr_context>([&] { return rfdetr_init_body(params, out_status); },
                                                 out_status, RFDETR_ERR_MODEL_LOAD);
}

extern "C" void rfdetr_free(rfdetr_context* ctx) { delete ctx; }

extern "C" const char* rfdetr_context_variant(const rfdetr_context* c) {
    return (c && c->model) ? c->model->cfg.variant.c_str() : "";
}
extern "C" uint32_t rfdetr_context_image_size(const rfdetr_context* c) { return (c && c->model) ? c->model->cfg.image_size : 0; }
extern "C" uint32_t rfdetr_context_num_queries(const rfdetr_context* c) { return (c && c->model) ? c->model->cfg.num_queries : 0; }
extern "C" uint32_t rfdetr_context_num_classes(const rfdetr_context* c) { return (c && c->model) ? c->model->cfg.num_classes : 0; }
extern "C" size_t rfdetr_context_n_tensors(const rfdetr_context* c) { return (c && c->model) ? c->n_tensors : 0; }

static rfdetr_status rfdetr_detect_body(rfdetr_context* ctx, const rfdetr_image* img,
                                        const rfdetr_detect_params* params, rfdetr_detection** out_detections,
                                        size_t* out_n) {
    if (out_detections) *out_detections = nullptr;
    if (out_n) *out_n = 0;
    if (!ctx || !img || !params || !out_detections || !out_n) return RFDETR_ERR_INVALID_ARG;
    if (!ctx->engine || !image_ok(img)) return RFDETR_ERR_INVALID_ARG;
    rfb::Engine& e = *ctx->engine;
    rfdetr_status s = e.reserve(1);
    if (s == RFDETR_OK) s = upload_images(ctx, &img, 1, img->rgb.size());
    if (s == RFDETR_OK) s = e.enqueue(1, e.d_rgb(), img->width, img->height);
    if (s == RFDETR_OK) {
        try {
            s = postprocess_device(ctx, 1, img->width, img->height, params, out_detections, out_n);
        } catch (...) {
            release_results(out_detections, out_n, 1);  // a failed call hands back no array
            throw;
        }
    }
    if (s != RFDETR_OK) {
        rfdetr_logf(RFDETR_LOG_ERROR, "rfdetr_detect: inference failed");
        return s == RFDETR_ERR_OUT_OF_MEMORY ? s : RFDETR_ERR_INFERENCE;
    }
    return RFDETR_OK;
}

extern "C" rfdetr_status rfdetr_detect(rfdetr_context* ctx, const rfdetr_image* img,
                                       const rfdetr_detect_params* params, rfdetr_detection** out_detections,
                                       size_t* out_n) {
    return rfdetr_c_boundary([&] { return rfdetr_detect_body(ctx, img, params, out_detections, out_n); },
                             RFDETR_ERR_OUT_OF_MEMORY, RFDETR_ERR_INFERENCE);
}

// ============================================================================
// rfdetr_b200.h
// ============================================================================

static rfdetr_context* rfdetr_b200_init_body(const rfdetr_params* params, const rfdetr_b200_params* b,
                                             rfdetr_status* out_status) {
    return init_impl(params, b ? b->device : 0, b && b->max_batch > 0 ? b->max_batch : 1, out_status,
                     b ? b->weight_type : 0);
}

extern "C" rfdetr_context* rfdetr_b200_init(const rfdetr_params* params, const rfdetr_b200_params* b,
                                            rfdetr_status* out_status) {
    return rfdetr_c_boundary_ptr<rfdetr_context>([&] { return rfdetr_b200_init_body(params, b, out_status); },
                                                 out_status, RFDETR_ERR_MODEL_LOAD);
}

static rfdetr_status rfdetr_b200_forward_rgb_body(rfdetr_context* ctx, const uint8_t* rgb, int batch, int width,
                                                  int height, float* out_logits, float* out_boxes, float* out_masks) {
    if (!ctx || !ctx->engine || !rgb || batch <= 0 || width <= 0 || height <= 0) return RFDETR_ERR_INVALID_ARG;
    rfdetr_status s = forward_rgb_impl(ctx, rgb, batch, width, height);
    if (s != RFDETR_OK) return s;
    return fetch_outputs(ctx, batch, out_logits, out_boxes, out_masks);
}

extern "C" rfdetr_status rfdetr_b200_forward_rgb(rfdetr_context* ctx, const uint8_t* rgb, int batch, int width,
                                                 int height, float* out_logits, float* out_boxes, float* out_masks) {
    return rfdetr_c_boundary(
        [&] { return rfdetr_b200_forward_rgb_body(ctx, rgb, batch, width, height, out_logits, out_boxes, out_masks); },
        RFDETR_ERR_OUT_OF_MEMORY, RFDETR_ERR_INFERENCE);
}

static rfdetr_status rfdetr_b200_submit_rgb_body(rfdetr_context* ctx, const uint8_t* rgb, int batch, int width,
                                                 int height, float* out_logits, float* out_boxes, float* out_masks) {
    if (!ctx || !ctx->engine || !rgb || batch <= 0 || width <= 0 || height <= 0) return RFDETR_ERR_INVALID_ARG;
    rfb::Engine& e = *ctx->engine;
    if (RFB_CUDA_FAIL(cudaSetDevice(e.device()))) return RFDETR_ERR_INFERENCE;
    rfdetr_status s = e.reserve(batch);  // synchronizes the engine stream before growing
    if (s != RFDETR_OK) return s;
    if (!ctx->copy_stream) {
        if (RFB_CUDA_FAIL(cudaStreamCreateWithFlags(&ctx->copy_stream, cudaStreamNonBlocking)) ||
            RFB_CUDA_FAIL(cudaStreamCreateWithFlags(&ctx->d2h_stream, cudaStreamNonBlocking)))
            return RFDETR_ERR_INFERENCE;
        for (int k = 0; k < 2; ++k)
            if (RFB_CUDA_FAIL(cudaEventCreateWithFlags(&ctx->slot_ready[k], cudaEventDisableTiming)) ||
                RFB_CUDA_FAIL(cudaEventCreateWithFlags(&ctx->slot_free[k], cudaEventDisableTiming)) ||
                RFB_CUDA_FAIL(cudaEventCreateWithFlags(&ctx->out_ready[k], cudaEventDisableTiming)) ||
                RFB_CUDA_FAIL(cudaEventCreateWithFlags(&ctx->out_free[k], cudaEventDisableTiming)))
                return RFDETR_ERR_INFERENCE;
    }
    const int k = ctx->next_slot;
    ctx->next_slot ^= 1;
    const size_t bytes = (size_t)batch * width * height * 3;
    if (bytes > ctx->slot_cap[k]) {
        // the slot's last reader must be done before it is replaced
        if (RFB_CUDA_FAIL(cudaEventSynchronize(ctx->slot_free[k]))) return RFDETR_ERR_INFERENCE;
        if (ctx->d_slot[k]) cudaFree(ctx->d_slot[k]);
        ctx->d_slot[k] = nullptr;
        ctx->slot_cap[k] = 0;
        if (RFB_CUDA_FAIL(cudaMalloc(&ctx->d_slot[k], bytes))) return RFDETR_ERR_OUT_OF_MEMORY;
        ctx->slot_cap[k] = bytes;
    }
    // upload behind the slot's previous reader, the forward behind the upload
    if (RFB_CUDA_FAIL(cudaStreamWaitEvent(ctx->copy_stream, ctx->slot_free[k], 0)) ||
        RFB_CUDA_FAIL(cudaMemcpyAsync(ctx->d_slot[k], rgb, bytes, cudaMemcpyHostToDevice, ctx->copy_stream)) ||
        RFB_CUDA_FAIL(cudaEventRecord(ctx->slot_ready[k], ctx->copy_stream)) ||
        RFB_CUDA_FAIL(cudaStreamWaitEvent(e.stream(), ctx->slot_ready[k], 0)))
        return RFDETR_ERR_INFERENCE;
    s = e.enqueue(batch, ctx->d_slot[k], width, height);
    if (s != RFDETR_OK) return s;
    if (RFB_CUDA_FAIL(cudaEventRecord(ctx->slot_free[k], e.stream()))) return RFDETR_ERR_INFERENCE;
    // outputs: device copy into output slot k behind the forward (once the slot's previous
    // transfer is done), then the transfer to the caller on d2h_stream
    const rfb::Config& c = e.cfg();
    const size_t nq = c.num_queries, nc = c.num_classes, hw = (size_t)e.mask_side() * e.mask_side();
    const size_t lb = out_logits ? (size_t)batch * nq * nc * 4 : 0, bb = out_boxes ? (size_t)batch * nq * 16 : 0;
    const size_t mb = out_masks && c.has_seg ? (size_t)batch * nq * hw * 4 : 0;
    if (lb + bb + mb > ctx->out_cap[k]) {
        if (RFB_CUDA_FAIL(cudaEventSynchronize(ctx->out_free[k]))) return RFDETR_ERR_INFERENCE;
        if (ctx->d_out[k]) cudaFree(ctx->d_out[k]);
        ctx->d_out[k] = nullptr;
        ctx->out_cap[k] = 0;
        if (RFB_CUDA_FAIL(cudaMalloc(&ctx->d_out[k], lb + bb + mb))) return RFDETR_ERR_OUT_OF_MEMORY;
        ctx->out_cap[k] = lb + bb + mb;
    }
    uint8_t* o = ctx->d_out[k];
    const cudaStream_t es = e.stream(), ds = ctx->d2h_stream;
    if (RFB_CUDA_FAIL(cudaStreamWaitEvent(es, ctx->out_free[k], 0)) ||
        (lb && RFB_CUDA_FAIL(cudaMemcpyAsync(o, e.logits(), lb, cudaMemcpyDeviceToDevice, es))) ||
        (bb && RFB_CUDA_FAIL(cudaMemcpyAsync(o + lb, e.boxes(), bb, cudaMemcpyDeviceToDevice, es))) ||
        (mb && RFB_CUDA_FAIL(cudaMemcpyAsync(o + lb + bb, e.masks(), mb, cudaMemcpyDeviceToDevice, es))) ||
        RFB_CUDA_FAIL(cudaEventRecord(ctx->out_ready[k], es)) || RFB_CUDA_FAIL(cudaStreamWaitEvent(ds, ctx->out_ready[k], 0)) ||
        (lb && RFB_CUDA_FAIL(cudaMemcpyAsync(out_logits, o, lb, cudaMemcpyDeviceToHost, ds))) ||
        (bb && RFB_CUDA_FAIL(cudaMemcpyAsync(out_boxes, o + lb, bb, cudaMemcpyDeviceToHost, ds))) ||
        (mb && RFB_CUDA_FAIL(cudaMemcpyAsync(out_masks, o + lb + bb, mb, cudaMemcpyDeviceToHost, ds))) ||
        RFB_CUDA_FAIL(cudaEventRecord(ctx->out_free[k], ds)))
        return RFDETR_ERR_INFERENCE;
    cudaEvent_t done = nullptr;
    if (!ctx->spare_events.empty()) {
        done = ctx->spare_events.back();
        ctx->spare_events.pop_back();
    } else if (RFB_CUDA_FAIL(cudaEventCreateWithFlags(&done, cudaEventDisableTiming))) {
        return RFDETR_ERR_INFERENCE;
    }
    if (RFB_CUDA_FAIL(cudaEventRecord(done, ds))) {
        ctx->spare_events.push_back(done);
        return RFDETR_ERR_INFERENCE;
    }
    try {
        ctx->inflight.push_back(done);
    } catch (...) {
        // not tracked: rfdetr_b200_wait still covers the submission (it synchronizes the streams)
        cudaEventDestroy(done);
        throw;
    }
    return RFDETR_OK;
}

extern "C" rfdetr_status rfdetr_b200_submit_rgb(rfdetr_context* ctx, const uint8_t* rgb, int batch, int width,
                                                int height, float* out_logits, float* out_boxes, float* out_masks) {
    return rfdetr_c_boundary(
        [&] { return rfdetr_b200_submit_rgb_body(ctx, rgb, batch, width, height, out_logits, out_boxes, out_masks); },
        RFDETR_ERR_OUT_OF_MEMORY, RFDETR_ERR_INFERENCE);
}

static rfdetr_status rfdetr_b200_wait_oldest_body(rfdetr_context* ctx) {
    if (!ctx || !ctx->engine) return RFDETR_ERR_INVALID_ARG;
    if (ctx->inflight.empty()) return RFDETR_OK;
    if (RFB_CUDA_FAIL(cudaSetDevice(ctx->engine->device()))) return RFDETR_ERR_INFERENCE;
    cudaEvent_t ev = ctx->inflight.front();
    // moved to the spares before it leaves the in-flight list, so a failing push leaves it owned
    ctx->spare_events.push_back(ev);
    ctx->inflight.pop_front();
    return RFB_CUDA_FAIL(cudaEventSynchronize(ev)) ? RFDETR_ERR_INFERENCE : RFDETR_OK;
}

extern "C" rfdetr_status rfdetr_b200_wait_oldest(rfdetr_context* ctx) {
    return rfdetr_c_boundary([&] { return rfdetr_b200_wait_oldest_body(ctx); },
                             RFDETR_ERR_OUT_OF_MEMORY, RFDETR_ERR_INFERENCE);
}

static rfdetr_status rfdetr_b200_wait_body(rfdetr_context* ctx) {
    if (!ctx || !ctx->engine) return RFDETR_ERR_INVALID_ARG;
    while (!ctx->inflight.empty()) {  // finished by the synchronizations below
        ctx->spare_events.push_back(ctx->inflight.front());
        ctx->inflight.pop_front();
    }
    if (ctx->copy_stream) {
        if (RFB_CUDA_FAIL(cudaSetDevice(ctx->engine->device())) ||
            RFB_CUDA_FAIL(cudaStreamSynchronize(ctx->copy_stream)) ||
            RFB_CUDA_FAIL(cudaStreamSynchronize(ctx->d2h_stream)))
            return RFDETR_ERR_INFERENCE;
    }
    return ctx->engine->finish();
}

extern "C" rfdetr_status rfdetr_b200_wait(rfdetr_context* ctx) {
    return rfdetr_c_boundary([&] { return rfdetr_b200_wait_body(ctx); },
                             RFDETR_ERR_OUT_OF_MEMORY, RFDETR_ERR_INFERENCE);
}

static rfdetr_status rfdetr_b200_forward_planar_body(rfdetr_context* ctx, const float* planar, int batch,
                                                     float* out_logits, float* out_boxes, float* out_masks) {
    if (!ctx || !ctx->engine || !planar || batch <= 0) return RFDETR_ERR_INVALID_ARG;
    rfb::Engine& e = *ctx->engine;
    rfdetr_status s = e.reserve(batch);
    if (s != RFDETR_OK) return s;
    const size_t S = e.cfg().image_size;
    if (RFB_CUDA_FAIL(cudaMemcpyAsync(e.d_planar(), planar, (size_t)batch * 3 * S * S * 4, cudaMemcpyHostToDevice,
                                      e.stream())))
        return RFDETR_ERR_INFERENCE;
    s = e.enqueue(batch, nullptr, 0, 0);
    if (s == RFDETR_OK) s = e.finish();
    if (s != RFDETR_OK) return s;
    return fetch_outputs(ctx, batch, out_logits, out_boxes, out_masks);
}

extern "C" rfdetr_status rfdetr_b200_forward_planar(rfdetr_context* ctx, const float* planar, int batch,
                                                    float* out_logits, float* out_boxes, float* out_masks) {
    return rfdetr_c_boundary(
        [&] { return rfdetr_b200_forward_planar_body(ctx, planar, batch, out_logits, out_boxes, out_masks); },
        RFDETR_ERR_OUT_OF_MEMORY, RFDETR_ERR_INFERENCE);
}

static rfdetr_status rfdetr_b200_enqueue_device_body(rfdetr_context* ctx, const uint8_t* d_rgb, int batch, int width,
                                                     int height) {
    if (!ctx || !ctx->engine || !d_rgb || batch <= 0 || width <= 0 || height <= 0) return RFDETR_ERR_INVALID_ARG;
    rfb::Engine& e = *ctx->engine;
    rfdetr_status s = e.reserve(batch);
    if (s != RFDETR_OK) return s;
    return e.enqueue(batch, d_rgb, width, height);
}

extern "C" rfdetr_status rfdetr_b200_enqueue_device(rfdetr_context* ctx, const uint8_t* d_rgb, int batch, int width,
                                                    int height) {
    return rfdetr_c_boundary([&] { return rfdetr_b200_enqueue_device_body(ctx, d_rgb, batch, width, height); },
                             RFDETR_ERR_OUT_OF_MEMORY, RFDETR_ERR_INFERENCE);
}

static rfdetr_status rfdetr_b200_sync_body(rfdetr_context* ctx) {
    if (!ctx || !ctx->engine) return RFDETR_ERR_INVALID_ARG;
    return ctx->engine->finish();
}

extern "C" rfdetr_status rfdetr_b200_sync(rfdetr_context* ctx) {
    return rfdetr_c_boundary([&] { return rfdetr_b200_sync_body(ctx); },
                             RFDETR_ERR_OUT_OF_MEMORY, RFDETR_ERR_INFERENCE);
}

extern "C" rfdetr_status rfdetr_b200_device_outputs(rfdetr_context* ctx, const float** l, const float** b,
                                                    const float** m) {
    if (!ctx || !ctx->engine) return RFDETR_ERR_INVALID_ARG;
    if (l) *l = ctx->engine->logits();
    if (b) *b = ctx->engine->boxes();
    if (m) *m = ctx->model->cfg.has_seg ? ctx->engine->masks() : nullptr;
    return RFDETR_OK;
}

static rfdetr_status rfdetr_b200_detect_batch_body(rfdetr_context* ctx, const rfdetr_image* const* imgs, size_t n,
                                                   const rfdetr_detect_params* params, rfdetr_detection** out_dets,
                                                   size_t* out_counts) {
    if (!ctx || !ctx->engine || !imgs || !params || !out_dets || !out_counts) return RFDETR_ERR_INVALID_ARG;
    for (size_t i = 0; i < n; ++i) { out_dets[i] = nullptr; out_counts[i] = 0; }
    if (n == 0) return RFDETR_OK;
    for (size_t i = 0; i < n; ++i)
        if (!image_ok(imgs[i])) return RFDETR_ERR_INVALID_ARG;
    // Same-sized runs go through one batched forward; the preprocess kernel
    // resizes each run to the model resolution on the GPU.  A failure releases
    // the arrays of the runs before it.
    size_t i = 0;
    while (i < n) {
        const int w = imgs[i]->width, h = imgs[i]->height;
        size_t j = i + 1;
        while (j < n && imgs[j]->width == w && imgs[j]->height == h) ++j;
        const int batch = (int)(j - i);
        rfb::Engine& e = *ctx->engine;
        rfdetr_status s = e.reserve(batch);
        if (s == RFDETR_OK) s = upload_images(ctx, imgs + i, (size_t)batch, (size_t)w * h * 3);
        if (s == RFDETR_OK) s = e.enqueue(batch, e.d_rgb(), w, h);
        if (s == RFDETR_OK) {
            try {
                s = postprocess_device(ctx, batch, w, h, params, out_dets + i, out_counts + i);
            } catch (...) {
                release_results(out_dets, out_counts, j);  // this run's arrays and those before it
                throw;
            }
        }
        if (s != RFDETR_OK && s != RFDETR_ERR_OUT_OF_MEMORY) s = RFDETR_ERR_INFERENCE;
        if (s != RFDETR_OK) {
            release_results(out_dets, out_counts, i);
            return s;
        }
        i = j;
    }
    return RFDETR_OK;
}

extern "C" rfdetr_status rfdetr_b200_detect_batch(rfdetr_context* ctx, const rfdetr_image* const* imgs, size_t n,
                                                  const rfdetr_detect_params* params, rfdetr_detection** out_dets,
                                                  size_t* out_counts) {
    return rfdetr_c_boundary(
        [&] { return rfdetr_b200_detect_batch_body(ctx, imgs, n, params, out_dets, out_counts); },
        RFDETR_ERR_OUT_OF_MEMORY, RFDETR_ERR_INFERENCE);
}

extern "C" int rfdetr_b200_device(const rfdetr_context* c) { return (c && c->engine) ? c->engine->device() : -1; }
extern "C" int rfdetr_b200_mask_side(const rfdetr_context* c) { return (c && c->engine) ? c->engine->mask_side() : 0; }
extern "C" int rfdetr_b200_kernels_per_forward(const rfdetr_context* c) {
    return (c && c->engine) ? c->engine->kernels_per_forward() : 0;
}
extern "C" void* rfdetr_b200_stream(const rfdetr_context* c) { return (c && c->engine) ? (void*)c->engine->stream() : nullptr; }

static long long rfdetr_b200_trace_body(rfdetr_context* ctx, const char* name, int batch, float* out, size_t cap) {
    if (!ctx || !ctx->engine || !name || !out || batch <= 0 || batch > ctx->engine->max_batch()) return -1;
    return ctx->engine->trace(name, batch, out, cap);
}

extern "C" long long rfdetr_b200_trace(rfdetr_context* ctx, const char* name, int batch, float* out, size_t cap) {
    return rfdetr_c_boundary([&] { return rfdetr_b200_trace_body(ctx, name, batch, out, cap); }, -1LL, -1LL);
}

extern "C" void rfdetr_b200_profile_enable(rfdetr_context* ctx, int on) {
    if (ctx && ctx->engine) ctx->engine->set_profiling(on != 0);
}

static int rfdetr_b200_profile_read_body(rfdetr_context* ctx, char* names, int name_len, float* ms, int cap) {
    if (!ctx || !ctx->engine) return -1;
    const auto prof = ctx->engine->profile();
    for (int i = 0; i < (int)prof.size() && i < cap; ++i) {
        if (names && name_len > 0) {
            std::strncpy(names + (size_t)i * name_len, prof[i].first.c_str(), (size_t)name_len - 1);
            names[(size_t)i * name_len + name_len - 1] = '\0';
        }
        if (ms) ms[i] = prof[i].second;
    }
    return (int)prof.size();
}

extern "C" int rfdetr_b200_profile_read(rfdetr_context* ctx, char* names, int name_len, float* ms, int cap) {
    return rfdetr_c_boundary([&] { return rfdetr_b200_profile_read_body(ctx, names, name_len, ms, cap); }, -1, -1);
}

static rfdetr_status rfdetr_b200_inspect_body(const char* path, rfdetr_b200_model_info* out) {
    if (!path || !out) return RFDETR_ERR_INVALID_ARG;
    rfdetr_status st;
    std::unique_ptr<rfb::Model> m(rfb::model_load(path, &st));
    if (!m) return st;
    st = rfb::model_validate(*m);
    if (st != RFDETR_OK) return st;
    st = rfb::engine_supports(m->cfg);
    const rfb::Config& c = m->cfg;
    std::memset(out, 0, sizeof(*out));
    out->image_size = c.image_size;
    out->patch_size = c.patch_size;
    out->num_queries = c.num_queries;
    out->num_classes = c.num_classes;
    out->dim = c.backbone.dim;
    out->depth = c.backbone.depth;
    out->num_windows = c.backbone.num_windows;
    out->dec_layers = c.decoder.layers;
    out->has_segmentation_head = c.has_seg ? 1 : 0;
    out->n_tensors = m->file.tensors.size();
    std::strncpy(out->variant, c.variant.c_str(), sizeof(out->variant) - 1);
    out->legacy_resize = c.bilinear_no_antialias ? 0 : 1;
    return st;
}

extern "C" rfdetr_status rfdetr_b200_inspect(const char* path, rfdetr_b200_model_info* out) {
    return rfdetr_c_boundary([&] { return rfdetr_b200_inspect_body(path, out); },
                             RFDETR_ERR_OUT_OF_MEMORY, RFDETR_ERR_MODEL_FORMAT);
}

extern "C" int rfdetr_b200_dequantize(uint32_t type, const void* src, long long n, float* dst) {
    if (!src || !dst || n < 0) return -1;
    return rfb::dequantize(type, src, n, dst) ? 0 : -1;
}

// ============================================================================
// rfdetr_capi.h
// ============================================================================

namespace {

struct CapiHandle {
    rfdetr_context* ctx = nullptr;
    struct Det {
        int class_id = 0;
        std::string class_name;
        float score = 0.f, x1 = 0, y1 = 0, x2 = 0, y2 = 0;
        std::vector<uint8_t> mask_png;
    };
    std::vector<Det> last;
    std::string last_json;
};

std::string make_json(int w, int h, const char* status, const rfdetr_detection* d, size_t n) {
    std::ostringstream o;
    o << "{\"status\":\"" << status << "\",\"image\":{\"width\":" << w << ",\"height\":" << h << "},\"detections\":[";
    for (size_t i = 0; i < n; ++i) {
        if (i) o << ",";
        o << "{\"class_id\":" << d[i].class_id << ",\"score\":" << d[i].score << ",\"x1\":" << d[i].x1
          << ",\"y1\":" << d[i].y1 << ",\"x2\":" << d[i].x2 << ",\"y2\":" << d[i].y2 << "}";
    }
    o << "]}";
    return o.str();
}

char* dup_c(const std::string& s) {
    char* b = static_cast<char*>(std::malloc(s.size() + 1));
    if (!b) return nullptr;
    std::memcpy(b, s.data(), s.size());
    b[s.size()] = '\0';
    return b;
}

int detect_common(rfdetr_handle_t handle, rfdetr_image* img, float threshold, uint32_t top_k, char** out_json) {
    auto* h = reinterpret_cast<CapiHandle*>(handle);
    if (!h || !h->ctx || !img || !out_json) return -1;
    *out_json = nullptr;
    h->last.clear();
    h->last_json.clear();
    rfdetr_detect_params dp{};
    dp.threshold = threshold;
    dp.top_k = top_k;
    rfdetr_detection* dets = nullptr;
    size_t n = 0;
    const rfdetr_status st = rfdetr_detect(h->ctx, img, &dp, &dets, &n);
    const char* status = st == RFDETR_OK ? "ok" : (st == RFDETR_ERR_NOT_IMPLEMENTED ? "not_implemented" : rfdetr_status_str(st));
    if (st == RFDETR_OK && dets) {
        h->last.reserve(n);
        for (size_t i = 0; i < n; ++i) {
            CapiHandle::Det s;
            s.class_id = (int)dets[i].class_id;
            s.class_name = dets[i].class_name ? dets[i].class_name : "";
            s.score = dets[i].score;
            s.x1 = dets[i].x1; s.y1 = dets[i].y1; s.x2 = dets[i].x2; s.y2 = dets[i].y2;
            if (dets[i].mask && dets[i].mask_width > 0 && dets[i].mask_height > 0)
                rfdetr_encode_png(dets[i].mask, dets[i].mask_width, dets[i].mask_height, 1, s.mask_png);
            h->last.push_back(std::move(s));
        }
    }
    std::string json = make_json(rfdetr_image_width(img), rfdetr_image_height(img), status, dets, n);
    rfdetr_detections_free(dets, n);
    h->last_json = json;
    *out_json = dup_c(json);
    if (!*out_json) return (int)RFDETR_ERR_OUT_OF_MEMORY;
    return 0;
}

}  // namespace

static int rfdetr_capi_load_body(const char* model_path, int n_threads, rfdetr_handle_t* out_handle) {
    if (!model_path || !out_handle) return -1;
    *out_handle = 0;
    rfdetr_params p{};
    p.model_path = model_path;
    p.n_threads = n_threads > 0 ? n_threads : 1;
    rfdetr_status st;
    rfdetr_context* ctx = rfdetr_init(&p, &st);
    if (!ctx) return (int)st;
    auto* h = new (std::nothrow) CapiHandle();
    if (!h) {
        rfdetr_free(ctx);
        return (int)RFDETR_ERR_OUT_OF_MEMORY;
    }
    h->ctx = ctx;
    *out_handle = reinterpret_cast<rfdetr_handle_t>(h);
    return 0;
}

extern "C" int rfdetr_capi_load(const char* model_path, int n_threads, rfdetr_handle_t* out_handle) {
    return rfdetr_c_boundary([&] { return rfdetr_capi_load_body(model_path, n_threads, out_handle); },
                             (int)RFDETR_ERR_OUT_OF_MEMORY, (int)RFDETR_ERR_MODEL_LOAD);
}

extern "C" int rfdetr_capi_unload(rfdetr_handle_t handle) {
    if (handle == 0) return 0;
    auto* h = reinterpret_cast<CapiHandle*>(handle);
    if (h->ctx) rfdetr_free(h->ctx);
    delete h;
    return 0;
}

static int rfdetr_capi_detect_path_body(rfdetr_handle_t handle, const char* path, float threshold, uint32_t top_k,
                                        char** out_json) {
    if (!handle || !path || !out_json) return -1;
    *out_json = nullptr;
    auto* h = reinterpret_cast<CapiHandle*>(handle);
    h->last.clear();
    h->last_json.clear();
    rfdetr_status st;
    rfdetr_image* img = rfdetr_image_load_file(path, &st);
    if (!img) return (int)st;
    const int rc = detect_common(handle, img, threshold, top_k, out_json);
    rfdetr_image_free(img);
    return rc;
}

extern "C" int rfdetr_capi_detect_path(rfdetr_handle_t handle, const char* path, float threshold, uint32_t top_k,
                                       char** out_json) {
    return rfdetr_c_boundary([&] { return rfdetr_capi_detect_path_body(handle, path, threshold, top_k, out_json); },
                             (int)RFDETR_ERR_OUT_OF_MEMORY, (int)RFDETR_ERR_INFERENCE);
}

static int rfdetr_capi_detect_buffer_body(rfdetr_handle_t handle, const uint8_t* bytes, size_t len, float threshold,
                                          uint32_t top_k, char** out_json) {
    if (!handle || !bytes || len == 0 || !out_json) return -1;
    *out_json = nullptr;
    auto* h = reinterpret_cast<CapiHandle*>(handle);
    h->last.clear();
    h->last_json.clear();
    rfdetr_status st;
    rfdetr_image* img = rfdetr_image_load_buffer(bytes, len, &st);
    if (!img) return (int)st;
    const int rc = detect_common(handle, img, threshold, top_k, out_json);
    rfdetr_image_free(img);
    return rc;
}

extern "C" int rfdetr_capi_detect_buffer(rfdetr_handle_t handle, const uint8_t* bytes, size_t len, float threshold,
                                         uint32_t top_k, char** out_json) {
    return rfdetr_c_boundary(
        [&] { return rfdetr_capi_detect_buffer_body(handle, bytes, len, threshold, top_k, out_json); },
        (int)RFDETR_ERR_OUT_OF_MEMORY, (int)RFDETR_ERR_INFERENCE);
}

extern "C" void rfdetr_capi_free_string(char* s) { std::free(s); }

extern "C" int rfdetr_capi_get_n_detections(rfdetr_handle_t handle) {
    auto* h = reinterpret_cast<CapiHandle*>(handle);
    return h ? (int)h->last.size() : -1;
}

extern "C" int rfdetr_capi_get_detection_class_id(rfdetr_handle_t handle, int i) {
    auto* h = reinterpret_cast<CapiHandle*>(handle);
    if (!h || i < 0 || (size_t)i >= h->last.size()) return -1;
    return h->last[i].class_id;
}

extern "C" int rfdetr_capi_get_detection_box(rfdetr_handle_t handle, int i, float out_xyxy[4]) {
    auto* h = reinterpret_cast<CapiHandle*>(handle);
    if (!h || i < 0 || (size_t)i >= h->last.size() || !out_xyxy) return -1;
    const auto& d = h->last[i];
    out_xyxy[0] = d.x1; out_xyxy[1] = d.y1; out_xyxy[2] = d.x2; out_xyxy[3] = d.y2;
    return 0;
}

extern "C" float rfdetr_capi_get_detection_score(rfdetr_handle_t handle, int i) {
    auto* h = reinterpret_cast<CapiHandle*>(handle);
    if (!h || i < 0 || (size_t)i >= h->last.size()) return -1.0f;
    return h->last[i].score;
}

extern "C" int rfdetr_capi_get_detection_class_name(rfdetr_handle_t handle, int i, char* buf, int buf_size) {
    auto* h = reinterpret_cast<CapiHandle*>(handle);
    if (!h || i < 0 || (size_t)i >= h->last.size()) return -1;
    const std::string& s = h->last[i].class_name;
    const int need = (int)s.size() + 1;
    if (!buf || buf_size < need) return need;
    std::memcpy(buf, s.data(), s.size());
    buf[s.size()] = '\0';
    return need;
}

extern "C" int rfdetr_capi_get_detection_mask_png(rfdetr_handle_t handle, int i, unsigned char* buf, int buf_size) {
    auto* h = reinterpret_cast<CapiHandle*>(handle);
    if (!h || i < 0 || (size_t)i >= h->last.size()) return -1;
    const auto& mp = h->last[i].mask_png;
    if (mp.empty()) return 0;
    const int need = (int)mp.size();
    if (!buf || buf_size < need) return need;
    std::memcpy(buf, mp.data(), (size_t)need);
    return need;
}
