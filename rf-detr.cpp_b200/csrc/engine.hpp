// The CUDA inference engine: one model's weights resident on one GPU, a
// persistent activation arena sized for a maximum batch, and the forward pass
// as a fixed sequence of kernel launches on one stream (capturable into a CUDA
// graph).  Replaces the reference's ggml graphs A/B + host top-K
// (src/rfdetr_model.cpp:77-451) for a batch of images.
#pragma once

#include "model.hpp"
#include "resize_legacy.hpp"

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <memory>
#include <string>
#include <utility>
#include <vector>

namespace rfb {

struct DLin {
    const __half* w = nullptr;  // [N][ldw] f16
    const float* b = nullptr;   // [N] f32 (may be null)
    int N = 0, K = 0, ldw = 0;
};
struct DNorm {
    const float* g = nullptr;
    const float* b = nullptr;
};

class Engine {
public:
    // Builds the engine on `device`; logs and returns nullptr on failure.
    static std::unique_ptr<Engine> create(const Model& m, int device, int max_batch, rfdetr_status* st);
    ~Engine();

    const Config& cfg() const { return cfg_; }
    int device() const { return device_; }
    cudaStream_t stream() const { return stream_; }
    int max_batch() const { return max_batch_; }
    int grid() const { return G_; }
    int mask_side() const { return Hm_; }

    // Grow the activation arena to hold `batch` images.
    rfdetr_status reserve(int batch);

    // Device-side input staging buffers (valid for max_batch images).
    uint8_t* d_rgb() { return rgb_u8_; }        // [B][src_h][src_w][3], capacity rgb_cap_ bytes
    size_t rgb_capacity() const { return rgb_cap_; }
    rfdetr_status reserve_rgb(size_t bytes);
    float* d_planar() { return img_; }          // [B][3][S][S]

    // Enqueue the forward pass on the engine stream.  If `d_src_rgb` is set
    // (device pointer, batch x src_h x src_w x 3 uint8) it is preprocessed
    // first; otherwise d_planar() holds the already-normalized input.
    // Asynchronous; call finish() to synchronize.
    // The launch sequence is captured into a CUDA graph the first time a
    // (batch, input pointer, input size) combination is seen and replayed
    // afterwards (RFDETR_NO_GRAPH=1 disables this; profiling forwards always
    // launch kernels individually).
    rfdetr_status enqueue(int batch, const uint8_t* d_src_rgb, int src_w, int src_h);
    // Synchronize the stream and check the device error word.
    rfdetr_status finish();
    // The same check in two halves, for callers that queue more work behind
    // the forward before they synchronize: enqueue_error_copy() copies the
    // device error word to `h_err` (pinned host memory) on the engine stream;
    // after the synchronization, device_error(*h_err) logs and clears a
    // nonzero word and reports it as RFDETR_ERR_INFERENCE.
    rfdetr_status enqueue_error_copy(int* h_err);
    rfdetr_status device_error(int err);

    // Outputs of the last forward (device pointers).
    const float* logits() const { return logits_; }   // [B*NQ][NC]
    const float* boxes() const { return boxes_; }     // [B*NQ][4] cxcywh
    const float* masks() const { return masks_; }     // [B][NQ][Hm*Hm] (seg only)

    // Copy a named intermediate of the last forward to host as f32 (debug and
    // parity tests).  Returns element count, or -1 for an unknown name.
    long long trace(const std::string& name, int batch, float* out, size_t cap);

    // Number of kernels one forward launches (for the benchmark record).
    int kernels_per_forward() const { return launches_; }

    // Per-launch timing: when enabled, the next forwards record a CUDA event
    // after every launch on the engine stream; profile() returns
    // (name, milliseconds) of each launch of the last forward (after finish()).
    void set_profiling(bool on) { profiling_ = on; }
    std::vector<std::pair<std::string, float>> profile();

private:
    Engine() = default;
    rfdetr_status enqueue_raw(int batch, const uint8_t* d_src_rgb, int src_w, int src_h);
    void drop_graphs();
    struct GraphEntry {
        int batch;
        const uint8_t* src;
        int w, h;
        cudaGraphExec_t exec;
    };
    std::vector<GraphEntry> graphs_;
    bool use_graphs_ = true;
    // Legacy preprocess resize (resize_mode legacy_stb): taps per source size,
    // uploaded outside any graph capture and kept for the engine's lifetime;
    // the resized batch goes through rsz_ [max_batch][S][S][3].
    struct LegacyEntry {
        int w, h;
        LegacyTapsDev taps;
    };
    std::vector<LegacyEntry> legacy_;
    bool legacy_resize(int w, int h) const { return !cfg_.bilinear_no_antialias && (w != S_ || h != S_); }
    rfdetr_status prepare_legacy(int w, int h);
    const LegacyTapsDev* legacy_taps(int w, int h) const;
    rfdetr_status upload_weights(const Model& m);
    rfdetr_status alloc_activations(int batch);
    void free_activations();

    Config cfg_;
    int device_ = 0;
    cudaStream_t stream_ = nullptr;
    int max_batch_ = 0;
    int launches_ = 0;
    bool profiling_ = false;
    std::vector<cudaEvent_t> prof_ev_;
    std::vector<std::string> prof_names_;
    int prof_used_ = 0;

    // dims
    int S_ = 0, P_ = 0, G_ = 0, nw_ = 0, ws_ = 0, Tp_ = 0, T_ = 0, NW_ = 0, Ntok_ = 0;
    int D_ = 0, H_ = 0, F_ = 0, L_ = 0, Kpatch_ = 0, Kpad_ = 0;
    int Dm_ = 0, NQ_ = 0, NC_ = 0, Fd_ = 0, Cb_ = 0, Hm_ = 0;
    int n_soaw_ = 0;

    // weights
    std::vector<void*> wallocs_;
    DLin patch_;
    float* posw_ = nullptr;    // [Ntok][D] windowed pos-embed (CLS rows included)
    float* clsrow_ = nullptr;  // [D] cls + pos[0]
    struct Block {
        DNorm ln1, ln2;
        DLin qkv, proj, fc1, fc2;
        const float* ls1 = nullptr;
        const float* ls2 = nullptr;
        bool global = false;
        int tap = -1;
    };
    std::vector<Block> blocks_;
    DNorm bbnorm_;
    DLin cv1_, cv2_;
    DNorm cv1n_, cv2n_, fnorm_;
    struct Bneck {
        DLin c1, c2;
        DNorm n1, n2;
    };
    std::vector<Bneck> bnecks_;
    DLin enc_, cls_, tb0_, tb1_, tb2_;
    DNorm encn_;
    const float* lrn_rp_ = nullptr;
    const float* feat_ = nullptr;
    DLin rph0_, rph1_;
    struct DecLayer {
        DLin qk, v, out, soaw, value, oproj, l1, l2;
        DNorm n1, n2, n3;
    };
    std::vector<DecLayer> dec_;
    DNorm dnorm_;
    DLin hcls_, hb0_, hb1_, hb2_;
    struct SegBlock {
        const float* dw_w = nullptr;
        const float* dw_b = nullptr;
        DNorm n;
        DLin pw;
    };
    std::vector<SegBlock> segb_;
    DLin sfp_, ql0_, ql2_, qfp_;
    DNorm qfn_;
    const float* segbias_ = nullptr;  // [Hm*Hm] broadcast of the scalar bias

    // activations
    void* arena_ = nullptr;
    int* d_err_ = nullptr;
    uint8_t* rgb_u8_ = nullptr;
    size_t rgb_cap_ = 0;
    uint8_t* rsz_ = nullptr;
    float* img_ = nullptr;
    __half* apatch_ = nullptr;
    float* x_ = nullptr;
    __half* h16_ = nullptr;
    __half* qkv_ = nullptr;
    __half* attn_ = nullptr;
    __half* f1_ = nullptr;
    __half* taps_ = nullptr;
    __half* cat_ = nullptr;
    __half* tmp128_ = nullptr;
    float* splitws_ = nullptr;  // split-K partial sums of the LayerNorm GEMMs with few row blocks
    float* p32a_ = nullptr;
    float* proj32_ = nullptr;
    __half* mem16_ = nullptr;
    __half* memm16_ = nullptr;
    __half* y16_ = nullptr;
    float* clsall_ = nullptr;
    __half* hb1_16_ = nullptr;
    __half* hb2_16_ = nullptr;
    float* tsdelta_ = nullptr;
    float* bboxall_ = nullptr;
    int32_t* topk_ = nullptr;
    float* refp_ = nullptr;
    __half* sine_ = nullptr;
    __half* q16a_ = nullptr;
    float* qpos_ = nullptr;
    float* tgt_ = nullptr;
    __half* tgt16_ = nullptr;
    __half* qk16_ = nullptr;
    __half* qkp_ = nullptr;
    __half* vp_ = nullptr;
    __half* sa16_ = nullptr;
    __half* value_ = nullptr;
    float* soaw_ = nullptr;
    __half* samp_ = nullptr;
    __half* ffn_ = nullptr;
    float* dec32_ = nullptr;
    __half* dec16_ = nullptr;
    float* logits_ = nullptr;
    __half* hh1_ = nullptr;
    __half* hh2_ = nullptr;
    float* bdelta_ = nullptr;
    float* boxes_ = nullptr;
    float* sp32_ = nullptr;
    __half* sln16_ = nullptr;
    __half* spp16_ = nullptr;
    __half* qn16_ = nullptr;
    __half* qh16_ = nullptr;
    float* qf32_ = nullptr;
    __half* qf16_ = nullptr;
    __half* qfp16_ = nullptr;
    float* masks_ = nullptr;
};

}  // namespace rfb
