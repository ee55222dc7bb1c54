// Engine: weight residency + forward orchestration.  The stage order and the
// arithmetic follow the reference forward (src/rfdetr_model.cpp:77-451) with
// its two ggml graphs and host top-K replaced by one stream of sm_100a
// kernels over a whole batch.
#include "engine.hpp"

#include "common.hpp"
#include "gemm.cuh"
#include "kernels.cuh"
#include "sm100.cuh"

#include <cmath>
#include <cstdlib>
#include <cstring>


namespace rfb {

// Scratch for the split-K partial sums of LayerNorm GEMMs with few row blocks.
constexpr size_t kSplitWsBytes = (size_t)8 << 20;

namespace {

uint16_t f2h_bits(float f) {
    const __half h = __float2half_rn(f);
    uint16_t u;
    std::memcpy(&u, &h, 2);
    return u;
}

}  // namespace

Engine::~Engine() {
    if (device_ >= 0) cudaSetDevice(device_);
    drop_graphs();
    free_activations();
    if (rgb_u8_) cudaFree(rgb_u8_);
    for (auto& l : legacy_) cudaFree(l.taps.base);
    for (void* p : wallocs_) cudaFree(p);
    if (d_err_) cudaFree(d_err_);
    for (cudaEvent_t e : prof_ev_) cudaEventDestroy(e);
    if (stream_) cudaStreamDestroy(stream_);
}

std::unique_ptr<Engine> Engine::create(const Model& m, int device, int max_batch, rfdetr_status* st) {
    auto set = [&](rfdetr_status s) { if (st) *st = s; };
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev <= 0) {
        rfdetr_logf(RFDETR_LOG_ERROR, "CUDA engine: no CUDA device available");
        set(RFDETR_ERR_INFERENCE);
        return nullptr;
    }
    if (device < 0 || device >= ndev) {
        rfdetr_logf(RFDETR_LOG_ERROR, "CUDA engine: device %d out of range (%d devices)", device, ndev);
        set(RFDETR_ERR_INVALID_ARG);
        return nullptr;
    }
    if (RFB_CUDA_FAIL(cudaSetDevice(device))) { set(RFDETR_ERR_INFERENCE); return nullptr; }
    cudaDeviceProp prop;
    if (RFB_CUDA_FAIL(cudaGetDeviceProperties(&prop, device))) { set(RFDETR_ERR_INFERENCE); return nullptr; }
    if (prop.major != 10) {
        rfdetr_logf(RFDETR_LOG_ERROR, "CUDA engine: device %d is sm_%d%d; this build targets sm_100a (B200)", device,
                    prop.major, prop.minor);
        set(RFDETR_ERR_INFERENCE);
        return nullptr;
    }
    gemm_set_num_sms(prop.multiProcessorCount);
    rfdetr_status s = engine_supports(m.cfg);
    if (s != RFDETR_OK) { set(s); return nullptr; }

    std::unique_ptr<Engine> e(new Engine());
    e->cfg_ = m.cfg;
    e->device_ = device;
    if (const char* ng = std::getenv("RFDETR_NO_GRAPH")) e->use_graphs_ = ng[0] == '0';
    if (RFB_CUDA_FAIL(cudaStreamCreateWithFlags(&e->stream_, cudaStreamNonBlocking))) {
        set(RFDETR_ERR_INFERENCE);
        return nullptr;
    }
    if (RFB_CUDA_FAIL(cudaMalloc(&e->d_err_, sizeof(int))) || RFB_CUDA_FAIL(cudaMemset(e->d_err_, 0, sizeof(int)))) {
        set(RFDETR_ERR_OUT_OF_MEMORY);
        return nullptr;
    }
    const Config& c = m.cfg;
    e->S_ = (int)c.image_size;
    e->P_ = (int)c.patch_size;
    e->G_ = c.grid();
    e->nw_ = (int)c.backbone.num_windows;
    e->ws_ = e->G_ / e->nw_;
    e->Tp_ = e->ws_ * e->ws_;
    e->T_ = e->Tp_ + 1;
    e->NW_ = e->nw_ * e->nw_;
    e->Ntok_ = e->NW_ * e->T_;
    e->D_ = (int)c.backbone.dim;
    e->H_ = (int)c.backbone.heads;
    e->F_ = (int)c.backbone.ffn_dim;
    e->L_ = (int)c.backbone.out_feature_indices.size();
    e->Kpatch_ = 3 * e->P_ * e->P_;
    e->Kpad_ = (e->Kpatch_ + 7) / 8 * 8;
    e->Dm_ = (int)c.decoder.model_dim;
    e->NQ_ = (int)c.num_queries;
    e->NC_ = (int)c.num_classes;
    e->Fd_ = (int)c.decoder.ffn_dim;
    e->Cb_ = (int)c.projector.bottleneck_dim;
    e->Hm_ = c.has_seg ? (int)(c.image_size / c.mask_downsample_ratio) : 0;
    e->n_soaw_ = (int)(c.decoder.cross_attn_heads * c.decoder.cross_attn_n_points * 3);
    s = e->upload_weights(m);
    if (s != RFDETR_OK) { set(s); return nullptr; }
    s = e->reserve(max_batch > 0 ? max_batch : 1);
    if (s != RFDETR_OK) { set(s); return nullptr; }
    set(RFDETR_OK);
    return e;
}

// ---------------------------------------------------------------------------
// weights
// ---------------------------------------------------------------------------

rfdetr_status Engine::upload_weights(const Model& m) {
    bool ok = true;
    auto dev_copy = [&](const void* src, size_t bytes) -> void* {
        void* p = nullptr;
        if (!ok) return nullptr;
        if (RFB_CUDA_FAIL(cudaMalloc(&p, bytes ? bytes : 16))) { ok = false; return nullptr; }
        wallocs_.push_back(p);
        if (bytes && RFB_CUDA_FAIL(cudaMemcpy(p, src, bytes, cudaMemcpyHostToDevice))) ok = false;
        return p;
    };
    auto f32 = [&](const std::string& n, size_t expect) -> std::vector<float> {
        std::vector<float> v = tensor_f32(m, n);
        if (v.empty() || (expect && v.size() != expect)) {
            rfdetr_logf(RFDETR_LOG_ERROR, "CUDA engine: tensor '%s' missing or has %zu elements (expected %zu)",
                        n.c_str(), v.size(), expect);
            ok = false;
        }
        return v;
    };
    auto upf = [&](const std::vector<float>& v) -> const float* {
        return static_cast<const float*>(dev_copy(v.data(), v.size() * 4));
    };
    // weight [N][K] f32 -> device f16 [N][ldw]
    auto uph = [&](const float* w, int N, int K, int ldw) -> const __half* {
        std::vector<uint16_t> h((size_t)N * ldw, 0);
        for (int n = 0; n < N; ++n)
            for (int k = 0; k < K; ++k) h[(size_t)n * ldw + k] = f2h_bits(w[(size_t)n * K + k]);
        return static_cast<const __half*>(dev_copy(h.data(), h.size() * 2));
    };
    auto lin = [&](const std::string& p, int N, int K) -> DLin {
        DLin l;
        std::vector<float> w = f32(p + ".weight", (size_t)N * K);
        std::vector<float> b = f32(p + ".bias", (size_t)N);
        if (!ok) return l;
        l.N = N;
        l.K = K;
        l.ldw = (K + 7) / 8 * 8;
        l.w = uph(w.data(), N, K, l.ldw);
        l.b = upf(b);
        return l;
    };
    auto norm = [&](const std::string& p, int n) -> DNorm {
        DNorm d;
        std::vector<float> g = f32(p + ".weight", n), b = f32(p + ".bias", n);
        if (!ok) return d;
        d.g = upf(g);
        d.b = upf(b);
        return d;
    };
    const Config& c = cfg_;
    const int D = D_, G = G_;

    // ---- patch embed + pos-embed (src/dinov2.cpp:339-408, model_loader.cpp:462-523)
    {
        std::vector<float> w = f32("backbone.patch_embed.weight", (size_t)D * Kpatch_);
        std::vector<float> b = f32("backbone.patch_embed.bias", D);
        std::vector<float> cls = f32("backbone.cls_token", D);
        const int ts = (int)c.backbone.pos_embed_train_size;
        std::vector<float> pe = f32("backbone.pos_embed", (size_t)(ts * ts + 1) * D);
        if (!ok) return RFDETR_ERR_MODEL_LOAD;
        patch_.N = D;
        patch_.K = Kpatch_;
        patch_.ldw = Kpad_;
        patch_.w = uph(w.data(), D, Kpatch_, Kpad_);
        patch_.b = upf(b);
        std::vector<float> pos((size_t)(G * G + 1) * D);
        std::memcpy(pos.data(), pe.data(), sizeof(float) * D);
        if (ts == G) std::memcpy(pos.data() + D, pe.data() + D, sizeof(float) * (size_t)G * G * D);
        else bicubic_resample(pe.data() + D, ts, D, pos.data() + D, G);
        std::vector<float> posw((size_t)Ntok_ * D);
        for (int win = 0; win < NW_; ++win) {
            std::memcpy(&posw[(size_t)win * T_ * D], pos.data(), sizeof(float) * D);
            for (int t = 0; t < Tp_; ++t) {
                const int gy = (win / nw_) * ws_ + t / ws_, gx = (win % nw_) * ws_ + t % ws_;
                std::memcpy(&posw[((size_t)win * T_ + 1 + t) * D], &pos[(size_t)(1 + gy * G + gx) * D],
                            sizeof(float) * D);
            }
        }
        posw_ = const_cast<float*>(upf(posw));
        std::vector<float> clsrow(D);
        for (int d = 0; d < D; ++d) clsrow[d] = cls[d] + pos[d];
        clsrow_ = const_cast<float*>(upf(clsrow));
    }
    // ---- backbone blocks
    blocks_.resize(c.backbone.depth);
    for (uint32_t i = 0; i < c.backbone.depth && ok; ++i) {
        const std::string p = "backbone.blocks." + std::to_string(i) + ".";
        Block& bk = blocks_[i];
        bk.ln1 = norm(p + "norm1", D);
        bk.ln2 = norm(p + "norm2", D);
        {
            std::vector<float> wq = f32(p + "attn.q.weight", (size_t)D * D), wk = f32(p + "attn.k.weight", (size_t)D * D),
                               wv = f32(p + "attn.v.weight", (size_t)D * D);
            std::vector<float> bq = f32(p + "attn.q.bias", D), bkk = f32(p + "attn.k.bias", D),
                               bv = f32(p + "attn.v.bias", D);
            if (!ok) break;
            std::vector<float> w((size_t)3 * D * D), b((size_t)3 * D);
            std::memcpy(w.data(), wq.data(), sizeof(float) * D * D);
            std::memcpy(w.data() + (size_t)D * D, wk.data(), sizeof(float) * D * D);
            std::memcpy(w.data() + (size_t)2 * D * D, wv.data(), sizeof(float) * D * D);
            std::memcpy(b.data(), bq.data(), sizeof(float) * D);
            std::memcpy(b.data() + D, bkk.data(), sizeof(float) * D);
            std::memcpy(b.data() + 2 * D, bv.data(), sizeof(float) * D);
            bk.qkv.N = 3 * D;
            bk.qkv.K = D;
            bk.qkv.ldw = D;
            bk.qkv.w = uph(w.data(), 3 * D, D, D);
            bk.qkv.b = upf(b);
        }
        bk.proj = lin(p + "attn.proj", D, D);
        bk.fc1 = lin(p + "mlp.fc1", F_, D);
        bk.fc2 = lin(p + "mlp.fc2", D, F_);
        bk.ls1 = upf(f32(p + "layer_scale1", D));
        bk.ls2 = upf(f32(p + "layer_scale2", D));
        for (uint32_t g : c.backbone.global_attn_indices)
            if (g == i) bk.global = true;
        for (size_t l = 0; l < c.backbone.out_feature_indices.size(); ++l)
            if (c.backbone.out_feature_indices[l] == i + 1) bk.tap = (int)l;
    }
    bbnorm_ = norm("backbone.norm", D);
    // ---- projector (src/projector.cpp): conv kernels F32 (OC, IC, kh, kw)
    const int C = (int)c.projector.out_dim, Cb = Cb_;
    {
        std::vector<float> w = f32("projector.cv1.conv.weight", (size_t)C * L_ * D);
        if (!ok) return RFDETR_ERR_MODEL_LOAD;
        cv1_.N = C; cv1_.K = L_ * D; cv1_.ldw = L_ * D;
        cv1_.w = uph(w.data(), C, L_ * D, L_ * D);
        const int Kc = (2 + (int)c.projector.n_bottlenecks) * Cb;
        std::vector<float> w2 = f32("projector.cv2.conv.weight", (size_t)C * Kc);
        if (!ok) return RFDETR_ERR_MODEL_LOAD;
        cv2_.N = C; cv2_.K = Kc; cv2_.ldw = Kc;
        cv2_.w = uph(w2.data(), C, Kc, Kc);
    }
    cv1n_ = norm("projector.cv1.norm", C);
    cv2n_ = norm("projector.cv2.norm", C);
    fnorm_ = norm("projector.final_norm", C);
    auto conv3 = [&](const std::string& n) -> DLin {
        DLin l;
        std::vector<float> w = f32(n, (size_t)Cb * Cb * 9);
        if (!ok) return l;
        std::vector<float> r((size_t)Cb * 9 * Cb);  // [oc][ky][kx][ic]
        for (int oc = 0; oc < Cb; ++oc)
            for (int ic = 0; ic < Cb; ++ic)
                for (int t = 0; t < 9; ++t) r[((size_t)oc * 9 + t) * Cb + ic] = w[((size_t)oc * Cb + ic) * 9 + t];
        l.N = Cb; l.K = 9 * Cb; l.ldw = 9 * Cb;
        l.w = uph(r.data(), Cb, 9 * Cb, 9 * Cb);
        return l;
    };
    bnecks_.resize(c.projector.n_bottlenecks);
    for (uint32_t j = 0; j < c.projector.n_bottlenecks && ok; ++j) {
        const std::string p = "projector.bottleneck." + std::to_string(j) + ".";
        bnecks_[j].c1 = conv3(p + "cv1.conv.weight");
        bnecks_[j].c2 = conv3(p + "cv2.conv.weight");
        bnecks_[j].n1 = norm(p + "cv1.norm", Cb);
        bnecks_[j].n2 = norm(p + "cv2.norm", Cb);
    }
    // ---- two-stage, group 0 (src/two_stage.cpp)
    const int Dm = Dm_;
    enc_ = lin("two_stage.enc_output.0", Dm, Dm);
    encn_ = norm("two_stage.enc_output_norm.0", Dm);
    cls_ = lin("two_stage.enc_out_class_embed.0", NC_, Dm);
    tb0_ = lin("two_stage.enc_out_bbox_embed.0.layers.0", Dm, Dm);
    tb1_ = lin("two_stage.enc_out_bbox_embed.0.layers.1", Dm, Dm);
    tb2_ = lin("two_stage.enc_out_bbox_embed.0.layers.2", 4, Dm);
    // ---- decoder
    {
        std::vector<float> rp = f32("decoder.queries.refpoints", 0);
        std::vector<float> ft = f32("decoder.queries.feat", 0);
        if (!ok) return RFDETR_ERR_MODEL_LOAD;
        if (rp.size() < (size_t)NQ_ * 4 || ft.size() < (size_t)NQ_ * Dm) {
            rfdetr_logf(RFDETR_LOG_ERROR, "CUDA engine: decoder queries hold fewer than num_queries rows");
            return RFDETR_ERR_MODEL_LOAD;
        }
        rp.resize((size_t)NQ_ * 4);
        ft.resize((size_t)NQ_ * Dm);
        lrn_rp_ = upf(rp);
        feat_ = upf(ft);
    }
    rph0_ = lin("decoder.ref_point_head.layers.0", Dm, 2 * Dm);
    rph1_ = lin("decoder.ref_point_head.layers.1", Dm, Dm);
    const int nso = (int)(c.decoder.cross_attn_heads * c.decoder.cross_attn_n_points * 2);
    const int naw = (int)(c.decoder.cross_attn_heads * c.decoder.cross_attn_n_points);
    dec_.resize(c.decoder.layers);
    for (uint32_t i = 0; i < c.decoder.layers && ok; ++i) {
        const std::string p = "decoder.layers." + std::to_string(i) + ".";
        DecLayer& L = dec_[i];
        {
            std::vector<float> w = f32(p + "self_attn.in_proj.weight", (size_t)3 * Dm * Dm);
            std::vector<float> b = f32(p + "self_attn.in_proj.bias", (size_t)3 * Dm);
            if (!ok) break;
            const __half* wd = uph(w.data(), 3 * Dm, Dm, Dm);
            const float* bd = upf(b);
            L.qk = DLin{wd, bd, 2 * Dm, Dm, Dm};
            L.v = DLin{wd + (size_t)2 * Dm * Dm, bd + 2 * Dm, Dm, Dm, Dm};
        }
        L.out = lin(p + "self_attn.out_proj", Dm, Dm);
        L.n1 = norm(p + "norm1", Dm);
        {
            std::vector<float> ws = f32(p + "cross_attn.sampling_offsets.weight", (size_t)nso * Dm);
            std::vector<float> bs = f32(p + "cross_attn.sampling_offsets.bias", nso);
            std::vector<float> wa = f32(p + "cross_attn.attention_weights.weight", (size_t)naw * Dm);
            std::vector<float> ba = f32(p + "cross_attn.attention_weights.bias", naw);
            if (!ok) break;
            std::vector<float> w(ws), b(bs);
            w.insert(w.end(), wa.begin(), wa.end());
            b.insert(b.end(), ba.begin(), ba.end());
            L.soaw = DLin{uph(w.data(), nso + naw, Dm, Dm), upf(b), nso + naw, Dm, Dm};
        }
        L.value = lin(p + "cross_attn.value_proj", Dm, Dm);
        L.oproj = lin(p + "cross_attn.output_proj", Dm, Dm);
        L.n2 = norm(p + "norm2", Dm);
        L.l1 = lin(p + "linear1", Fd_, Dm);
        L.l2 = lin(p + "linear2", Dm, Fd_);
        L.n3 = norm(p + "norm3", Dm);
    }
    dnorm_ = norm("decoder.norm", Dm);
    hcls_ = lin("heads.class_embed", NC_, Dm);
    hb0_ = lin("heads.bbox_embed.layers.0", Dm, Dm);
    hb1_ = lin("heads.bbox_embed.layers.1", Dm, Dm);
    hb2_ = lin("heads.bbox_embed.layers.2", 4, Dm);
    // ---- segmentation head (src/segmentation.cpp)
    if (c.has_seg) {
        segb_.resize(c.decoder.layers);
        for (uint32_t b = 0; b < c.decoder.layers && ok; ++b) {
            const std::string p = "segmentation_head.blocks." + std::to_string(b) + ".";
            segb_[b].dw_w = upf(f32(p + "dwconv.weight", (size_t)Dm * 9));
            segb_[b].dw_b = upf(f32(p + "dwconv.bias", Dm));
            segb_[b].n = norm(p + "norm", Dm);
            segb_[b].pw = lin(p + "pwconv1", Dm, Dm);
        }
        sfp_ = lin("segmentation_head.spatial_features_proj", Dm, Dm);
        qfn_ = norm("segmentation_head.query_features_block.norm_in", Dm);
        ql0_ = lin("segmentation_head.query_features_block.layers.0", 4 * Dm, Dm);
        ql2_ = lin("segmentation_head.query_features_block.layers.2", Dm, 4 * Dm);
        qfp_ = lin("segmentation_head.query_features_proj", Dm, Dm);
        std::vector<float> sb = f32("segmentation_head.bias", 1);
        if (ok) segbias_ = upf(std::vector<float>((size_t)Hm_ * Hm_, sb[0]));
    }
    return ok ? RFDETR_OK : RFDETR_ERR_MODEL_LOAD;
}

// ---------------------------------------------------------------------------
// activations
// ---------------------------------------------------------------------------

void Engine::free_activations() {
    if (arena_) cudaFree(arena_);
    arena_ = nullptr;
}

rfdetr_status Engine::reserve(int batch) {
    if (batch <= max_batch_) return RFDETR_OK;
    if (RFB_CUDA_FAIL(cudaSetDevice(device_))) return RFDETR_ERR_INFERENCE;
    cudaStreamSynchronize(stream_);
    return alloc_activations(batch);
}

rfdetr_status Engine::reserve_rgb(size_t bytes) {
    if (bytes <= rgb_cap_) return RFDETR_OK;
    if (RFB_CUDA_FAIL(cudaSetDevice(device_))) return RFDETR_ERR_INFERENCE;
    cudaStreamSynchronize(stream_);
    if (rgb_u8_) cudaFree(rgb_u8_);
    rgb_u8_ = nullptr;
    rgb_cap_ = 0;
    if (RFB_CUDA_FAIL(cudaMalloc(&rgb_u8_, bytes))) return RFDETR_ERR_OUT_OF_MEMORY;
    rgb_cap_ = bytes;
    return RFDETR_OK;
}

rfdetr_status Engine::alloc_activations(int B) {
    drop_graphs();  // captured graphs hold the old buffer addresses
    free_activations();
    const size_t Mb = (size_t)B * Ntok_;       // backbone rows
    const size_t Mp = (size_t)B * G_ * G_;      // spatial rows
    const size_t Mq = (size_t)B * NQ_;          // query rows
    const size_t HW = (size_t)Hm_ * Hm_;
    struct Req { void** p; size_t bytes; };
    std::vector<Req> reqs = {
        {(void**)&img_, (size_t)B * 3 * S_ * S_ * 4},
        {(void**)&apatch_, (size_t)B * NW_ * Tp_ * Kpad_ * 2},
        {(void**)&x_, Mb * D_ * 4},
        {(void**)&h16_, Mb * D_ * 2},
        {(void**)&qkv_, Mb * 3 * D_ * 2},
        {(void**)&attn_, Mb * D_ * 2},
        {(void**)&f1_, Mb * F_ * 2},
        {(void**)&taps_, Mp * L_ * D_ * 2},
        {(void**)&cat_, Mp * (2 + bnecks_.size()) * Cb_ * 2},
        {(void**)&tmp128_, Mp * Cb_ * 2},
        // split-K LayerNorm GEMMs run only with at most 74 tiles, so their partial sums never exceed
        // 148 splits x 128 rows x 64 columns of floats, whatever the batch
        {(void**)&splitws_, kSplitWsBytes},
        {(void**)&p32a_, Mp * Dm_ * 4},
        {(void**)&proj32_, Mp * Dm_ * 4},
        {(void**)&mem16_, Mp * Dm_ * 2},
        {(void**)&memm16_, Mp * Dm_ * 2},
        {(void**)&y16_, Mp * Dm_ * 2},
        {(void**)&clsall_, Mp * NC_ * 4},
        {(void**)&hb1_16_, Mp * Dm_ * 2},
        {(void**)&hb2_16_, Mp * Dm_ * 2},
        {(void**)&tsdelta_, Mp * 4 * 4},
        {(void**)&bboxall_, Mp * 4 * 4},
        {(void**)&topk_, Mq * 4},
        {(void**)&refp_, Mq * 4 * 4},
        {(void**)&sine_, Mq * 2 * Dm_ * 2},
        {(void**)&q16a_, Mq * Dm_ * 2},
        {(void**)&qpos_, Mq * Dm_ * 4},
        {(void**)&tgt_, Mq * Dm_ * 4},
        {(void**)&tgt16_, Mq * Dm_ * 2},
        {(void**)&qk16_, Mq * Dm_ * 2},
        {(void**)&qkp_, Mq * 2 * Dm_ * 2},
        {(void**)&vp_, Mq * Dm_ * 2},
        {(void**)&sa16_, Mq * Dm_ * 2},
        {(void**)&value_, Mp * Dm_ * 2},
        {(void**)&soaw_, Mq * n_soaw_ * 4},
        {(void**)&samp_, Mq * Dm_ * 2},
        {(void**)&ffn_, Mq * Fd_ * 2},
        {(void**)&dec32_, Mq * Dm_ * 4},
        {(void**)&dec16_, Mq * Dm_ * 2},
        {(void**)&logits_, Mq * NC_ * 4},
        {(void**)&hh1_, Mq * Dm_ * 2},
        {(void**)&hh2_, Mq * Dm_ * 2},
        {(void**)&bdelta_, Mq * 4 * 4},
        {(void**)&boxes_, Mq * 4 * 4},
    };
    rsz_ = nullptr;
    if (!cfg_.bilinear_no_antialias) reqs.push_back({(void**)&rsz_, (size_t)B * S_ * S_ * 3});
    if (cfg_.has_seg) {
        reqs.push_back({(void**)&sp32_, (size_t)B * HW * Dm_ * 4});
        reqs.push_back({(void**)&sln16_, (size_t)B * HW * Dm_ * 2});
        reqs.push_back({(void**)&spp16_, (size_t)B * HW * Dm_ * 2});
        reqs.push_back({(void**)&qn16_, Mq * Dm_ * 2});
        reqs.push_back({(void**)&qh16_, Mq * 4 * Dm_ * 2});
        reqs.push_back({(void**)&qf32_, Mq * Dm_ * 4});
        reqs.push_back({(void**)&qf16_, Mq * Dm_ * 2});
        reqs.push_back({(void**)&qfp16_, Mq * Dm_ * 2});
        reqs.push_back({(void**)&masks_, (size_t)B * NQ_ * HW * 4});
    }
    size_t total = 0;
    for (auto& r : reqs) total += (r.bytes + 255) / 256 * 256;
    if (RFB_CUDA_FAIL(cudaMalloc(&arena_, total))) {
        arena_ = nullptr;
        max_batch_ = 0;
        return RFDETR_ERR_OUT_OF_MEMORY;
    }
    char* p = static_cast<char*>(arena_);
    for (auto& r : reqs) {
        *r.p = p;
        p += (r.bytes + 255) / 256 * 256;
    }
    max_batch_ = B;
    return RFDETR_OK;
}

// ---------------------------------------------------------------------------
// forward
// ---------------------------------------------------------------------------

namespace {

struct Launcher {
    cudaStream_t st;
    int* err;
    float* splitws = nullptr;  // scratch for split-K LayerNorm GEMMs (kSplitWsBytes)
    int count = 0;
    bool ok = true;
    // optional per-launch events (profiling)
    std::vector<cudaEvent_t>* ev = nullptr;
    std::vector<std::string>* names = nullptr;
    int* used = nullptr;
    void mark(const char* what) {
        if (!ev) return;
        if (*used >= (int)ev->size()) {
            cudaEvent_t e;
            if (cudaEventCreate(&e) != cudaSuccess) return;
            ev->push_back(e);
            names->emplace_back();
        }
        cudaEventRecord((*ev)[*used], st);
        (*names)[*used] = what;
        ++*used;
    }
    void check(cudaError_t e, const char* what) {
        ++count;
        if (e != cudaSuccess && ok) {
            rfdetr_logf(RFDETR_LOG_ERROR, "forward: %s failed: %s", what, cudaGetErrorString(e));
            ok = false;
        }
        mark(what);
    }
    void gemm(const char* what, const __half* A, int lda, int M, const DLin& W, int epi, int act, float* out32,
              int ld32, __half* out16, int ld16, const float* colscale = nullptr, const DNorm* ln = nullptr,
              float eps = 1e-5f, const float* resid = nullptr, int ldr = 0) {
        GemmArgs a;
        a.A = A; a.lda = lda; a.B = W.w; a.ldb = W.ldw;
        a.M = M; a.N = W.N; a.K = W.K;
        a.epi = epi; a.act = act; a.bias = W.b; a.colscale = colscale;
        if (ln) { a.ln_g = ln->g; a.ln_b = ln->b; a.ln_eps = eps; }
        a.resid = resid; a.ldr = ldr;
        a.out32 = out32; a.ld32 = ld32; a.out16 = out16; a.ld16 = ld16;
        a.err = err;
        if (splitws) { a.split_ws = splitws; a.split_ws_bytes = kSplitWsBytes; }
        check(rfb::gemm(a, st), what);
    }
    // ConvX: 3x3 convolution (implicit GEMM over the channels-last map `src`,
    // B images of h x w pixels, c channels at pitch lds) + LayerNorm + SiLU.
    void conv3(const char* what, const __half* src, int lds, int B, int h, int w, int c, const DLin& W,
               __half* out16, int ld16, const DNorm* ln, float eps) {
        GemmArgs a;
        a.conv_src = src; a.conv_lds = lds; a.conv_h = h; a.conv_w = w; a.conv_c = c;
        a.B = W.w; a.ldb = W.ldw;
        a.M = B * h * w; a.N = W.N; a.K = W.K;
        a.epi = EPI_LN; a.act = ACT_SILU; a.bias = W.b;
        a.ln_g = ln->g; a.ln_b = ln->b; a.ln_eps = eps;
        a.out16 = out16; a.ld16 = ld16;
        a.err = err;
        if (splitws) { a.split_ws = splitws; a.split_ws_bytes = kSplitWsBytes; }
        check(rfb::gemm(a, st), what);
    }
};

}  // namespace

void Engine::drop_graphs() {
    for (auto& g : graphs_) cudaGraphExecDestroy(g.exec);
    graphs_.clear();
}

rfdetr_status Engine::prepare_legacy(int w, int h) {
    if (legacy_taps(w, h)) return RFDETR_OK;
    if (RFB_CUDA_FAIL(cudaSetDevice(device_))) return RFDETR_ERR_INFERENCE;
    LegacyEntry e{w, h, {}};
    const cudaError_t ce = upload_legacy_taps(w, h, S_, S_, &e.taps);
    if (ce == cudaErrorMemoryAllocation) return RFDETR_ERR_OUT_OF_MEMORY;
    if (RFB_CUDA_FAIL(ce)) return RFDETR_ERR_INFERENCE;
    legacy_.push_back(e);
    return RFDETR_OK;
}

const LegacyTapsDev* Engine::legacy_taps(int w, int h) const {
    for (const auto& l : legacy_)
        if (l.w == w && l.h == h) return &l.taps;
    return nullptr;
}

rfdetr_status Engine::enqueue(int B, const uint8_t* src_rgb, int src_w, int src_h) {
    if (src_rgb && legacy_resize(src_w, src_h)) {
        // taps are uploaded here, before any capture, so that replays reuse them
        const rfdetr_status s = prepare_legacy(src_w, src_h);
        if (s != RFDETR_OK) return s;
    }
    if (!use_graphs_ || profiling_) return enqueue_raw(B, src_rgb, src_w, src_h);
    if (RFB_CUDA_FAIL(cudaSetDevice(device_))) return RFDETR_ERR_INFERENCE;
    for (auto& g : graphs_) {
        if (g.batch == B && g.src == src_rgb && g.w == src_w && g.h == src_h) {
            return RFB_CUDA_FAIL(cudaGraphLaunch(g.exec, stream_)) ? RFDETR_ERR_INFERENCE : RFDETR_OK;
        }
    }
    // First time for this shape / input: run it directly (this also performs
    // any one-time per-device kernel set-up), then capture the same sequence
    // for the next calls.
    rfdetr_status s = enqueue_raw(B, src_rgb, src_w, src_h);
    if (s != RFDETR_OK) return s;
    cudaGraph_t graph = nullptr;
    if (cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        cudaGetLastError();
        return RFDETR_OK;  // capture unavailable: keep launching directly
    }
    const int launches = launches_;
    const rfdetr_status cs = enqueue_raw(B, src_rgb, src_w, src_h);
    const cudaError_t ce = cudaStreamEndCapture(stream_, &graph);
    launches_ = launches;
    if (cs != RFDETR_OK || ce != cudaSuccess || !graph) {
        if (graph) cudaGraphDestroy(graph);
        cudaGetLastError();
        return RFDETR_OK;
    }
    cudaGraphExec_t exec = nullptr;
    const cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (ie != cudaSuccess) {
        cudaGetLastError();
        return RFDETR_OK;
    }
    if (graphs_.size() >= 16) {
        cudaGraphExecDestroy(graphs_.front().exec);
        graphs_.erase(graphs_.begin());
    }
    graphs_.push_back({B, src_rgb, src_w, src_h, exec});
    return RFDETR_OK;
}


rfdetr_status Engine::enqueue_raw(int B, const uint8_t* src_rgb, int src_w, int src_h) {
    if (B <= 0 || B > max_batch_) return RFDETR_ERR_INVALID_ARG;
    if (RFB_CUDA_FAIL(cudaSetDevice(device_))) return RFDETR_ERR_INFERENCE;
    Launcher L{stream_, d_err_};
    L.splitws = splitws_;
    if (profiling_) {
        L.ev = &prof_ev_;
        L.names = &prof_names_;
        L.used = &prof_used_;
        prof_used_ = 0;
        L.mark("start");
    }
    cudaStream_t st = stream_;
    const int D = D_, G = G_, Dm = Dm_, NQ = NQ_;
    const int Mb = B * Ntok_, Mp = B * G * G, Mq = B * NQ;

    // ---- input
    // ---- preprocess + patch im2col in windowed order (one kernel from uint8)
    if (src_rgb) {
        if (src_w <= 0 || src_h <= 0) return RFDETR_ERR_INVALID_ARG;
        const uint8_t* pix = src_rgb;
        int pw = src_w, ph = src_h;
        if (legacy_resize(src_w, src_h)) {
            // legacy_stb models: the library resize to S x S (uint8), then the identity path
            const LegacyTapsDev* t = legacy_taps(src_w, src_h);
            if (!t || !rsz_) return RFDETR_ERR_INFERENCE;
            L.check(resize_legacy_rgb(src_rgb, B, src_w, src_h, *t, S_, S_, rsz_, st), "resize_legacy");
            pix = rsz_;
            pw = ph = S_;
        }
        L.check(patch_from_rgb(pix, B, pw, ph, S_, P_, nw_, Kpad_, cfg_.mean, cfg_.std, apatch_, st),
                "patch_from_rgb");
    } else {
        L.check(patch_im2col(img_, B, S_, P_, nw_, Kpad_, apatch_, st), "patch_im2col");
    }
    // ---- patch embed into windowed tokens (+ pos), CLS rows
    {
        GemmArgs a;
        a.A = apatch_; a.lda = Kpad_; a.B = patch_.w; a.ldb = patch_.ldw;
        a.M = B * NW_ * Tp_; a.N = D; a.K = Kpatch_;
        a.epi = EPI_PATCH; a.bias = patch_.b; a.out32 = x_; a.ld32 = D;
        a.patch_tp = Tp_; a.patch_t = T_; a.patch_rows = NW_ * Tp_; a.patch_ntok = Ntok_; a.posw = posw_;
        a.err = d_err_;
        L.check(gemm(a, st), "patch_embed");
    }
    L.check(write_cls_rows(x_, clsrow_, B, NW_, T_, D, st), "cls_rows");

    // ---- backbone blocks (src/dinov2.cpp:432-538)
    const float scale = 1.0f / std::sqrt((float)(D / H_));
    // a tapped block's output is normalised once for its tap and the next block's norm1
    // (RFDETR_LN_TAP=0: two launches; the outputs are the same bit for bit)
    const char* ln_tap_env = std::getenv("RFDETR_LN_TAP");
    const bool fuse_tap = !(ln_tap_env && ln_tap_env[0] == '0');
    bool ln1_done = false;
    for (size_t i = 0; i < blocks_.size(); ++i) {
        const Block& bk = blocks_[i];
        if (!ln1_done) L.check(layernorm(x_, Mb, D, bk.ln1.g, bk.ln1.b, 1e-6f, nullptr, h16_, st), "ln1");
        ln1_done = false;
        L.gemm("qkv", h16_, D, Mb, bk.qkv, EPI_F16, ACT_NONE, nullptr, 0, qkv_, 3 * D);
        if (bk.global)
            L.check(attention_tc(qkv_, qkv_ + D, qkv_ + 2 * D, 3 * D, 3 * D, 3 * D, attn_, D, Ntok_, B, H_, scale, d_err_,
                                 st),
                    "attn_global");
        else
            L.check(attention_tc(qkv_, qkv_ + D, qkv_ + 2 * D, 3 * D, 3 * D, 3 * D, attn_, D, T_, B * NW_, H_, scale,
                                 d_err_, st),
                    "attn_window");
        L.gemm("proj", attn_, D, Mb, bk.proj, EPI_RESID, ACT_NONE, x_, D, nullptr, 0, bk.ls1);
        L.check(layernorm(x_, Mb, D, bk.ln2.g, bk.ln2.b, 1e-6f, nullptr, h16_, st), "ln2");
        L.gemm("fc1", h16_, D, Mb, bk.fc1, EPI_F16, ACT_GELU, nullptr, 0, f1_, F_);
        L.gemm("fc2", f1_, F_, Mb, bk.fc2, EPI_RESID, ACT_NONE, x_, D, nullptr, 0, bk.ls2);
        if (bk.tap >= 0 && fuse_tap && i + 1 < blocks_.size()) {
            const Block& nb = blocks_[i + 1];
            L.check(layernorm_and_tap(x_, B, G, nw_, D, nb.ln1.g, nb.ln1.b, h16_, bbnorm_.g, bbnorm_.b, taps_, L_ * D,
                                      bk.tap * D, st),
                    "ln1+tap");
            ln1_done = true;
        } else if (bk.tap >= 0) {
            L.check(backbone_tap(x_, B, G, nw_, D, bbnorm_.g, bbnorm_.b, taps_, L_ * D, bk.tap * D, st), "tap");
        }
    }

    // ---- projector (src/projector.cpp:85-189), token-major
    const int Cb = Cb_, Ccat = (2 + (int)bnecks_.size()) * Cb;
    L.gemm("proj.cv1", taps_, L_ * D, Mp, cv1_, EPI_LN, ACT_SILU, nullptr, 0, cat_, Ccat, nullptr, &cv1n_, 1e-6f);
    const __half* cur = cat_ + Cb;
    for (size_t j = 0; j < bnecks_.size(); ++j) {
        L.conv3("bneck.cv1", cur, Ccat, B, G, G, Cb, bnecks_[j].c1, tmp128_, Cb, &bnecks_[j].n1, 1e-6f);
        __half* dst = cat_ + (2 + j) * Cb;
        L.conv3("bneck.cv2", tmp128_, Cb, B, G, G, Cb, bnecks_[j].c2, dst, Ccat, &bnecks_[j].n2, 1e-6f);
        cur = dst;
    }
    L.gemm("proj.cv2", cat_, Ccat, Mp, cv2_, EPI_LN, ACT_SILU, p32a_, Dm, nullptr, 0, nullptr, &cv2n_, 1e-6f);
    L.check(layernorm(p32a_, Mp, Dm, fnorm_.g, fnorm_.b, 1e-6f, proj32_, mem16_, st), "final_norm");

    // ---- two-stage (src/two_stage.cpp:91-236)
    const __half* ts_in = mem16_;
    if (G >= 50) {
        L.check(mask_memory(proj32_, B, G, Dm, memm16_, st), "mask_memory");
        ts_in = memm16_;
    }
    L.gemm("enc_output", ts_in, Dm, Mp, enc_, EPI_LN, ACT_NONE, nullptr, 0, y16_, Dm, nullptr, &encn_, 1e-5f);
    L.gemm("enc_class", y16_, Dm, Mp, cls_, EPI_F32, ACT_NONE, clsall_, NC_, nullptr, 0);
    L.gemm("enc_bbox0", y16_, Dm, Mp, tb0_, EPI_F16, ACT_RELU, nullptr, 0, hb1_16_, Dm);
    L.gemm("enc_bbox1", hb1_16_, Dm, Mp, tb1_, EPI_F16, ACT_RELU, nullptr, 0, hb2_16_, Dm);
    L.gemm("enc_bbox2", hb2_16_, Dm, Mp, tb2_, EPI_F32, ACT_NONE, tsdelta_, 4, nullptr, 0);
    L.check(two_stage_boxes(tsdelta_, B, G, bboxall_, st), "two_stage_boxes");

    // ---- top-K + decoder inputs (src/rfdetr_model.cpp:222-271)
    L.check(topk_tokens(clsall_, B, G * G, NC_, NQ, topk_, st), "topk");
    L.check(query_init(bboxall_, topk_, lrn_rp_, feat_, B, G * G, NQ, Dm, refp_, sine_, tgt_, tgt16_, st),
            "query_init");
    L.gemm("ref_point_head0", sine_, 2 * Dm, Mq, rph0_, EPI_F16, ACT_RELU, nullptr, 0, q16a_, Dm);
    L.gemm("ref_point_head1", q16a_, Dm, Mq, rph1_, EPI_F32, ACT_NONE, qpos_, Dm, nullptr, 0);

    // ---- decoder layers (src/decoder.cpp:293-379)
    const int sa_h = (int)cfg_.decoder.self_attn_heads;
    const float sa_scale = 1.0f / std::sqrt((float)(Dm / sa_h));
    for (size_t li = 0; li < dec_.size(); ++li) {
        const DecLayer& Ly = dec_[li];
        L.check(add_to_f16(tgt_, qpos_, (size_t)Mq * Dm, qk16_, st), "tgt+pos");
        L.gemm("sa.qk", qk16_, Dm, Mq, Ly.qk, EPI_F16, ACT_NONE, nullptr, 0, qkp_, 2 * Dm);
        L.gemm("sa.v", tgt16_, Dm, Mq, Ly.v, EPI_F16, ACT_NONE, nullptr, 0, vp_, Dm);
        L.check(attention(qkp_, qkp_ + Dm, vp_, 2 * Dm, 2 * Dm, Dm, sa16_, Dm, NQ, B, sa_h, Dm / sa_h, sa_scale, st),
                "self_attn");
        L.gemm("sa.out+norm1", sa16_, Dm, Mq, Ly.out, EPI_LN, ACT_NONE, tgt_, Dm, nullptr, 0, nullptr, &Ly.n1, 1e-5f,
               tgt_, Dm);
        L.check(add_to_f16(tgt_, qpos_, (size_t)Mq * Dm, qk16_, st), "x+pos");
        L.gemm("value_proj", mem16_, Dm, Mp, Ly.value, EPI_F16, ACT_NONE, nullptr, 0, value_, Dm);
        // sampling offsets + attention weights (src/decoder.cpp:238-259) as one N = 96 GEMM, then the
        // bilinear gather (:127-207)
        L.gemm("so_aw", qk16_, Dm, Mq, Ly.soaw, EPI_F32, ACT_NONE, soaw_, n_soaw_, nullptr, 0);
        L.check(deform_sample(value_, soaw_, n_soaw_, refp_, B, NQ, G, (int)cfg_.decoder.cross_attn_heads,
                              (int)cfg_.decoder.cross_attn_n_points, Dm, samp_, st),
                "deform");
        L.gemm("ca.out+norm2", samp_, Dm, Mq, Ly.oproj, EPI_LN, ACT_NONE, tgt_, Dm, tgt16_, Dm, nullptr, &Ly.n2, 1e-5f,
               tgt_, Dm);
        L.gemm("linear1", tgt16_, Dm, Mq, Ly.l1, EPI_F16, ACT_RELU, nullptr, 0, ffn_, Fd_);
        L.gemm("linear2+norm3", ffn_, Fd_, Mq, Ly.l2, EPI_LN, ACT_NONE, tgt_, Dm, tgt16_, Dm, nullptr, &Ly.n3, 1e-5f,
               tgt_, Dm);
    }
    L.check(layernorm(tgt_, Mq, Dm, dnorm_.g, dnorm_.b, 1e-5f, dec32_, dec16_, st), "decoder.norm");

    // ---- heads (src/heads.cpp:31-56) + reparam (src/rfdetr_model.cpp:438-448)
    L.gemm("class_embed", dec16_, Dm, Mq, hcls_, EPI_F32, ACT_NONE, logits_, NC_, nullptr, 0);
    L.gemm("bbox0", dec16_, Dm, Mq, hb0_, EPI_F16, ACT_RELU, nullptr, 0, hh1_, Dm);
    L.gemm("bbox1", hh1_, Dm, Mq, hb1_, EPI_F16, ACT_RELU, nullptr, 0, hh2_, Dm);
    L.gemm("bbox2", hh2_, Dm, Mq, hb2_, EPI_F32, ACT_NONE, bdelta_, 4, nullptr, 0);
    L.check(box_reparam(bdelta_, refp_, Mq, boxes_, st), "box_reparam");

    // ---- segmentation head (src/segmentation.cpp:170-309); only the last
    // block's mask is consumed, so only its projection + einsum are computed.
    if (cfg_.has_seg) {
        const int Hm = Hm_, HW = Hm * Hm;
        L.check(resize_bilinear(proj32_, B, G, Hm, Dm, sp32_, st), "seg.resize");
        for (size_t bi = 0; bi < segb_.size(); ++bi) {
            const SegBlock& sb = segb_[bi];
            L.check(dwconv_ln(sp32_, B, Hm, Hm, Dm, sb.dw_w, sb.dw_b, sb.n.g, sb.n.b, 1e-6f, sln16_, st), "seg.dwconv");
            L.gemm("seg.pwconv", sln16_, Dm, B * HW, sb.pw, EPI_RESID, ACT_GELU, sp32_, Dm, nullptr, 0);
        }
        L.check(to_f16(sp32_, (size_t)B * HW * Dm, sln16_, st), "seg.to16");
        L.gemm("seg.spatial_proj", sln16_, Dm, B * HW, sfp_, EPI_F16, ACT_NONE, nullptr, 0, spp16_, Dm);
        L.check(layernorm(dec32_, Mq, Dm, qfn_.g, qfn_.b, 1e-6f, nullptr, qn16_, st), "seg.qf_norm");
        L.gemm("seg.qf0", qn16_, Dm, Mq, ql0_, EPI_F16, ACT_GELU, nullptr, 0, qh16_, 4 * Dm);
        L.check(cudaMemcpyAsync(qf32_, dec32_, (size_t)Mq * Dm * 4, cudaMemcpyDeviceToDevice, st), "copy");
        L.gemm("seg.qf2", qh16_, 4 * Dm, Mq, ql2_, EPI_RESID, ACT_NONE, qf32_, Dm, nullptr, 0);
        L.check(to_f16(qf32_, (size_t)Mq * Dm, qf16_, st), "seg.qf16");
        L.gemm("seg.qf_proj", qf16_, Dm, Mq, qfp_, EPI_F16, ACT_NONE, nullptr, 0, qfp16_, Dm);
        GemmArgs a;
        a.A = qfp16_; a.lda = Dm; a.B = spp16_; a.ldb = Dm;
        a.M = NQ; a.N = HW; a.K = Dm;
        a.batches = B; a.a_batch_rows = NQ; a.b_batch_rows = HW; a.out_batch_stride = (long long)NQ * HW;
        a.epi = EPI_F32; a.bias = segbias_; a.out32 = masks_; a.ld32 = HW; a.err = d_err_;
        L.check(gemm(a, st), "seg.masks");
    }
    launches_ = L.count;
    return L.ok ? RFDETR_OK : RFDETR_ERR_INFERENCE;
}

std::vector<std::pair<std::string, float>> Engine::profile() {
    std::vector<std::pair<std::string, float>> out;
    for (int i = 1; i < prof_used_; ++i) {
        float ms = 0.f;
        if (cudaEventElapsedTime(&ms, prof_ev_[i - 1], prof_ev_[i]) != cudaSuccess) ms = -1.f;
        out.emplace_back(prof_names_[i], ms);
    }
    return out;
}

rfdetr_status Engine::finish() {
    if (RFB_CUDA_FAIL(cudaSetDevice(device_))) return RFDETR_ERR_INFERENCE;
    if (RFB_CUDA_FAIL(cudaStreamSynchronize(stream_))) return RFDETR_ERR_INFERENCE;
    int err = 0;
    if (RFB_CUDA_FAIL(cudaMemcpy(&err, d_err_, sizeof(int), cudaMemcpyDeviceToHost))) return RFDETR_ERR_INFERENCE;
    return device_error(err);
}

rfdetr_status Engine::enqueue_error_copy(int* h_err) {
    return RFB_CUDA_FAIL(cudaMemcpyAsync(h_err, d_err_, sizeof(int), cudaMemcpyDeviceToHost, stream_))
               ? RFDETR_ERR_INFERENCE
               : RFDETR_OK;
}

rfdetr_status Engine::device_error(int err) {
    if (!err) return RFDETR_OK;
    if ((err & 0xFF) == kErrWaitTimeout)
        rfdetr_logf(RFDETR_LOG_ERROR,
                    "forward: a kernel's bounded wait expired (mbarrier at shared offset 0x%x, cluster rank %d)",
                    (unsigned)((err >> 8) & 0xFFFFF), (err >> 28) & 1);
    else
        rfdetr_logf(RFDETR_LOG_ERROR, "forward: device error word %d", err);
    cudaMemset(d_err_, 0, sizeof(int));
    return RFDETR_ERR_INFERENCE;
}

long long Engine::trace(const std::string& name, int B, float* out, size_t cap) {
    struct Src { const void* p; size_t n; bool half; size_t ld; size_t off; size_t cols; };
    const size_t Mp = (size_t)B * G_ * G_, Mq = (size_t)B * NQ_, Mb = (size_t)B * Ntok_;
    Src s{nullptr, 0, false, 0, 0, 0};
    if (name == "backbone.x") s = {x_, Mb * D_, false, 0, 0, 0};
    else if (name.rfind("backbone.multiscale.level", 0) == 0) {
        const int l = std::atoi(name.c_str() + 25);
        if (l < 0 || l >= L_) return -1;
        s = {taps_, Mp, true, (size_t)L_ * D_, (size_t)l * D_, (size_t)D_};
    } else if (name == "projector.output") s = {proj32_, Mp * Dm_, false, 0, 0, 0};
    else if (name == "two_stage.cls_all") s = {clsall_, Mp * NC_, false, 0, 0, 0};
    else if (name == "two_stage.bbox_all") s = {bboxall_, Mp * 4, false, 0, 0, 0};
    else if (name == "decoder.refpoints") s = {refp_, Mq * 4, false, 0, 0, 0};
    else if (name == "decoder.query_pos") s = {qpos_, Mq * Dm_, false, 0, 0, 0};
    else if (name == "decoder.norm.output") s = {dec32_, Mq * Dm_, false, 0, 0, 0};
    else if (name == "heads.class_logits") s = {logits_, Mq * NC_, false, 0, 0, 0};
    else if (name == "boxes") s = {boxes_, Mq * 4, false, 0, 0, 0};
    else if (name == "topk") {
        if (cap < Mq) return -1;
        std::vector<int32_t> t(Mq);
        if (cudaMemcpy(t.data(), topk_, Mq * 4, cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
        for (size_t i = 0; i < Mq; ++i) out[i] = (float)t[i];
        return (long long)Mq;
    } else if (name == "seg.masks.final" && cfg_.has_seg) s = {masks_, (size_t)B * NQ_ * Hm_ * Hm_, false, 0, 0, 0};
    else return -1;
    if (s.half) {
        const size_t n = s.n * s.cols;
        if (cap < n) return -1;
        std::vector<__half> h(s.n * s.ld);
        if (cudaMemcpy(h.data(), s.p, h.size() * 2, cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
        for (size_t r = 0; r < s.n; ++r)
            for (size_t c = 0; c < s.cols; ++c) out[r * s.cols + c] = __half2float(h[r * s.ld + s.off + c]);
        return (long long)n;
    }
    if (cap < s.n) return -1;
    if (cudaMemcpy(out, s.p, s.n * 4, cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
    return (long long)s.n;
}

}  // namespace rfb
