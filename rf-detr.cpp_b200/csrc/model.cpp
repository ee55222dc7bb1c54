#include "model.hpp"

#include "common.hpp"

#include <algorithm>
#include <cmath>
#include <cstring>
#include <new>

namespace rfb {

namespace {

const GgufValue* kv(const GgufFile& f, const char* k) {
    auto it = f.kv.find(k);
    return it == f.kv.end() ? nullptr : &it->second;
}
bool get_u32(const GgufFile& f, const char* k, uint32_t& out) {
    const GgufValue* v = kv(f, k);
    if (!v || v->type > 12 || v->type == 8 || v->type == 9) return false;
    out = (uint32_t)v->u;
    return true;
}
bool get_str(const GgufFile& f, const char* k, std::string& out) {
    const GgufValue* v = kv(f, k);
    if (!v || v->type != 8) return false;
    out = v->s;
    return true;
}
bool get_u32_arr(const GgufFile& f, const char* k, std::vector<uint32_t>& out) {
    const GgufValue* v = kv(f, k);
    if (!v || v->type != 9 || v->arr_type == 8) return false;
    out.clear();
    for (double d : v->nums) out.push_back((uint32_t)(int64_t)d);
    return true;
}
bool get_f32_arr(const GgufFile& f, const char* k, float* out, size_t n) {
    const GgufValue* v = kv(f, k);
    if (!v || v->type != 9 || v->nums.size() != n) return false;
    for (size_t i = 0; i < n; ++i) out[i] = (float)v->nums[i];
    return true;
}

}  // namespace

Model* model_load(const std::string& path, rfdetr_status* st) {
    auto set = [&](rfdetr_status s) { if (st) *st = s; };
    Model* m = new (std::nothrow) Model();
    if (!m) { set(RFDETR_ERR_OUT_OF_MEMORY); return nullptr; }
    auto fail = [&](rfdetr_status s, const char* msg) -> Model* {
        rfdetr_logf(RFDETR_LOG_ERROR, "model_load: %s", msg);
        delete m;
        set(s);
        return nullptr;
    };
    std::string err;
    const int rc = gguf_read(path, &m->file, &err);
    if (rc == -2) {
        rfdetr_logf(RFDETR_LOG_ERROR, "model_load: file not found '%s'", path.c_str());
        delete m;
        set(RFDETR_ERR_FILE_NOT_FOUND);
        return nullptr;
    }
    if (rc != 0) return fail(rc == -3 ? RFDETR_ERR_IO : RFDETR_ERR_MODEL_FORMAT, err.c_str());
    m->path = path;
    const GgufFile& f = m->file;
    Config& c = m->cfg;
    std::string fmt;
    if (!get_str(f, "rfdetr.format.version", fmt) || fmt != "2")
        return fail(RFDETR_ERR_MODEL_FORMAT, "unsupported rfdetr.format.version");
    if (!get_str(f, "rfdetr.variant", c.variant)) return fail(RFDETR_ERR_MODEL_FORMAT, "rfdetr.variant missing");
    if (!get_u32(f, "rfdetr.image_size", c.image_size)) return fail(RFDETR_ERR_MODEL_FORMAT, "rfdetr.image_size missing");
    if (!get_u32(f, "rfdetr.patch_size", c.patch_size)) return fail(RFDETR_ERR_MODEL_FORMAT, "rfdetr.patch_size missing");
    if (!get_u32(f, "rfdetr.num_queries", c.num_queries)) return fail(RFDETR_ERR_MODEL_FORMAT, "rfdetr.num_queries missing");
    if (!get_u32(f, "rfdetr.group_detr", c.group_detr)) return fail(RFDETR_ERR_MODEL_FORMAT, "rfdetr.group_detr missing");
    if (!get_u32(f, "rfdetr.num_classes", c.num_classes)) return fail(RFDETR_ERR_MODEL_FORMAT, "rfdetr.num_classes missing");
    {
        const GgufValue* v = kv(f, "rfdetr.class_names");
        if (!v || v->type != 9 || v->arr_type != 8) return fail(RFDETR_ERR_MODEL_FORMAT, "rfdetr.class_names missing");
        c.class_names = v->strs;
        if (c.class_names.size() != c.num_classes)
            return fail(RFDETR_ERR_MODEL_FORMAT, "class_names length != num_classes");
    }
    if (!get_f32_arr(f, "rfdetr.preprocess.mean", c.mean, 3))
        return fail(RFDETR_ERR_MODEL_FORMAT, "rfdetr.preprocess.mean missing or wrong shape");
    if (!get_f32_arr(f, "rfdetr.preprocess.std", c.std, 3))
        return fail(RFDETR_ERR_MODEL_FORMAT, "rfdetr.preprocess.std missing or wrong shape");
    std::string mode;
    if (get_str(f, "rfdetr.preprocess.resize_mode", mode)) {
        if (mode == "bilinear_no_antialias") c.bilinear_no_antialias = true;
        else if (mode == "legacy_stb") c.bilinear_no_antialias = false;
        else return fail(RFDETR_ERR_MODEL_FORMAT, "unsupported rfdetr.preprocess.resize_mode");
    }
    auto& b = c.backbone;
    if (!get_u32(f, "rfdetr.backbone.dim", b.dim) || !get_u32(f, "rfdetr.backbone.depth", b.depth) ||
        !get_u32(f, "rfdetr.backbone.heads", b.heads) || !get_u32(f, "rfdetr.backbone.ffn_dim", b.ffn_dim) ||
        !get_u32(f, "rfdetr.backbone.num_windows", b.num_windows) ||
        !get_u32(f, "rfdetr.backbone.pos_embed_train_size", b.pos_embed_train_size))
        return fail(RFDETR_ERR_MODEL_FORMAT, "rfdetr.backbone.* incomplete");
    if (!get_u32_arr(f, "rfdetr.backbone.global_attn_indices", b.global_attn_indices))
        return fail(RFDETR_ERR_MODEL_FORMAT, "rfdetr.backbone.global_attn_indices missing");
    if (!get_u32_arr(f, "rfdetr.backbone.out_feature_indices", b.out_feature_indices))
        return fail(RFDETR_ERR_MODEL_FORMAT, "rfdetr.backbone.out_feature_indices missing");
    auto& p = c.projector;
    if (!get_u32(f, "rfdetr.projector.in_dim", p.in_dim) || !get_u32(f, "rfdetr.projector.out_dim", p.out_dim) ||
        !get_u32(f, "rfdetr.projector.bottleneck_dim", p.bottleneck_dim) ||
        !get_u32(f, "rfdetr.projector.n_bottlenecks", p.n_bottlenecks))
        return fail(RFDETR_ERR_MODEL_FORMAT, "rfdetr.projector.* incomplete");
    auto& d = c.decoder;
    if (!get_u32(f, "rfdetr.decoder.layers", d.layers) || !get_u32(f, "rfdetr.decoder.model_dim", d.model_dim) ||
        !get_u32(f, "rfdetr.decoder.ffn_dim", d.ffn_dim) ||
        !get_u32(f, "rfdetr.decoder.self_attn_heads", d.self_attn_heads) ||
        !get_u32(f, "rfdetr.decoder.cross_attn_heads", d.cross_attn_heads) ||
        !get_u32(f, "rfdetr.decoder.cross_attn_n_levels", d.cross_attn_n_levels) ||
        !get_u32(f, "rfdetr.decoder.cross_attn_n_points", d.cross_attn_n_points))
        return fail(RFDETR_ERR_MODEL_FORMAT, "rfdetr.decoder.* incomplete");
    if (!get_u32(f, "rfdetr.two_stage.n_groups", c.two_stage_groups))
        return fail(RFDETR_ERR_MODEL_FORMAT, "rfdetr.two_stage.n_groups missing");
    {
        const GgufValue* v = kv(f, "rfdetr.has_segmentation_head");
        c.has_seg = v && v->type == 7 && v->u != 0;
    }
    if (c.has_seg) {
        if (!get_u32(f, "rfdetr.mask_downsample_ratio", c.mask_downsample_ratio))
            return fail(RFDETR_ERR_MODEL_FORMAT, "rfdetr.mask_downsample_ratio missing for seg model");
        if (c.mask_downsample_ratio == 0) return fail(RFDETR_ERR_MODEL_FORMAT, "rfdetr.mask_downsample_ratio must be > 0");
    }
    set(RFDETR_OK);
    return m;
}

std::vector<std::string> expected_tensor_names(const Config& c) {
    std::vector<std::string> n;
    auto lin = [&](const std::string& p) { n.push_back(p + ".weight"); n.push_back(p + ".bias"); };
    n.push_back("backbone.patch_embed.weight");
    n.push_back("backbone.patch_embed.bias");
    n.push_back("backbone.cls_token");
    n.push_back("backbone.pos_embed");
    for (uint32_t i = 0; i < c.backbone.depth; ++i) {
        const std::string p = "backbone.blocks." + std::to_string(i) + ".";
        lin(p + "norm1");
        lin(p + "attn.q");
        lin(p + "attn.k");
        lin(p + "attn.v");
        lin(p + "attn.proj");
        n.push_back(p + "layer_scale1");
        lin(p + "norm2");
        lin(p + "mlp.fc1");
        lin(p + "mlp.fc2");
        n.push_back(p + "layer_scale2");
    }
    lin("backbone.norm");
    n.push_back("projector.cv1.conv.weight");
    lin("projector.cv1.norm");
    n.push_back("projector.cv2.conv.weight");
    lin("projector.cv2.norm");
    for (uint32_t j = 0; j < c.projector.n_bottlenecks; ++j) {
        const std::string p = "projector.bottleneck." + std::to_string(j) + ".";
        n.push_back(p + "cv1.conv.weight");
        lin(p + "cv1.norm");
        n.push_back(p + "cv2.conv.weight");
        lin(p + "cv2.norm");
    }
    lin("projector.final_norm");
    for (uint32_t g = 0; g < c.two_stage_groups; ++g) {
        const std::string gi = std::to_string(g);
        lin("two_stage.enc_output." + gi);
        lin("two_stage.enc_output_norm." + gi);
        lin("two_stage.enc_out_class_embed." + gi);
        for (int j = 0; j < 3; ++j) lin("two_stage.enc_out_bbox_embed." + gi + ".layers." + std::to_string(j));
    }
    n.push_back("decoder.queries.feat");
    n.push_back("decoder.queries.refpoints");
    lin("decoder.ref_point_head.layers.0");
    lin("decoder.ref_point_head.layers.1");
    for (uint32_t i = 0; i < c.decoder.layers; ++i) {
        const std::string p = "decoder.layers." + std::to_string(i) + ".";
        lin(p + "self_attn.in_proj");
        lin(p + "self_attn.out_proj");
        lin(p + "norm1");
        lin(p + "cross_attn.sampling_offsets");
        lin(p + "cross_attn.attention_weights");
        lin(p + "cross_attn.value_proj");
        lin(p + "cross_attn.output_proj");
        lin(p + "norm2");
        lin(p + "linear1");
        lin(p + "linear2");
        lin(p + "norm3");
    }
    lin("decoder.norm");
    lin("heads.class_embed");
    for (int j = 0; j < 3; ++j) lin("heads.bbox_embed.layers." + std::to_string(j));
    if (c.has_seg) {
        for (uint32_t b = 0; b < c.decoder.layers; ++b) {
            const std::string p = "segmentation_head.blocks." + std::to_string(b) + ".";
            lin(p + "dwconv");
            lin(p + "norm");
            lin(p + "pwconv1");
        }
        lin("segmentation_head.spatial_features_proj");
        lin("segmentation_head.query_features_block.norm_in");
        lin("segmentation_head.query_features_block.layers.0");
        lin("segmentation_head.query_features_block.layers.2");
        lin("segmentation_head.query_features_proj");
        n.push_back("segmentation_head.bias");
    }
    return n;
}

rfdetr_status model_validate(const Model& m) {
    const Config& c = m.cfg;
    if (c.has_seg) {
        uint32_t have = 0;
        while (m.file.find("segmentation_head.blocks." + std::to_string(have) + ".dwconv.weight")) ++have;
        if (have == 0 && c.decoder.layers > 0) {
            rfdetr_logf(RFDETR_LOG_ERROR,
                        "model_validate_tensors: the metadata declares a segmentation head, which needs %u head "
                        "block(s) for %u decoder layers, but this file has 0 of them: no segmentation_head.blocks.* "
                        "tensors are present at all. The conversion did not complete, or the metadata does not match "
                        "the weights.",
                        c.decoder.layers, c.decoder.layers);
            return RFDETR_ERR_MODEL_LOAD;
        }
        if (have < c.decoder.layers) {
            rfdetr_logf(RFDETR_LOG_ERROR,
                        "model_validate_tensors: this segmentation GGUF has %u head block(s) but the model has %u "
                        "decoder layers and needs one block per layer. It was converted before the segmentation-head "
                        "block-count fix and its masks are incorrect. Re-convert the model.",
                        have, c.decoder.layers);
            return RFDETR_ERR_MODEL_LOAD;
        }
    }
    std::vector<std::string> missing;
    for (const auto& n : expected_tensor_names(c))
        if (!m.file.find(n)) missing.push_back(n);
    if (!missing.empty()) {
        rfdetr_logf(RFDETR_LOG_ERROR, "model_validate_tensors: %zu missing tensor(s); first: '%s'", missing.size(),
                    missing.front().c_str());
        return RFDETR_ERR_MODEL_LOAD;
    }
    return RFDETR_OK;
}

rfdetr_status engine_supports(const Config& c) {
    auto bad = [](const char* why) {
        rfdetr_logf(RFDETR_LOG_ERROR, "CUDA engine: unsupported model configuration: %s", why);
        return RFDETR_ERR_MODEL_FORMAT;
    };
    const auto& b = c.backbone;
    if (c.patch_size == 0 || c.image_size % c.patch_size) return bad("image_size not a multiple of patch_size");
    const int G = c.grid();
    if (b.num_windows == 0 || G % b.num_windows) return bad("grid not divisible by num_windows");
    if (b.heads == 0 || b.dim % b.heads || b.dim / b.heads != 64) return bad("backbone head_dim must be 64");
    if (b.dim % 64 || b.dim > 384) return bad("backbone dim must be a multiple of 64 and <= 384");
    if (b.ffn_dim % 64) return bad("backbone ffn_dim must be a multiple of 64");
    if (b.out_feature_indices.empty() || b.out_feature_indices.size() > 4) return bad("1..4 feature taps");
    if (c.projector.in_dim != b.dim * b.out_feature_indices.size()) return bad("projector.in_dim != taps * dim");
    const auto& d = c.decoder;
    if (d.model_dim != 256 || c.projector.out_dim != 256) return bad("decoder / projector width must be 256");
    if (c.projector.bottleneck_dim * 2 != c.projector.out_dim) return bad("bottleneck_dim must be out_dim / 2");
    if (d.self_attn_heads == 0 || d.model_dim / d.self_attn_heads != 32) return bad("decoder self-attn head_dim must be 32");
    if (d.cross_attn_heads == 0 || d.model_dim % d.cross_attn_heads || (d.model_dim / d.cross_attn_heads) % 8)
        return bad("cross-attn head_dim must be a multiple of 8");
    if (d.cross_attn_n_levels != 1) return bad("one feature level");
    if (d.ffn_dim % 64) return bad("decoder ffn_dim must be a multiple of 64");
    if ((int)c.num_queries > G * G) return bad("num_queries exceeds the token count");
    if (G * G > 4096) return bad("grid larger than 64 x 64");
    if (c.two_stage_groups == 0) return bad("no two-stage group");
    if (c.has_seg && (c.image_size % c.mask_downsample_ratio)) return bad("mask size not integral");
    return RFDETR_OK;
}

std::vector<float> tensor_f32(const Model& m, const std::string& name) {
    const GgufTensor* t = m.file.find(name);
    if (!t) return {};
    std::vector<float> out((size_t)t->nelements());
    if (!dequantize(t->type, m.file.tensor_data(*t), t->nelements(), out.data())) return {};
    return out;
}

void bicubic_resample(const float* src, int src_side, int dim, float* dst, int dst_side) {
    constexpr float A = -0.5f;
    auto kern = [](float x) -> float {
        const float ax = std::fabs(x);
        if (ax < 1.0f) return ((A + 2.0f) * ax - (A + 3.0f)) * ax * ax + 1.0f;
        if (ax < 2.0f) return ((A * ax - 5.0f * A) * ax + 8.0f * A) * ax - 4.0f * A;
        return 0.0f;
    };
    const float scale = (float)src_side / (float)dst_side;
    const float invscale = scale >= 1.0f ? 1.0f / scale : 1.0f;
    const float support = scale >= 1.0f ? 2.0f * scale : 2.0f;
    const int taps = (int)std::ceil(support) * 2 + 1;
    std::vector<float> w((size_t)dst_side * taps, 0.f);
    std::vector<int> idx((size_t)dst_side * taps, 0), cnt(dst_side, 0);
    for (int o = 0; o < dst_side; ++o) {
        const float center = scale * ((float)o + 0.5f);
        const int lo = std::max((int)(center - support + 0.5f), 0);
        const int hi = std::min((int)(center + support + 0.5f), src_side);
        const int n = std::min(std::max(hi - lo, 0), taps);
        float tot = 0.f;
        for (int j = 0; j < n; ++j) {
            const float v = kern(((float)j + (float)lo - center + 0.5f) * invscale);
            w[(size_t)o * taps + j] = v;
            idx[(size_t)o * taps + j] = lo + j;
            tot += v;
        }
        if (tot != 0.f)
            for (int j = 0; j < n; ++j) w[(size_t)o * taps + j] /= tot;
        cnt[o] = n;
    }
    for (int oy = 0; oy < dst_side; ++oy)
        for (int ox = 0; ox < dst_side; ++ox) {
            float* dd = dst + ((size_t)oy * dst_side + ox) * dim;
            std::fill(dd, dd + dim, 0.f);
            for (int ky = 0; ky < cnt[oy]; ++ky) {
                const float wy = w[(size_t)oy * taps + ky];
                if (wy == 0.f) continue;
                const int sy = idx[(size_t)oy * taps + ky];
                for (int kx = 0; kx < cnt[ox]; ++kx) {
                    const float wx = w[(size_t)ox * taps + kx];
                    if (wx == 0.f) continue;
                    const int sx = idx[(size_t)ox * taps + kx];
                    const float ww = wx * wy;
                    const float* s = src + ((size_t)sy * src_side + sx) * dim;
                    for (int i = 0; i < dim; ++i) dd[i] += ww * s[i];
                }
            }
        }
}

}  // namespace rfb
