// Model configuration and host-side tensor inventory, read from a GGUF file
// (format v2).  Mirrors the reference loader's metadata contract and its
// error behaviour: src/model_loader.hpp:25-79, src/model_loader.cpp:212-371,
// 541-750.
#pragma once

#include "gguf.hpp"
#include "rfdetr.h"

#include <cstdint>
#include <string>
#include <vector>

namespace rfb {

struct Config {
    std::string variant;
    uint32_t image_size = 0, patch_size = 0, num_queries = 0, group_detr = 0, num_classes = 0;
    std::vector<std::string> class_names;
    float mean[3] = {0, 0, 0}, std[3] = {1, 1, 1};
    bool bilinear_no_antialias = false;  // rfdetr.preprocess.resize_mode
    struct {
        uint32_t dim = 0, depth = 0, heads = 0, ffn_dim = 0, num_windows = 0, pos_embed_train_size = 0;
        std::vector<uint32_t> global_attn_indices, out_feature_indices;
    } backbone;
    struct {
        uint32_t in_dim = 0, out_dim = 0, bottleneck_dim = 0, n_bottlenecks = 0;
    } projector;
    struct {
        uint32_t layers = 0, model_dim = 0, ffn_dim = 0, self_attn_heads = 0, cross_attn_heads = 0,
                 cross_attn_n_levels = 0, cross_attn_n_points = 0;
    } decoder;
    uint32_t two_stage_groups = 0;
    bool has_seg = false;
    uint32_t mask_downsample_ratio = 4;

    int grid() const { return (int)(image_size / patch_size); }
};

struct Model {
    Config cfg;
    GgufFile file;
    std::string path;
};

// Parse + validate.  Returns nullptr and sets *st on failure (log messages go
// through the log callback, like the reference).
Model* model_load(const std::string& path, rfdetr_status* st);

// Names the reference expects for this config (src/model_loader.cpp:541-689).
std::vector<std::string> expected_tensor_names(const Config& c);

// Seg-head block check + expected-name check (src/model_loader.cpp:703-750).
rfdetr_status model_validate(const Model& m);

// Checks the configuration is one the CUDA engine's kernels implement
// (head sizes, widths, grid limits).  Logs and returns RFDETR_ERR_MODEL_FORMAT
// otherwise: there is no fallback path.
rfdetr_status engine_supports(const Config& c);

// Dequantized f32 copy of a tensor (empty on failure).
std::vector<float> tensor_f32(const Model& m, const std::string& name);

// Antialiased bicubic (A = -0.5) patch-grid resample: src [src*src][dim] ->
// dst [dst*dst][dim] (src/model_loader.cpp:117-208).
void bicubic_resample(const float* src, int src_side, int dim, float* dst, int dst_side);

}  // namespace rfb
