// Minimal GGUF (v2/v3) reader: metadata key/values and the tensor table,
// with the tensor data read into host memory.  Replaces the gguf_* calls the
// reference makes through ggml (src/model_loader.cpp:212-371).
#pragma once

#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

namespace rfb {

// ggml tensor type ids (GGUF on-disk values)
enum GgmlType : uint32_t {
    GT_F32 = 0, GT_F16 = 1, GT_Q4_0 = 2, GT_Q4_1 = 3, GT_Q5_0 = 6, GT_Q5_1 = 7, GT_Q8_0 = 8,
    GT_Q4_K = 12, GT_Q5_K = 13, GT_Q6_K = 14, GT_BF16 = 30,
};

const char* ggml_type_name(uint32_t t);
// bytes per block and elements per block; false for unsupported types
bool ggml_type_block(uint32_t t, size_t* block_bytes, int* block_elems);

struct GgufValue {
    uint32_t type = 0;           // GGUF value type
    uint32_t arr_type = 0;       // element type for arrays
    uint64_t u = 0;              // unsigned/bool scalars
    int64_t i = 0;               // signed scalars
    double f = 0;                // float scalars
    std::string s;               // strings
    std::vector<double> nums;    // numeric arrays
    std::vector<std::string> strs;
};

struct GgufTensor {
    std::string name;
    uint32_t type = 0;
    int n_dims = 0;
    int64_t ne[4] = {1, 1, 1, 1};  // ggml order: ne[0] fastest
    uint64_t offset = 0;           // relative to the data section
    size_t nbytes = 0;
    int64_t nelements() const { return ne[0] * ne[1] * ne[2] * ne[3]; }
};

struct GgufFile {
    uint32_t version = 0;
    uint64_t n_kv = 0;
    std::vector<uint8_t> kv_raw;    // the metadata section exactly as stored (for rewriting the file)
    uint64_t alignment = 32;        // general.alignment
    std::unordered_map<std::string, GgufValue> kv;
    std::vector<GgufTensor> tensors;
    std::unordered_map<std::string, size_t> index;  // name -> tensors[]
    std::vector<uint8_t> data;                      // whole data section

    const GgufTensor* find(const std::string& n) const {
        auto it = index.find(n);
        return it == index.end() ? nullptr : &tensors[it->second];
    }
    const uint8_t* tensor_data(const GgufTensor& t) const { return data.data() + t.offset; }
};

// Parse the file.  Returns 0 on success, a negative rfdetr_status otherwise
// (-2 file not found, -3 I/O, -6 malformed / unsupported format).
int gguf_read(const std::string& path, GgufFile* out, std::string* err);

// Write `f` as a GGUF file: the same version, metadata (kv_raw copied byte for
// byte) and tensor order, tensor `i` of type tensors[i].type with its bytes at
// f.data + tensors[i].offset; offsets are recomputed, every tensor's data is
// aligned to f.alignment and zero-padded (the layout of gguf-py's GGUFWriter).
// Returns 0 or a negative rfdetr_status (-3 I/O).
int gguf_write(const std::string& path, const GgufFile& f, std::string* err);

// Dequantize `n` elements of a tensor of type `t` to f32 (ggml's to_float
// arithmetic for each block format).  Returns false for unsupported types.
bool dequantize(uint32_t t, const void* src, int64_t n, float* dst);

float half_to_float(uint16_t h);

}  // namespace rfb
