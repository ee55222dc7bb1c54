// GGUF reader and block dequantizers.  The block layouts and the dequant
// arithmetic are those of the ggml block formats (ggml-common.h / ggml-quants.c
// of the ggml library the reference builds on), restated here.
#include "gguf.hpp"

#include <cstdio>
#include <cstring>
#include <memory>
#include <new>

namespace rfb {

namespace {

enum : uint32_t {
    V_U8 = 0, V_I8 = 1, V_U16 = 2, V_I16 = 3, V_U32 = 4, V_I32 = 5, V_F32 = 6, V_BOOL = 7,
    V_STR = 8, V_ARR = 9, V_U64 = 10, V_I64 = 11, V_F64 = 12,
};

struct Reader {
    FILE* f;
    uint64_t size = 0;  // file size: no length read from the file may exceed what is left of it
    bool ok = true;
    uint64_t left() const {
        const long p = std::ftell(f);
        return p < 0 || (uint64_t)p > size ? 0 : size - (uint64_t)p;
    }
    template <class T>
    T get() {
        T v{};
        if (ok && std::fread(&v, sizeof(T), 1, f) != 1) ok = false;
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (!ok || n > left()) { ok = false; return {}; }
        std::string s(n, '\0');
        if (n && std::fread(&s[0], 1, n, f) != n) ok = false;
        return s;
    }
};

size_t scalar_size(uint32_t t) {
    switch (t) {
        case V_U8: case V_I8: case V_BOOL: return 1;
        case V_U16: case V_I16: return 2;
        case V_U32: case V_I32: case V_F32: return 4;
        case V_U64: case V_I64: case V_F64: return 8;
        default: return 0;
    }
}

double read_scalar(Reader& r, uint32_t t, GgufValue* v) {
    switch (t) {
        case V_U8: { auto x = r.get<uint8_t>(); v->u = x; v->i = x; return x; }
        case V_I8: { auto x = r.get<int8_t>(); v->i = x; v->u = (uint64_t)x; return x; }
        case V_U16: { auto x = r.get<uint16_t>(); v->u = x; v->i = x; return x; }
        case V_I16: { auto x = r.get<int16_t>(); v->i = x; v->u = (uint64_t)x; return x; }
        case V_U32: { auto x = r.get<uint32_t>(); v->u = x; v->i = x; return x; }
        case V_I32: { auto x = r.get<int32_t>(); v->i = x; v->u = (uint64_t)x; return x; }
        case V_F32: { auto x = r.get<float>(); v->f = x; return x; }
        case V_BOOL: { auto x = r.get<uint8_t>(); v->u = x != 0; v->i = x != 0; return x != 0; }
        case V_U64: { auto x = r.get<uint64_t>(); v->u = x; v->i = (int64_t)x; return (double)x; }
        case V_I64: { auto x = r.get<int64_t>(); v->i = x; v->u = (uint64_t)x; return (double)x; }
        case V_F64: { auto x = r.get<double>(); v->f = x; return x; }
        default: r.ok = false; return 0;
    }
}

}  // namespace

float half_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000) << 16;
    const uint32_t exp = (h >> 10) & 0x1F;
    const uint32_t man = h & 0x3FF;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {  // subnormal
            int e = -1;
            uint32_t m = man;
            do { ++e; m <<= 1; } while ((m & 0x400) == 0);
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((m & 0x3FF) << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7F800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

const char* ggml_type_name(uint32_t t) {
    switch (t) {
        case GT_F32: return "F32"; case GT_F16: return "F16"; case GT_BF16: return "BF16";
        case GT_Q4_0: return "Q4_0"; case GT_Q4_1: return "Q4_1"; case GT_Q5_0: return "Q5_0";
        case GT_Q5_1: return "Q5_1"; case GT_Q8_0: return "Q8_0"; case GT_Q4_K: return "Q4_K";
        case GT_Q5_K: return "Q5_K"; case GT_Q6_K: return "Q6_K";
        default: return "unsupported";
    }
}

bool ggml_type_block(uint32_t t, size_t* bb, int* be) {
    switch (t) {
        case GT_F32: *bb = 4; *be = 1; return true;
        case GT_F16: case GT_BF16: *bb = 2; *be = 1; return true;
        case GT_Q4_0: *bb = 18; *be = 32; return true;
        case GT_Q4_1: *bb = 20; *be = 32; return true;
        case GT_Q5_0: *bb = 22; *be = 32; return true;
        case GT_Q5_1: *bb = 24; *be = 32; return true;
        case GT_Q8_0: *bb = 34; *be = 32; return true;
        case GT_Q4_K: *bb = 144; *be = 256; return true;
        case GT_Q5_K: *bb = 176; *be = 256; return true;
        case GT_Q6_K: *bb = 210; *be = 256; return true;
        default: return false;
    }
}

namespace {

int gguf_read_impl(const std::string& path, GgufFile* out, std::string* err) {
    auto fail = [&](int code, const char* m) { if (err) *err = m; return code; };
    std::unique_ptr<FILE, int (*)(FILE*)> fp(std::fopen(path.c_str(), "rb"), &std::fclose);
    if (!fp) return fail(-2, "file not found");
    Reader r{fp.get()};
    if (std::fseek(r.f, 0, SEEK_END) != 0) return fail(-3, "seek failed");
    const long fsize = std::ftell(r.f);
    if (fsize < 0 || std::fseek(r.f, 0, SEEK_SET) != 0) return fail(-3, "seek failed");
    r.size = (uint64_t)fsize;
    char magic[4];
    if (std::fread(magic, 1, 4, r.f) != 4 || std::memcmp(magic, "GGUF", 4) != 0) return fail(-6, "bad GGUF magic");
    out->version = r.get<uint32_t>();
    if (out->version < 2 || out->version > 3) return fail(-6, "unsupported GGUF version");
    const uint64_t n_tensors = r.get<uint64_t>();
    const uint64_t n_kv = r.get<uint64_t>();
    if (!r.ok || n_tensors > 100000 || n_kv > 100000) return fail(-6, "corrupt GGUF header");
    out->n_kv = n_kv;
    const long kv_begin = std::ftell(r.f);
    for (uint64_t i = 0; i < n_kv; ++i) {
        std::string key = r.str();
        GgufValue v;
        v.type = r.get<uint32_t>();
        if (!r.ok) return fail(-6, "truncated GGUF metadata");
        if (v.type == V_STR) {
            v.s = r.str();
        } else if (v.type == V_ARR) {
            v.arr_type = r.get<uint32_t>();
            const uint64_t n = r.get<uint64_t>();
            // every element takes at least one byte of the file (a string at least its 8-byte length)
            const uint64_t min_elem = v.arr_type == V_STR ? 8 : (scalar_size(v.arr_type) ? scalar_size(v.arr_type) : 1);
            if (!r.ok || n > r.left() / min_elem) return fail(-6, "corrupt GGUF array");
            if (v.arr_type == V_STR) {
                v.strs.reserve(n);
                for (uint64_t j = 0; j < n && r.ok; ++j) v.strs.push_back(r.str());
            } else if (scalar_size(v.arr_type)) {
                v.nums.reserve(n);
                for (uint64_t j = 0; j < n && r.ok; ++j) {
                    GgufValue tmp;
                    v.nums.push_back(read_scalar(r, v.arr_type, &tmp));
                }
            } else {
                return fail(-6, "unsupported GGUF array type");
            }
        } else if (scalar_size(v.type)) {
            v.f = read_scalar(r, v.type, &v);
            if (v.type != V_F32 && v.type != V_F64) v.f = (double)v.i;
        } else {
            return fail(-6, "unsupported GGUF value type");
        }
        if (!r.ok) return fail(-6, "truncated GGUF metadata");
        out->kv.emplace(std::move(key), std::move(v));
    }
    {
        // keep the metadata section verbatim (it is copied when the file is rewritten)
        const long kv_end = std::ftell(r.f);
        if (kv_begin < 0 || kv_end < kv_begin) return fail(-3, "ftell failed");
        out->kv_raw.resize((size_t)(kv_end - kv_begin));
        if (std::fseek(r.f, kv_begin, SEEK_SET) != 0 ||
            (!out->kv_raw.empty() && std::fread(out->kv_raw.data(), 1, out->kv_raw.size(), r.f) != out->kv_raw.size()) ||
            std::fseek(r.f, kv_end, SEEK_SET) != 0)
            return fail(-3, "read failed");
    }
    out->tensors.resize(n_tensors);
    for (uint64_t i = 0; i < n_tensors; ++i) {
        GgufTensor& t = out->tensors[i];
        t.name = r.str();
        t.n_dims = (int)r.get<uint32_t>();
        if (!r.ok || t.n_dims < 1 || t.n_dims > 4) return fail(-6, "corrupt GGUF tensor info");
        uint64_t elems = 1;
        for (int d = 0; d < t.n_dims; ++d) {
            const uint64_t n = r.get<uint64_t>();
            if (n >= (1ull << 32)) return fail(-6, "corrupt GGUF tensor shape");
            t.ne[d] = (int64_t)n;
            elems *= n;  // < 2^48 after each step: no overflow
            if (elems >= (1ull << 48)) return fail(-6, "corrupt GGUF tensor shape");
        }
        t.type = r.get<uint32_t>();
        t.offset = r.get<uint64_t>();
        if (!r.ok) return fail(-6, "truncated GGUF tensor info");
        size_t bb;
        int be;
        if (!ggml_type_block(t.type, &bb, &be)) return fail(-6, "unsupported tensor type");
        if (t.ne[0] % be) return fail(-6, "tensor row not a multiple of its block size");
        t.nbytes = (size_t)(t.nelements() / be) * bb;
        out->index[t.name] = i;
    }
    uint64_t align = 32;
    auto ita = out->kv.find("general.alignment");
    if (ita != out->kv.end()) align = ita->second.u ? ita->second.u : 32;
    if (align > (1u << 20) || (align & (align - 1))) return fail(-6, "corrupt GGUF alignment");
    out->alignment = align;
    long pos = std::ftell(r.f);
    if (pos < 0) return fail(-3, "ftell failed");
    const uint64_t data_start = ((uint64_t)pos + align - 1) / align * align;
    if (std::fseek(r.f, 0, SEEK_END) != 0) return fail(-3, "seek failed");
    const long end = std::ftell(r.f);
    if (end < 0 || (uint64_t)end < data_start) return fail(-6, "GGUF data section missing");
    const uint64_t data_size = (uint64_t)end - data_start;
    for (const auto& t : out->tensors)
        if (t.offset > data_size || t.nbytes > data_size - t.offset)
            return fail(-6, "tensor data out of file bounds (truncated file?)");
    out->data.resize(data_size);
    if (std::fseek(r.f, (long)data_start, SEEK_SET) != 0) return fail(-3, "seek failed");
    if (data_size && std::fread(out->data.data(), 1, data_size, r.f) != data_size) return fail(-3, "read failed");
    return 0;
}

}  // namespace

int gguf_read(const std::string& path, GgufFile* out, std::string* err) {
    try {
        return gguf_read_impl(path, out, err);
    } catch (const std::bad_alloc&) {
        if (err) *err = "out of memory reading the GGUF file";
        return -4;
    }
}

int gguf_write(const std::string& path, const GgufFile& f, std::string* err) {
    std::unique_ptr<FILE, int (*)(FILE*)> fp(std::fopen(path.c_str(), "wb"), &std::fclose);
    if (!fp) {
        if (err) *err = "cannot open " + path + " for writing";
        return -3;
    }
    FILE* o = fp.get();
    bool ok = true;
    auto put = [&](const void* p, size_t n) { ok = ok && (n == 0 || std::fwrite(p, 1, n, o) == n); };
    auto put64 = [&](uint64_t v) { put(&v, 8); };
    auto put32 = [&](uint32_t v) { put(&v, 4); };
    const uint64_t al = f.alignment ? f.alignment : 32;
    put("GGUF", 4);
    put32(f.version);
    put64(f.tensors.size());
    put64(f.n_kv);
    put(f.kv_raw.data(), f.kv_raw.size());
    std::vector<uint64_t> offs(f.tensors.size());
    uint64_t off = 0;
    for (size_t i = 0; i < f.tensors.size(); ++i) {
        const GgufTensor& t = f.tensors[i];
        offs[i] = off;
        put64(t.name.size());
        put(t.name.data(), t.name.size());
        put32((uint32_t)t.n_dims);
        for (int d = 0; d < t.n_dims; ++d) put64((uint64_t)t.ne[d]);
        put32(t.type);
        put64(off);
        off += (t.nbytes + al - 1) / al * al;
    }
    static const uint8_t zeros[256] = {};
    auto pad_to = [&](uint64_t pos) {
        const uint64_t p = (pos + al - 1) / al * al - pos;
        for (uint64_t k = 0; k < p; k += sizeof(zeros)) put(zeros, std::min<uint64_t>(sizeof(zeros), p - k));
    };
    const long hdr = std::ftell(o);
    if (hdr < 0) ok = false;
    pad_to((uint64_t)hdr);
    for (size_t i = 0; i < f.tensors.size() && ok; ++i) {
        const GgufTensor& t = f.tensors[i];
        if (t.offset + t.nbytes > f.data.size()) {
            if (err) *err = "tensor " + t.name + " has no data";
            return -3;
        }
        put(f.data.data() + t.offset, t.nbytes);
        pad_to(t.nbytes);
    }
    if (!ok) {
        if (err) *err = "write failed: " + path;
        return -3;
    }
    return 0;
}

namespace {

inline float h2f(const uint8_t* p) {
    uint16_t h;
    std::memcpy(&h, p, 2);
    return half_to_float(h);
}

inline void scale_min_k4(int j, const uint8_t* q, uint8_t* d, uint8_t* m) {
    if (j < 4) {
        *d = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *d = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

}  // namespace

bool dequantize(uint32_t t, const void* srcv, int64_t n, float* y) {
    const uint8_t* s = static_cast<const uint8_t*>(srcv);
    switch (t) {
        case GT_F32:
            std::memcpy(y, s, (size_t)n * 4);
            return true;
        case GT_F16:
            for (int64_t i = 0; i < n; ++i) y[i] = h2f(s + 2 * i);
            return true;
        case GT_BF16:
            for (int64_t i = 0; i < n; ++i) {
                uint32_t b = (uint32_t)(s[2 * i] | (s[2 * i + 1] << 8)) << 16;
                std::memcpy(&y[i], &b, 4);
            }
            return true;
        case GT_Q8_0:
            for (int64_t b = 0; b < n / 32; ++b, s += 34) {
                const float d = h2f(s);
                for (int j = 0; j < 32; ++j) y[b * 32 + j] = (float)(int8_t)s[2 + j] * d;
            }
            return true;
        case GT_Q4_0:
            for (int64_t b = 0; b < n / 32; ++b, s += 18) {
                const float d = h2f(s);
                for (int j = 0; j < 16; ++j) {
                    y[b * 32 + j] = (float)((s[2 + j] & 0x0F) - 8) * d;
                    y[b * 32 + j + 16] = (float)((s[2 + j] >> 4) - 8) * d;
                }
            }
            return true;
        case GT_Q4_1:
            for (int64_t b = 0; b < n / 32; ++b, s += 20) {
                const float d = h2f(s), m = h2f(s + 2);
                for (int j = 0; j < 16; ++j) {
                    y[b * 32 + j] = (float)(s[4 + j] & 0x0F) * d + m;
                    y[b * 32 + j + 16] = (float)(s[4 + j] >> 4) * d + m;
                }
            }
            return true;
        case GT_Q5_0:
            for (int64_t b = 0; b < n / 32; ++b, s += 22) {
                const float d = h2f(s);
                uint32_t qh;
                std::memcpy(&qh, s + 2, 4);
                for (int j = 0; j < 16; ++j) {
                    const uint8_t xh0 = ((qh >> (j + 0)) << 4) & 0x10;
                    const uint8_t xh1 = ((qh >> (j + 12))) & 0x10;
                    const int x0 = ((s[6 + j] & 0x0F) | xh0) - 16;
                    const int x1 = ((s[6 + j] >> 4) | xh1) - 16;
                    y[b * 32 + j] = (float)x0 * d;
                    y[b * 32 + j + 16] = (float)x1 * d;
                }
            }
            return true;
        case GT_Q5_1:
            for (int64_t b = 0; b < n / 32; ++b, s += 24) {
                const float d = h2f(s), m = h2f(s + 2);
                uint32_t qh;
                std::memcpy(&qh, s + 4, 4);
                for (int j = 0; j < 16; ++j) {
                    const uint8_t xh0 = ((qh >> (j + 0)) << 4) & 0x10;
                    const uint8_t xh1 = ((qh >> (j + 12))) & 0x10;
                    const int x0 = (s[8 + j] & 0x0F) | xh0;
                    const int x1 = (s[8 + j] >> 4) | xh1;
                    y[b * 32 + j] = (float)x0 * d + m;
                    y[b * 32 + j + 16] = (float)x1 * d + m;
                }
            }
            return true;
        case GT_Q4_K:
            for (int64_t b = 0; b < n / 256; ++b, s += 144) {
                const float d = h2f(s), dmin = h2f(s + 2);
                const uint8_t* sc = s + 4;
                const uint8_t* q = s + 16;
                float* yy = y + b * 256;
                int is = 0;
                for (int j = 0; j < 256; j += 64) {
                    uint8_t a, m;
                    scale_min_k4(is + 0, sc, &a, &m);
                    const float d1 = d * a, m1 = dmin * m;
                    scale_min_k4(is + 1, sc, &a, &m);
                    const float d2 = d * a, m2 = dmin * m;
                    for (int l = 0; l < 32; ++l) *yy++ = d1 * (q[l] & 0xF) - m1;
                    for (int l = 0; l < 32; ++l) *yy++ = d2 * (q[l] >> 4) - m2;
                    q += 32;
                    is += 2;
                }
            }
            return true;
        case GT_Q5_K:
            for (int64_t b = 0; b < n / 256; ++b, s += 176) {
                const float d = h2f(s), dmin = h2f(s + 2);
                const uint8_t* sc = s + 4;
                const uint8_t* qh = s + 16;
                const uint8_t* ql = s + 48;
                float* yy = y + b * 256;
                int is = 0;
                uint8_t u1 = 1, u2 = 2;
                for (int j = 0; j < 256; j += 64) {
                    uint8_t a, m;
                    scale_min_k4(is + 0, sc, &a, &m);
                    const float d1 = d * a, m1 = dmin * m;
                    scale_min_k4(is + 1, sc, &a, &m);
                    const float d2 = d * a, m2 = dmin * m;
                    for (int l = 0; l < 32; ++l) *yy++ = d1 * ((ql[l] & 0xF) + (qh[l] & u1 ? 16 : 0)) - m1;
                    for (int l = 0; l < 32; ++l) *yy++ = d2 * ((ql[l] >> 4) + (qh[l] & u2 ? 16 : 0)) - m2;
                    ql += 32;
                    is += 2;
                    u1 <<= 2;
                    u2 <<= 2;
                }
            }
            return true;
        case GT_Q6_K:
            for (int64_t b = 0; b < n / 256; ++b, s += 210) {
                const uint8_t* ql = s;
                const uint8_t* qh = s + 128;
                const int8_t* sc = reinterpret_cast<const int8_t*>(s + 192);
                const float d = h2f(s + 208);
                float* yy = y + b * 256;
                for (int nn = 0; nn < 256; nn += 128) {
                    for (int l = 0; l < 32; ++l) {
                        const int is = l / 16;
                        const int8_t q1 = (int8_t)((ql[l + 0] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
                        const int8_t q2 = (int8_t)((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                        const int8_t q3 = (int8_t)((ql[l + 0] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                        const int8_t q4 = (int8_t)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                        yy[l + 0] = d * sc[is + 0] * q1;
                        yy[l + 32] = d * sc[is + 2] * q2;
                        yy[l + 64] = d * sc[is + 4] * q3;
                        yy[l + 96] = d * sc[is + 6] * q4;
                    }
                    yy += 128;
                    ql += 64;
                    qh += 32;
                    sc += 8;
                }
            }
            return true;
        default:
            return false;
    }
}

}  // namespace rfb
