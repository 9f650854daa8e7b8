// q38_gguf.cpp -- GGUF checkpoint reader for the attention-core weights.
//
// Reads the GGUF container (versions 2 and 3) with the checks the
// reference's loader applies (src/gguf/mod.rs:459-533, Gguf::open): magic,
// version 2..3, at least one tensor, metadata entries of the 13 known value
// types (no nested arrays), tensor descriptors of 1..8 non-zero dimensions
// of a known ggml type whose element count is a whole number of blocks, a
// power-of-two `general.alignment` (default 32), and every tensor's bytes
// inside the file. Only F32 tensors are ever read out: the norms, conv, dt
// and A vectors that full_core and linear_core consume (ops.rs:456-467,
// 665-740, 813-940); quantized matrices are only sized.
//
// Host code, no GPU: the file is memory-mapped and the requested tensors are
// copied out; q38_bind_gguf then hands them to q38_bind_full_layer /
// q38_bind_linear_layer.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <exception>
#include <string>
#include <vector>

#include "q38_internal.h"

namespace {

constexpr uint32_t kGgufMagic = 0x46554747u;  // "GGUF", little-endian
constexpr int kGgufMaxDims = 8;
constexpr uint32_t kGgmlF32 = 0;

// Elements per block and bytes per block of the ggml tensor types a GGUF
// file may hold (the table of src/gguf/mod.rs:136-178); 0 = unknown type.
struct BlockSize {
    uint32_t elements, bytes;
};
BlockSize ggml_block(uint32_t type) {
    switch (type) {
        case 0: return {1, 4};      // F32
        case 1: return {1, 2};      // F16
        case 30: return {1, 2};     // BF16
        case 2: return {32, 18};    // Q4_0
        case 3: return {32, 20};    // Q4_1
        case 6: return {32, 22};    // Q5_0
        case 7: return {32, 24};    // Q5_1
        case 8: return {32, 34};    // Q8_0
        case 20: return {32, 18};   // IQ4_NL
        case 10: return {256, 84};  // Q2_K
        case 11: return {256, 110}; // Q3_K
        case 12: return {256, 144}; // Q4_K
        case 13: return {256, 176}; // Q5_K
        case 14: return {256, 210}; // Q6_K
        case 16: return {256, 66};  // IQ2_XXS
        case 17: return {256, 74};  // IQ2_XS
        case 18: return {256, 98};  // IQ3_XXS
        case 19: return {256, 50};  // IQ1_S
        case 21: return {256, 110}; // IQ3_S
        case 22: return {256, 82};  // IQ2_S
        case 23: return {256, 136}; // IQ4_XS
        case 29: return {256, 56};  // IQ1_M
        default: return {0, 0};
    }
}

// Scalar size of a metadata value type (0 for string, array, unknown).
uint64_t meta_scalar_size(uint32_t type) {
    switch (type) {
        case 0: case 1: case 7: return 1;   // u8, i8, bool
        case 2: case 3: return 2;           // u16, i16
        case 4: case 5: case 6: return 4;   // u32, i32, f32
        case 10: case 11: case 12: return 8;  // u64, i64, f64
        default: return 0;
    }
}
constexpr uint32_t kMetaU32 = 4, kMetaString = 8, kMetaArray = 9, kMetaTypes = 13;

struct Tensor {
    std::string name;
    uint32_t n_dims = 0;
    uint64_t shape[kGgufMaxDims] = {};
    uint32_t type = 0;
    uint64_t offset = 0, elements = 0, nbytes = 0;
    const unsigned char *data = nullptr;
};

// Little-endian cursor over the mapped bytes; any read past the end fails
// the whole parse.
struct Cursor {
    const unsigned char *base;
    uint64_t size, at = 0;
    bool failed = false;
    const unsigned char *take(uint64_t n) {
        if (failed || n > size - at) {
            failed = true;
            return nullptr;
        }
        const unsigned char *p = base + at;
        at += n;
        return p;
    }
    uint32_t u32() {
        const unsigned char *p = take(4);
        uint32_t v = 0;
        if (p) std::memcpy(&v, p, 4);
        return v;
    }
    uint64_t u64() {
        const unsigned char *p = take(8);
        uint64_t v = 0;
        if (p) std::memcpy(&v, p, 8);
        return v;
    }
    bool string(std::string *out) {
        const uint64_t n = u64();
        const unsigned char *p = take(n);
        if (!p) return false;
        if (out) out->assign(reinterpret_cast<const char *>(p), size_t(n));
        return true;
    }
    bool skip_values(uint32_t type, uint64_t count) {
        if (const uint64_t sz = meta_scalar_size(type)) {
            if (count > UINT64_MAX / sz) return false;
            return take(count * sz) != nullptr || count == 0;
        }
        if (type != kMetaString) return false;
        for (uint64_t i = 0; i < count; ++i)
            if (!string(nullptr)) return false;
        return true;
    }
};

class GgufFile {
  public:
    ~GgufFile() {
        if (map_ && map_ != MAP_FAILED) munmap(map_, size_);
        if (fd_ >= 0) close(fd_);
    }
    // Returns an empty string on success, else the reason.
    std::string open(const char *path) {
        fd_ = ::open(path, O_RDONLY);
        if (fd_ < 0) return std::string("cannot open ") + path;
        struct stat sb;
        if (fstat(fd_, &sb) != 0) return "cannot stat the file";
        size_ = uint64_t(sb.st_size);
        if (size_ < 24) return "file smaller than 24 bytes";
        map_ = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
        if (map_ == MAP_FAILED) return "cannot map the file";
        Cursor c{static_cast<const unsigned char *>(map_), size_};
        const uint32_t magic = c.u32(), version = c.u32();
        const uint64_t n_tensors = c.u64(), n_meta = c.u64();
        if (magic != kGgufMagic || version < 2 || version > 3 || n_tensors == 0)
            return "unsupported or corrupt GGUF header";
        uint32_t alignment = 32;
        for (uint64_t m = 0; m < n_meta; ++m) {
            std::string key;
            if (!c.string(&key)) return "metadata key";
            const uint32_t type = c.u32();
            if (c.failed || type >= kMetaTypes) return "unknown meta type";
            if (type == kMetaArray) {
                const uint32_t elem = c.u32();
                const uint64_t n = c.u64();
                if (c.failed || elem >= kMetaTypes) return "unknown array type";
                if (elem == kMetaArray) return "nested arrays not allowed";
                if (!c.skip_values(elem, n)) return "array value";
            } else if (type == kMetaString) {
                if (!c.string(nullptr)) return "meta string";
            } else {
                const unsigned char *p = c.take(meta_scalar_size(type));
                if (!p) return "scalar value";
                if (key == "general.alignment" && type == kMetaU32) {
                    uint32_t a;
                    std::memcpy(&a, p, 4);
                    if (a == 0 || (a & (a - 1)) != 0) return "invalid GGUF alignment";
                    alignment = a;
                }
            }
        }
        // A descriptor takes at least 32 bytes, which bounds a corrupt count.
        if (n_tensors > (size_ - c.at) / 32) return "tensor descriptors past end of file";
        tensors_.resize(size_t(n_tensors));
        for (Tensor &t : tensors_) {
            if (!c.string(&t.name)) return "tensor name";
            t.n_dims = c.u32();
            if (c.failed || t.n_dims == 0 || t.n_dims > kGgufMaxDims) return "tensor n_dims";
            t.elements = 1;
            for (uint32_t d = 0; d < t.n_dims; ++d) {
                t.shape[d] = c.u64();
                if (t.shape[d] == 0 || t.elements > UINT64_MAX / t.shape[d])
                    return "tensor shape overflow";
                t.elements *= t.shape[d];
            }
            t.type = c.u32();
            t.offset = c.u64();
            if (c.failed) return "tensor trailer";
            const BlockSize b = ggml_block(t.type);
            if (b.elements == 0) return "unknown tensor type";
            if (t.shape[0] % b.elements != 0 || t.elements % b.elements != 0 ||
                t.elements / b.elements > UINT64_MAX / b.bytes)
                return "tensor bytes overflow";
            t.nbytes = t.elements / b.elements * b.bytes;
        }
        const uint64_t data_offset = (c.at + alignment - 1) & ~uint64_t(alignment - 1);
        if (data_offset > size_) return "tensor data begins past end of file";
        for (Tensor &t : tensors_) {
            if (t.offset > size_ - data_offset || t.nbytes > size_ - data_offset - t.offset)
                return "tensor outside GGUF file";
            t.data = static_cast<const unsigned char *>(map_) + data_offset + t.offset;
        }
        return {};
    }
    const Tensor *find(const std::string &name) const {
        for (const Tensor &t : tensors_)
            if (t.name == name) return &t;
        return nullptr;
    }

  private:
    int fd_ = -1;
    void *map_ = nullptr;
    uint64_t size_ = 0;
    std::vector<Tensor> tensors_;
};

int gguf_fail(const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    q38::record_error(buf);
    return Q38_ERR_ARG;
}

// Copies F32 tensor `name` (exactly n elements) to dst.
int read_f32(const GgufFile &f, const std::string &name, float *dst, uint64_t n) {
    const Tensor *t = f.find(name);
    if (!t) return gguf_fail("tensor %s not found", name.c_str());
    if (t->type != kGgmlF32) return gguf_fail("tensor %s is not F32 (type %u)", name.c_str(), t->type);
    if (t->elements != n)
        return gguf_fail("tensor %s has %llu elements, expected %llu", name.c_str(),
                         static_cast<unsigned long long>(t->elements),
                         static_cast<unsigned long long>(n));
    std::memcpy(dst, t->data, size_t(n) * sizeof(float));
    return Q38_OK;
}

}  // namespace

extern "C" int q38_gguf_read_f32(const char *path, const char *name, float *dst, int64_t n) {
    if (!path || !name || !dst || n <= 0) return gguf_fail("null argument or non-positive count");
    try {
        GgufFile f;
        const std::string err = f.open(path);
        if (!err.empty()) return gguf_fail("invalid GGUF: %s", err.c_str());
        return read_f32(f, name, dst, uint64_t(n));
    } catch (const std::exception &e) {
        return gguf_fail("GGUF read failed: %s", e.what());
    }
}

namespace {
int bind_gguf(q38_ctx *ctx, const char *path, int first_layer, int last_layer);
}

extern "C" int q38_bind_gguf(q38_ctx *ctx, const char *path, int first_layer, int last_layer) {
    try {
        return bind_gguf(ctx, path, first_layer, last_layer);
    } catch (const std::exception &e) {
        return gguf_fail("GGUF binding failed: %s", e.what());
    }
}

namespace {
int bind_gguf(q38_ctx *ctx, const char *path, int first_layer, int last_layer) {
    if (!ctx || !path) return gguf_fail("null argument");
    if (first_layer < 0 || last_layer > 64 || first_layer > last_layer)
        return gguf_fail("layer range [%d, %d] outside 0..64", first_layer, last_layer);
    GgufFile f;
    const std::string err = f.open(path);
    if (!err.empty()) return gguf_fail("invalid GGUF: %s", err.c_str());
    const q38_geom &g = ctx->geom;
    const uint64_t qkv_dim = uint64_t(2 * g.linear_qk_heads + g.linear_v_heads) * g.linear_head_dim;
    for (int layer = first_layer; layer <= last_layer; ++layer) {
        // Tensor names of bind_layer (ops.rs:53-100).
        const std::string pre = "blk." + std::to_string(layer) + ".";
        if (q38::is_full_attention(layer)) {
            std::vector<float> qn(g.attn_head_dim), kn(g.attn_head_dim);
            if (int rc = read_f32(f, pre + "attn_q_norm.weight", qn.data(), qn.size())) return rc;
            if (int rc = read_f32(f, pre + "attn_k_norm.weight", kn.data(), kn.size())) return rc;
            if (int rc = q38_bind_full_layer(ctx, layer, qn.data(), kn.data())) return rc;
        } else {
            std::vector<float> conv(qkv_dim * g.conv_kernel), dt(g.linear_v_heads),
                a(g.linear_v_heads), norm(g.linear_head_dim);
            if (int rc = read_f32(f, pre + "ssm_conv1d.weight", conv.data(), conv.size())) return rc;
            if (int rc = read_f32(f, pre + "ssm_dt.bias", dt.data(), dt.size())) return rc;
            if (int rc = read_f32(f, pre + "ssm_a", a.data(), a.size())) return rc;
            if (int rc = read_f32(f, pre + "ssm_norm.weight", norm.data(), norm.size())) return rc;
            if (int rc = q38_bind_linear_layer(ctx, layer, conv.data(), dt.data(), a.data(),
                                               norm.data()))
                return rc;
        }
    }
    return Q38_OK;
}
}  // namespace

// A projection matrix straight from the checkpoint: the 2-D tensor `name`
// (shape [width, rows], as tensor_gemv_* require, src/kernel/tensor.rs:
// 1095-1110) handed to q38_weight_create.
extern "C" int q38_weight_from_gguf(q38_ctx *ctx, const char *path, const char *name,
                                    q38_weight **out) {
    if (!ctx || !path || !name || !out) return gguf_fail("null argument");
    *out = nullptr;
    try {
        GgufFile f;
        const std::string err = f.open(path);
        if (!err.empty()) return gguf_fail("invalid GGUF: %s", err.c_str());
        const Tensor *t = f.find(name);
        if (!t) return gguf_fail("tensor %s not found", name);
        if (t->n_dims != 2) return gguf_fail("tensor %s is not 2-dimensional", name);
        return q38_weight_create(ctx, int(t->type), int64_t(t->shape[0]), int64_t(t->shape[1]),
                                 t->data, size_t(t->nbytes), out);
    } catch (const std::exception &e) {
        return gguf_fail("GGUF read failed: %s", e.what());
    }
}
