// On-disk formats of the reference's weights and tensors:
//
//  * GGUF weight files (GGUFModel::load / get / metadata getters,
//    src/objects_runtime/gguf_loader.{hpp,cpp}): header, metadata and tensor
//    directory parsed on the host; tensor bytes read on demand and dequantised
//    on the device to f32 / bf16 (F32, F16, BF16, Q8_0, Q4_0, Q4_1, Q4_K --
//    every dtype the reference's converter writes, gguf_schema.py:204-300),
//    or loaded straight into a convolution's packed layout.
//  * SAMT raw tensors (save_raw_tensor / load_raw_tensor,
//    src/objects_runtime/common.cpp:59-119): "SAMT" | int32 ndims | int64
//    ne[ndims] | int32 ggml type | data.
//
// Dequantisation follows GGML's per-block definitions (ggml-quants.c, the
// published block formats of ggml-org/ggml) in f32 with separate multiply
// and add, as GGML's portable build computes them:
//   Q8_0 {f16 d, int8 q[32]}:               y = q * d
//   Q4_0 {f16 d, u8 q[16]}:                 y[j] = (lo(q[j]) - 8) * d, y[j+16] = (hi(q[j]) - 8) * d
//   Q4_1 {f16 d, f16 m, u8 q[16]}:          y[j] = lo(q[j]) * d + m, y[j+16] = hi(q[j]) * d + m
//   Q4_K {f16 d, f16 dmin, u8 sc[12], u8 q[128]}: 8 sub-blocks of 32 with 6-bit scale s and min m,
//       y = (d * s) * nibble - (dmin * m); sub-block 2i takes the low nibbles of q[32i..32i+31],
//       sub-block 2i+1 the high ones.
#include "s3dsp_internal.h"

#include <cstdio>
#include <memory>
#include <string>
#include <unordered_map>
#include <vector>

using namespace s3dsp;

namespace {

// ggml type ids (ggml.h of the pinned ggml; gguf-py GGMLQuantizationType)
enum : int32_t {
    kF32 = 0, kF16 = 1, kQ4_0 = 2, kQ4_1 = 3, kQ8_0 = 8, kQ4_K = 12,
    kI8 = 24, kI16 = 25, kI32 = 26, kI64 = 27, kF64 = 28, kBF16 = 30
};

// {bytes per block, elements per block} of a ggml type, {0, 0} when unknown
struct TypeSize {
    int64_t bytes, block;
};
TypeSize type_size(int32_t t) {
    switch (t) {
        case kF32: return {4, 1};
        case kF16: return {2, 1};
        case kBF16: return {2, 1};
        case kQ8_0: return {34, 32};
        case kQ4_0: return {18, 32};
        case kQ4_1: return {20, 32};
        case kQ4_K: return {144, 256};
        case kI8: return {1, 1};
        case kI16: return {2, 1};
        case kI32: return {4, 1};
        case kI64: return {8, 1};
        case kF64: return {8, 1};
        default: return {0, 0};
    }
}
bool dequantisable(int32_t t) {
    return t == kF32 || t == kF16 || t == kBF16 || t == kQ8_0 || t == kQ4_0 || t == kQ4_1 || t == kQ4_K;
}

// ---------------------------------------------------------------------------
// device dequantisation: one thread per output element
// ---------------------------------------------------------------------------
__device__ __forceinline__ float h2f(const uint8_t* p) {
    return __half2float(__ushort_as_half((unsigned short)(p[0] | p[1] << 8)));
}

template <typename OutT>
__device__ __forceinline__ void put(OutT* out, int64_t i, float v);
template <>
__device__ __forceinline__ void put<float>(float* out, int64_t i, float v) { out[i] = v; }
template <>
__device__ __forceinline__ void put<__nv_bfloat16>(__nv_bfloat16* out, int64_t i, float v) {
    out[i] = __float2bfloat16_rn(v);
}

template <typename OutT>
__global__ void dequant_kernel(const uint8_t* __restrict__ src, int32_t type, int64_t n, OutT* __restrict__ out) {
    pdl_wait();
    pdl_trigger();
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        float v;
        switch (type) {
            case kF32: v = reinterpret_cast<const float*>(src)[i]; break;
            case kF16: v = h2f(src + 2 * i); break;
            case kBF16:
                v = __uint_as_float((uint32_t)(src[2 * i] | src[2 * i + 1] << 8) << 16);
                break;
            case kQ8_0: {
                const uint8_t* b = src + (i >> 5) * 34;
                v = __fmul_rn((float)(int8_t)b[2 + (i & 31)], h2f(b));
                break;
            }
            case kQ4_0: {
                const uint8_t* b = src + (i >> 5) * 18;
                const int j = (int)(i & 31);
                const int q = j < 16 ? (b[2 + j] & 15) : (b[2 + j - 16] >> 4);
                v = __fmul_rn((float)(q - 8), h2f(b));
                break;
            }
            case kQ4_1: {
                const uint8_t* b = src + (i >> 5) * 20;
                const int j = (int)(i & 31);
                const int q = j < 16 ? (b[4 + j] & 15) : (b[4 + j - 16] >> 4);
                v = __fadd_rn(__fmul_rn((float)q, h2f(b)), h2f(b + 2));
                break;
            }
            default: {  // kQ4_K
                const uint8_t* b = src + (i >> 8) * 144;
                const int j = (int)(i & 255);
                const int sub = j >> 5, l = j & 31;
                const uint8_t* sc = b + 4;
                int s, m;
                if (sub < 4) {
                    s = sc[sub] & 63;
                    m = sc[sub + 4] & 63;
                } else {
                    s = (sc[sub + 4] & 15) | (sc[sub - 4] >> 6) << 4;
                    m = (sc[sub + 4] >> 4) | (sc[sub] >> 6) << 4;
                }
                const uint8_t qb = b[16 + (sub >> 1) * 32 + l];
                const int q = (sub & 1) ? (qb >> 4) : (qb & 15);
                v = __fsub_rn(__fmul_rn(__fmul_rn(h2f(b), (float)s), (float)q), __fmul_rn(h2f(b + 2), (float)m));
                break;
            }
        }
        put(out, i, v);
    }
}

// ---------------------------------------------------------------------------
// GGUF parsing (little-endian, versions 2 and 3)
// ---------------------------------------------------------------------------
enum : uint32_t {
    kU8 = 0, kI8v = 1, kU16 = 2, kI16v = 3, kU32 = 4, kI32v = 5, kF32v = 6, kBool = 7, kStr = 8, kArr = 9,
    kU64 = 10, kI64v = 11, kF64v = 12
};
int64_t scalar_size(uint32_t t) {
    switch (t) {
        case kU8: case kI8v: case kBool: return 1;
        case kU16: case kI16v: return 2;
        case kU32: case kI32v: case kF32v: return 4;
        case kU64: case kI64v: case kF64v: return 8;
        default: return 0;
    }
}

struct Value {
    uint32_t type = 0;
    uint32_t elem_type = 0;            // arrays
    std::vector<uint8_t> raw;          // scalar bytes, or the packed array of scalars
    std::string str;                   // string
    std::vector<std::string> strs;     // array of strings
    uint64_t count = 0;                // array length
};

struct Reader {
    FILE* f;
    uint64_t size;
    bool ok = true;
    bool get(void* p, uint64_t n) {
        if (!ok || n > size || fread(p, 1, n, f) != n) ok = false;
        return ok;
    }
    template <typename T>
    T val() {
        T v{};
        get(&v, sizeof v);
        return v;
    }
    std::string str() {
        const uint64_t n = val<uint64_t>();
        if (!ok || n > size) {
            ok = false;
            return {};
        }
        std::string s(n, '\0');
        get(s.data(), n);
        return s;
    }
};

}  // namespace

struct s3dsp_gguf {
    std::string path;
    uint32_t version = 0;
    uint64_t alignment = 32, data_offset = 0, file_size = 0;
    std::unordered_map<std::string, Value> kv;
    struct Tensor {
        std::string name;
        int32_t type = 0, n_dims = 0;
        int64_t ne[4] = {1, 1, 1, 1};
        uint64_t offset = 0, nbytes = 0;
    };
    std::vector<Tensor> tensors;
    std::unordered_map<std::string, int64_t> index;
};

namespace {

s3d_status parse_gguf(s3dsp_gguf& g, FILE* f, char* error, uint64_t error_capacity) {
    Reader r{f, g.file_size};
    const uint32_t magic = r.val<uint32_t>();
    if (!r.ok || magic != 0x46554747u) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "%s: not a GGUF file", g.path.c_str());
    g.version = r.val<uint32_t>();
    if (g.version != 2 && g.version != 3)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "%s: GGUF version %u", g.path.c_str(), g.version);
    const uint64_t n_tensors = r.val<uint64_t>(), n_kv = r.val<uint64_t>();
    if (!r.ok || n_tensors > g.file_size / 16 || n_kv > g.file_size / 8)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "%s: corrupt header", g.path.c_str());
    for (uint64_t i = 0; i < n_kv && r.ok; ++i) {
        std::string key = r.str();
        Value v;
        v.type = r.val<uint32_t>();
        if (v.type == kStr) {
            v.str = r.str();
        } else if (v.type == kArr) {
            v.elem_type = r.val<uint32_t>();
            v.count = r.val<uint64_t>();
            if (!r.ok || v.count > g.file_size) break;
            if (v.elem_type == kStr) {
                v.strs.reserve(v.count);
                for (uint64_t k = 0; k < v.count && r.ok; ++k) v.strs.push_back(r.str());
            } else {
                const int64_t es = scalar_size(v.elem_type);
                if (es == 0 || v.count * es > g.file_size) {
                    r.ok = false;
                    break;
                }
                v.raw.resize(v.count * es);
                r.get(v.raw.data(), v.raw.size());
            }
        } else {
            const int64_t es = scalar_size(v.type);
            if (es == 0) {
                r.ok = false;
                break;
            }
            v.raw.resize(es);
            r.get(v.raw.data(), es);
        }
        g.kv[key] = std::move(v);
    }
    if (!r.ok) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "%s: corrupt metadata", g.path.c_str());
    const auto al = g.kv.find("general.alignment");
    if (al != g.kv.end() && al->second.type == kU32) {
        uint32_t a;
        std::memcpy(&a, al->second.raw.data(), 4);
        if (a == 0 || (a & (a - 1)))
            return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "%s: alignment %u", g.path.c_str(), a);
        g.alignment = a;
    }
    g.tensors.resize(n_tensors);
    for (uint64_t i = 0; i < n_tensors && r.ok; ++i) {
        s3dsp_gguf::Tensor& t = g.tensors[i];
        t.name = r.str();
        t.n_dims = (int32_t)r.val<uint32_t>();
        if (!r.ok || t.n_dims < 1 || t.n_dims > 4)
            return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "%s: tensor %llu has %d dims", g.path.c_str(),
                        (unsigned long long)i, t.n_dims);
        int64_t n = 1;
        for (int d = 0; d < t.n_dims; ++d) {
            t.ne[d] = (int64_t)r.val<uint64_t>();
            if (t.ne[d] < 0 || (t.ne[d] > 0 && n > INT64_MAX / t.ne[d])) r.ok = false;
            else n *= t.ne[d];
        }
        t.type = (int32_t)r.val<uint32_t>();
        t.offset = r.val<uint64_t>();
        const TypeSize ts = type_size(t.type);
        if (!r.ok || ts.block == 0 || t.ne[0] % ts.block)
            return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "%s: tensor '%s' type %d / shape unsupported",
                        g.path.c_str(), t.name.c_str(), t.type);
        t.nbytes = (uint64_t)(n / ts.block * ts.bytes);
        if (!g.index.emplace(t.name, (int64_t)i).second)
            return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "%s: duplicate tensor '%s'", g.path.c_str(),
                        t.name.c_str());
    }
    if (!r.ok) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "%s: corrupt tensor directory", g.path.c_str());
    const long pos = ftell(f);
    g.data_offset = ((uint64_t)pos + g.alignment - 1) / g.alignment * g.alignment;
    for (const auto& t : g.tensors)
        if (t.offset % g.alignment || g.data_offset + t.offset + t.nbytes > g.file_size)
            return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "%s: tensor '%s' outside the file", g.path.c_str(),
                        t.name.c_str());
    return S3D_OK;
}

const Value* find_kv(const s3dsp_gguf* g, const char* key) {
    if (!g || !key) return nullptr;
    const auto it = g->kv.find(key);
    return it == g->kv.end() ? nullptr : &it->second;
}

s3d_status read_bytes(const std::string& path, uint64_t offset, void* dst, uint64_t n, char* error,
                      uint64_t error_capacity) {
    FILE* f = fopen(path.c_str(), "rb");
    if (!f) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "cannot open %s", path.c_str());
    const bool ok = fseeko(f, (off_t)offset, SEEK_SET) == 0 && fread(dst, 1, n, f) == n;
    fclose(f);
    return ok ? S3D_OK : fail(error, error_capacity, S3D_INTERNAL_ERROR, "short read of %s", path.c_str());
}

s3d_status dequantize_device(s3dsp_context* ctx, int32_t type, const void* d_src, int64_t n, uint32_t dtype,
                             void* d_out, char* error, uint64_t error_capacity) {
    if (!dequantisable(type))
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "ggml type %d cannot be converted to float", type);
    if (dtype != S3DSP_F32 && dtype != S3DSP_BF16)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "output dtype must be F32 or BF16");
    if (n % type_size(type).block)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "%lld elements are not whole blocks", (long long)n);
    if (n == 0) return S3D_OK;
    const int64_t g = (n + 255) / 256;
    const int grid = (int)(g < ctx->sm_count * 16 ? g : ctx->sm_count * 16);
    const uint8_t* src = static_cast<const uint8_t*>(d_src);
    if (dtype == S3DSP_F32)
        launch_pdl(dequant_kernel<float>, dim3(grid), dim3(256), 0, ctx->stream, src, type, n,
                   static_cast<float*>(d_out));
    else
        launch_pdl(dequant_kernel<__nv_bfloat16>, dim3(grid), dim3(256), 0, ctx->stream, src, type, n,
                   static_cast<__nv_bfloat16*>(d_out));
    S3DSP_LAUNCH_CHECK("dequant_kernel");
    return S3D_OK;
}

constexpr uint32_t kSamtMagic = 0x544D4153u;  // "SAMT" little-endian

}  // namespace

extern "C" {

S3DSP_API s3d_status s3dsp_gguf_open(const char* path, s3dsp_gguf** out, char* error, uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!path || !out) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    *out = nullptr;
    FILE* f = fopen(path, "rb");
    if (!f) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "failed to load GGUF: %s", path);
    std::unique_ptr<s3dsp_gguf> g(new (std::nothrow) s3dsp_gguf);
    if (!g) {
        fclose(f);
        return fail(error, error_capacity, S3D_OUT_OF_MEMORY, "host allocation");
    }
    g->path = path;
    fseeko(f, 0, SEEK_END);
    g->file_size = (uint64_t)ftello(f);
    fseeko(f, 0, SEEK_SET);
    const s3d_status st = parse_gguf(*g, f, error, error_capacity);
    fclose(f);
    if (st != S3D_OK) return st;
    *out = g.release();
    return S3D_OK;
}

S3DSP_API void s3dsp_gguf_close(s3dsp_gguf* g) { delete g; }

S3DSP_API int64_t s3dsp_gguf_n_tensors(const s3dsp_gguf* g) { return g ? (int64_t)g->tensors.size() : -1; }

S3DSP_API int64_t s3dsp_gguf_find(const s3dsp_gguf* g, const char* name) {
    if (!g || !name) return -1;
    const auto it = g->index.find(name);
    return it == g->index.end() ? -1 : it->second;
}

S3DSP_API s3d_status s3dsp_gguf_tensor_info(const s3dsp_gguf* g, int64_t index, const char** name, int32_t* type,
                                            int32_t* n_dims, int64_t* ne, uint64_t* nbytes) {
    if (!g || index < 0 || index >= (int64_t)g->tensors.size()) return S3D_INVALID_ARGUMENT;
    const auto& t = g->tensors[(size_t)index];
    if (name) *name = t.name.c_str();
    if (type) *type = t.type;
    if (n_dims) *n_dims = t.n_dims;
    if (ne)
        for (int d = 0; d < 4; ++d) ne[d] = t.ne[d];
    if (nbytes) *nbytes = t.nbytes;
    return S3D_OK;
}

// Integer metadata as GGUFModel::u32 reads it (gguf_loader.cpp:89-99): the
// four 32/64-bit integer types convert, anything else gives the default.
S3DSP_API uint32_t s3dsp_gguf_u32(const s3dsp_gguf* g, const char* key, uint32_t def) {
    const Value* v = find_kv(g, key);
    if (!v) return def;
    switch (v->type) {
        case kU32: case kI32v: {
            uint32_t x;
            std::memcpy(&x, v->raw.data(), 4);
            return x;
        }
        case kU64: case kI64v: {
            uint64_t x;
            std::memcpy(&x, v->raw.data(), 8);
            return (uint32_t)x;
        }
        default: return def;
    }
}

S3DSP_API int32_t s3dsp_gguf_i32(const s3dsp_gguf* g, const char* key, int32_t def) {
    return (int32_t)s3dsp_gguf_u32(g, key, (uint32_t)def);
}

S3DSP_API float s3dsp_gguf_f32(const s3dsp_gguf* g, const char* key, float def) {
    const Value* v = find_kv(g, key);
    if (!v || v->type != kF32v) return def;
    float x;
    std::memcpy(&x, v->raw.data(), 4);
    return x;
}

// String metadata: copies up to cap - 1 bytes and a NUL; returns the full
// length, or -1 when the key is missing or not a string.
S3DSP_API int64_t s3dsp_gguf_str(const s3dsp_gguf* g, const char* key, char* buf, uint64_t cap) {
    const Value* v = find_kv(g, key);
    if (!v || v->type != kStr) return -1;
    if (buf && cap) {
        const size_t n = v->str.size() < cap - 1 ? v->str.size() : (size_t)(cap - 1);
        std::memcpy(buf, v->str.data(), n);
        buf[n] = '\0';
    }
    return (int64_t)v->str.size();
}

// Length of an array, or -1 when the key is missing or not an array.
S3DSP_API int64_t s3dsp_gguf_array_len(const s3dsp_gguf* g, const char* key) {
    const Value* v = find_kv(g, key);
    return v && v->type == kArr ? (int64_t)v->count : -1;
}

// Element `i` of a string array (as s3dsp_gguf_str).
S3DSP_API int64_t s3dsp_gguf_str_array(const s3dsp_gguf* g, const char* key, int64_t i, char* buf, uint64_t cap) {
    const Value* v = find_kv(g, key);
    if (!v || v->type != kArr || v->elem_type != kStr || i < 0 || i >= (int64_t)v->strs.size()) return -1;
    const std::string& s = v->strs[(size_t)i];
    if (buf && cap) {
        const size_t n = s.size() < cap - 1 ? s.size() : (size_t)(cap - 1);
        std::memcpy(buf, s.data(), n);
        buf[n] = '\0';
    }
    return (int64_t)s.size();
}

// An int32 / uint32 array (GGUFModel::i32_array, gguf_loader.cpp:128-141):
// copies up to cap values, returns the length, or -1 (missing or other type).
S3DSP_API int64_t s3dsp_gguf_i32_array(const s3dsp_gguf* g, const char* key, int32_t* out, int64_t cap) {
    const Value* v = find_kv(g, key);
    if (!v || v->type != kArr || (v->elem_type != kI32v && v->elem_type != kU32)) return -1;
    const int64_t n = (int64_t)v->count;
    if (out) std::memcpy(out, v->raw.data(), 4 * (size_t)(n < cap ? n : cap));
    return n;
}

S3DSP_API s3d_status s3dsp_gguf_read(const s3dsp_gguf* g, int64_t index, void* h_dst, uint64_t capacity, char* error,
                                     uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!g || !h_dst || index < 0 || index >= (int64_t)g->tensors.size())
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "bad tensor index or NULL argument");
    const auto& t = g->tensors[(size_t)index];
    if (capacity < t.nbytes)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "'%s' needs %llu bytes", t.name.c_str(),
                    (unsigned long long)t.nbytes);
    return read_bytes(g->path, g->data_offset + t.offset, h_dst, t.nbytes, error, error_capacity);
}

S3DSP_API s3d_status s3dsp_dequantize(s3dsp_context* ctx, int32_t ggml_type, const void* d_src, int64_t n,
                                      uint32_t dtype, void* d_out, char* error, uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || (n > 0 && (!d_src || !d_out)) || n < 0)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument or negative count");
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    return dequantize_device(ctx, ggml_type, d_src, n, dtype, d_out, error, error_capacity);
}

S3DSP_API s3d_status s3dsp_gguf_load(s3dsp_context* ctx, const s3dsp_gguf* g, int64_t index, uint32_t dtype,
                                     void* d_out, int64_t capacity, char* error, uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || !g || !d_out || index < 0 || index >= (int64_t)g->tensors.size())
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "bad tensor index or NULL argument");
    const auto& t = g->tensors[(size_t)index];
    const int64_t n = t.ne[0] * t.ne[1] * t.ne[2] * t.ne[3];
    if (capacity < n)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "'%s' has %lld elements, capacity %lld",
                    t.name.c_str(), (long long)n, (long long)capacity);
    if (!dequantisable(t.type))
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "'%s': ggml type %d is not a float type",
                    t.name.c_str(), t.type);
    std::vector<uint8_t> host(t.nbytes);
    S3DSP_TRY(read_bytes(g->path, g->data_offset + t.offset, host.data(), t.nbytes, error, error_capacity));
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    void* staged = nullptr;
    S3DSP_CUDA(s3dsp::malloc_async(&staged, t.nbytes > 0 ? t.nbytes : 16, ctx->stream), "cudaMallocAsync");
    cudaError_t e = cudaMemcpyAsync(staged, host.data(), t.nbytes, cudaMemcpyHostToDevice, ctx->stream);
    s3d_status st = S3D_OK;
    if (e == cudaSuccess) st = dequantize_device(ctx, t.type, staged, n, dtype, d_out, error, error_capacity);
    cudaFreeAsync(staged, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);  // the host buffer dies on return
    if (e != cudaSuccess) return cuda_fail(error, error_capacity, e, "gguf load");
    return st;
}

// A GGUF conv / linear weight straight into the layout a conv of `precision`
// consumes (s3dsp_weights_pack), after checking the stored shape against the
// layout: MESH_PACKED ne = {cout*cin, kvol}, SLAT_ROW ne = {27*cin, cout},
// LINEAR ne = {cin, cout}.
S3DSP_API s3d_status s3dsp_gguf_load_weights(s3dsp_context* ctx, const s3dsp_gguf* g, const char* name,
                                             uint32_t layout, int32_t kvol, int64_t cin, int64_t cout,
                                             uint32_t precision, void* d_dst, char* error,
                                             uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!ctx || !g || !name || !d_dst) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    const int64_t index = s3dsp_gguf_find(g, name);
    if (index < 0) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "tensor '%s' not in %s", name, g->path.c_str());
    const auto& t = g->tensors[(size_t)index];
    int64_t want0, want1;
    if (layout == S3DSP_LAYOUT_MESH_PACKED) want0 = cout * cin, want1 = kvol;
    else if (layout == S3DSP_LAYOUT_SLAT_ROW) want0 = 27 * cin, want1 = cout;
    else if (layout == S3DSP_LAYOUT_LINEAR) want0 = cin, want1 = cout;
    else return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "layout %u is not a GGUF layout", layout);
    if (t.ne[0] != want0 || t.ne[1] != want1 || t.ne[2] != 1 || t.ne[3] != 1)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "'%s' has ne {%lld, %lld}, layout wants {%lld, %lld}",
                    name, (long long)t.ne[0], (long long)t.ne[1], (long long)want0, (long long)want1);
    const int64_t n = want0 * want1;
    S3DSP_CUDA(cudaSetDevice(ctx->device), "cudaSetDevice");
    float* f32 = nullptr;
    S3DSP_CUDA(s3dsp::malloc_async(&f32, 4 * (size_t)n, ctx->stream), "cudaMallocAsync");
    s3d_status st = s3dsp_gguf_load(ctx, g, index, S3DSP_F32, f32, n, error, error_capacity);
    if (st == S3D_OK)
        st = s3dsp_weights_pack(ctx, f32, S3DSP_F32, 0, layout, kvol, cin, cout, precision, d_dst, error,
                                error_capacity);
    cudaFreeAsync(f32, ctx->stream);
    return st;
}

S3DSP_API s3d_status s3dsp_samt_info(const char* path, int32_t* n_dims, int64_t* ne, int32_t* ggml_type,
                                     uint64_t* nbytes, char* error, uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!path) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "NULL argument");
    FILE* f = fopen(path, "rb");
    if (!f) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "cannot open %s", path);
    uint32_t magic = 0;
    int32_t nd = 0, type = 0;
    int64_t dims[8] = {0};
    bool ok = fread(&magic, 4, 1, f) == 1 && magic == kSamtMagic && fread(&nd, 4, 1, f) == 1 && nd > 0 && nd <= 8;
    ok = ok && fread(dims, 8, (size_t)nd, f) == (size_t)nd && fread(&type, 4, 1, f) == 1;
    fclose(f);
    if (!ok) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "%s: not a SAMT tensor", path);
    if (type == 30) type = kI32;  // writers used both ids for int32 (common.cpp:108-110)
    const TypeSize ts = type_size(type);
    int64_t n = 1;
    for (int d = 0; d < nd; ++d) {
        if (dims[d] < 0) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "%s: negative extent", path);
        n *= dims[d];
    }
    if (ts.block == 0 || n % ts.block)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "%s: ggml type %d unsupported", path, type);
    if (n_dims) *n_dims = nd;
    if (ne)
        for (int d = 0; d < nd; ++d) ne[d] = dims[d];
    if (ggml_type) *ggml_type = type;
    if (nbytes) *nbytes = (uint64_t)(n / ts.block * ts.bytes);
    return S3D_OK;
}

S3DSP_API s3d_status s3dsp_samt_read(const char* path, void* h_dst, uint64_t capacity, char* error,
                                     uint64_t error_capacity) {
    int32_t nd = 0;
    uint64_t nbytes = 0;
    S3DSP_TRY(s3dsp_samt_info(path, &nd, nullptr, nullptr, &nbytes, error, error_capacity));
    if (!h_dst || capacity < nbytes)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "%s needs %llu bytes", path, (unsigned long long)nbytes);
    return read_bytes(path, 12 + 8 * (uint64_t)nd, h_dst, nbytes, error, error_capacity);
}

S3DSP_API s3d_status s3dsp_samt_write(const char* path, int32_t n_dims, const int64_t* ne, int32_t ggml_type,
                                      const void* data, uint64_t nbytes, char* error, uint64_t error_capacity) {
    clear_error(error, error_capacity);
    if (!path || !ne || (nbytes && !data) || n_dims <= 0 || n_dims > 8)
        return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "bad SAMT arguments");
    FILE* f = fopen(path, "wb");
    if (!f) return fail(error, error_capacity, S3D_INVALID_ARGUMENT, "cannot create %s", path);
    bool ok = fwrite(&kSamtMagic, 4, 1, f) == 1 && fwrite(&n_dims, 4, 1, f) == 1;
    ok = ok && fwrite(ne, 8, (size_t)n_dims, f) == (size_t)n_dims && fwrite(&ggml_type, 4, 1, f) == 1;
    ok = ok && (nbytes == 0 || fwrite(data, 1, nbytes, f) == nbytes);
    ok = (fclose(f) == 0) && ok;
    return ok ? S3D_OK : fail(error, error_capacity, S3D_INTERNAL_ERROR, "short write of %s", path);
}

}  // extern "C"
