// gguf.cpp -- GGUF v2/v3 reader for the engine, plus error and buffer helpers.
//
// Follows src/gguf.rs:127-182: header magic and version check (v1 rejected), the 13
// metadata value types of rd_value (:94-124) with the 16 MiB string limit (:81-92),
// the tensor table, and the data start aligned to general.alignment (default 32).
// type_bytes mirrors :288-298 and its Unsupported error :280-285. Tensors are read
// straight out of the caller's image (a mapped file or a buffer), like tensor_raw
// (:436-450) without the copy.
#include <algorithm>
#include <cstring>

#include "engine.hpp"

namespace evl {

// ------------------------------------------------------------------ errors
namespace {
thread_local std::string g_last_error;
}

void set_last_error(const std::string& msg) { g_last_error = msg; }
const char* last_error() { return g_last_error.c_str(); }

[[noreturn]] void raise(evl_status code, const std::string& msg) { throw Error{code, msg}; }

void cuda_check(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return;
    cudaGetLastError();  // clear a non-sticky launch error so later calls report their own
    raise(e == cudaErrorMemoryAllocation ? EVL_ERR_OUT_OF_MEMORY : EVL_ERR_CUDA,
          std::string(what) + ": " + cudaGetErrorString(e));
}

DeviceGuard::DeviceGuard(int device) {
    cudaGetDevice(&prev);
    if (device >= 0 && device != prev) cuda_check(cudaSetDevice(device), "cudaSetDevice");
}
DeviceGuard::~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
}

DeviceBuffer::~DeviceBuffer() {
    if (p) cudaFree(p);
}
void DeviceBuffer::alloc(size_t n) {
    if (p) cudaFree(p);
    p = nullptr;
    bytes = n;
    if (n) cuda_check(cudaMalloc(&p, n), "cudaMalloc");
}

PinnedBuffer::~PinnedBuffer() {
    if (p) cudaFreeHost(p);
}
void PinnedBuffer::alloc(size_t n) {
    if (p) cudaFreeHost(p);
    p = nullptr;
    bytes = n;
    if (n) cuda_check(cudaMallocHost(&p, n), "cudaMallocHost");
}

// ------------------------------------------------------------------ gguf.rs
const char* type_name(uint32_t t) {
    switch (t) {
        case 0: return "F32";
        case 1: return "F16";
        case 2: return "Q4_0";
        case 3: return "Q4_1";
        case 6: return "Q5_0";
        case 7: return "Q5_1";
        case 8: return "Q8_0";
        case 10: return "Q2_K";
        case 11: return "Q3_K";
        case 12: return "Q4_K";
        case 13: return "Q5_K";
        case 14: return "Q6_K";
        case 30: return "BF16";
        default: return "other";
    }
}

size_t type_bytes(uint32_t t, size_t n) {
    switch (t) {
        case GGML_F32: return n * 4;
        case GGML_F16:
        case GGML_BF16: return n * 2;
        case GGML_Q8_0: return n / 32 * 34;
        case GGML_Q4_K: return n / 256 * 144;
        case GGML_Q5_K: return n / 256 * 176;
        case GGML_Q6_K: return n / 256 * 210;
        default:
            raise(EVL_ERR_UNSUPPORTED,
                  "ggml type " + std::to_string(t) + " (" + type_name(t) + ") not supported yet");
    }
}

bool GgufValue::as_u64(uint64_t* o) const {
    if (kind == U64) { *o = u; return true; }
    if (kind == I64 && i >= 0) { *o = (uint64_t)i; return true; }
    return false;
}
bool GgufValue::as_f64(double* o) const {
    if (kind == F64) { *o = f; return true; }
    if (kind == U64) { *o = (double)u; return true; }
    if (kind == I64) { *o = (double)i; return true; }
    return false;
}

uint64_t GgufTensor::elements() const {
    uint64_t n = 1;
    for (auto d : dims) n *= d;
    return n;
}

namespace {
class Cursor {
public:
    Cursor(const uint8_t* p, size_t n) : p_(p), n_(n) {}
    void need(size_t k) {
        if (k > n_ - pos_) raise(EVL_ERR_IO, "failed to fill whole buffer");
    }
    template <class T> T get() {
        need(sizeof(T));
        T v;
        std::memcpy(&v, p_ + pos_, sizeof(T));
        pos_ += sizeof(T);
        return v;
    }
    std::string str() {
        uint64_t n = get<uint64_t>();
        if (n > (1u << 24)) raise(EVL_ERR_INVALID_DATA, "string too long");
        need(n);
        std::string s((const char*)p_ + pos_, n);
        pos_ += n;
        return s;
    }
    GgufValue value(uint32_t ty, int depth = 0) {
        GgufValue v;
        switch (ty) {
            case 0: v.kind = GgufValue::U64; v.u = get<uint8_t>(); break;
            case 1: v.kind = GgufValue::I64; v.i = get<int8_t>(); break;
            case 2: v.kind = GgufValue::U64; v.u = get<uint16_t>(); break;
            case 3: v.kind = GgufValue::I64; v.i = get<int16_t>(); break;
            case 4: v.kind = GgufValue::U64; v.u = get<uint32_t>(); break;
            case 5: v.kind = GgufValue::I64; v.i = get<int32_t>(); break;
            case 6: v.kind = GgufValue::F64; v.f = (double)get<float>(); break;
            case 7: v.kind = GgufValue::BOOL; v.b = get<uint8_t>() != 0; break;
            case 8: v.kind = GgufValue::STR; v.s = str(); break;
            case 9: {
                if (depth > 8) raise(EVL_ERR_INVALID_DATA, "GGUF arrays nested too deeply");
                uint32_t et = get<uint32_t>();
                uint64_t n = get<uint64_t>();
                v.kind = GgufValue::ARRAY;
                v.arr.reserve((size_t)std::min<uint64_t>(n, 1u << 20));
                for (uint64_t k = 0; k < n; ++k) v.arr.push_back(value(et, depth + 1));
                break;
            }
            case 10: v.kind = GgufValue::U64; v.u = get<uint64_t>(); break;
            case 11: v.kind = GgufValue::I64; v.i = get<int64_t>(); break;
            case 12: v.kind = GgufValue::F64; v.f = get<double>(); break;
            default: raise(EVL_ERR_INVALID_DATA, "unknown GGUF value type " + std::to_string(ty));
        }
        return v;
    }
    size_t pos() const { return pos_; }

private:
    const uint8_t* p_;
    size_t n_;
    size_t pos_ = 0;
};
}  // namespace

void Gguf::open(const uint8_t* data, size_t len) {
    base_ = data;
    len_ = len;
    Cursor c(data, len);
    c.need(4);
    if (std::memcmp(data, "GGUF", 4) != 0) raise(EVL_ERR_INVALID_DATA, "not a GGUF file");
    c.get<uint32_t>();
    uint32_t version = c.get<uint32_t>();
    if (version < 2) raise(EVL_ERR_INVALID_DATA, "GGUF v1 unsupported");
    uint64_t n_tensors = c.get<uint64_t>();
    uint64_t n_kv = c.get<uint64_t>();
    for (uint64_t k = 0; k < n_kv; ++k) {
        std::string key = c.str();
        uint32_t ty = c.get<uint32_t>();
        meta_[key] = c.value(ty);
    }
    for (uint64_t k = 0; k < n_tensors; ++k) {
        GgufTensor t;
        t.name = c.str();
        uint32_t nd = c.get<uint32_t>();
        if (nd > 8) raise(EVL_ERR_INVALID_DATA, t.name + ": too many dimensions");
        for (uint32_t d = 0; d < nd; ++d) t.dims.push_back(c.get<uint64_t>());
        t.type = c.get<uint32_t>();
        t.offset = c.get<uint64_t>();
        tensors_[t.name] = t;
    }
    uint64_t align = 32;
    if (const GgufValue* a = meta("general.alignment")) a->as_u64(&align);
    if (align == 0) raise(EVL_ERR_INVALID_DATA, "general.alignment is zero");
    data_start_ = (c.pos() + align - 1) / align * align;
}

const GgufValue* Gguf::meta(const std::string& key) const {
    auto it = meta_.find(key);
    return it == meta_.end() ? nullptr : &it->second;
}

std::string Gguf::architecture() const {
    const GgufValue* v = meta("general.architecture");
    return v && v->kind == GgufValue::STR ? v->s : std::string();
}

const GgufTensor& Gguf::tensor(const std::string& name) const {
    auto it = tensors_.find(name);
    if (it == tensors_.end()) raise(EVL_ERR_NOT_FOUND, "tensor " + name + " not found");
    return it->second;
}

const uint8_t* Gguf::raw(const GgufTensor& t, size_t* nbytes) const {
    size_t n = type_bytes(t.type, (size_t)t.elements());
    uint64_t off = data_start_ + t.offset;
    if (off > len_ || n > len_ - off) raise(EVL_ERR_IO, "failed to fill whole buffer");
    *nbytes = n;
    return base_ + off;
}

}  // namespace evl
