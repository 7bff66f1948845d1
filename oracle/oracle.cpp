// oracle.cpp -- CPU oracle for Evelyn's decode token loop.
//
// TEST INFRASTRUCTURE ONLY: the checker the CUDA engine is compared against,
// and the "port" arm of the CPU baseline. The product never links it.
//
// It restates, operation for operation in f32, the reference's
//   * GGUF reader            src/gguf.rs:127-182 (header, metadata, tensor table, alignment)
//   * type sizes/dequantise  src/gguf.rs:288-298, 300-320, 327-336, 338-430
//   * QMatrix / matvec       src/runtime.rs:23-89 (per-row dequantise, sequential f32 dot,
//                            64-row chunks spread over worker threads like rayon's par_chunks_mut)
//   * rms_norm               src/runtime.rs:193-196
//   * Model::load            src/runtime.rs:199-406 (metadata keys, defaults, tied LM head)
//   * dense_ffn / SiLU       src/runtime.rs:409-418, src/activation.rs:50
//   * rope_neox / interleave src/runtime.rs:437-474
//   * full_attention         src/runtime.rs:663-768 (f32 KV, softmax order, w/sum*v; the
//                            gated query of qwen35, :684-695, :753-761)
//   * gated-delta layers     src/runtime.rs:476-630 (sigmoid, softplus, SiLU x*sigmoid(x),
//                            causal depthwise conv, gated delta rule, per-head norm and gate)
//   * Session::step          src/runtime.rs:773-808
//   * argmax / log_prob      src/runtime.rs:897-912, validate_token_ids :125-135
//
// Built with -ffp-contract=off so that a*b-c*d is two roundings and a subtraction,
// exactly like the Rust source (rustc never contracts to FMA). Transcendentals call
// glibc's powf/sinf/cosf/expf/sqrtf, which are what Rust's f32 methods lower to on
// Linux (log1pf for `ln_1p`).

#include "oracle.h"

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <cmath>
#include <condition_variable>
#include <cstdio>
#include <cstring>
#include <fcntl.h>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <sys/mman.h>
#include <sys/stat.h>
#include <thread>
#include <unistd.h>
#include <vector>

namespace {

enum Status { OK = 0, INVALID_INPUT = 1, INVALID_DATA = 2, NOT_FOUND = 3, UNSUPPORTED = 4, IO = 5 };

thread_local std::string g_err;

int fail(int code, const std::string& msg) {
    g_err = msg;
    return code;
}

struct Error {
    int code;
    std::string msg;
};

[[noreturn]] void raise(int code, const std::string& msg) { throw Error{code, msg}; }

// ---------------------------------------------------------------- thread pool
// A fixed pool that runs `fn(task)` for task in [0, n) -- the role rayon plays
// in the reference (par_chunks_mut(64), into_par_iter over heads).
class Pool {
public:
    explicit Pool(int n) { resize(n); }
    ~Pool() { stop(); }

    void resize(int n) {
        if (n < 1) n = 1;
        std::lock_guard<std::mutex> job_lock(job_mu_);
        stop();
        quit_ = false;
        nthreads_ = n;
        for (int i = 1; i < n; ++i) workers_.emplace_back([this] { loop(); });
    }
    int size() const { return nthreads_; }

    // Each call owns its task counters; a worker joins a job only while holding mu_
    // and while the job is published, and run() returns only after every worker that
    // joined has left it, so no worker can carry an index or the task function of one
    // job into the next.
    void run(size_t ntasks, const std::function<void(size_t)>& fn) {
        if (ntasks == 0) return;
        if (nthreads_ == 1 || ntasks == 1) {
            for (size_t t = 0; t < ntasks; ++t) fn(t);
            return;
        }
        std::lock_guard<std::mutex> job_lock(job_mu_);  // one parallel job at a time
        Job job{&fn, ntasks};
        {
            std::lock_guard<std::mutex> g(mu_);
            job_ = &job;
            ++gen_;
        }
        cv_.notify_all();
        job.work();
        std::unique_lock<std::mutex> g(mu_);
        job_ = nullptr;  // no worker joins from here on
        done_cv_.wait(g, [&] { return job.active == 0; });
    }

private:
    struct Job {
        const std::function<void(size_t)>* fn;
        size_t ntasks;
        std::atomic<size_t> next{0};
        int active = 0;  // workers inside work(), guarded by the pool's mu_
        Job(const std::function<void(size_t)>* f, size_t n) : fn(f), ntasks(n) {}
        void work() {
            for (size_t t = next.fetch_add(1); t < ntasks; t = next.fetch_add(1)) (*fn)(t);
        }
    };

    void loop() {
        uint64_t seen = 0;
        for (;;) {
            Job* job;
            {
                std::unique_lock<std::mutex> g(mu_);
                cv_.wait(g, [&] { return quit_ || gen_ != seen; });
                if (quit_) return;
                seen = gen_;
                job = job_;
                if (!job) continue;  // woke after that job was already finished
                ++job->active;
            }
            job->work();
            std::lock_guard<std::mutex> g(mu_);
            if (--job->active == 0) done_cv_.notify_all();
        }
    }
    void stop() {
        {
            std::lock_guard<std::mutex> g(mu_);
            quit_ = true;
        }
        cv_.notify_all();
        for (auto& w : workers_) w.join();
        workers_.clear();
    }

    std::vector<std::thread> workers_;
    std::mutex mu_, job_mu_;
    std::condition_variable cv_, done_cv_;
    Job* job_ = nullptr;
    uint64_t gen_ = 0;
    bool quit_ = false;
    int nthreads_ = 1;
};

Pool& pool() {
    static Pool p(std::max(1u, std::thread::hardware_concurrency()));
    return p;
}

// ---------------------------------------------------------------- gguf.rs
constexpr uint32_t GGML_F32 = 0, GGML_F16 = 1, GGML_Q8_0 = 8, GGML_Q4_K = 12, GGML_Q5_K = 13,
                   GGML_Q6_K = 14, GGML_BF16 = 30;

const char* type_name(uint32_t t) {  // gguf.rs:261-278
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

[[noreturn]] void unsupported(uint32_t t) {  // gguf.rs:280-285
    raise(UNSUPPORTED, "ggml type " + std::to_string(t) + " (" + type_name(t) + ") not supported yet");
}

// gguf.rs:288-298 (integer division truncates like the Rust source)
size_t type_bytes(uint32_t t, size_t n) {
    switch (t) {
        case GGML_F32: return n * 4;
        case GGML_F16:
        case GGML_BF16: return n * 2;
        case GGML_Q8_0: return n / 32 * 34;
        case GGML_Q4_K: return n / 256 * 144;
        case GGML_Q5_K: return n / 256 * 176;
        case GGML_Q6_K: return n / 256 * 210;
        default: unsupported(t);
    }
}

float bits_to_f32(uint32_t b) {
    float f;
    std::memcpy(&f, &b, 4);
    return f;
}

// gguf.rs:300-320
float f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31;
    uint32_t exp = (h >> 10) & 0x1f;
    uint32_t frac = h & 0x3ff;
    uint32_t bits;
    if (exp == 0 && frac == 0) {
        bits = sign;
    } else if (exp == 0) {
        int32_t e = 127 - 15 + 1;
        uint32_t f = frac;
        while ((f & 0x400) == 0) {
            f <<= 1;
            e -= 1;
        }
        bits = sign | ((uint32_t)e << 23) | ((f & 0x3ff) << 13);
    } else if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (frac << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (frac << 13);
    }
    return bits_to_f32(bits);
}

inline float hf(const uint8_t* b, size_t i) { return f16_to_f32((uint16_t)(b[i] | (b[i + 1] << 8))); }

// gguf.rs:327-336 get_scale_min_k4
inline void scale_min_k4(int j, const uint8_t* q, float* s, float* m) {
    if (j < 4) {
        *s = (float)(q[j] & 63);
        *m = (float)(q[j + 4] & 63);
    } else {
        *s = (float)((q[j + 4] & 0xf) | ((q[j - 4] >> 6) << 4));
        *m = (float)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

// gguf.rs:338-430. `y` must have room for n values; the count check mirrors :423-428.
void dequantize(uint32_t t, const uint8_t* raw, size_t nbytes, size_t n, float* y) {
    size_t produced = 0;
    switch (t) {
        case GGML_F32:
            for (size_t i = 0; i + 4 <= nbytes; i += 4) {
                uint32_t b = raw[i] | (raw[i + 1] << 8) | (raw[i + 2] << 16) | ((uint32_t)raw[i + 3] << 24);
                if (produced < n) y[produced] = bits_to_f32(b);
                ++produced;
            }
            break;
        case GGML_F16:
            for (size_t i = 0; i + 2 <= nbytes; i += 2) {
                if (produced < n) y[produced] = hf(raw, i);
                ++produced;
            }
            break;
        case GGML_BF16:
            for (size_t i = 0; i + 2 <= nbytes; i += 2) {
                uint32_t b = (uint32_t)(raw[i] | (raw[i + 1] << 8)) << 16;
                if (produced < n) y[produced] = bits_to_f32(b);
                ++produced;
            }
            break;
        case GGML_Q8_0:
            for (size_t o = 0; o + 34 <= nbytes; o += 34) {
                const uint8_t* b = raw + o;
                float d = hf(b, 0);
                for (int i = 0; i < 32; ++i) {
                    if (produced < n) y[produced] = d * (float)(int8_t)b[2 + i];
                    ++produced;
                }
            }
            break;
        case GGML_Q4_K:
            for (size_t o = 0; o + 144 <= nbytes; o += 144) {
                const uint8_t* b = raw + o;
                float d = hf(b, 0), dmin = hf(b, 2);
                const uint8_t* sc = b + 4;
                const uint8_t* qs = b + 16;
                for (int blk = 0, is = 0; blk < 4; ++blk, is += 2) {
                    const uint8_t* q = qs + blk * 32;
                    float s1, m1, s2, m2;
                    scale_min_k4(is, sc, &s1, &m1);
                    scale_min_k4(is + 1, sc, &s2, &m2);
                    for (int l = 0; l < 32; ++l) {
                        if (produced < n) y[produced] = d * s1 * (float)(q[l] & 0xf) - dmin * m1;
                        ++produced;
                    }
                    for (int l = 0; l < 32; ++l) {
                        if (produced < n) y[produced] = d * s2 * (float)(q[l] >> 4) - dmin * m2;
                        ++produced;
                    }
                }
            }
            break;
        case GGML_Q5_K:
            for (size_t o = 0; o + 176 <= nbytes; o += 176) {
                const uint8_t* b = raw + o;
                float d = hf(b, 0), dmin = hf(b, 2);
                const uint8_t* sc = b + 4;
                const uint8_t* qh = b + 16;
                const uint8_t* qs = b + 48;
                uint8_t u1 = 1, u2 = 2;
                for (int blk = 0, is = 0; blk < 4; ++blk, is += 2) {
                    const uint8_t* q = qs + blk * 32;
                    float s1, m1, s2, m2;
                    scale_min_k4(is, sc, &s1, &m1);
                    scale_min_k4(is + 1, sc, &s2, &m2);
                    for (int l = 0; l < 32; ++l) {
                        int v = (q[l] & 0xf) + ((qh[l] & u1) ? 16 : 0);
                        if (produced < n) y[produced] = d * s1 * (float)v - dmin * m1;
                        ++produced;
                    }
                    for (int l = 0; l < 32; ++l) {
                        int v = (q[l] >> 4) + ((qh[l] & u2) ? 16 : 0);
                        if (produced < n) y[produced] = d * s2 * (float)v - dmin * m2;
                        ++produced;
                    }
                    u1 = (uint8_t)(u1 << 2);
                    u2 = (uint8_t)(u2 << 2);
                }
            }
            break;
        case GGML_Q6_K:
            for (size_t o = 0; o + 210 <= nbytes; o += 210) {
                const uint8_t* b = raw + o;
                const uint8_t* ql_all = b;
                const uint8_t* qh_all = b + 128;
                const uint8_t* sc_all = b + 192;
                float d = hf(b, 208);
                for (int half = 0; half < 2; ++half) {
                    const uint8_t* ql = ql_all + half * 64;
                    const uint8_t* qh = qh_all + half * 32;
                    const uint8_t* sc = sc_all + half * 8;
                    float out[128];
                    for (int l = 0; l < 32; ++l) {
                        int is = l / 16;
                        int q1 = (int)((ql[l] & 0xf) | ((qh[l] & 3) << 4)) - 32;
                        int q2 = (int)((ql[l + 32] & 0xf) | (((qh[l] >> 2) & 3) << 4)) - 32;
                        int q3 = (int)((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                        int q4 = (int)((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                        out[l] = d * (float)(int8_t)sc[is] * (float)q1;
                        out[l + 32] = d * (float)(int8_t)sc[is + 2] * (float)q2;
                        out[l + 64] = d * (float)(int8_t)sc[is + 4] * (float)q3;
                        out[l + 96] = d * (float)(int8_t)sc[is + 6] * (float)q4;
                    }
                    for (int i = 0; i < 128; ++i) {
                        if (produced < n) y[produced] = out[i];
                        ++produced;
                    }
                }
            }
            break;
        default: unsupported(t);
    }
    if (produced != n)
        raise(INVALID_DATA, "dequantised " + std::to_string(produced) + " of " + std::to_string(n) + " values");
}

// GGUF metadata value (gguf.rs:13-45)
struct Value {
    enum Kind { U64, I64, F64, BOOL, STR, ARRAY } kind = U64;
    uint64_t u = 0;
    int64_t i = 0;
    double f = 0;
    bool b = false;
    std::string s;
    std::vector<Value> arr;

    bool as_u64(uint64_t* out) const {
        if (kind == U64) { *out = u; return true; }
        if (kind == I64 && i >= 0) { *out = (uint64_t)i; return true; }
        return false;
    }
    bool as_f64(double* out) const {
        if (kind == F64) { *out = f; return true; }
        if (kind == U64) { *out = (double)u; return true; }
        if (kind == I64) { *out = (double)i; return true; }
        return false;
    }
};

struct TensorInfo {
    std::string name;
    std::vector<uint64_t> dims;  // dims[0] innermost
    uint32_t type = 0;
    uint64_t offset = 0;
    uint64_t elements() const {
        uint64_t n = 1;
        for (auto d : dims) n *= d;
        return n;
    }
};

class Reader {
public:
    Reader(const uint8_t* p, size_t n) : p_(p), n_(n) {}
    void need(size_t k) {
        if (k > n_ - pos_) raise(IO, "failed to fill whole buffer");
    }
    template <class T> T rd() {
        need(sizeof(T));
        T v;
        std::memcpy(&v, p_ + pos_, sizeof(T));
        pos_ += sizeof(T);
        return v;
    }
    std::string rd_str() {  // gguf.rs:81-92
        uint64_t n = rd<uint64_t>();
        if (n > (1u << 24)) raise(INVALID_DATA, "string too long");
        need(n);
        std::string s((const char*)p_ + pos_, n);
        pos_ += n;
        return s;
    }
    Value rd_value(uint32_t ty) {  // gguf.rs:94-124
        Value v;
        switch (ty) {
            case 0: v.kind = Value::U64; v.u = rd<uint8_t>(); break;
            case 1: v.kind = Value::I64; v.i = rd<int8_t>(); break;
            case 2: v.kind = Value::U64; v.u = rd<uint16_t>(); break;
            case 3: v.kind = Value::I64; v.i = rd<int16_t>(); break;
            case 4: v.kind = Value::U64; v.u = rd<uint32_t>(); break;
            case 5: v.kind = Value::I64; v.i = rd<int32_t>(); break;
            case 6: v.kind = Value::F64; v.f = (double)rd<float>(); break;
            case 7: v.kind = Value::BOOL; v.b = rd<uint8_t>() != 0; break;
            case 8: v.kind = Value::STR; v.s = rd_str(); break;
            case 9: {
                uint32_t et = rd<uint32_t>();
                uint64_t n = rd<uint64_t>();
                v.kind = Value::ARRAY;
                for (uint64_t k = 0; k < n; ++k) v.arr.push_back(rd_value(et));
                break;
            }
            case 10: v.kind = Value::U64; v.u = rd<uint64_t>(); break;
            case 11: v.kind = Value::I64; v.i = rd<int64_t>(); break;
            case 12: v.kind = Value::F64; v.f = rd<double>(); break;
            default: raise(INVALID_DATA, "unknown GGUF value type " + std::to_string(ty));
        }
        return v;
    }
    size_t pos() const { return pos_; }

private:
    const uint8_t* p_;
    size_t n_;
    size_t pos_ = 0;
};

struct Gguf {  // gguf.rs:62-68, opened from an in-memory image
    const uint8_t* base = nullptr;
    size_t len = 0;
    uint32_t version = 0;
    std::map<std::string, Value> metadata;
    std::map<std::string, TensorInfo> tensors;
    uint64_t data_start = 0;

    void open(const uint8_t* p, size_t n) {  // gguf.rs:127-182
        base = p;
        len = n;
        Reader r(p, n);
        r.need(4);
        if (std::memcmp(p, "GGUF", 4) != 0) raise(INVALID_DATA, "not a GGUF file");
        r.rd<uint32_t>();
        version = r.rd<uint32_t>();
        if (version < 2) raise(INVALID_DATA, "GGUF v1 unsupported");
        uint64_t n_tensors = r.rd<uint64_t>();
        uint64_t n_kv = r.rd<uint64_t>();
        for (uint64_t k = 0; k < n_kv; ++k) {
            std::string key = r.rd_str();
            uint32_t ty = r.rd<uint32_t>();
            metadata[key] = r.rd_value(ty);
        }
        for (uint64_t k = 0; k < n_tensors; ++k) {
            TensorInfo t;
            t.name = r.rd_str();
            uint32_t nd = r.rd<uint32_t>();
            for (uint32_t d = 0; d < nd; ++d) t.dims.push_back(r.rd<uint64_t>());
            t.type = r.rd<uint32_t>();
            t.offset = r.rd<uint64_t>();
            tensors[t.name] = t;
        }
        uint64_t align = 32;
        auto it = metadata.find("general.alignment");
        if (it != metadata.end()) it->second.as_u64(&align);
        uint64_t pos = r.pos();
        data_start = (pos + align - 1) / align * align;
    }
    const Value* meta(const std::string& k) const {
        auto it = metadata.find(k);
        return it == metadata.end() ? nullptr : &it->second;
    }
    std::string architecture() const {
        const Value* v = meta("general.architecture");
        return (v && v->kind == Value::STR) ? v->s : std::string();
    }
    const TensorInfo& info(const std::string& name) const {
        auto it = tensors.find(name);
        if (it == tensors.end()) raise(NOT_FOUND, "tensor " + name + " not found");
        return it->second;
    }
    // gguf.rs:436-450 tensor_raw (borrowed view into the image)
    const uint8_t* tensor_raw(const TensorInfo& t, size_t* nbytes) const {
        size_t bytes = type_bytes(t.type, (size_t)t.elements());
        uint64_t off = data_start + t.offset;
        if (off > len || bytes > len - off) raise(IO, "failed to fill whole buffer");
        *nbytes = bytes;
        return base + off;
    }
    // gguf.rs:199-215 tensor_f32
    std::vector<float> tensor_f32(const std::string& name) const {
        const TensorInfo& t = info(name);
        size_t nbytes;
        const uint8_t* raw = tensor_raw(t, &nbytes);
        std::vector<float> y((size_t)t.elements());
        dequantize(t.type, raw, nbytes, y.size(), y.data());
        return y;
    }
};

// ---------------------------------------------------------------- runtime.rs
struct QMatrix {  // runtime.rs:23-51
    size_t rows = 0, cols = 0, row_bytes = 0;
    uint32_t type = 0;
    const uint8_t* data = nullptr;

    static QMatrix from_raw(const TensorInfo& t, const uint8_t* raw) {
        QMatrix m;
        if (t.dims.size() == 2) {
            m.cols = t.dims[0];
            m.rows = t.dims[1];
        } else if (t.dims.size() == 1) {
            m.cols = t.dims[0];
            m.rows = 1;
        } else {
            raise(INVALID_DATA, t.name + ": unsupported rank");
        }
        m.row_bytes = type_bytes(t.type, m.cols);
        m.type = t.type;
        m.data = raw;
        return m;
    }

    // runtime.rs:54-69
    std::vector<float> row(size_t r) const {
        if (r >= rows)
            raise(INVALID_INPUT, "embedding row " + std::to_string(r) + " is outside matrix vocabulary " +
                                     std::to_string(rows));
        std::vector<float> y(cols);
        dequantize(type, data + r * row_bytes, row_bytes, cols, y.data());
        return y;
    }

    // runtime.rs:72-88: 64-row chunks in parallel; per row a fresh dequantised
    // row and a sequential f32 sum starting at zero.
    void matvec(const float* x, float* y) const {
        size_t chunks = (rows + 63) / 64;
        pool().run(chunks, [&](size_t chunk) {
            std::vector<float> rowbuf(cols);
            size_t end = std::min(rows, chunk * 64 + 64);
            for (size_t r = chunk * 64; r < end; ++r) {
                dequantize(type, data + r * row_bytes, row_bytes, cols, rowbuf.data());
                float acc = 0.0f;
                for (size_t c = 0; c < cols; ++c) acc += rowbuf[c] * x[c];
                y[r] = acc;
            }
        });
    }
};

struct SsmConfig {  // runtime.rs:112-120
    size_t conv_kernel = 0, inner = 0, state = 0, groups = 0, value_heads = 0;
};

struct Config {  // runtime.rs:93-110
    std::string arch;
    size_t layers = 0, dim = 0, ffn = 0, heads = 0, kv_heads = 0, head_dim = 0, rope_dim = 0, vocab = 0;
    float rope_base = 10000.0f, eps = 1e-6f;
    bool rope_interleaved = false;
    size_t full_attention_interval = 4;
    bool has_ssm = false;
    SsmConfig ssm;
    int64_t eos = -1;
};

struct GatedDelta {  // runtime.rs:155-170
    QMatrix qkv, z, alpha, beta, out;
    std::vector<float> conv, a, dt, norm;
    size_t conv_kernel = 0, key_dim = 0, key_heads = 0, value_dim = 0, value_heads = 0;
};

struct Layer {  // runtime.rs:142-181
    std::vector<float> attn_norm, ffn_norm, q_norm, k_norm;
    bool has_q_norm = false, has_k_norm = false;
    bool delta = false;  // Attention::GatedDelta (else Attention::Full)
    bool gated = false;  // Full: the q projection interleaves a sigmoid gate per head (qwen35)
    QMatrix q, k, v, o, gate, up, down;
    GatedDelta gd;
};

// runtime.rs:193-196
std::vector<float> rms_norm(const float* x, size_t n, const float* w, float eps) {
    float ss = 0.0f;
    for (size_t i = 0; i < n; ++i) ss += x[i] * x[i];
    float inv = 1.0f / sqrtf(ss / (float)n + eps);
    std::vector<float> y(n);
    for (size_t i = 0; i < n; ++i) y[i] = x[i] * inv * w[i];
    return y;
}

// activation.rs:50 (SiLU, the activation import.rs:31-40 picks for qwen3/llama)
inline float silu(float z) { return z / (1.0f + expf(-z)); }

// runtime.rs:437-450
void rope_neox(float* v, size_t heads, size_t hd, size_t rotary_dim, size_t pos, float base) {
    rotary_dim = std::min(rotary_dim, hd) & ~(size_t)1;
    size_t half = rotary_dim / 2;
    for (size_t h = 0; h < heads; ++h) {
        float* s = v + h * hd;
        for (size_t i = 0; i < half; ++i) {
            float theta = (float)pos * powf(base, -2.0f * (float)i / (float)rotary_dim);
            float sn = sinf(theta), cs = cosf(theta);
            float a = s[i], b = s[i + half];
            s[i] = a * cs - b * sn;
            s[i + half] = a * sn + b * cs;
        }
    }
}

// runtime.rs:455-474
void rope_interleaved(float* v, size_t heads, size_t hd, size_t rotary_dim, size_t pos, float base) {
    rotary_dim = std::min(rotary_dim, hd) & ~(size_t)1;
    for (size_t h = 0; h < heads; ++h) {
        float* s = v + h * hd;
        for (size_t i = 0; i < rotary_dim; i += 2) {
            float theta = (float)pos * powf(base, -((float)i) / (float)rotary_dim);
            float sn = sinf(theta), cs = cosf(theta);
            float a = s[i], b = s[i + 1];
            s[i] = a * cs - b * sn;
            s[i + 1] = a * sn + b * cs;
        }
    }
}

// runtime.rs:476-483
inline float sigmoid(float x) {
    if (x >= 0.0f) return 1.0f / (1.0f + expf(-x));
    const float e = expf(x);
    return e / (1.0f + e);
}

// runtime.rs:485-487
inline float softplus(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

// runtime.rs:489-491: the SiLU of the gated-delta layers, x * sigmoid(x) (the FFN's is
// activation.rs's z / (1 + e^-z))
inline float silu_sigmoid(float x) { return x * sigmoid(x); }

// runtime.rs:493-528: state [width][nv] row-major (key, value); decay, then the delta
// rule's correction, then the read-out by q over sqrt(width).
void gated_delta_step(float* state, const float* q, const float* k, const float* v, size_t width, size_t nv,
                      float decay, float beta, float* out) {
    for (size_t value = 0; value < nv; ++value)
        for (size_t key = 0; key < width; ++key) state[key * nv + value] *= decay;
    std::vector<float> delta(nv);
    for (size_t value = 0; value < nv; ++value) {
        float predicted = 0.0f;
        for (size_t key = 0; key < width; ++key) predicted += state[key * nv + value] * k[key];
        delta[value] = (v[value] - predicted) * beta;
    }
    for (size_t key = 0; key < width; ++key)
        for (size_t value = 0; value < nv; ++value) state[key * nv + value] += k[key] * delta[value];
    const float root = sqrtf((float)width);
    for (size_t value = 0; value < nv; ++value) {
        float acc = 0.0f;
        for (size_t key = 0; key < width; ++key) acc += state[key * nv + value] * q[key];
        out[value] = acc / root;
    }
}

}  // namespace

struct orc_model {
    void* map = nullptr;
    size_t map_len = 0;
    Gguf g;
    Config cfg;
    QMatrix embed, lm_head;
    std::vector<Layer> layers;
    std::vector<float> out_norm;

    ~orc_model() {
        if (map) munmap(map, map_len);
    }

    // runtime.rs:199-406
    void load() {
        std::string arch = g.architecture();
        if (arch.empty()) arch = "llama";
        auto need = [&](const std::string& k) -> uint64_t {
            uint64_t v;
            const Value* val = g.meta(arch + "." + k);
            if (!val || !val->as_u64(&v)) raise(INVALID_DATA, "missing " + arch + "." + k);
            return v;
        };
        cfg.arch = arch;
        cfg.dim = need("embedding_length");
        cfg.heads = need("attention.head_count");
        uint64_t kvh;
        const Value* kvv = g.meta(arch + ".attention.head_count_kv");
        if (kvv && kvv->as_u64(&kvh)) {
            cfg.kv_heads = kvh;
        } else if (kvv && kvv->kind == Value::ARRAY) {
            cfg.kv_heads = cfg.heads;
            for (const auto& e : kvv->arr) {
                uint64_t u;
                if (e.as_u64(&u) && u > 0) {
                    cfg.kv_heads = u;
                    break;
                }
            }
        } else {
            cfg.kv_heads = cfg.heads;
        }
        uint64_t hd;
        const Value* kl = g.meta(arch + ".attention.key_length");
        cfg.head_dim = (kl && kl->as_u64(&hd)) ? hd : cfg.dim / cfg.heads;
        if (arch == "qwen35") {  // runtime.rs:225-235
            cfg.has_ssm = true;
            cfg.ssm.conv_kernel = need("ssm.conv_kernel");
            cfg.ssm.inner = need("ssm.inner_size");
            cfg.ssm.state = need("ssm.state_size");
            cfg.ssm.groups = need("ssm.group_count");
            cfg.ssm.value_heads = need("ssm.time_step_rank");
        }
        cfg.layers = need("block_count");
        cfg.ffn = need("feed_forward_length");
        double f;
        const Value* rb = g.meta(arch + ".rope.freq_base");
        cfg.rope_base = (rb && rb->as_f64(&f)) ? (float)f : 10000.0f;
        uint64_t rd;
        const Value* rdv = g.meta(arch + ".rope.dimension_count");
        cfg.rope_dim = (rdv && rdv->as_u64(&rd)) ? rd : cfg.head_dim;
        const Value* ri = g.meta(arch + ".rope.mrope_interleaved");
        cfg.rope_interleaved = ri && ri->kind == Value::BOOL && ri->b;
        uint64_t fai;
        const Value* fav = g.meta(arch + ".full_attention_interval");
        cfg.full_attention_interval = (fav && fav->as_u64(&fai)) ? fai : 4;  // runtime.rs:258
        const Value* ep = g.meta(arch + ".attention.layer_norm_rms_epsilon");
        cfg.eps = (ep && ep->as_f64(&f)) ? (float)f : 1e-6f;
        auto te = g.tensors.find("token_embd.weight");
        cfg.vocab = te == g.tensors.end() ? 0 : (size_t)te->second.dims.at(1);
        const Value* eos = g.meta("tokenizer.ggml.eos_token_id");
        uint64_t e;
        cfg.eos = (eos && eos->as_u64(&e) && e <= 0xffffffffu) ? (int64_t)e : -1;

        auto mat = [&](const std::string& n) {
            const TensorInfo& t = g.info(n);
            size_t nb;
            const uint8_t* raw = g.tensor_raw(t, &nb);
            return QMatrix::from_raw(t, raw);
        };
        embed = mat("token_embd.weight");
        layers.resize(cfg.layers);
        for (size_t i = 0; i < cfg.layers; ++i) {
            std::string p = "blk." + std::to_string(i) + ".";
            Layer& L = layers[i];
            const bool has_gated_delta = g.tensors.count(p + "attn_qkv.weight") != 0;
            if (arch == "qwen35" && cfg.full_attention_interval > 0) {  // runtime.rs:278-290
                const bool expected = (i + 1) % cfg.full_attention_interval != 0;
                if (has_gated_delta != expected)
                    raise(INVALID_DATA, p + "attention type does not match qwen35.full_attention_interval=" +
                                            std::to_string(cfg.full_attention_interval));
            }
            if (has_gated_delta) {  // runtime.rs:298-356
                if (!cfg.has_ssm) raise(INVALID_DATA, "gated-delta tensors found without SSM architecture metadata");
                GatedDelta& d = L.gd;
                L.delta = true;
                d.key_dim = cfg.ssm.state;
                d.key_heads = cfg.ssm.groups;
                d.value_heads = cfg.ssm.value_heads;
                if (d.value_heads == 0 || cfg.ssm.inner % d.value_heads != 0)
                    raise(INVALID_DATA, "Qwen3.5 SSM inner size must divide evenly across value heads");
                d.value_dim = cfg.ssm.inner / d.value_heads;
                d.conv_kernel = cfg.ssm.conv_kernel;
                d.qkv = mat(p + "attn_qkv.weight");
                d.z = mat(p + "attn_gate.weight");
                d.conv = g.tensor_f32(p + "ssm_conv1d.weight");
                d.alpha = mat(p + "ssm_alpha.weight");
                d.beta = mat(p + "ssm_beta.weight");
                d.a = g.tensor_f32(p + "ssm_a");
                d.dt = g.tensor_f32(p + "ssm_dt");
                d.norm = g.tensor_f32(p + "ssm_norm.weight");
                d.out = mat(p + "ssm_out.weight");
                const size_t channels = 2 * d.key_dim * d.key_heads + d.value_dim * d.value_heads;
                if (d.qkv.rows != channels || d.z.rows != d.value_dim * d.value_heads ||
                    d.conv.size() != d.conv_kernel * channels || d.alpha.rows != d.value_heads ||
                    d.beta.rows != d.value_heads || d.a.size() != d.value_heads || d.dt.size() != d.value_heads ||
                    d.norm.size() != d.value_dim || d.out.cols != d.value_dim * d.value_heads ||
                    d.out.rows != cfg.dim)
                    raise(INVALID_DATA, p + "gated-delta tensor shapes do not match Qwen3.5 metadata");
            } else {
                L.q = mat(p + "attn_q.weight");
                L.k = mat(p + "attn_k.weight");
                L.v = mat(p + "attn_v.weight");
                L.o = mat(p + "attn_output.weight");
                if (g.tensors.count(p + "attn_q_norm.weight")) {
                    L.q_norm = g.tensor_f32(p + "attn_q_norm.weight");
                    L.has_q_norm = true;
                }
                if (g.tensors.count(p + "attn_k_norm.weight")) {
                    L.k_norm = g.tensor_f32(p + "attn_k_norm.weight");
                    L.has_k_norm = true;
                }
                L.gated = arch == "qwen35";  // runtime.rs:371
            }
            std::string ffn_norm_name = g.tensors.count(p + "post_attention_norm.weight")
                                            ? p + "post_attention_norm.weight"
                                            : p + "ffn_norm.weight";
            L.attn_norm = g.tensor_f32(p + "attn_norm.weight");
            L.ffn_norm = g.tensor_f32(ffn_norm_name);
            L.gate = mat(p + "ffn_gate.weight");
            L.up = mat(p + "ffn_up.weight");
            L.down = mat(p + "ffn_down.weight");
        }
        out_norm = g.tensor_f32("output_norm.weight");
        lm_head = g.tensors.count("output.weight") ? mat("output.weight") : mat("token_embd.weight");
    }

    // runtime.rs:409-418 (rayon::join of gate and up is two independent matvecs)
    std::vector<float> dense_ffn(size_t i, const float* x) const {
        const Layer& l = layers.at(i);
        std::vector<float> g(l.gate.rows), u(l.up.rows);
        l.gate.matvec(x, g.data());
        l.up.matvec(x, u.data());
        std::vector<float> h(g.size());
        for (size_t k = 0; k < g.size(); ++k) h[k] = silu(g[k]) * u[k];
        std::vector<float> y(l.down.rows);
        l.down.matvec(h.data(), y.data());
        return y;
    }
};

struct GatedDeltaState {  // runtime.rs:532-549
    std::vector<float> conv_history;  // the last kernel - 1 un-convolved projection rows
    std::vector<float> recurrent;     // [value_heads][key_dim][value_dim]
};

struct orc_session {  // runtime.rs:634-661
    const orc_model* model;
    std::vector<std::vector<float>> k_cache, v_cache;
    std::vector<GatedDeltaState> delta;  // per layer (empty for full-attention layers)
    size_t pos = 0;
};

namespace {

// runtime.rs:551-630
std::vector<float> gated_delta_attention(const GatedDelta& d, GatedDeltaState& st, const float* x, float eps) {
    const size_t key_width = d.key_dim * d.key_heads, value_width = d.value_dim * d.value_heads;
    const size_t channels = 2 * key_width + value_width;
    std::vector<float> projection(channels), z(value_width);
    d.qkv.matvec(x, projection.data());
    d.z.matvec(x, z.data());
    // the previous kernel - 1 projections, then this token; one depthwise causal
    // convolution per channel
    const size_t history_len = st.conv_history.size();
    std::vector<float> conv_input(st.conv_history);
    conv_input.insert(conv_input.end(), projection.begin(), projection.end());
    std::vector<float> conv_output(channels);
    for (size_t ch = 0; ch < channels; ++ch) {
        float sum = 0.0f;
        for (size_t tap = 0; tap < d.conv_kernel; ++tap)
            sum += conv_input[tap * channels + ch] * d.conv[ch * d.conv_kernel + tap];
        conv_output[ch] = silu_sigmoid(sum);
    }
    if (history_len > 0)
        std::copy(conv_input.end() - (std::ptrdiff_t)history_len, conv_input.end(), st.conv_history.begin());
    std::vector<float> alpha(d.value_heads), beta(d.value_heads);
    d.alpha.matvec(x, alpha.data());
    d.beta.matvec(x, beta.data());
    std::vector<float> output(value_width, 0.0f);
    for (size_t head = 0; head < d.value_heads; ++head) {
        const size_t key_head = head % d.key_heads;
        std::vector<float> q(conv_output.begin() + key_head * d.key_dim,
                             conv_output.begin() + (key_head + 1) * d.key_dim);
        std::vector<float> k(conv_output.begin() + key_width + key_head * d.key_dim,
                             conv_output.begin() + key_width + (key_head + 1) * d.key_dim);
        const float* v = conv_output.data() + 2 * key_width + head * d.value_dim;
        float qs = 0.0f, ks = 0.0f;
        for (float e : q) qs += e * e;
        for (float e : k) ks += e * e;
        const float q_norm = sqrtf(qs + eps), k_norm = sqrtf(ks + eps);
        for (auto& e : q) e /= q_norm;
        for (auto& e : k) e /= k_norm;
        const float decay = expf(softplus(alpha[head] + d.dt[head]) * d.a[head]);
        const float b = sigmoid(beta[head]);
        float* state = st.recurrent.data() + head * d.key_dim * d.value_dim;
        gated_delta_step(state, q.data(), k.data(), v, d.key_dim, d.value_dim, decay, b,
                         output.data() + head * d.value_dim);
    }
    // per-head RMSNorm and the projected SiLU gate after the recurrent update
    for (size_t head = 0; head < d.value_heads; ++head) {
        float* o = output.data() + head * d.value_dim;
        std::vector<float> normalized = rms_norm(o, d.value_dim, d.norm.data(), eps);
        for (size_t i = 0; i < d.value_dim; ++i) o[i] = normalized[i] * silu_sigmoid(z[head * d.value_dim + i]);
    }
    std::vector<float> y(d.out.rows);
    d.out.matvec(output.data(), y.data());
    return y;
}

// runtime.rs:663-768
std::vector<float> full_attention(const Layer& layer, const float* xn, const Config& c, size_t pos,
                                  std::vector<float>& k_cache, std::vector<float>& v_cache) {
    std::vector<float> projected(layer.q.rows), kv(layer.k.rows), vv(layer.v.rows);
    layer.q.matvec(xn, projected.data());
    layer.k.matvec(xn, kv.data());
    layer.v.matvec(xn, vv.data());
    size_t query_width = c.heads * c.head_dim;
    std::vector<float> qv, query_gate;
    if (layer.gated) {  // runtime.rs:687-693: per head [query | gate]
        for (size_t h = 0; h < c.heads; ++h) {
            const float* st = projected.data() + h * c.head_dim * 2;
            qv.insert(qv.end(), st, st + c.head_dim);
            query_gate.insert(query_gate.end(), st + c.head_dim, st + 2 * c.head_dim);
        }
    } else {
        qv = std::move(projected);
    }
    size_t kv_heads = layer.k.rows / c.head_dim;
    size_t group = c.heads / kv_heads;
    if (layer.has_q_norm) {
        for (size_t h = 0; h < c.heads; ++h) {
            size_t st = h * c.head_dim;
            std::vector<float> n = rms_norm(qv.data() + st, c.head_dim, layer.q_norm.data(), c.eps);
            std::copy(n.begin(), n.end(), qv.begin() + st);
        }
    }
    if (layer.has_k_norm) {
        for (size_t h = 0; h < kv_heads; ++h) {
            size_t st = h * c.head_dim;
            std::vector<float> n = rms_norm(kv.data() + st, c.head_dim, layer.k_norm.data(), c.eps);
            std::copy(n.begin(), n.end(), kv.begin() + st);
        }
    }
    if (c.rope_interleaved) {
        rope_interleaved(qv.data(), c.heads, c.head_dim, c.rope_dim, pos, c.rope_base);
        rope_interleaved(kv.data(), kv_heads, c.head_dim, c.rope_dim, pos, c.rope_base);
    } else {
        rope_neox(qv.data(), c.heads, c.head_dim, c.rope_dim, pos, c.rope_base);
        rope_neox(kv.data(), kv_heads, c.head_dim, c.rope_dim, pos, c.rope_base);
    }
    k_cache.insert(k_cache.end(), kv.begin(), kv.end());
    v_cache.insert(v_cache.end(), vv.begin(), vv.end());
    size_t t = pos + 1;
    size_t kv_width = kv_heads * c.head_dim;
    float scale = 1.0f / sqrtf((float)c.head_dim);
    std::vector<float> att(query_width, 0.0f);
    size_t hd = c.head_dim;
    pool().run(c.heads, [&](size_t head) {
        size_t kv_head = head / group;
        const float* qh = qv.data() + head * hd;
        std::vector<float> scores(t);
        for (size_t p = 0; p < t; ++p) {
            const float* kp = k_cache.data() + p * kv_width + kv_head * hd;
            float s = 0.0f;
            for (size_t d = 0; d < hd; ++d) s += qh[d] * kp[d];
            scores[p] = s * scale;
        }
        float maximum = -3.40282347e38f;  // f32::MIN
        for (float s : scores) maximum = std::fmax(maximum, s);
        float sum = 0.0f;
        for (auto& s : scores) {
            s = expf(s - maximum);
            sum += s;
        }
        float* out = att.data() + head * hd;
        for (size_t p = 0; p < t; ++p) {
            const float* vp = v_cache.data() + p * kv_width + kv_head * hd;
            float w = scores[p];
            for (size_t d = 0; d < hd; ++d) out[d] += w / sum * vp[d];
        }
        if (layer.gated)  // runtime.rs:753-761
            for (size_t d = 0; d < hd; ++d) out[d] *= sigmoid(query_gate[head * hd + d]);
    });
    std::vector<float> y(layer.o.rows);
    layer.o.matvec(att.data(), y.data());
    return y;
}

template <class F> int guarded(F&& f) {
    try {
        f();
        return OK;
    } catch (const Error& e) {
        return fail(e.code, e.msg);
    } catch (const std::bad_alloc&) {
        return fail(IO, "out of memory");
    } catch (const std::exception& e) {
        return fail(INVALID_DATA, e.what());
    }
}

}  // namespace

extern "C" {

const char* orc_last_error(void) { return g_err.c_str(); }
void orc_set_threads(int n) { pool().resize(n); }
int orc_get_threads(void) { return pool().size(); }

int64_t orc_type_bytes(uint32_t t, uint64_t n) {
    int64_t out = -1;
    guarded([&] { out = (int64_t)type_bytes(t, n); });
    return out;
}

float orc_f16_to_f32(uint16_t h) { return f16_to_f32(h); }

int orc_dequantize(uint32_t t, const uint8_t* raw, size_t nbytes, size_t n, float* out) {
    return guarded([&] { dequantize(t, raw, nbytes, n, out); });
}

static int finish_load(orc_model* m, orc_model** out) {
    int rc = guarded([&] {
        m->g.open(m->map ? (const uint8_t*)m->map : m->g.base, m->map ? m->map_len : m->g.len);
        m->load();
    });
    if (rc != OK) {
        delete m;
        return rc;
    }
    *out = m;
    return OK;
}

int orc_model_load(const char* path, orc_model** out) {
    int fd = open(path, O_RDONLY);
    if (fd < 0) return fail(errno == ENOENT ? NOT_FOUND : IO, std::string(path) + ": " + strerror(errno));
    struct stat st;
    if (fstat(fd, &st) != 0) {
        close(fd);
        return fail(IO, strerror(errno));
    }
    void* p = st.st_size ? mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0) : nullptr;
    close(fd);
    if (!st.st_size) return fail(IO, "failed to fill whole buffer");
    if (p == MAP_FAILED) return fail(IO, strerror(errno));
    orc_model* m = new orc_model();
    m->map = p;
    m->map_len = (size_t)st.st_size;
    return finish_load(m, out);
}

int orc_model_load_memory(const uint8_t* data, size_t len, orc_model** out) {
    orc_model* m = new orc_model();
    m->g.base = data;
    m->g.len = len;
    return finish_load(m, out);
}

void orc_model_free(orc_model* m) { delete m; }

int orc_model_config(const orc_model* m, orc_config* o) {
    std::memset(o, 0, sizeof(*o));
    std::snprintf(o->arch, sizeof(o->arch), "%s", m->cfg.arch.c_str());
    o->layers = m->cfg.layers;
    o->dim = m->cfg.dim;
    o->ffn = m->cfg.ffn;
    o->heads = m->cfg.heads;
    o->kv_heads = m->cfg.kv_heads;
    o->head_dim = m->cfg.head_dim;
    o->rope_dim = m->cfg.rope_dim;
    o->vocab = m->cfg.vocab;
    o->rope_base = m->cfg.rope_base;
    o->eps = m->cfg.eps;
    o->rope_interleaved = m->cfg.rope_interleaved;
    o->full_attention_interval = m->cfg.full_attention_interval;
    o->ssm_conv_kernel = m->cfg.ssm.conv_kernel;
    o->ssm_inner = m->cfg.ssm.inner;
    o->ssm_state = m->cfg.ssm.state;
    o->ssm_groups = m->cfg.ssm.groups;
    o->ssm_value_heads = m->cfg.ssm.value_heads;
    o->eos_token_id = m->cfg.eos;
    return OK;
}

int orc_dense_ffn(const orc_model* m, size_t layer, const float* x, float* y) {
    return guarded([&] {
        if (layer >= m->layers.size()) raise(INVALID_INPUT, "layer out of range");
        auto r = m->dense_ffn(layer, x);
        std::copy(r.begin(), r.end(), y);
    });
}

int orc_ffn_input(const orc_model* m, size_t layer, const float* x, float* y) {
    return guarded([&] {
        if (layer >= m->layers.size()) raise(INVALID_INPUT, "layer out of range");
        auto r = rms_norm(x, m->cfg.dim, m->layers[layer].ffn_norm.data(), m->cfg.eps);
        std::copy(r.begin(), r.end(), y);
    });
}

int orc_matvec(const orc_model* m, const char* tensor, const float* x, size_t xn, float* y, size_t yn) {
    return guarded([&] {
        const TensorInfo& t = m->g.info(tensor);
        size_t nb;
        QMatrix q = QMatrix::from_raw(t, m->g.tensor_raw(t, &nb));
        if (xn != q.cols || yn != q.rows) raise(INVALID_INPUT, "matvec shape mismatch");
        q.matvec(x, y);
    });
}

int orc_tensor_f32(const orc_model* m, const char* tensor, float* out, size_t n) {
    return guarded([&] {
        auto v = m->g.tensor_f32(tensor);
        if (v.size() != n) raise(INVALID_INPUT, "tensor size mismatch");
        std::copy(v.begin(), v.end(), out);
    });
}

int orc_tensor_info(const orc_model* m, const char* tensor, uint32_t* type, uint64_t* dims, uint32_t* ndims) {
    return guarded([&] {
        const TensorInfo& t = m->g.info(tensor);
        *type = t.type;
        *ndims = (uint32_t)t.dims.size();
        for (size_t i = 0; i < t.dims.size() && i < 4; ++i) dims[i] = t.dims[i];
    });
}

int orc_session_new(const orc_model* m, orc_session** out) {
    auto* s = new orc_session();
    s->model = m;
    s->k_cache.resize(m->cfg.layers);
    s->v_cache.resize(m->cfg.layers);
    s->delta.resize(m->cfg.layers);
    for (size_t i = 0; i < m->layers.size(); ++i) {  // runtime.rs:539-548
        const Layer& L = m->layers[i];
        if (!L.delta) continue;
        const GatedDelta& d = L.gd;
        const size_t channels = 2 * d.key_dim * d.key_heads + d.value_dim * d.value_heads;
        s->delta[i].conv_history.assign((d.conv_kernel - 1) * channels, 0.0f);
        s->delta[i].recurrent.assign(d.value_heads * d.key_dim * d.value_dim, 0.0f);
    }
    *out = s;
    return OK;
}

void orc_session_free(orc_session* s) { delete s; }
uint64_t orc_session_pos(const orc_session* s) { return s->pos; }

int orc_validate_token_ids(const uint32_t* ids, size_t n, size_t vocab) {
    for (size_t i = 0; i < n; ++i)
        if (ids[i] >= vocab)
            return fail(INVALID_INPUT, "token ID " + std::to_string(ids[i]) + " is outside model vocabulary (" +
                                           std::to_string(vocab) + "); check that tokenizer and GGUF match");
    return OK;
}

// runtime.rs:773-808
int orc_session_step(orc_session* s, uint32_t token, orc_ffn_fn ffn, void* ctx, float* logits) {
    const orc_model* m = s->model;
    const Config& c = m->cfg;
    int rc = orc_validate_token_ids(&token, 1, c.vocab);
    if (rc != OK) return rc;
    return guarded([&] {
        std::vector<float> x = m->embed.row(token);
        std::vector<float> fy(c.dim);
        for (size_t li = 0; li < m->layers.size(); ++li) {
            const Layer& layer = m->layers[li];
            std::vector<float> normalized = rms_norm(x.data(), c.dim, layer.attn_norm.data(), c.eps);
            std::vector<float> a =
                layer.delta ? gated_delta_attention(layer.gd, s->delta[li], normalized.data(), c.eps)
                            : full_attention(layer, normalized.data(), c, s->pos, s->k_cache[li], s->v_cache[li]);
            for (size_t i = 0; i < x.size(); ++i) x[i] += a[i];
            std::vector<float> fin = rms_norm(x.data(), c.dim, layer.ffn_norm.data(), c.eps);
            const float* fo;
            std::vector<float> dense;
            if (ffn && ffn(ctx, li, fin.data(), c.dim, fy.data()) == 0) {
                fo = fy.data();
            } else {
                dense = m->dense_ffn(li, fin.data());
                fo = dense.data();
            }
            for (size_t i = 0; i < x.size(); ++i) x[i] += fo[i];
        }
        s->pos += 1;
        std::vector<float> xn = rms_norm(x.data(), c.dim, m->out_norm.data(), c.eps);
        m->lm_head.matvec(xn.data(), logits);
    });
}

int orc_session_fill_kv(orc_session* s, uint64_t n, uint64_t seed) {
    const Config& c = s->model->cfg;
    uint64_t st = seed ? seed : 1;
    auto next = [&]() {  // xorshift64* (lib.rs:53-60)
        st ^= st >> 12;
        st ^= st << 25;
        st ^= st >> 27;
        return st * 0x2545F4914F6CDD1DULL;
    };
    for (size_t li = 0; li < c.layers; ++li) {
        size_t w = s->model->layers[li].k.rows;
        for (uint64_t p = 0; p < n; ++p)
            for (size_t i = 0; i < w; ++i) {
                s->k_cache[li].push_back((float)(next() >> 40) / 16777216.0f - 0.5f);
                s->v_cache[li].push_back((float)(next() >> 40) / 16777216.0f - 0.5f);
            }
    }
    s->pos += n;
    return OK;
}

void orc_gated_delta_step(float* state, const float* q, const float* k, const float* v, size_t width, size_t nv,
                          float decay, float beta, float* out) {
    gated_delta_step(state, q, k, v, width, nv, decay, beta, out);
}

void orc_rope_interleaved(float* v, size_t heads, size_t hd, size_t rotary_dim, size_t pos, float base) {
    rope_interleaved(v, heads, hd, rotary_dim, pos, base);
}

uint32_t orc_argmax(const float* v, size_t n) {  // runtime.rs:897-905: strict '>' keeps the first max
    size_t bi = 0;
    float bv = -3.40282347e38f;
    for (size_t i = 0; i < n; ++i)
        if (v[i] > bv) {
            bi = i;
            bv = v[i];
        }
    return (uint32_t)bi;
}

// server.rs:326-352 (sample_token): temperature <= f32::EPSILON -> argmax; else the f32
// weights exp((v - max) / T) summed in f64 in index order, one xorshift64* draw of 53
// bits, and the first index whose running f64 sum reaches draw * total (argmax when the
// total is not finite and positive, or no index reaches it).
uint32_t orc_sample_token(const float* logits, size_t n, float temperature, uint64_t* state) {
    if (temperature <= 1.1920929e-7f) return orc_argmax(logits, n);
    float maximum = -INFINITY;
    for (size_t i = 0; i < n; ++i) maximum = std::fmax(maximum, logits[i]);  // f32::max ignores NaN
    std::vector<double> w(n);
    for (size_t i = 0; i < n; ++i) w[i] = (double)std::exp((logits[i] - maximum) / temperature);
    double total = 0.0;
    for (size_t i = 0; i < n; ++i) total += w[i];
    if (!std::isfinite(total) || total <= 0.0) return orc_argmax(logits, n);
    uint64_t x = *state;
    x ^= x >> 12;
    x ^= x << 25;
    x ^= x >> 27;
    *state = x;
    const double unit = (double)((x * 0x2545F4914F6CDD1Dull) >> 11) / (double)(1ull << 53);
    const double threshold = unit * total;
    double cumulative = 0.0;
    for (size_t i = 0; i < n; ++i) {
        cumulative += w[i];
        if (cumulative >= threshold) return (uint32_t)i;
    }
    return orc_argmax(logits, n);
}

float orc_log_prob(const float* logits, size_t n, uint32_t target) {  // runtime.rs:908-912
    float mx = -3.40282347e38f;
    for (size_t i = 0; i < n; ++i) mx = std::fmax(mx, logits[i]);
    float sum = 0.0f;
    for (size_t i = 0; i < n; ++i) sum += expf(logits[i] - mx);
    float lse = mx + logf(sum);
    return logits[target] - lse;
}

}  // extern "C"
