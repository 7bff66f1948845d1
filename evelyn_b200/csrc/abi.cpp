// abi.cpp -- the extern "C" surface declared in include/evelyn.h.
//
// Each entry point catches every C++ exception at the boundary and turns it into an
// evl_status plus a thread-local message, the way the reference surfaces
// io::Error values (src/runtime.rs, src/gguf.rs).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#if defined(__x86_64__)
#include <immintrin.h>
#endif

#include <algorithm>
#include <cerrno>
#include <cfloat>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <new>
#include <thread>

#include "engine.hpp"

using namespace evl;

namespace {

template <class F> evl_status guarded(F&& f) {
    try {
        f();
        return EVL_OK;
    } catch (const Error& e) {
        set_last_error(e.msg);
        return e.code;
    } catch (const std::bad_alloc&) {
        set_last_error("out of host memory");
        return EVL_ERR_OUT_OF_MEMORY;
    } catch (const std::exception& e) {
        set_last_error(e.what());
        return EVL_ERR_IO;
    }
}

void require(bool ok, const char* msg) {
    if (!ok) raise(EVL_ERR_INVALID_INPUT, msg);
}

evl_model_options defaults() {
    evl_model_options o;
    std::memset(&o, 0, sizeof(o));
    o.struct_size = sizeof(o);
    o.device = -1;
    o.tp_rank = 0;
    o.tp_size = 1;
    return o;
}

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

}  // namespace

extern "C" {

const char* evl_last_error(void) { return last_error(); }
uint32_t evl_abi_version(void) { return EVL_ABI_VERSION; }
void evl_model_options_init(evl_model_options* o) {
    if (o) *o = defaults();
}

evl_status evl_validate_token_ids(const uint32_t* ids, size_t n, size_t vocab) {
    return guarded([&] {
        require(ids || n == 0, "null ids");
        for (size_t i = 0; i < n; ++i)
            if (ids[i] >= vocab)
                raise(EVL_ERR_INVALID_INPUT, "token ID " + std::to_string(ids[i]) + " is outside model vocabulary (" +
                                                 std::to_string(vocab) + "); check that tokenizer and GGUF match");
    });
}

}  // extern "C"

namespace {
// The first index of the maximum under a strict '>' scan from -FLT_MAX (NaN never
// wins; nothing above -FLT_MAX gives 0). Blocks of 256 values reduce to their maximum;
// the strict '>' across blocks keeps the first block that holds the maximum, which is
// then searched for its first occurrence. `blockmax` is the block's maximum under the
// same '>' (a NaN never replaces a number).
template <class BlockMax>
uint32_t argmax_blocks(const float* v, size_t n, BlockMax blockmax) {
    constexpr size_t B = 256;
    float mx = -FLT_MAX;
    size_t best = SIZE_MAX, i = 0;
    for (; i + B <= n; i += B) {
        const float bm = blockmax(v + i);
        if (bm > mx) {
            mx = bm;
            best = i;
        }
    }
    for (size_t k = i; k < n; ++k)  // a tail value above every block's is the first maximum
        if (v[k] > mx) {
            mx = v[k];
            best = k;
        }
    if (best == SIZE_MAX) return 0;
    if (best >= i) return (uint32_t)best;
    for (size_t k = best; k < best + B; ++k)
        if (v[k] == mx) return (uint32_t)k;
    return (uint32_t)best;
}

uint32_t argmax_base(const float* v, size_t n) {
    return argmax_blocks(v, n, [](const float* b) {
        float lm[16];
        for (int j = 0; j < 16; ++j) lm[j] = -FLT_MAX;
        for (int k = 0; k < 256; k += 16)
            for (int j = 0; j < 16; ++j) lm[j] = b[k + j] > lm[j] ? b[k + j] : lm[j];
        float m = -FLT_MAX;
        for (int j = 0; j < 16; ++j) m = lm[j] > m ? lm[j] : m;
        return m;
    });
}

#if defined(__x86_64__)
// vmaxps(a, b) is (a > b) ? a : b per lane, the scan's own comparison
__attribute__((target("avx2"))) float blockmax_avx2(const float* b) {
    __m256 a0 = _mm256_set1_ps(-FLT_MAX), a1 = a0, a2 = a0, a3 = a0;
    for (int k = 0; k < 256; k += 32) {
        a0 = _mm256_max_ps(_mm256_loadu_ps(b + k), a0);
        a1 = _mm256_max_ps(_mm256_loadu_ps(b + k + 8), a1);
        a2 = _mm256_max_ps(_mm256_loadu_ps(b + k + 16), a2);
        a3 = _mm256_max_ps(_mm256_loadu_ps(b + k + 24), a3);
    }
    a0 = _mm256_max_ps(_mm256_max_ps(a0, a1), _mm256_max_ps(a2, a3));
    alignas(32) float t[8];
    _mm256_store_ps(t, a0);
    float m = -FLT_MAX;
    for (int j = 0; j < 8; ++j) m = t[j] > m ? t[j] : m;
    return m;
}
__attribute__((target("avx2"))) uint32_t argmax_avx2(const float* v, size_t n) {
    return argmax_blocks(v, n, blockmax_avx2);
}
#endif
}  // namespace

extern "C" {

uint32_t evl_argmax(const float* v, size_t n) {
#if defined(__x86_64__)
    static const bool avx2 = __builtin_cpu_supports("avx2");
    if (avx2) return argmax_avx2(v, n);
#endif
    return argmax_base(v, n);
}

float evl_log_prob(const float* logits, size_t n, uint32_t target) {
    float mx = -FLT_MAX;
    for (size_t i = 0; i < n; ++i) mx = std::fmax(mx, logits[i]);
    float sum = 0.f;
    for (size_t i = 0; i < n; ++i) sum += std::exp(logits[i] - mx);
    return logits[target] - (mx + std::log(sum));
}

evl_status evl_tp_shard_plan(const evl_config* cfg, int32_t tp_size, int32_t rank, evl_tp_shard* out) {
    return guarded([&] {
        require(cfg && out, "null argument");
        Config c;
        c.heads = cfg->heads;
        c.kv_heads = cfg->kv_heads;
        c.head_dim = cfg->head_dim;
        c.ffn = cfg->ffn;
        c.vocab = cfg->vocab;
        const TpShard s = tp_shard_plan(c, tp_size, rank);
        for (int i = 0; i < 2; ++i) {
            out->q_rows[i] = s.q[i];
            out->kv_rows[i] = s.kv[i];
            out->ffn_rows[i] = s.ffn[i];
            out->vocab_rows[i] = s.vocab[i];
        }
    });
}

evl_status evl_tp_unique_id(uint8_t out[128]) {
    return guarded([&] {
        require(out, "null output");
        ncclUniqueId id;
        nccl_check(nccl().GetUniqueId(&id), "ncclGetUniqueId");
        std::memcpy(out, id.internal, 128);
    });
}

// ------------------------------------------------------------------ model
evl_status evl_model_load_memory(const void* data, size_t len, const evl_model_options* opts, evl_model** out) {
    return guarded([&] {
        require(data && out, "null argument");
        evl_model_options o = opts ? *opts : defaults();
        auto* m = new evl_model();
        try {
            m->m = load_model(static_cast<const uint8_t*>(data), len, o);
        } catch (...) {
            delete m;
            throw;
        }
        *out = m;
    });
}

evl_status evl_model_load(const char* path, const evl_model_options* opts, evl_model** out) {
    return guarded([&] {
        require(path && out, "null argument");
        const int fd = ::open(path, O_RDONLY);
        if (fd < 0) raise(errno == ENOENT ? EVL_ERR_NOT_FOUND : EVL_ERR_IO, std::string(path) + ": " + strerror(errno));
        struct stat st;
        if (fstat(fd, &st) != 0) {
            ::close(fd);
            raise(EVL_ERR_IO, strerror(errno));
        }
        const size_t len = (size_t)st.st_size;
        void* p = len ? mmap(nullptr, len, PROT_READ, MAP_PRIVATE, fd, 0) : nullptr;
        ::close(fd);
        if (!len) raise(EVL_ERR_IO, "failed to fill whole buffer");
        if (p == MAP_FAILED) raise(EVL_ERR_IO, strerror(errno));
        evl_model_options o = opts ? *opts : defaults();
        auto* m = new evl_model();
        try {
            m->m = load_model(static_cast<const uint8_t*>(p), len, o);
        } catch (...) {
            munmap(p, len);
            delete m;
            throw;
        }
        munmap(p, len);
        *out = m;
    });
}

void evl_model_free(evl_model* m) {
    if (!m) return;
    DeviceGuard g(m->m->device);
    delete m;
}

evl_status evl_model_config(const evl_model* model, evl_config* o) {
    return guarded([&] {
        require(model && o, "null argument");
        const Config& c = model->m->cfg;
        std::memset(o, 0, sizeof(*o));
        std::snprintf(o->arch, sizeof(o->arch), "%s", c.arch.c_str());
        o->layers = c.layers;
        o->dim = c.dim;
        o->ffn = c.ffn;
        o->heads = c.heads;
        o->kv_heads = c.kv_heads;
        o->head_dim = c.head_dim;
        o->rope_dim = c.rope_dim;
        o->vocab = c.vocab;
        o->rope_base = c.rope_base;
        o->eps = c.eps;
        o->rope_interleaved = c.rope_interleaved;
        o->eos_token_id = c.eos;
    });
}

evl_status evl_model_ssm_config(const evl_model* model, evl_ssm_config* o) {
    return guarded([&] {
        require(model && o, "null argument");
        const Model& m = *model->m;
        const Config& c = m.cfg;
        std::memset(o, 0, sizeof(*o));
        o->has_ssm = c.has_ssm;
        o->delta_layers = m.delta_layers;
        o->full_attention_interval = c.full_attention_interval;
        o->conv_kernel = c.ssm_conv_kernel;
        o->inner = c.ssm_inner;
        o->state = c.ssm_state;
        o->groups = c.ssm_groups;
        o->value_heads = c.ssm_value_heads;
    });
}

uint64_t evl_model_weight_bytes(const evl_model* model) { return model ? model->m->weight_bytes_per_step : 0; }

evl_status evl_model_dense_ffn(evl_model* model, size_t layer, const float* x, float* y) {
    return guarded([&] {
        require(model && x && y, "null argument");
        Model& m = *model->m;
        require(layer < m.cfg.layers, "layer out of range");
        std::lock_guard<std::mutex> lk(m.mu);
        DeviceGuard g(m.device);
        const size_t dim = m.cfg.dim;
        float* s = m.scratch.as<float>();
        float* dx = s;
        float* dy = s + dim;
        float* ybuf = s + 2 * dim;
        float* h = s + 3 * dim;
        cuda_check(cudaMemcpyAsync(dx, x, dim * 4, cudaMemcpyHostToDevice, m.stream), "H2D");
        run_dense_ffn(m, layer, dx, nullptr, dy, false, 1, h, ybuf, m.d_err, nullptr, m.stream, false);
        cuda_check(cudaMemcpyAsync(y, dy, dim * 4, cudaMemcpyDeviceToHost, m.stream), "D2H");
        cuda_check(cudaStreamSynchronize(m.stream), "dense_ffn");
    });
}

evl_status evl_model_ffn_input(evl_model* model, size_t layer, const float* x, float* y) {
    return guarded([&] {
        require(model && x && y, "null argument");
        Model& m = *model->m;
        require(layer < m.cfg.layers, "layer out of range");
        std::lock_guard<std::mutex> lk(m.mu);
        DeviceGuard g(m.device);
        const size_t dim = m.cfg.dim;
        float* s = m.scratch.as<float>();
        cuda_check(cudaMemcpyAsync(s, x, dim * 4, cudaMemcpyHostToDevice, m.stream), "H2D");
        cuda_check(launch_rmsnorm(s, m.layers[layer].ffn_norm, s + dim, (uint32_t)dim, 1, m.cfg.eps, m.stream, false),
                   "rmsnorm");
        cuda_check(cudaMemcpyAsync(y, s + dim, dim * 4, cudaMemcpyDeviceToHost, m.stream), "D2H");
        cuda_check(cudaStreamSynchronize(m.stream), "ffn_input");
    });
}

evl_status evl_model_dequantize(evl_model* model, const char* tensor, float* out, size_t n) {
    return guarded([&] {
        require(model && tensor && out, "null argument");
        Model& m = *model->m;
        std::lock_guard<std::mutex> lk(m.mu);
        DeviceGuard g(m.device);
        auto vit = m.vecs.find(tensor);
        if (vit != m.vecs.end()) {
            require(n == vit->second.second, "element count mismatch");
            cuda_check(cudaMemcpy(out, vit->second.first, n * 4, cudaMemcpyDeviceToHost), "D2H");
            return;
        }
        auto it = m.matrices.find(tensor);
        if (it == m.matrices.end()) raise(EVL_ERR_NOT_FOUND, std::string("tensor ") + tensor + " not found");
        const QMatrix& q = *it->second;
        require(n == (size_t)q.rows * q.cols, "element count mismatch");
        DeviceBuffer buf;
        const uint32_t chunk_rows = std::max<uint32_t>(1, (uint32_t)((256ull << 20) / (4ull * q.cols)));
        buf.alloc((size_t)std::min<uint32_t>(chunk_rows, q.rows) * q.cols * 4);
        for (uint32_t r0 = 0; r0 < q.rows; r0 += chunk_rows) {
            const uint32_t nr = std::min(chunk_rows, q.rows - r0);
            cuda_check(launch_dequant_repacked(q.dev, r0, nr, buf.as<float>(), m.stream), "dequantize");
            cuda_check(cudaMemcpyAsync(out + (size_t)r0 * q.cols, buf.p, (size_t)nr * q.cols * 4,
                                       cudaMemcpyDeviceToHost, m.stream),
                       "D2H");
            cuda_check(cudaStreamSynchronize(m.stream), "dequantize");
        }
    });
}

evl_status evl_model_matvec(evl_model* model, const char* tensor, const float* x, size_t xn, float* y, size_t yn) {
    return guarded([&] {
        require(model && tensor && x && y, "null argument");
        Model& m = *model->m;
        auto it = m.matrices.find(tensor);
        if (it == m.matrices.end()) raise(EVL_ERR_NOT_FOUND, std::string("tensor ") + tensor + " not found");
        const QMatrix& q = *it->second;
        require(xn == q.cols && yn == q.rows, "matvec shape mismatch");
        std::lock_guard<std::mutex> lk(m.mu);
        DeviceGuard g(m.device);
        DeviceBuffer bx, by;
        bx.alloc(xn * 4);
        by.alloc(yn * 4);
        cuda_check(cudaMemcpyAsync(bx.p, x, xn * 4, cudaMemcpyHostToDevice, m.stream), "H2D");
        MatvecArgs a;
        a.nseg = 1;
        a.seg[0].m = q.dev;
        a.seg[0].y = by.as<float>();
        a.x = bx.as<float>();
        a.cols = q.cols;
        a.err = m.d_err;
        cuda_check(launch_qmatvec(a, m.stream, false), "matvec");
        cuda_check(cudaMemcpyAsync(y, by.p, yn * 4, cudaMemcpyDeviceToHost, m.stream), "D2H");
        cuda_check(cudaStreamSynchronize(m.stream), "matvec");
    });
}

// ------------------------------------------------------------------ sessions
evl_status evl_session_new(evl_model* model, uint32_t max_ctx, evl_session** out) {
    return guarded([&] {
        require(model && out, "null argument");
        DeviceGuard g(model->m->device);
        auto* s = new evl_session();
        try {
            s->d.init(model->m.get(), 1, max_ctx);
        } catch (...) {
            delete s;
            throw;
        }
        *out = s;
    });
}

void evl_session_free(evl_session* s) { delete s; }
uint64_t evl_session_pos(const evl_session* s) { return s ? s->d.host_pos[0] : 0; }

evl_status evl_session_step(evl_session* s, uint32_t token, const evl_ffn_backend* ffn, float* logits_out,
                            uint32_t* argmax_out) {
    return guarded([&] {
        require(s, "null session");
        s->d.step(&token, ffn, logits_out, argmax_out);
    });
}

evl_status evl_session_generate(evl_session* s, uint32_t token, uint32_t n, uint32_t* tokens_out) {
    return guarded([&] {
        require(s && (tokens_out || n == 0), "null argument");
        s->d.generate(token, n, tokens_out);
    });
}

evl_status evl_session_prefill(evl_session* s, const uint32_t* tokens, size_t n, float* logits_out,
                               uint32_t* argmax_out) {
    return guarded([&] {
        require(s && (tokens || n == 0), "null argument");
        s->d.prefill(0, tokens, n, logits_out, argmax_out);
    });
}

evl_status evl_session_sample(evl_session* s, float temperature, uint64_t* rng_state, uint32_t* token_out) {
    return guarded([&] {
        require(s && rng_state && token_out, "null argument");
        s->d.sample(temperature, rng_state, token_out);
    });
}

evl_status evl_batch_prefill(evl_batch* b, uint32_t seq, const uint32_t* tokens, size_t n, float* logits_out,
                             uint32_t* argmax_out) {
    return guarded([&] {
        require(b && (tokens || n == 0), "null argument");
        b->d.prefill(seq, tokens, n, logits_out, argmax_out);
    });
}

evl_status evl_batch_sample(evl_batch* b, float temperature, uint64_t* rng_states, uint32_t* tokens_out) {
    return guarded([&] {
        require(b && rng_states && tokens_out, "null argument");
        b->d.sample(temperature, rng_states, tokens_out);
    });
}

void* evl_session_stream(evl_session* s) { return s ? (void*)s->d.stream : nullptr; }
uint32_t evl_session_kernels_per_step(const evl_session* s) { return s ? s->d.kernels_per_step : 0; }
const char* evl_session_notes(const evl_session* s) {
    if (!s) return "";
    s->notes = s->d.step_note;
    return s->notes.c_str();
}

evl_status evl_batch_new(evl_model* model, uint32_t n_seqs, uint32_t max_ctx, evl_batch** out) {
    return guarded([&] {
        require(model && out, "null argument");
        DeviceGuard g(model->m->device);
        auto* b = new evl_batch();
        try {
            b->d.init(model->m.get(), n_seqs, max_ctx);
        } catch (...) {
            delete b;
            throw;
        }
        *out = b;
    });
}

void evl_batch_free(evl_batch* b) { delete b; }
uint64_t evl_batch_pos(const evl_batch* b, uint32_t seq) {
    return (b && seq < b->d.host_pos.size()) ? b->d.host_pos[seq] : 0;
}
evl_status evl_batch_step(evl_batch* b, const uint32_t* tokens, float* logits_out, uint32_t* argmax_out) {
    return guarded([&] {
        require(b && tokens, "null argument");
        b->d.step(tokens, nullptr, logits_out, argmax_out);
    });
}
void* evl_batch_stream(evl_batch* b) { return b ? (void*)b->d.stream : nullptr; }

// ------------------------------------------------------------------ kernels on caller buffers
evl_status evl_dequantize_raw(uint32_t type, const void* d_raw, size_t n, float* d_out, void* stream) {
    return guarded([&] {
        require(d_raw && d_out, "null argument");
        type_bytes(type, n);  // Unsupported for unknown types
        cuda_check(launch_dequant_raw(type, d_raw, n, d_out, as_stream(stream)), "dequantize");
    });
}

evl_status evl_qmatrix_create(uint32_t type, uint32_t rows, uint32_t cols, const void* host_raw, int device,
                              evl_qmatrix** out) {
    return guarded([&] {
        require(host_raw && out && rows && cols, "null argument or empty matrix");
        auto* q = new evl_qmatrix();
        try {
            q->device = device;
            DeviceGuard g(device);
            q->m.name = "matrix";
            q->m.type = type;
            q->m.rows = rows;
            q->m.cols = cols;
            repack_sizes(q->m);
            q->buf.alloc(q->m.bytes());
            q->err.alloc(4);
            cuda_check(cudaMemset(q->err.p, 0, 4), "memset");
            place(q->m, q->buf.as<uint8_t>());
            const uint64_t stride = type_bytes(type, cols);
            DeviceBuffer raw;
            raw.alloc(stride * rows);
            cuda_check(cudaMemcpy(raw.p, host_raw, stride * rows, cudaMemcpyHostToDevice), "upload");
            cuda_check(launch_repack(q->m.dev, q->buf.as<uint8_t>(), q->m.bytes(), raw.p, stride, 0), "repack");
            cuda_check(cudaDeviceSynchronize(), "repack");
        } catch (...) {
            delete q;
            throw;
        }
        *out = q;
    });
}

void evl_qmatrix_free(evl_qmatrix* q) {
    if (!q) return;
    DeviceGuard g(q->device);
    delete q;
}
uint64_t evl_qmatrix_bytes(const evl_qmatrix* q) { return q ? q->m.bytes() : 0; }

evl_status evl_qmatrix_matvec(const evl_qmatrix* q, const float* d_x, float* d_y, void* stream) {
    return guarded([&] {
        require(q && d_x && d_y, "null argument");
        require((reinterpret_cast<uintptr_t>(d_x) & 15) == 0, "x must be 16-byte aligned");
        MatvecArgs a;
        a.nseg = 1;
        a.seg[0].m = q->m.dev;
        a.seg[0].y = d_y;
        a.x = d_x;
        a.cols = q->m.cols;
        a.err = q->err.as<int>();
        // programmatic dependent launch on a caller's stream: the kernel streams weights
        // while the previous kernel finishes and reads x, writes y only after
        // griddepcontrol.wait
        cuda_check(launch_qmatvec(a, as_stream(stream), stream != nullptr), "matvec");
    });
}

evl_status evl_qmatrix_matmul(evl_qmatrix* q, const float* d_x, uint32_t nvec, float* d_y, void* stream) {
    return guarded([&] {
        require(q && d_x && d_y, "null argument");
        require(nvec >= 1 && nvec <= 32, "nvec must be 1..32");
        const QMatrix& m = q->m;
        const uint64_t gb = gemm_layout_bytes(m.type, m.rows, m.cols);
        if (!gb) raise(EVL_ERR_UNSUPPORTED, "batched product needs Q4_K, Q6_K or Q8_0 with cols a multiple of 256");
        DeviceGuard g(q->device);
        cudaStream_t s = as_stream(stream);
        if (!q->gemm_buf.p) {
            q->gemm_buf.alloc(gb);
            q->gemm = gemm_view(m.type, m.rows, m.cols, q->gemm_buf.as<uint8_t>());
            cuda_check(launch_gemm_repack(m.dev, q->gemm, s), "gemm repack");
        }
        int sms = 148;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, q->device);
        const uint32_t ksplit = gemm_ksplit(q->gemm, sms), rows_pad = q->gemm.mtiles * 128;
        const uint64_t xb = gemm_x_bytes(32, m.cols), pb = (uint64_t)ksplit * 32 * rows_pad * 4;
        if (q->bx.bytes < xb) q->bx.alloc(xb);
        if (q->xinv.bytes < 3 * 128) q->xinv.alloc(3 * 128);  // xinv[32] | stats[32][2]
        if (q->part.bytes < pb) q->part.alloc(pb);
        GemmX gx;
        gx.x = d_x;
        gx.nseq = nvec;
        gx.cols = m.cols;
        gx.x_stride = m.cols;
        gx.bx = q->bx.as<uint8_t>();
        gx.xinv = q->xinv.as<float>();
        gx.stats = q->xinv.as<float>() + 32;
        cuda_check(launch_gemm_stage_x(gx, s, false), "stage x");
        GemmArgs ga;
        ga.w = q->gemm;
        ga.bx = gx.bx;
        ga.xinv = gx.xinv;
        ga.nseq = nvec;
        ga.ksplit = ksplit;
        ga.rows_pad = rows_pad;
        ga.part = q->part.as<float>();
        ga.err = q->err.as<int>();
        cuda_check(launch_qgemm(ga, s, false), "gemm");
        GemmReduce r;
        r.part = ga.part;
        r.ksplit = ksplit;
        r.rows_pad = rows_pad;
        r.nseq = nvec;
        r.rows = m.rows;
        r.y = d_y;
        r.y_stride = m.rows;
        cuda_check(launch_gemm_reduce(r, s, false), "gemm reduce");
        int32_t err = 0;
        cuda_check(cudaMemcpyAsync(&err, q->err.p, 4, cudaMemcpyDeviceToHost, s), "D2H");
        cuda_check(cudaStreamSynchronize(s), "matmul");
        if (err) {
            cudaMemset(q->err.p, 0, 4);
            raise(EVL_ERR_TIMEOUT, "a device wait in the batched product timed out");
        }
    });
}

evl_status evl_qmatrix_dequantize(const evl_qmatrix* q, float* d_out, void* stream) {
    return guarded([&] {
        require(q && d_out, "null argument");
        cuda_check(launch_dequant_repacked(q->m.dev, 0, q->m.rows, d_out, as_stream(stream)), "dequantize");
    });
}

}  // extern "C"

namespace evl {

void check_attention_args(const float* d_q, const void* d_k_pages, const void* d_v_pages, const int32_t* d_page_table,
                          uint32_t t, uint32_t heads, uint32_t kv_heads, uint32_t head_dim, uint32_t page_size,
                          const float* d_out) {
    require(d_q && d_k_pages && d_v_pages && d_page_table && d_out, "null argument");
    require(t > 0, "no positions to attend");
    require(head_dim == 128 || head_dim == 64 || head_dim == 256, "head_dim must be 64, 128 or 256");
    require(page_size == 16, "page_size must be 16");
    require(kv_heads && heads % kv_heads == 0, "heads must be a multiple of kv_heads");
    const uint32_t g = heads / kv_heads;
    require(g == 1 || g == 2 || g == 4 || g == 8, "heads / kv_heads must be 1, 2, 4 or 8");
}

// Splits over the sequence: enough (kv_head, split) CTAs to cover the SMs twice.
uint32_t attention_splits(uint32_t t, uint32_t kv_heads, uint32_t page_size) {
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const uint32_t pages = (t + page_size - 1) / page_size;
    return std::max<uint32_t>(1, std::min<uint32_t>((2u * sms) / kv_heads, pages));
}

size_t attention_part_bytes(uint32_t heads, uint32_t nsplit, uint32_t head_dim) {
    return (size_t)heads * nsplit * (head_dim + 2) * 4;
}

// One standalone decode attention with caller-provided partials (`part`) and error flag.
void attention_standalone(const float* d_q, const void* d_k_pages, const void* d_v_pages, const int32_t* d_page_table,
                          uint32_t t, uint32_t heads, uint32_t kv_heads, uint32_t head_dim, uint32_t page_size,
                          float* d_out, float* part, uint32_t nsplit, int32_t* d_err, cudaStream_t s) {
    AttnArgs a;
    a.q = d_q;
    a.out = d_out;
    a.kv.pool = const_cast<void*>(d_k_pages);
    a.kv.head_stride = (uint64_t)page_size * head_dim * 2;
    a.kv.page_stride = a.kv.head_stride * kv_heads;
    a.kv.layer_stride = 0;
    a.kv.v_offset = static_cast<const uint8_t*>(d_v_pages) - static_cast<const uint8_t*>(d_k_pages);
    a.kv.page_size = page_size;
    a.kv.elem_bytes = 2;
    a.page_table = d_page_table;
    a.max_pages = (t + page_size - 1) / page_size;
    a.pos = nullptr;
    a.pos_value = (int32_t)(t - 1);
    a.heads = heads;
    a.kv_heads = kv_heads;
    a.head_dim = head_dim;
    a.nsplit = nsplit;
    a.part = part;
    a.scale = 1.0f / sqrtf((float)head_dim);
    a.err = d_err;
    // 16-row f16 pages of head_dim 64 / 128 and a GQA group of 1, 2, 4 or 8: the cluster
    // kernel (split-K over 8 CTAs per kv head, tensor-core loop, on-chip merge, one
    // launch) in its standalone mode (q ready, k and v already in the pages). K and V
    // share one tensor map based at the lower of the two buffers; the map's extent is a
    // bound, the loads only touch the pages the table names.
    const uint32_t G = heads / kv_heads;
    const uint32_t ring = attention_cluster_pages(a.max_pages, 8, page_size, head_dim, 2, G, 16);
    if (page_size == 16 && ring) {
        const uint8_t* k8 = static_cast<const uint8_t*>(d_k_pages);
        const uint8_t* v8 = static_cast<const uint8_t*>(d_v_pages);
        const uint8_t* base = std::min(k8, v8);
        const uint64_t row = 2ull * head_dim;
        KvTmap tmap;
        if ((uint64_t)(k8 - base) % row == 0 && (uint64_t)(v8 - base) % row == 0 &&
            make_kv_tmap(base, (1ull << 30) * row, head_dim, &tmap)) {
            AttnArgs c = a;
            c.kv.pool = const_cast<uint8_t*>(base);
            c.kv.k_offset = k8 - base;
            c.nsplit = 8;
            RopeArgs r;
            r.q = const_cast<float*>(d_q);
            r.kv = c.kv;
            r.page_table = d_page_table;
            r.max_pages = a.max_pages;
            r.batch = 1;
            r.heads = heads;
            r.kv_heads = kv_heads;
            r.head_dim = head_dim;
            r.err = d_err;
            // two stages: 8-page chunks keep every warp of a group on a page (the
            // double-buffered 4-stage ring measured slower here: 83 vs 66 us at 32K)
            cuda_check(launch_attention_cluster(r, c, ring, 2, s, false, &tmap), "attention");
            return;
        }
    }
    cuda_check(launch_attention(a, s, false), "attention");
}

}  // namespace evl

namespace {
constexpr size_t kWsHeader = 256;  // error flag, padded so the partials stay aligned
}  // namespace

extern "C" {

evl_status evl_attention_decode(const float* d_q, const void* d_k_pages, const void* d_v_pages,
                                const int32_t* d_page_table, uint32_t t, uint32_t heads, uint32_t kv_heads,
                                uint32_t head_dim, uint32_t page_size, float* d_out, void* stream) {
    return guarded([&] {
        check_attention_args(d_q, d_k_pages, d_v_pages, d_page_table, t, heads, kv_heads, head_dim, page_size, d_out);
        cudaStream_t s = as_stream(stream);
        const uint32_t nsplit = attention_splits(t, kv_heads, page_size);
        DeviceBuffer scratch;
        scratch.alloc(kWsHeader + attention_part_bytes(heads, nsplit, head_dim));
        int32_t* d_err = scratch.as<int32_t>();
        cuda_check(cudaMemsetAsync(d_err, 0, 4, s), "memset");
        attention_standalone(d_q, d_k_pages, d_v_pages, d_page_table, t, heads, kv_heads, head_dim, page_size, d_out,
                             reinterpret_cast<float*>(scratch.as<uint8_t>() + kWsHeader), nsplit, d_err, s);
        int32_t err = 0;
        cuda_check(cudaMemcpyAsync(&err, d_err, 4, cudaMemcpyDeviceToHost, s), "D2H");
        cuda_check(cudaStreamSynchronize(s), "attention");
        if (err == DEV_ERR_WAIT_TIMEOUT) raise(EVL_ERR_TIMEOUT, "a device wait for KV pages timed out");
    });
}

size_t evl_attention_workspace_bytes(uint32_t t_max, uint32_t heads, uint32_t kv_heads, uint32_t head_dim) {
    if (!t_max || !kv_heads) return 0;
    return kWsHeader + attention_part_bytes(heads, attention_splits(t_max, kv_heads, 16), head_dim);
}

evl_status evl_attention_decode_ws(const float* d_q, const void* d_k_pages, const void* d_v_pages,
                                   const int32_t* d_page_table, uint32_t t, uint32_t heads, uint32_t kv_heads,
                                   uint32_t head_dim, uint32_t page_size, float* d_out, void* d_workspace,
                                   size_t workspace_bytes, void* stream) {
    return guarded([&] {
        check_attention_args(d_q, d_k_pages, d_v_pages, d_page_table, t, heads, kv_heads, head_dim, page_size, d_out);
        require(d_workspace, "null workspace");
        require((reinterpret_cast<uintptr_t>(d_workspace) & 255) == 0, "workspace must be 256-byte aligned");
        const uint32_t nsplit = attention_splits(t, kv_heads, page_size);
        if (workspace_bytes < kWsHeader + attention_part_bytes(heads, nsplit, head_dim))
            raise(EVL_ERR_INVALID_INPUT, "workspace too small; size it with evl_attention_workspace_bytes");
        attention_standalone(d_q, d_k_pages, d_v_pages, d_page_table, t, heads, kv_heads, head_dim, page_size, d_out,
                             reinterpret_cast<float*>(static_cast<uint8_t*>(d_workspace) + kWsHeader), nsplit,
                             static_cast<int32_t*>(d_workspace), as_stream(stream));
    });
}

}  // extern "C"
