// engine.hpp -- internal host-side types of the decode engine (not part of the ABI).
//
// Model   ~ runtime.rs Model (:184-425): config, device-resident repacked weights.
// Decoder ~ runtime.rs Session (:634-808): per-sequence paged KV cache, work buffers,
//           the captured CUDA graph of one dense step. evl_session wraps one with a
//           single sequence, evl_batch one with n sequences.
#pragma once

#include <cuda_runtime.h>
#include <nccl.h>

#include <algorithm>
#include <cstdint>
#include <cstdlib>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/evelyn.h"
#include "kernels.h"

namespace evl {

// ------------------------------------------------------------------ errors
struct Error {
    evl_status code;
    std::string msg;
};
[[noreturn]] void raise(evl_status code, const std::string& msg);
void cuda_check(cudaError_t e, const char* what);
void set_last_error(const std::string& msg);
const char* last_error();

// Makes `device` current for the lifetime of the guard.
struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int device);
    ~DeviceGuard();
};

struct DeviceBuffer {
    void* p = nullptr;
    size_t bytes = 0;
    DeviceBuffer() = default;
    DeviceBuffer(const DeviceBuffer&) = delete;
    DeviceBuffer& operator=(const DeviceBuffer&) = delete;
    ~DeviceBuffer();
    void alloc(size_t n);
    template <class T> T* as() const { return static_cast<T*>(p); }
};

struct PinnedBuffer {
    void* p = nullptr;
    size_t bytes = 0;
    PinnedBuffer() = default;
    PinnedBuffer(const PinnedBuffer&) = delete;
    PinnedBuffer& operator=(const PinnedBuffer&) = delete;
    ~PinnedBuffer();
    void alloc(size_t n);
    template <class T> T* as() const { return static_cast<T*>(p); }
};

// ------------------------------------------------------------------ NCCL (resolved at run time)
struct Nccl {
    bool loaded = false;
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*AllReduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*Broadcast)(const void*, void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
};
const Nccl& nccl();  // raises EVL_ERR_NCCL when no libnccl can be loaded
void nccl_check(ncclResult_t r, const char* what);

// ------------------------------------------------------------------ GGUF (src/gguf.rs)
size_t type_bytes(uint32_t t, size_t n);  // gguf.rs:288-298; raises Unsupported
const char* type_name(uint32_t t);

struct GgufValue {
    enum Kind { U64, I64, F64, BOOL, STR, ARRAY } kind = U64;
    uint64_t u = 0;
    int64_t i = 0;
    double f = 0;
    bool b = false;
    std::string s;
    std::vector<GgufValue> arr;
    bool as_u64(uint64_t* o) const;
    bool as_f64(double* o) const;
};

struct GgufTensor {
    std::string name;
    std::vector<uint64_t> dims;
    uint32_t type = 0;
    uint64_t offset = 0;
    uint64_t elements() const;
};

class Gguf {
public:
    // Parses an image that stays alive for the parser's lifetime.
    void open(const uint8_t* data, size_t len);
    const GgufValue* meta(const std::string& key) const;
    std::string architecture() const;
    bool has(const std::string& tensor) const { return tensors_.count(tensor) != 0; }
    const GgufTensor& tensor(const std::string& name) const;  // NotFound
    const uint8_t* raw(const GgufTensor& t, size_t* nbytes) const;
    const std::map<std::string, GgufTensor>& tensors() const { return tensors_; }

private:
    const uint8_t* base_ = nullptr;
    size_t len_ = 0;
    std::map<std::string, GgufValue> meta_;
    std::map<std::string, GgufTensor> tensors_;
    uint64_t data_start_ = 0;
};

// ------------------------------------------------------------------ repacked matrices
// Host-side description of one repacked matrix (or one tensor-parallel shard of it).
struct QMatrix {
    std::string name;
    uint32_t type = 0, rows = 0, cols = 0;
    size_t total_bytes = 0;  // rows * row_bytes, rounded up to 256
    size_t offset = 0;       // inside the model's weight buffer
    QMatDev dev;             // device view once placed
    QGemmDev gemm;           // GEMM-layout copy for batched steps (q == null until built)
    size_t bytes() const { return total_bytes; }
};

// Sizes of the repacked form of a [rows][cols] tensor of `type`; raises Unsupported.
void repack_sizes(QMatrix& m);
// Points m.dev at base + m.offset.
void place(QMatrix& m, uint8_t* base);

// ------------------------------------------------------------------ model
struct Config {
    std::string arch;
    uint64_t layers = 0, dim = 0, ffn = 0, heads = 0, kv_heads = 0, head_dim = 0, rope_dim = 0, vocab = 0;
    float rope_base = 10000.f, eps = 1e-6f;
    bool rope_interleaved = false;
    int64_t eos = -1;
    // Qwen3.5 (runtime.rs:106-120, 225-235, 258)
    uint64_t full_attention_interval = 4;
    bool has_ssm = false;
    uint64_t ssm_conv_kernel = 0, ssm_inner = 0, ssm_state = 0, ssm_groups = 0, ssm_value_heads = 0;
};

// A Qwen3.5 gated-delta layer (runtime.rs:155-170): key_dim = ssm_state, key_heads =
// ssm_groups, value_dim = ssm_inner / value_heads.
struct DeltaWeights {
    QMatrix qkv, z, alpha, beta, out;
    QMatrix ab;             // alpha rows then beta rows, when the two share a type (else empty)
    float* conv = nullptr;  // [channels][kernel]
    float* a = nullptr;     // [value_heads]
    float* dt = nullptr;    // [value_heads]
    float* norm = nullptr;  // [value_dim]
    uint32_t index = 0;     // among the model's gated-delta layers (its state slot)
};

struct LayerWeights {
    QMatrix q, k, v, o, gate, up, down;
    float* attn_norm = nullptr;
    float* ffn_norm = nullptr;
    float* q_norm = nullptr;  // null when the GGUF has no attn_q_norm
    float* k_norm = nullptr;
    bool delta = false;       // Attention::GatedDelta: `d` holds it and q/k/v/o are empty
    bool gated = false;       // qwen35 full attention: `qg` is the query gate
    QMatrix qg;               // the gate rows of the interleaved attn_q (runtime.rs:687-693)
    DeltaWeights d;
};

struct Model {
    Config cfg;
    int device = 0;
    int tp_rank = 0, tp_size = 1;
    ncclComm_t comm = nullptr;
    bool kv_f32 = false;
    // this rank's shard sizes
    uint32_t lheads = 0, lkv_heads = 0, lffn = 0, lvocab = 0, vocab0 = 0;

    DeviceBuffer weights;  // every repacked matrix
    DeviceBuffer vectors;  // norms + rope table (f32)
    QMatrix embed, lm_head;
    std::vector<LayerWeights> layers;
    float* out_norm = nullptr;
    float* rope_inv_freq = nullptr;
    std::map<std::string, QMatrix*> matrices;
    std::map<std::string, std::pair<float*, size_t>> vecs;
    uint64_t weight_bytes_per_step = 0;
    // Qwen3.5: gated-delta layer count and sizes (0 for other models)
    uint32_t delta_layers = 0, delta_channels = 0, delta_value_width = 0;

    // GEMM-layout copies of every layer matrix and the LM head, built on the device the
    // first time a batch of more than one sequence is created (build_gemm_weights)
    DeviceBuffer gemm_weights;
    bool gemm_ready = false;

    // model-level calls (dense_ffn, matvec, dequantize) run on this stream
    std::mutex mu;
    cudaStream_t stream = nullptr;
    DeviceBuffer scratch;  // x[dim] | y[dim] | ybuf[dim] | h[lffn] | spare
    int32_t* d_err = nullptr;

    ~Model();
};

std::unique_ptr<Model> load_model(const uint8_t* data, size_t len, const evl_model_options& opts);

// The tensor-parallel shard of rank R of T: [first, last) rows of attn_q (and columns
// of attn_output), attn_k / attn_v, ffn_gate / ffn_up (columns of ffn_down, on
// 256-value super-block boundaries, uneven when the block count does not divide) and
// the LM head. Raises InvalidInput / Unsupported like load_model.
struct TpShard {
    uint64_t q[2], kv[2], ffn[2], vocab[2];
};
TpShard tp_shard_plan(const Config& c, int T, int R);

void allreduce_sum(Model& m, float* buf, size_t n, cudaStream_t s);

// Makes the GEMM-layout copies (QMatrix::gemm) of the layer matrices and the LM head;
// returns false (nothing built) when some matrix has no GEMM layout.
bool build_gemm_weights(Model& m);

// Per-CTA budget of a matvec's L2 prefetch of the next launches' weights, in KB:
// `dflt` scaled by the percentage in EVELYN_PREFETCH (0 turns the prefetch off).
inline uint32_t prefetch_kb(uint32_t dflt) {
    static const int pct = [] {
        const char* e = std::getenv("EVELYN_PREFETCH");
        return e ? std::max(0, std::atoi(e)) : 100;
    }();
    return (uint32_t)((uint64_t)dflt * (uint32_t)pct / 100);
}

// Device launch sequence of one dense FFN on `x` (already normalised when norm_w is
// null) writing y; add=true accumulates into y (residual). TP: partial + all-reduce.
// `next` (may be null) holds the three matrices the launch after the FFN reads
// (unused entries have q == null), warmed into L2.
// peers (tensor parallelism inside a step) sums the down-proj partials through the
// ranks' peer-memory inboxes at tag slot `slot`; null uses an NCCL all-reduce.
void run_dense_ffn(Model& m, size_t layer, const float* x, const float* norm_w, float* y, bool add, uint32_t batch,
                   float* h_buf, float* y_buf, int* err, const QMatDev* next, cudaStream_t s, bool pdl,
                   const TpPeers* peers = nullptr, uint32_t slot = 0);

// ------------------------------------------------------------------ decode attention on caller buffers
// Shared by the evl_attention_decode* entry points (abi.cpp, attention_noalloc.cu):
// argument checks (InvalidInput), the split count over the sequence, the size of the
// split partials, and one split-K attention launch with caller-provided partials and
// device error flag.
void check_attention_args(const float* d_q, const void* d_k_pages, const void* d_v_pages, const int32_t* d_page_table,
                          uint32_t t, uint32_t heads, uint32_t kv_heads, uint32_t head_dim, uint32_t page_size,
                          const float* d_out);
uint32_t attention_splits(uint32_t t, uint32_t kv_heads, uint32_t page_size);
size_t attention_part_bytes(uint32_t heads, uint32_t nsplit, uint32_t head_dim);
void attention_standalone(const float* d_q, const void* d_k_pages, const void* d_v_pages, const int32_t* d_page_table,
                          uint32_t t, uint32_t heads, uint32_t kv_heads, uint32_t head_dim, uint32_t page_size,
                          float* d_out, float* part, uint32_t nsplit, int32_t* d_err, cudaStream_t s);

// ------------------------------------------------------------------ sessions
struct StepBuffers {
    uint32_t batch = 1;
    uint32_t max_ctx = 0, pages_per_seq = 0;
    DeviceBuffer kv, page_table, pos, tokens, argmax, hist, err;
    DeviceBuffer x, q, k, v, att, h, y, logits, xn, part, amax_v, amax_i;
    // Qwen3.5: query gate; gated-delta projections (qkv channels, z, alpha | beta), the
    // recurrent output, and per sequence the conv history (two copies) and states
    DeviceBuffer qgate, dproj, dz, dab, dout, dhist, dstate;
    cudaEvent_t routed_ev = nullptr;  // routed FFN: the D2H of its input, waited on alone
    DeviceBuffer gbx, gxinv, gpart, gpart2, gpart3;  // batched products: staged x, 2^-e, partial sums
    uint32_t cluster_splits = 0, cluster_ring = 0;  // single-sequence cluster attention (ring 0: off)
    KvTmap kv_tmap{};             // the KV pool for the attention's tensor-core path
    uint32_t cluster_stages = 2;  // ring stages of the cluster attention
    uint32_t qkv_ctas = 0;        // grid cap of the QKV matvec (0: all SMs)
    bool kv_tmap_ok = false;
    uint32_t nsplit = 1, amax_parts = 1;
    PinnedBuffer h_tokens, h_argmax, h_logits, h_xn, h_y, h_err;
    // persistent step kernel (decode_step.cu): its tagged vectors (x, q, k, v, attention
    // partials, attention output, h) and the step counter their tags derive from
    DeviceBuffer tagpool, epoch;
    // tensor parallelism: this rank's inbox for the step's exchanges (tp_comm.cu), the
    // peers' inboxes and logits buffers mapped into this process
    DeviceBuffer smp_rng, smp_out, smp_m, smp_s;  // sampling: states, picks, per-part max and sums
    PinnedBuffer h_rng;
    DeviceBuffer tpinbox;
    TpPeers tp;
    const float* peer_logits[kMaxPeers] = {};
    std::vector<void*> ipc_open;
    uint64_t *xt = nullptr, *qt = nullptr, *kt = nullptr, *vt = nullptr, *partt = nullptr, *attt = nullptr,
             *ht = nullptr;
    uint32_t tag_period = 0;
};

struct Decoder {  // shared by Session (batch 1) and Batch (batch n)
    Model* model = nullptr;
    StepBuffers b;
    KvCacheDev kv;
    cudaStream_t stream = nullptr;
    cudaGraphExec_t graph = nullptr;
    bool graph_pdl = true;
    std::vector<uint64_t> host_pos;
    uint32_t kernels = 0, kernels_per_step = 0;
    StepKernel* step_k = nullptr;  // persistent whole-step kernel (single sequence)
    bool step_tried = false;
    std::string step_note;        // why the step kernel is not used, if it is not

    ~Decoder();
    // share_kv: a prefill child whose rows are positions of one sequence of that decoder
    void init(Model* m, uint32_t batch, uint32_t max_ctx, const Decoder* share_kv = nullptr);
    void init_tp();  // collective over the model's ranks: inboxes, peer mappings
    MatvecArgs qkv_args(uint32_t layer) const;
    RopeArgs rope_args(uint32_t layer) const;
    AttnArgs attn_args(uint32_t layer, uint32_t nsplit) const;
    void build_step_kernel();
    bool use_gemm = false;  // batch > 1 on one GPU: tensor-core products
    void enqueue_batched(bool pdl);
    void gemm_stage(const float* x, uint32_t cols, uint32_t stride, const float* norm_w, bool pdl);
    void gemm_product(const QMatrix& w, float* part, uint32_t& ksplit, bool pdl);
    GemmReduce reduce_args(const QMatrix& w, const float* part, uint32_t ksplit, float* y, uint32_t y_stride, int epi,
                           const float* part2, uint32_t ksplit2) const;
    void gemm_reduce(const QMatrix& w, const float* part, uint32_t ksplit, float* y, uint32_t y_stride, int epi,
                     const float* part2, uint32_t ksplit2, bool pdl);
    // Enqueue one dense step (every kernel) on `stream`.
    void enqueue_dense(bool pdl);
    void enqueue_layer_attention(uint32_t layer, bool pdl);
    void enqueue_delta(uint32_t layer, bool pdl);  // a Qwen3.5 gated-delta layer's attention half
    void enqueue_head(bool pdl);
    void gather_peer_logits();
    // A step with a routed-FFN hook (eager, synchronising at routed layers).
    void run_routed(const evl_ffn_backend& ffn);
    void launch_graph();
    void check_device_error();
    // Session::step for every sequence: host tokens in, optional host logits/argmax out.
    void step(const uint32_t* tokens, const evl_ffn_backend* ffn, float* logits_out, uint32_t* argmax_out);
    // On-device greedy loop of n steps (single sequence).
    void generate(uint32_t token, uint32_t n, uint32_t* tokens_out);
    // Temperature sampling of every sequence from the last step's logits (host states
    // in/out, host tokens out).
    void sample(float temperature, uint64_t* states, uint32_t* tokens_out);
    // Batched prompt processing of sequence `seq`: n tokens, optional logits [n][vocab]
    // and argmax [n] (host).
    void prefill(uint32_t seq, const uint32_t* tokens, size_t n, float* logits_out, uint32_t* argmax_out);
    std::unique_ptr<Decoder> pf;  // prefill child (made on first use)
    bool pf_stepwise = false;     // no tensor-core products for this model: a single
                                  // session's prefill runs one step per prompt token
    bool prefill_child = false;
    // what the child's device page table holds: its rows [0, pf_rows) map sequence
    // pf_seq's pages, the rest the spare page (pf_rows = 0: not written yet)
    uint32_t pf_rows = 0, pf_seq = 0;
};

}  // namespace evl

struct evl_model {
    std::unique_ptr<evl::Model> m;
};
struct evl_session {
    evl::Decoder d;
    mutable std::string notes;  // evl_session_notes' text
};
struct evl_batch {
    evl::Decoder d;
};
struct evl_qmatrix {
    evl::QMatrix m;
    evl::DeviceBuffer buf;
    evl::DeviceBuffer err;  // device error flag of this matrix's launches
    int device = 0;
    // batched products (made on first use): GEMM-layout copy, staged x, partial sums
    evl::DeviceBuffer gemm_buf, bx, xinv, part;
    evl::QGemmDev gemm;
};
