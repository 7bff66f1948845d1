// kernels.h -- host-side launchers of the decode kernels.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "common.cuh"

namespace evl {

// ---------------------------------------------------------------- dequant.cu
cudaError_t launch_dequant_raw(uint32_t type, const void* raw, uint64_t n, float* out, cudaStream_t s);
cudaError_t launch_dequant_repacked(const QMatDev& m, uint32_t row0, uint32_t nrows, float* out, cudaStream_t s);
// Repack raw GGUF rows (device memory, `stride` bytes apart) into the matvec layout of
// `d` at dst (dst_bytes, zeroed first: the padding rows of the last slab).
cudaError_t launch_repack(const QMatDev& d, uint8_t* dst, uint64_t dst_bytes, const void* raw, uint64_t stride,
                          cudaStream_t s);

// ---------------------------------------------------------------- qmatvec.cu
enum MatvecEpilogue : int {
    EPI_STORE = 0,   // y[r] = W x
    EPI_ADD = 1,     // y[r] += W x          (residual add after o-proj / down-proj)
    EPI_SWIGLU = 2,  // y[r] = silu(Wg x) * (Wu x)   (m = gate, m2 = up)
};

struct MatvecSeg {
    QMatDev m;
    QMatDev m2;          // up matrix for EPI_SWIGLU
    float* y = nullptr;
    int epi = EPI_STORE;
};

constexpr int kMaxSegs = 3;

struct MatvecArgs {
    MatvecSeg seg[kMaxSegs];
    int nseg = 0;
    const float* x = nullptr;      // input vector, cols floats
    uint32_t cols = 0;
    const float* norm_w = nullptr; // fused RMSNorm weight (null: x used as is)
    float eps = 1e-6f;
    QMatDev prefetch[3];           // matrices the next launches read, in order (q == null:
                                   // none); this CTA's share of each is warmed into L2 at
                                   // the end, up to prefetch_bytes per CTA
    uint32_t prefetch_bytes = 96u << 10;
    uint32_t max_ctas = 0;         // grid cap (0: one CTA per SM), leaving SMs to the next launch
    int* err = nullptr;            // device error flag (DeviceError), required
};

// One fused launch over up to three matrices that share the input vector (all of
// the same width). Types Q4_K, Q5_K, Q6_K, Q8_0; a launch with any F16, BF16 or F32
// matrix, or a gate and up of two types, runs as launch_plain_matvec.
cudaError_t launch_qmatvec(const MatvecArgs& a, cudaStream_t s, bool pdl);

// ---------------------------------------------------------------- gated_delta.cu
// The recurrent half of a Qwen3.5 gated-delta layer (runtime.rs:551-630) between its
// projections and ssm_out: conv, q/k normalisation, the delta rule on the state, the
// per-head norm and SiLU(z) gate. A cluster of up to 4 CTAs per (value head, sequence),
// each on a slice of the head's value columns (one CTA per head where the slice does
// not fit in shared memory).
struct GatedDeltaArgs {
    const float* proj = nullptr;   // [batch][channels] attn_qkv output (q | k | v channels)
    const float* z = nullptr;      // [batch][value_heads * value_dim] attn_gate output
    const float* ab = nullptr;     // [batch][2 * value_heads] ssm_alpha | ssm_beta outputs
    const float* conv = nullptr;   // [channels][kernel]
    const float* a = nullptr;      // [value_heads]
    const float* dt = nullptr;     // [value_heads]
    const float* norm = nullptr;   // [value_dim]
    float* hist = nullptr;         // per sequence [2][kernel - 1][channels] (copy pos % 2 read)
    float* state = nullptr;        // per sequence [value_heads][key_dim][value_dim]
    float* out = nullptr;          // [batch][value_heads * value_dim]
    const int32_t* pos = nullptr;  // [batch] this token's position
    uint32_t batch = 1, channels = 0, kernel = 0, key_dim = 0, key_heads = 0, value_dim = 0, value_heads = 0;
    uint64_t hist_stride = 0, state_stride = 0;  // floats per sequence
    float eps = 1e-6f;
};
size_t gated_delta_smem(uint32_t key_dim, uint32_t value_dim);
cudaError_t launch_gated_delta(const GatedDeltaArgs& a, cudaStream_t s, bool pdl);

// plain_matvec.cu: the same launch, warp per row, for unquantised matrices (a
// quantised matrix in it is read through the exact dequantiser).
bool matvec_has_plain(const MatvecArgs& a);
cudaError_t launch_plain_matvec(const MatvecArgs& a, cudaStream_t s, bool pdl);

// ---------------------------------------------------------------- attention.cu
// Paged KV cache. The K tile of (page, layer, head) starts at
//   pool + page*page_stride + layer*layer_stride + head*head_stride
// and its V tile v_offset bytes further on. The engine's own pool is
// [pages][layers][k|v][kv_heads][page_size][head_dim] (v_offset = kv_heads*head_stride).
struct KvCacheDev {
    void* pool = nullptr;
    uint64_t page_stride = 0;      // bytes per page (all layers)
    uint64_t layer_stride = 0;     // bytes per layer inside a page
    uint64_t head_stride = 0;      // bytes per (k|v, head) tile
    int64_t v_offset = 0;          // bytes from a K tile to its V tile
    int64_t k_offset = 0;          // bytes from pool to the K tiles (0 for the engine's pool)
    uint32_t page_size = 16;
    uint32_t elem_bytes = 2;       // 2 = f16, 4 = f32
};

struct RopeArgs {
    float* q = nullptr;            // [batch][heads*hd]   in/out
    const float* k = nullptr;      // [batch][kv_heads*hd]
    const float* v = nullptr;
    const float* q_norm = nullptr; // per-head RMSNorm weights (null: none)
    const float* k_norm = nullptr;
    KvCacheDev kv;
    uint32_t layer = 0;
    const int32_t* page_table = nullptr;  // [batch][max_pages]
    uint32_t max_pages = 0;
    const int32_t* pos = nullptr;  // [batch] position of the new token
    uint32_t batch = 1, heads = 0, kv_heads = 0, head_dim = 0, rope_dim = 0;
    float rope_base = 1e6f, eps = 1e-6f;
    int interleaved = 0;
    const float* rope_inv_freq = nullptr;  // [rope_dim/2] base^(-2i/rope_dim), host-computed
    int* err = nullptr;            // device error flag (DeviceError)
};
cudaError_t launch_qk_norm_rope_append(const RopeArgs& a, cudaStream_t s, bool pdl);

struct AttnArgs {
    const float* q = nullptr;      // [batch][heads*hd] (normed + rotated)
    float* out = nullptr;          // [batch][heads*hd]
    KvCacheDev kv;
    uint32_t layer = 0;
    const int32_t* page_table = nullptr;
    uint32_t max_pages = 0;
    const int32_t* pos = nullptr;  // attend to positions [0, pos]; null: use pos_value
    int32_t pos_value = 0;         // (single sequence)
    uint32_t batch = 1, heads = 0, kv_heads = 0, head_dim = 0;
    uint32_t nsplit = 1;           // fixed grid split count; each split covers
                                   // ceil(t / nsplit) positions rounded up to whole pages
    float* part = nullptr;         // scratch [batch][heads][nsplit][head_dim + 2]
    float scale = 0.f;
    int* err = nullptr;            // device error flag (DeviceError)
    const float* gate = nullptr;   // [batch][heads*hd] or null: out *= sigmoid(gate), the
                                   // gated query of Qwen3.5 (runtime.rs:753-761)
};
cudaError_t launch_attention(const AttnArgs& a, cudaStream_t s, bool pdl);
// QK-norm + RoPE + append, split-K attention and the split merge in one launch of one
// thread-block cluster of a.nsplit (1, 2, 4 or 8) CTAs per (sequence, kv head)
// (attention_cluster.cu); each CTA streams its split's pages through a shared ring of
// `ring_pages` pages. attention_cluster_pages: the ring for a cache of max_pages pages
// per sequence (at most cap pages), 0 when this path does not apply.
uint32_t attention_cluster_pages(uint32_t max_pages, uint32_t nsplit, uint32_t page_size, uint32_t head_dim,
                                 uint32_t elem_bytes, uint32_t group, uint32_t cap = 16);
// The KV pool viewed as [rows][head_dim] f16 rows (16-row x 64-value boxes, 128-byte
// swizzle), for the tensor-core path of launch_attention_cluster. Opaque copy of a
// CUtensorMap; false when the driver call or the shape is not available.
struct alignas(64) KvTmap {
    unsigned long long w[16];
};
bool make_kv_tmap(const void* pool, uint64_t bytes, uint32_t head_dim, KvTmap* out);
// The ring streams in `stages` chunks (2 or 4, dividing ring_pages), each read by its
// own warp group. tmap (optional):
// f16 pages of 16 rows run on the tensor cores (mma.sync), else the scalar loop.
cudaError_t launch_attention_cluster(const RopeArgs& r, const AttnArgs& a, uint32_t ring_pages, uint32_t stages,
                                     cudaStream_t s, bool pdl, const KvTmap* tmap = nullptr);

// ---------------------------------------------------------------- decode_step.cu
// A whole single-sequence decode step as one persistent kernel (decode_step.cu). Its
// phases hand vectors to one another as tagged pairs: each element is one 8-byte word,
// (tag << 32) | f32 bits, stored in a single access; a reader waits until the words it
// needs carry the tag it expects. Tags are `epoch * period + 1 + slot`, where epoch is
// the number of completed steps (a device counter the step's argmax advances) and
// slot names the (layer, vector) the word belongs to.
constexpr int kMaxPeers = 8;  // tensor-parallel ranks a phase writes its rows to

// Where the rows of a matvec segment (or the attention output) go: the same rows
// [row0, row0 + rows) of ndst full-length vectors -- this rank's copy first, then the
// peers' copies (tensor parallelism) -- as tagged words (dst) or plain floats (plain).
struct TaggedOut {
    uint64_t* dst[kMaxPeers] = {};
    float* plain[kMaxPeers] = {};
    uint32_t ndst = 0, row0 = 0, tag = 0;
    const uint64_t* resid = nullptr;  // EPI_ADD: the residual (this rank's full vector, tagged)
    uint32_t resid_tag = 0;
};

// QK-norm, RoPE, KV append, split-K GQA attention and the split merge of one layer.
struct StepAttn {
    const uint64_t *q = nullptr, *k = nullptr, *v = nullptr;  // tagged [lheads*hd], [lkv*hd], [lkv*hd]
    uint32_t qkv_tag = 0;
    uint64_t* part = nullptr;  // tagged partials [lkv][nsplit][G][hd + 2] (o..., m, l)
    uint32_t part_tag = 0;
    TaggedOut out;             // attention output rows [lheads * hd] at row0 of [heads * hd]
    RopeArgs rope;             // norms, RoPE table, KV cache, layer, page table, position, shape
    uint32_t nsplit = 1;       // splits per kv head (one CTA each)
    uint32_t ring_pages = 2;   // K/V page pairs a split stages at a time (even)
    float scale = 0.f;
};

enum StepPhaseKind : uint32_t { STEP_MATVEC = 0, STEP_ATTN = 1 };
struct StepPhaseDesc {
    uint32_t kind = STEP_MATVEC;
    MatvecArgs mv;                 // segments, cols, norm_w, eps (x and seg[].y unused)
    const uint64_t* xt = nullptr;  // tagged input [cols]
    uint32_t x_tag = 0;
    TaggedOut out[kMaxSegs];
    StepAttn at;
};
struct StepKernel;
// Builds the persistent step kernel over `n` phases (one cooperative CTA per SM);
// `epoch` is read at the start of every launch, `period` the tag slots per step.
// cudaErrorInvalidValue / cudaErrorNotSupported when the phases do not fit it.
cudaError_t step_kernel_create(const StepPhaseDesc* phases, uint32_t n, const uint32_t* epoch, uint32_t period,
                               int* err, StepKernel** out);
cudaError_t step_kernel_launch(const StepKernel* k, cudaStream_t s);
// Clears the grid abort flag (after a step that reported an error).
cudaError_t step_kernel_reset(const StepKernel* k, cudaStream_t s);
void step_kernel_destroy(StepKernel* k);
// Splits and page-ring size the step kernel's attention phase uses for a cache of
// max_pages pages per sequence on a GPU with `sms` SMs.
uint32_t step_attn_splits(uint32_t kv_heads, uint32_t max_pages, int sms);
// The embedding row of tokens[0] (QMatrix::row, src/runtime.rs:54-69) as tagged words
// with slot 0 of the current epoch.
cudaError_t launch_embed_tagged(const QMatDev& embed, const int32_t* tokens, uint64_t* xt, const uint32_t* epoch,
                                uint32_t period, int32_t* err, cudaStream_t s);

// ---------------------------------------------------------------- tp_comm.cu
// Tensor-parallel exchanges of a step through inboxes in peer memory (tp_comm.cu).
// inbox[r] is rank r's inbox as mapped into this process: [purpose][sender][cap] tagged
// words. Tags are epoch * period + 1 + slot, as in decode_step.cu.
enum TpPurpose : uint32_t { TP_O = 0, TP_DOWN = 1, TP_PICK = 2, TP_PURPOSES = 3 };
struct TpPeers {
    uint64_t* inbox[kMaxPeers] = {};
    uint32_t rank = 0, size = 1;
    uint32_t cap = 0;  // words per (purpose, sender)
    const uint32_t* epoch = nullptr;
    uint32_t period = 0;  // tag slots per step
};
// x[i] += (sum over ranks in rank order of each rank's part[i]) for i < n.
cudaError_t launch_tp_allreduce_add(const TpPeers& P, uint32_t purpose, uint32_t slot, float* x, const float* part,
                                    uint32_t n, int* err, cudaStream_t s, bool pdl);
// Greedy pick (src/runtime.rs:897-905) over the ranks' vocabulary shards: this rank's
// shard is logits[b * stride + v0 + i], i < n; ends the step like launch_argmax and
// advances epoch.
cudaError_t launch_tp_argmax(const TpPeers& P, uint32_t slot, const float* logits, uint32_t stride, uint32_t v0,
                             uint32_t n, uint32_t batch, float* part_v, int32_t* part_i, uint32_t parts, int32_t* out,
                             int32_t* next_tokens, int32_t* pos, int32_t* hist, uint32_t hist_stride, uint32_t* epoch,
                             int* err, cudaStream_t s, bool pdl);

// ---------------------------------------------------------------- qgemm.cu
// A matrix in the GEMM layout (per 128-row M tile and 256-value K chunk, one block of
// the original quant bytes split by field), made on the device from the matvec layout.
struct QGemmDev {
    uint32_t type = 0, rows = 0, cols = 0;
    uint32_t mtiles = 0, nchunks = 0, block_bytes = 0;
    const uint8_t* q = nullptr;
};
uint64_t gemm_layout_bytes(uint32_t type, uint32_t rows, uint32_t cols);  // 0: unsupported
QGemmDev gemm_view(uint32_t type, uint32_t rows, uint32_t cols, const uint8_t* q);
cudaError_t launch_gemm_repack(const QMatDev& src, const QGemmDev& dst, cudaStream_t s);

// x of nseq <= 32 sequences -> the MMA B operand (gemm_x_bytes) and per-sequence 2^-e
struct GemmX {
    const float* x = nullptr;  // [nseq][x_stride]
    uint32_t nseq = 0, cols = 0, x_stride = 0, nsp = 0;
    const float* norm_w = nullptr;  // fused RMSNorm (null: none)
    float eps = 1e-6f;
    uint8_t* bx = nullptr;
    float* xinv = nullptr;          // [nseq]
    float* stats = nullptr;         // [nseq][2] scratch: RMS scale, 2^e
};
uint64_t gemm_x_bytes(uint32_t nseq, uint32_t cols);
cudaError_t launch_gemm_stage_x(GemmX a, cudaStream_t s, bool pdl);
// rows up to this many values are staged in one launch (else two)
uint32_t gemm_stage_one_launch_cols();

// part[kr][seq][rows_pad] = sum over K range kr of W x (ksplit ranges per M tile)
struct GemmArgs {
    QGemmDev w;
    const uint8_t* bx = nullptr;
    const float* xinv = nullptr;
    uint32_t nseq = 0, ksplit = 1, rows_pad = 0;
    float* part = nullptr;
    int* err = nullptr;
};
uint32_t gemm_ksplit(const QGemmDev& w, int sms);
cudaError_t launch_qgemm(const GemmArgs& a, cudaStream_t s, bool pdl);

// y[seq][r] (op)= sum_kr part[kr][seq][r]; EPI_SWIGLU: silu(sum part) * sum part2
struct GemmReduce {
    const float* part = nullptr;
    const float* part2 = nullptr;
    uint32_t ksplit = 1, ksplit2 = 1, rows_pad = 0, rows_pad2 = 0;
    uint32_t nseq = 0, rows = 0;
    float* y = nullptr;
    uint32_t y_stride = 0;
    int epi = EPI_STORE;
};
cudaError_t launch_gemm_reduce(const GemmReduce& a, cudaStream_t s, bool pdl);
// up to three independent reductions in one launch (e.g. the Q, K and V products)
cudaError_t launch_gemm_reduce_n(const GemmReduce* a, uint32_t n, cudaStream_t s, bool pdl);

// ---------------------------------------------------------------- misc.cu
cudaError_t launch_embed(const QMatDev& embed, const int32_t* tokens, uint32_t batch, float* x, int32_t* err,
                         cudaStream_t s, bool pdl);
cudaError_t launch_rmsnorm(const float* x, const float* w, float* y, uint32_t n, uint32_t batch, float eps,
                           cudaStream_t s, bool pdl);
cudaError_t launch_add(float* x, const float* y, uint64_t n, cudaStream_t s, bool pdl);
// Warm up to four device ranges into L2 (bulk prefetches of 16 KB, 16-byte aligned
// starts; a null base is skipped): the device's work while the host waits on something.
struct L2Ranges {
    const uint8_t* base[4] = {};
    uint64_t bytes[4] = {};
};
cudaError_t launch_l2_prefetch(const L2Ranges& r, cudaStream_t s);
// Greedy pick over [batch][n] logits: first maximum wins (strict '>' like src/runtime.rs:897-905).
// Optionally writes the pick to next_tokens, logs it at hist[b*hist_stride + pos[b]] and
// advances pos[b] (null pointers skip each part).
// Temperature sampling of each of `batch` logits rows (src/server.rs:326-352): rng[b] is
// the xorshift64* state (device), advanced as the reference advances it; argmax[b] is
// the greedy pick of the same row (the fallback). part_m [batch][parts] and part_s
// (doubles) are scratch. temperature > FLT_EPSILON (the caller takes argmax otherwise).
cudaError_t launch_sample(const float* logits, uint32_t n, uint32_t batch, float temperature, uint64_t* rng,
                          const int32_t* argmax, float* part_m, double* part_s, uint32_t parts, int32_t* out,
                          cudaStream_t s);
// epoch (optional) is advanced once the pick is made: the step's last kernel.
cudaError_t launch_argmax(const float* logits, uint32_t n, uint32_t batch, float* part_v, int32_t* part_i,
                          uint32_t parts, int32_t* out, int32_t* next_tokens, int32_t* pos, int32_t* hist,
                          uint32_t hist_stride, cudaStream_t s, bool pdl, uint32_t* epoch = nullptr);

}  // namespace evl
