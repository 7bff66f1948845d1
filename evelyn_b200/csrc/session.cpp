// session.cpp -- Session::step on the device (src/runtime.rs:634-808).
//
// One dense step is a fixed launch sequence over device-resident state:
//   embed row -> per layer { RMSNorm+QKV matvec (one launch over Wq, Wk, Wv),
//   QK-norm + RoPE + paged-KV append, split-K GQA attention + merge,
//   o-proj matvec with the residual add fused, RMSNorm + gate/up matvec with the
//   SwiGLU fused, down matvec with the residual add fused } -> final RMSNorm +
//   LM-head matvec -> argmax (which also feeds the next token and advances pos).
// Token, position and page table live in device memory, so the sequence is
// captured once as a CUDA graph (with programmatic dependent launches between
// kernels) and replayed every step. Layers routed through an FfnBackend hook
// (runtime.rs:801-804) break the graph: the step then runs eagerly and crosses to
// the host only at those layers.
#include <algorithm>
#include <cfloat>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "engine.hpp"

namespace evl {

namespace {
constexpr uint32_t kPageSize = 16;

// One launch of a fused matvec per sequence.
void matvec_each(const MatvecArgs& base, uint32_t batch, uint64_t x_stride, const uint64_t* y_strides, cudaStream_t s,
                 bool pdl, const char* what) {
    for (uint32_t bi = 0; bi < batch; ++bi) {
        MatvecArgs a = base;
        a.x = base.x + bi * x_stride;
        for (int k = 0; k < a.nseg; ++k) a.seg[k].y = base.seg[k].y + bi * y_strides[k];
        cuda_check(launch_qmatvec(a, s, pdl), what);
    }
}
}  // namespace

Decoder::~Decoder() {
    if (model) {
        DeviceGuard g(model->device);
        if (graph) cudaGraphExecDestroy(graph);
        if (step_k) step_kernel_destroy(step_k);
        if (b.routed_ev) cudaEventDestroy(b.routed_ev);
        if (stream) cudaStreamDestroy(stream);
        for (void* p : b.ipc_open) cudaIpcCloseMemHandle(p);
    }
}

void Decoder::init(Model* m, uint32_t batch, uint32_t max_ctx, const Decoder* share_kv) {
    model = m;
    const Config& c = m->cfg;
    if (batch == 0) raise(EVL_ERR_INVALID_INPUT, "batch must be at least 1");
    if (max_ctx == 0) raise(EVL_ERR_INVALID_INPUT, "max_ctx must be at least 1");
    prefill_child = share_kv != nullptr;
    b.batch = batch;
    b.max_ctx = max_ctx;
    b.pages_per_seq = (max_ctx + kPageSize - 1) / kPageSize;
    const uint64_t hd = c.head_dim, L = c.layers;
    const uint64_t elem = m->kv_f32 ? 4 : 2;
    const uint64_t head_stride = (uint64_t)kPageSize * hd * elem;
    const uint64_t layer_stride = 2ull * m->lkv_heads * head_stride;
    const uint64_t page_stride = L * layer_stride;
    const uint64_t pages = (uint64_t)batch * b.pages_per_seq;
    if (share_kv) {
        // the prompt rows of a prefill write and read their parent's cache; the page
        // table is written per prefill call (Decoder::prefill)
        kv = share_kv->kv;
        b.pages_per_seq = share_kv->b.pages_per_seq;
        b.page_table.alloc((uint64_t)batch * b.pages_per_seq * 4);
    } else {
        // one spare page past the sequences' own: a prefill's padding rows write there
        b.kv.alloc((pages + 1) * page_stride);
        // zeroed: the tensor-core attention multiplies whole 16-position page tiles by
        // the softmax weights, 0 for the positions not written yet, so those must hold
        // finite values (0 * NaN would poison the sum)
        cuda_check(cudaMemset(b.kv.p, 0, b.kv.bytes), "memset KV cache");
        kv.pool = b.kv.p;
        kv.page_stride = page_stride;
        kv.layer_stride = layer_stride;
        kv.head_stride = head_stride;
        kv.v_offset = (int64_t)(m->lkv_heads * head_stride);
        kv.page_size = kPageSize;
        kv.elem_bytes = (uint32_t)elem;
        // every sequence owns a contiguous run of pages
        std::vector<int32_t> pt(pages);
        for (uint64_t i = 0; i < pages; ++i) pt[i] = (int32_t)i;
        b.page_table.alloc(pages * 4);
        cuda_check(cudaMemcpy(b.page_table.p, pt.data(), pages * 4, cudaMemcpyHostToDevice), "page table");
    }
    const uint64_t qw = (uint64_t)m->lheads * hd, kw = (uint64_t)m->lkv_heads * hd;
    b.pos.alloc(batch * 4);
    b.tokens.alloc(batch * 4);
    b.argmax.alloc(batch * 4);
    b.hist.alloc((uint64_t)batch * max_ctx * 4);
    b.err.alloc(4);
    cuda_check(cudaMemset(b.pos.p, 0, batch * 4), "memset");
    cuda_check(cudaMemset(b.tokens.p, 0, batch * 4), "memset");
    cuda_check(cudaMemset(b.err.p, 0, 4), "memset");
    b.x.alloc(batch * c.dim * 4);
    b.q.alloc(batch * qw * 4);
    b.k.alloc(batch * kw * 4);
    b.v.alloc(batch * kw * 4);
    b.att.alloc(batch * qw * 4);
    b.h.alloc((uint64_t)batch * m->lffn * 4);
    b.y.alloc(batch * std::max<uint64_t>(c.dim, m->lvocab) * 4);
    b.logits.alloc(batch * c.vocab * 4);
    b.xn.alloc(batch * c.dim * 4);
    if (c.has_ssm) {  // Qwen3.5: query gates; gated-delta projections and per-sequence state
        b.qgate.alloc(batch * qw * 4);
        if (m->delta_layers) {
            const uint64_t CH = m->delta_channels, VW = m->delta_value_width, VH = c.ssm_value_heads;
            b.dproj.alloc(batch * CH * 4);
            b.dz.alloc(batch * VW * 4);
            b.dab.alloc(batch * 2 * VH * 4);
            b.dout.alloc(batch * VW * 4);
            // zero at the start of every sequence (runtime.rs:539-548)
            b.dhist.alloc(std::max<uint64_t>(4, batch * m->delta_layers * 2 * (c.ssm_conv_kernel - 1) * CH * 4));
            b.dstate.alloc((uint64_t)batch * m->delta_layers * VH * c.ssm_state * (c.ssm_inner / VH) * 4);
            cuda_check(cudaMemset(b.dhist.p, 0, b.dhist.bytes), "memset");
            cuda_check(cudaMemset(b.dstate.p, 0, b.dstate.bytes), "memset");
        }
    }
    // enough (kv_head, split) CTAs to cover the SMs twice
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, m->device);
    // splits per (kv head, sequence): enough CTAs to cover the SMs twice; a batch keeps
    // at least 32 pages (512 positions) of each sequence per split so long contexts
    // still spread over many CTAs
    const uint32_t want = (uint32_t)(2 * sms) / std::max<uint32_t>(1, m->lkv_heads * batch);
    const uint32_t by_len = batch > 1 ? (b.pages_per_seq + 31) / 32 : 1;
    b.nsplit = std::max<uint32_t>(1, std::min<uint32_t>(std::max<uint32_t>({want, by_len, 1u}), b.pages_per_seq));
    b.part.alloc((uint64_t)batch * m->lheads * b.nsplit * (hd + 2) * 4);
    {  // attention with QK-norm/RoPE/append and the split merge in one cluster launch
        // f16 pages take the tensor-core loop (EVELYN_ATTN_MMA=0: the scalar one). A batch
        // without it uses the split kernels, which run its many (sequence, kv head) pairs
        // faster than the scalar loop.
        const char* fe = std::getenv("EVELYN_FUSED_ATTN");
        const char* me = std::getenv("EVELYN_ATTN_MMA");
        const bool mma_ok = elem == 2 && !(me && me[0] == '0');
        // (a prefill's rows append before any of them reads: the split kernels, whose
        // append is a launch of its own)
        if ((batch == 1 || mma_ok) && !(fe && fe[0] == '0') && !prefill_child) {
            // one sequence: 8 splits per kv head; a batch: as few as keep ~2 CTAs per SM busy
            uint32_t C = 8;
            while (C > 1 && m->lkv_heads * batch * C > 2u * (uint32_t)sms) C /= 2;
            if (const char* ce = std::getenv("EVELYN_ATTN_SPLITS"))  // 1, 2, 4 or 8 (tests)
                for (C = 8; C > 1 && C > (uint32_t)std::strtoul(ce, nullptr, 10);) C /= 2;
            // EVELYN_ATTN_RING caps the ring (even, >= 2), so tests reach the streamed
            // multi-chunk case at small contexts
            const char* re = std::getenv("EVELYN_ATTN_RING");
            // (a batch's long splits take the largest ring: the copies in flight bound them)
            const uint32_t cap = re ? (uint32_t)std::strtoul(re, nullptr, 10) & ~1u : (batch > 1 ? 24u : 16u);
            const uint32_t ring = attention_cluster_pages(b.pages_per_seq, C, kPageSize, (uint32_t)hd, (uint32_t)elem,
                                                          m->lheads / std::max<uint32_t>(1, m->lkv_heads),
                                                          std::max<uint32_t>(cap, 2));
            if (ring) {
                b.cluster_splits = C;
                b.cluster_ring = ring;
                // one sequence: two stages (double buffering; more, smaller chunks measured
                // slower, the chunk's compute rather than its copy bounds a split); a batch:
                // four (two warp groups double-buffered, measured 2914 against 2874 tok/s at
                // 32 sequences); EVELYN_ATTN_STAGES (2 .. 4) overrides
                const char* se = std::getenv("EVELYN_ATTN_STAGES");
                uint32_t st = se ? (uint32_t)std::strtoul(se, nullptr, 10) : (batch > 1 ? 4u : 2u);
                st = st >= 4 && ring % 4 == 0 && ring >= 8 ? 4u : 2u;
                b.cluster_stages = st;
                // EVELYN_QKV_CTAS caps the QKV matvec's grid so the attention's CTAs can
                // start on the SMs it leaves free (measured slower than the full grid: off)
                if (const char* qe = std::getenv("EVELYN_QKV_CTAS")) b.qkv_ctas = (uint32_t)std::strtoul(qe, nullptr, 10);
                if (mma_ok) b.kv_tmap_ok = make_kv_tmap(b.kv.p, b.kv.bytes, (uint32_t)hd, &b.kv_tmap);
                if (batch > 1 && !b.kv_tmap_ok) b.cluster_ring = 0;  // no tensor map: split kernels
            }
        }
    }
    b.amax_parts = (uint32_t)sms;
    b.amax_v.alloc((uint64_t)batch * b.amax_parts * 4);
    b.amax_i.alloc((uint64_t)batch * b.amax_parts * 4);
    b.h_tokens.alloc(batch * 4);
    b.h_argmax.alloc(batch * 4);
    b.h_logits.alloc(batch * c.vocab * 4);
    b.h_xn.alloc(c.dim * 4);
    b.h_y.alloc(c.dim * 4);
    b.h_err.alloc(4);
    *b.h_err.as<int>() = 0;
    cuda_check(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "cudaStreamCreate");
    host_pos.assign(batch, 0);
    // a batch of sequences on one GPU runs its products on the tensor cores
    const char* env = std::getenv("EVELYN_BATCH_GEMM");
    // (not for the Qwen3.5 hybrid layers, which run as matvecs per sequence)
    if (batch > 1 && batch <= 32 && !(env && env[0] == '0') && !c.has_ssm && build_gemm_weights(*m)) {
        use_gemm = true;
        const uint64_t kmax = std::max<uint64_t>({c.dim, (uint64_t)m->lffn, qw});
        b.gbx.alloc(gemm_x_bytes(32, (uint32_t)kmax));
        b.gxinv.alloc(3 * 32 * 4);  // xinv[32] | stats[32][2]
        uint64_t pmax = 0;
        std::vector<const QMatrix*> mats = {&m->lm_head};
        for (const auto& L : m->layers)
            for (const QMatrix* q : {&L.q, &L.k, &L.v, &L.o, &L.gate, &L.up, &L.down}) mats.push_back(q);
        for (const QMatrix* q : mats)
            pmax = std::max<uint64_t>(pmax, (uint64_t)gemm_ksplit(q->gemm, sms) * batch * q->gemm.mtiles * 128 * 4);
        b.gpart.alloc(pmax);
        b.gpart2.alloc(pmax);
        b.gpart3.alloc(pmax);
    }
    if (m->tp_size > 1) init_tp();
}

// Tensor parallelism: this rank's inbox for the step's exchanges and the mappings of
// every peer's inbox and logits buffer (CUDA IPC handles swapped with one NCCL
// all-gather). Every rank creates its session or batch together with the others.
void Decoder::init_tp() {
    Model& m = *model;
    const uint32_t T = (uint32_t)m.tp_size, R = (uint32_t)m.tp_rank, L = (uint32_t)m.cfg.layers;
    if (T > (uint32_t)kMaxPeers) raise(EVL_ERR_UNSUPPORTED, "tensor parallelism over more than 8 ranks");
    const uint64_t cap = ((std::max<uint64_t>((uint64_t)b.batch * m.cfg.dim, 2ull * b.batch)) + 31) & ~31ull;
    b.tpinbox.alloc((uint64_t)TP_PURPOSES * T * cap * 8);
    cuda_check(cudaMemset(b.tpinbox.p, 0xff, b.tpinbox.bytes), "memset");  // tag 0xffffffff: never expected
    if (!b.epoch.p) {
        b.epoch.alloc(4);
        cuda_check(cudaMemset(b.epoch.p, 0, 4), "memset");
    }
    cudaIpcMemHandle_t mine[2];
    cuda_check(cudaIpcGetMemHandle(&mine[0], b.tpinbox.p), "cudaIpcGetMemHandle");
    cuda_check(cudaIpcGetMemHandle(&mine[1], b.logits.p), "cudaIpcGetMemHandle");
    DeviceBuffer send, all;
    send.alloc(sizeof(mine));
    all.alloc(sizeof(mine) * T);
    cuda_check(cudaMemcpy(send.p, mine, sizeof(mine), cudaMemcpyHostToDevice), "H2D handles");
    nccl_check(nccl().AllGather(send.p, all.p, sizeof(mine), ncclUint8, m.comm, stream), "ncclAllGather");
    std::vector<cudaIpcMemHandle_t> hs(2 * T);
    cuda_check(cudaMemcpyAsync(hs.data(), all.p, sizeof(mine) * T, cudaMemcpyDeviceToHost, stream), "D2H handles");
    cuda_check(cudaStreamSynchronize(stream), "handle exchange");
    b.tp = TpPeers{};
    for (uint32_t r = 0; r < T; ++r) {
        if (r == R) {
            b.tp.inbox[r] = b.tpinbox.as<uint64_t>();
            b.peer_logits[r] = b.logits.as<float>();
            continue;
        }
        void* pi = nullptr;
        void* pl = nullptr;
        cuda_check(cudaIpcOpenMemHandle(&pi, hs[2 * r], cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
        b.ipc_open.push_back(pi);
        cuda_check(cudaIpcOpenMemHandle(&pl, hs[2 * r + 1], cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
        b.ipc_open.push_back(pl);
        b.tp.inbox[r] = static_cast<uint64_t*>(pi);
        b.peer_logits[r] = static_cast<const float*>(pl);
    }
    b.tp.rank = R;
    b.tp.size = T;
    b.tp.cap = (uint32_t)cap;
    b.tp.epoch = b.epoch.as<uint32_t>();
    b.tp.period = 2 * L + 1;  // slots: o of layer l 2l, down 2l + 1, the pick 2L
}

void Decoder::gemm_stage(const float* x, uint32_t cols, uint32_t stride, const float* norm_w, bool pdl) {
    GemmX g;
    g.x = x;
    g.nseq = b.batch;
    g.cols = cols;
    g.x_stride = stride;
    g.norm_w = norm_w;
    g.eps = model->cfg.eps;
    g.bx = b.gbx.as<uint8_t>();
    g.xinv = b.gxinv.as<float>();
    g.stats = b.gxinv.as<float>() + 32;
    cuda_check(launch_gemm_stage_x(g, stream, pdl), "stage x");
    kernels += cols <= gemm_stage_one_launch_cols() ? 1 : 2;
}

void Decoder::gemm_product(const QMatrix& w, float* part, uint32_t& ksplit, bool pdl) {
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, model->device);
    GemmArgs a;
    a.w = w.gemm;
    a.bx = b.gbx.as<uint8_t>();
    a.xinv = b.gxinv.as<float>();
    a.nseq = b.batch;
    a.ksplit = ksplit = gemm_ksplit(w.gemm, sms);
    a.rows_pad = w.gemm.mtiles * 128;
    a.part = part;
    a.err = b.err.as<int>();
    cuda_check(launch_qgemm(a, stream, pdl), "gemm");
    kernels += 1;
}

GemmReduce Decoder::reduce_args(const QMatrix& w, const float* part, uint32_t ksplit, float* y, uint32_t y_stride,
                                int epi, const float* part2, uint32_t ksplit2) const {
    GemmReduce r;
    r.part = part;
    r.ksplit = ksplit;
    r.rows_pad = w.gemm.mtiles * 128;
    r.part2 = part2;
    r.ksplit2 = ksplit2;
    r.rows_pad2 = r.rows_pad;
    r.nseq = b.batch;
    r.rows = w.rows;
    r.y = y;
    r.y_stride = y_stride;
    r.epi = epi;
    return r;
}

void Decoder::gemm_reduce(const QMatrix& w, const float* part, uint32_t ksplit, float* y, uint32_t y_stride, int epi,
                          const float* part2, uint32_t ksplit2, bool pdl) {
    GemmReduce r;
    r.part = part;
    r.ksplit = ksplit;
    r.rows_pad = w.gemm.mtiles * 128;
    r.part2 = part2;
    r.ksplit2 = ksplit2;
    r.rows_pad2 = r.rows_pad;
    r.nseq = b.batch;
    r.rows = w.rows;
    r.y = y;
    r.y_stride = y_stride;
    r.epi = epi;
    cuda_check(launch_gemm_reduce(r, stream, pdl), "gemm reduce");
    kernels += 1;
}

// A step for 2..32 sequences on one GPU: every matrix is read once per step by the
// tensor-core products (qgemm.cu); attention and the small kernels are the batched
// ones of the single-sequence path.
void Decoder::enqueue_batched(bool pdl) {
    Model& m = *model;
    const Config& c = m.cfg;
    const bool tp = m.tp_size > 1;
    const uint32_t dim = (uint32_t)c.dim, hd = (uint32_t)c.head_dim;
    const uint32_t qw = m.lheads * hd, kw = m.lkv_heads * hd, F = m.lffn;
    float* x = b.x.as<float>();
    float* p1 = b.gpart.as<float>();
    float* p2 = b.gpart2.as<float>();
    uint32_t k1 = 1, k2 = 1;
    for (uint32_t li = 0; li < c.layers; ++li) {
        const LayerWeights& L = m.layers[li];
        gemm_stage(x, dim, dim, L.attn_norm, pdl);
        {  // Q, K, V products into three partial buffers, then one reduction launch
            uint32_t kq = 1, kk = 1, kv = 1;
            float* p3 = b.gpart3.as<float>();
            gemm_product(L.q, p1, kq, pdl);
            gemm_product(L.k, p2, kk, pdl);
            gemm_product(L.v, p3, kv, pdl);
            const GemmReduce r[3] = {reduce_args(L.q, p1, kq, b.q.as<float>(), qw, EPI_STORE, nullptr, 0),
                                     reduce_args(L.k, p2, kk, b.k.as<float>(), kw, EPI_STORE, nullptr, 0),
                                     reduce_args(L.v, p3, kv, b.v.as<float>(), kw, EPI_STORE, nullptr, 0)};
            cuda_check(launch_gemm_reduce_n(r, 3, stream, pdl), "gemm reduce");
            kernels += 1;
        }
        if (b.cluster_ring) {
            cuda_check(launch_attention_cluster(rope_args(li), attn_args(li, b.cluster_splits), b.cluster_ring, b.cluster_stages, stream,
                                                pdl, b.kv_tmap_ok ? &b.kv_tmap : nullptr),
                       "attention");
            kernels += 1;
        } else {
            cuda_check(launch_qk_norm_rope_append(rope_args(li), stream, pdl), "qk-norm/rope/append");
            cuda_check(launch_attention(attn_args(li, b.nsplit), stream, pdl), "attention");
            kernels += 3;
        }
        gemm_stage(b.att.as<float>(), qw, qw, nullptr, pdl);
        gemm_product(L.o, p1, k1, pdl);
        if (tp) {  // partial sums through the peer inboxes, residual add fused
            gemm_reduce(L.o, p1, k1, b.y.as<float>(), dim, EPI_STORE, nullptr, 0, pdl);
            cuda_check(launch_tp_allreduce_add(b.tp, TP_O, 2 * li, x, b.y.as<float>(), b.batch * dim,
                                               b.err.as<int>(), stream, pdl),
                       "o sum");
            kernels += 1;
        } else {
            gemm_reduce(L.o, p1, k1, x, dim, EPI_ADD, nullptr, 0, pdl);
        }
        gemm_stage(x, dim, dim, L.ffn_norm, pdl);
        gemm_product(L.gate, p1, k1, pdl);
        gemm_product(L.up, p2, k2, pdl);
        gemm_reduce(L.gate, p1, k1, b.h.as<float>(), F, EPI_SWIGLU, p2, k2, pdl);
        gemm_stage(b.h.as<float>(), F, F, nullptr, pdl);
        gemm_product(L.down, p1, k1, pdl);
        if (tp) {
            gemm_reduce(L.down, p1, k1, b.y.as<float>(), dim, EPI_STORE, nullptr, 0, pdl);
            cuda_check(launch_tp_allreduce_add(b.tp, TP_DOWN, 2 * li + 1, x, b.y.as<float>(), b.batch * dim,
                                               b.err.as<int>(), stream, pdl),
                       "ffn sum");
            kernels += 1;
        } else {
            gemm_reduce(L.down, p1, k1, x, dim, EPI_ADD, nullptr, 0, pdl);
        }
    }
    gemm_stage(x, dim, dim, m.out_norm, pdl);
    gemm_product(m.lm_head, p1, k1, pdl);
    // this rank's vocabulary shard into its columns of the [batch][vocab] logits
    gemm_reduce(m.lm_head, p1, k1, b.logits.as<float>() + m.vocab0, (uint32_t)c.vocab, EPI_STORE, nullptr, 0, pdl);
    if (tp) {
        cuda_check(launch_tp_argmax(b.tp, 2 * (uint32_t)c.layers, b.logits.as<float>(), (uint32_t)c.vocab, m.vocab0,
                                    m.lvocab, b.batch, b.amax_v.as<float>(), b.amax_i.as<int32_t>(), b.amax_parts,
                                    b.argmax.as<int32_t>(), b.tokens.as<int32_t>(), b.pos.as<int32_t>(),
                                    b.hist.as<int32_t>(), b.max_ctx, b.epoch.as<uint32_t>(), b.err.as<int>(), stream,
                                    pdl),
                   "argmax");
    } else {
        cuda_check(launch_argmax(b.logits.as<float>(), (uint32_t)c.vocab, b.batch, b.amax_v.as<float>(),
                                 b.amax_i.as<int32_t>(), b.amax_parts, b.argmax.as<int32_t>(), b.tokens.as<int32_t>(),
                                 b.pos.as<int32_t>(), b.hist.as<int32_t>(), b.max_ctx, stream, pdl),
                   "argmax");
    }
    kernels += 2;
}

MatvecArgs Decoder::qkv_args(uint32_t li) const {
    const Model& m = *model;
    const Config& c = m.cfg;
    const LayerWeights& L = m.layers[li];
    MatvecArgs a;  // attn RMSNorm + Q/K/V in one launch
    a.nseg = 3;
    a.seg[0].m = L.q.dev;
    a.seg[0].y = b.q.as<float>();
    a.seg[1].m = L.k.dev;
    a.seg[1].y = b.k.as<float>();
    a.seg[2].m = L.v.dev;
    a.seg[2].y = b.v.as<float>();
    a.x = b.x.as<float>();
    a.cols = (uint32_t)c.dim;
    a.norm_w = L.attn_norm;
    a.eps = c.eps;
    a.err = b.err.as<int>();
    // read after the attention kernels, which leave HBM idle
    a.prefetch[0] = L.o.dev;
    a.prefetch[1] = L.gate.dev;
    a.prefetch[2] = L.up.dev;
    a.prefetch_bytes = prefetch_kb(96) << 10;
    a.max_ctas = b.qkv_ctas;
    return a;
}

RopeArgs Decoder::rope_args(uint32_t li) const {
    const Model& m = *model;
    const Config& c = m.cfg;
    const LayerWeights& L = m.layers[li];
    RopeArgs r;
    r.q = b.q.as<float>();
    r.k = b.k.as<float>();
    r.v = b.v.as<float>();
    r.q_norm = L.q_norm;
    r.k_norm = L.k_norm;
    r.kv = kv;
    r.layer = li;
    r.page_table = b.page_table.as<int32_t>();
    r.max_pages = b.pages_per_seq;
    r.pos = b.pos.as<int32_t>();
    r.batch = b.batch;
    r.heads = m.lheads;
    r.kv_heads = m.lkv_heads;
    r.head_dim = (uint32_t)c.head_dim;
    r.rope_dim = (uint32_t)c.rope_dim;
    r.rope_base = c.rope_base;
    r.eps = c.eps;
    r.interleaved = c.rope_interleaved;
    r.rope_inv_freq = m.rope_inv_freq;
    r.err = b.err.as<int>();
    return r;
}

AttnArgs Decoder::attn_args(uint32_t li, uint32_t nsplit) const {
    const Model& m = *model;
    const uint64_t hd = m.cfg.head_dim;
    AttnArgs at;
    at.q = b.q.as<float>();
    at.out = b.att.as<float>();
    at.kv = kv;
    at.layer = li;
    at.page_table = b.page_table.as<int32_t>();
    at.max_pages = b.pages_per_seq;
    at.pos = b.pos.as<int32_t>();
    at.batch = b.batch;
    at.heads = m.lheads;
    at.kv_heads = m.lkv_heads;
    at.head_dim = (uint32_t)hd;
    at.nsplit = nsplit;
    at.part = b.part.as<float>();
    at.scale = 1.0f / sqrtf((float)hd);
    at.err = b.err.as<int>();
    if (m.layers[li].gated) at.gate = b.qgate.as<float>();  // the sigmoid query gate on the output
    return at;
}

void Decoder::enqueue_layer_attention(uint32_t li, bool pdl) {
    Model& m = *model;
    const Config& c = m.cfg;
    const LayerWeights& L = m.layers[li];
    const uint32_t B = b.batch;
    const uint64_t hd = c.head_dim, qw = (uint64_t)m.lheads * hd, kw = (uint64_t)m.lkv_heads * hd;
    float* x = b.x.as<float>();
    if (L.delta) {
        enqueue_delta(li, pdl);
        return;
    }
    {
        const uint64_t ys[3] = {qw, kw, kw};
        matvec_each(qkv_args(li), B, c.dim, ys, stream, pdl, "qkv matvec");
        kernels += B;
    }
    if (L.gated) {  // the query gate rows of attn_q (runtime.rs:687-693)
        MatvecArgs a;
        a.nseg = 1;
        a.seg[0].m = L.qg.dev;
        a.seg[0].y = b.qgate.as<float>();
        a.x = x;
        a.cols = (uint32_t)c.dim;
        a.norm_w = L.attn_norm;
        a.eps = c.eps;
        a.err = b.err.as<int>();
        const uint64_t ys[1] = {qw};
        matvec_each(a, B, c.dim, ys, stream, pdl, "query gate matvec");
        kernels += B;
    }
    if (b.cluster_ring) {
        cuda_check(launch_attention_cluster(rope_args(li), attn_args(li, b.cluster_splits), b.cluster_ring, b.cluster_stages, stream, pdl,
                                            b.kv_tmap_ok ? &b.kv_tmap : nullptr),
                   "attention");
        kernels += 1;
    } else {
        cuda_check(launch_qk_norm_rope_append(rope_args(li), stream, pdl), "qk-norm/rope/append");
        kernels += 1;
        cuda_check(launch_attention(attn_args(li, b.nsplit), stream, pdl), "attention");
        kernels += 2;
    }
    {  // o-proj, residual add fused (TP: partial sums, all-reduce, then add)
        const bool tp = m.tp_size > 1;
        MatvecArgs a;
        a.nseg = 1;
        a.seg[0].m = L.o.dev;
        a.seg[0].y = tp ? b.y.as<float>() : x;
        a.seg[0].epi = tp ? EPI_STORE : EPI_ADD;
        a.x = b.att.as<float>();
        a.cols = (uint32_t)qw;
        a.err = b.err.as<int>();
        a.prefetch[0] = L.gate.dev;
        a.prefetch[1] = L.up.dev;
        a.prefetch_bytes = prefetch_kb(96) << 10;
        const uint64_t ys[1] = {c.dim};
        matvec_each(a, B, qw, ys, stream, pdl, "o-proj matvec");
        kernels += B;
        if (tp) {  // partial sums through the peer inboxes, residual add fused
            cuda_check(launch_tp_allreduce_add(b.tp, TP_O, 2 * li, x, b.y.as<float>(), B * (uint32_t)c.dim,
                                               b.err.as<int>(), stream, pdl),
                       "o sum");
            kernels += 1;
        }
    }
}

// A Qwen3.5 gated-delta layer (runtime.rs:551-630): attn RMSNorm fused into the
// attn_qkv + attn_gate launch and the ssm_alpha + ssm_beta launch, the recurrent kernel
// (gated_delta.cu), then ssm_out with the residual add.
void Decoder::enqueue_delta(uint32_t li, bool pdl) {
    Model& m = *model;
    const Config& c = m.cfg;
    const LayerWeights& L = m.layers[li];
    const DeltaWeights& D = L.d;
    const uint32_t B = b.batch, CH = m.delta_channels, VW = m.delta_value_width;
    const uint32_t VH = (uint32_t)c.ssm_value_heads, KD = (uint32_t)c.ssm_state, VD = VW / VH;
    float* x = b.x.as<float>();
    MatvecArgs a;
    a.x = x;
    a.cols = (uint32_t)c.dim;
    a.norm_w = L.attn_norm;
    a.eps = c.eps;
    a.err = b.err.as<int>();
    const bool stacked = D.ab.rows != 0;  // alpha | beta as one matrix: a third segment
    {
        MatvecArgs p = a;
        p.nseg = stacked ? 3 : 2;
        p.seg[0].m = D.qkv.dev;
        p.seg[0].y = b.dproj.as<float>();
        p.seg[1].m = D.z.dev;
        p.seg[1].y = b.dz.as<float>();
        p.seg[2].m = D.ab.dev;
        p.seg[2].y = b.dab.as<float>();
        p.prefetch[0] = D.out.dev;
        p.prefetch[1] = L.gate.dev;
        p.prefetch_bytes = prefetch_kb(96) << 10;
        const uint64_t ys[3] = {CH, VW, 2ull * VH};
        matvec_each(p, B, c.dim, ys, stream, pdl, "gated-delta projections matvec");
        kernels += B;
    }
    if (!stacked) {
        MatvecArgs p = a;
        p.nseg = 2;
        p.seg[0].m = D.alpha.dev;
        p.seg[0].y = b.dab.as<float>();
        p.seg[1].m = D.beta.dev;
        p.seg[1].y = b.dab.as<float>() + VH;
        const uint64_t ys[2] = {2ull * VH, 2ull * VH};
        matvec_each(p, B, c.dim, ys, stream, pdl, "gated-delta alpha/beta matvec");
        kernels += B;
    }
    {
        GatedDeltaArgs g;
        g.proj = b.dproj.as<float>();
        g.z = b.dz.as<float>();
        g.ab = b.dab.as<float>();
        g.conv = D.conv;
        g.a = D.a;
        g.dt = D.dt;
        g.norm = D.norm;
        g.batch = B;
        g.channels = CH;
        g.kernel = (uint32_t)c.ssm_conv_kernel;
        g.key_dim = KD;
        g.key_heads = (uint32_t)c.ssm_groups;
        g.value_dim = VD;
        g.value_heads = VH;
        g.hist_stride = (uint64_t)m.delta_layers * 2 * (g.kernel - 1) * CH;
        g.state_stride = (uint64_t)m.delta_layers * VH * KD * VD;
        g.hist = b.dhist.as<float>() + (uint64_t)D.index * 2 * (g.kernel - 1) * CH;
        g.state = b.dstate.as<float>() + (uint64_t)D.index * VH * KD * VD;
        g.out = b.dout.as<float>();
        g.pos = b.pos.as<int32_t>();
        g.eps = c.eps;
        // launched after the projections complete, not early under programmatic
        // dependent launch: measured 941 against 722 tok/s on the 2B-class hybrid shape
        // (the one-CTA-per-head kernel), 1099 against 997 (the cluster kernel)
        cuda_check(launch_gated_delta(g, stream, false), "gated delta");
        kernels += 1;
    }
    {  // ssm_out, residual add fused
        MatvecArgs p;
        p.nseg = 1;
        p.seg[0].m = D.out.dev;
        p.seg[0].y = x;
        p.seg[0].epi = EPI_ADD;
        p.x = b.dout.as<float>();
        p.cols = VW;
        p.err = b.err.as<int>();
        p.prefetch[0] = L.gate.dev;
        p.prefetch[1] = L.up.dev;
        p.prefetch_bytes = prefetch_kb(96) << 10;
        const uint64_t ys[1] = {c.dim};
        matvec_each(p, B, VW, ys, stream, pdl, "ssm_out matvec");
        kernels += B;
    }
}

// The persistent whole-step kernel for a single sequence (decode_step.cu): every layer
// and the LM head in one cooperative launch, phases handing vectors on as tagged words.
// Opt-in with EVELYN_STEP_KERNEL=1: it is correct (tested against the launch sequence
// and the oracle) but measured slower than the launch sequence on the 8B shape (343 vs
// 596 tok/s), whose kernels stay the default. When it cannot be built (or captured)
// the step runs as the launch sequence below, and step_note says why.
void Decoder::build_step_kernel() {
    Model& m = *model;
    const Config& c = m.cfg;
    step_tried = true;
    const char* env = std::getenv("EVELYN_STEP_KERNEL");
    if (!env || env[0] != '1') return;
    if (b.batch != 1) return;
    if (m.tp_size != 1) {
        step_note = "step kernel not used: tensor parallelism";
        return;
    }
    if (c.has_ssm) {
        step_note = "step kernel not used: Qwen3.5 gated-delta and gated-query layers";
        return;
    }
    int sms = 148;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, m.device);
    const uint32_t hd = (uint32_t)c.head_dim, G = m.lheads / std::max<uint32_t>(1, m.lkv_heads);
    const uint32_t L = (uint32_t)c.layers, T = (uint32_t)m.tp_size, R = (uint32_t)m.tp_rank;
    const uint32_t nsplit = step_attn_splits(m.lkv_heads, b.pages_per_seq, sms);
    const uint32_t eb = m.kv_f32 ? 4 : 2;
    // page pairs staged per split at a time: as many as the per-warp partials' bytes hold
    uint32_t ring = (uint32_t)((16ull * G * (hd + 2) * 4) / (2ull * 16 * hd * eb)) & ~1u;
    ring = std::max<uint32_t>(2, std::min<uint32_t>(16, ring));
    // tagged vectors, each on a 256-byte boundary (words)
    auto up = [](uint64_t n) { return (n + 31) & ~31ull; };
    const uint64_t nx = up(c.dim), nq = up((uint64_t)m.lheads * hd), nk = up((uint64_t)m.lkv_heads * hd);
    const uint64_t np = up((uint64_t)m.lkv_heads * nsplit * G * (hd + 2)), na = up(c.heads * hd), nh = up(c.ffn);
    b.tagpool.alloc((nx + nq + 2 * nk + np + na + nh) * 8);
    cuda_check(cudaMemset(b.tagpool.p, 0xff, b.tagpool.bytes), "memset");  // tag 0xffffffff: never expected
    uint64_t* w = b.tagpool.as<uint64_t>();
    b.xt = w, w += nx;
    b.qt = w, w += nq;
    b.kt = w, w += nk;
    b.vt = w, w += nk;
    b.partt = w, w += np;
    b.attt = w, w += na;
    b.ht = w;
    b.epoch.alloc(4);
    cuda_check(cudaMemset(b.epoch.p, 0, 4), "memset");
    b.tag_period = 8 * (L + 1);
    // slots per layer l: x entering it 8l, q/k/v 8l+1, partials 8l+2, attention 8l+3,
    // x after o 8l+4, h 8l+5; x entering the LM head 8L
    auto out1 = [](uint64_t* dst, uint32_t row0, uint32_t slot) {
        TaggedOut o;
        o.dst[0] = dst;
        o.ndst = 1;
        o.row0 = row0;
        o.tag = slot;
        return o;
    };
    const uint32_t o_row0 = R * (uint32_t)(c.dim / T);
    uint64_t f0 = 0;
    {  // this rank's first FFN row (the gate/up shard)
        const uint64_t nb = c.ffn / 256, base = nb / T, rem = nb % T;
        f0 = T > 1 ? (R * base + std::min<uint64_t>(R, rem)) * 256 : 0;
    }
    std::vector<StepPhaseDesc> ph;
    for (uint32_t li = 0; li < L; ++li) {
        const LayerWeights& LW = m.layers[li];
        StepPhaseDesc d;
        d.mv = qkv_args(li);
        d.xt = b.xt;
        d.x_tag = 8 * li;
        d.out[0] = out1(b.qt, 0, 8 * li + 1);
        d.out[1] = out1(b.kt, 0, 8 * li + 1);
        d.out[2] = out1(b.vt, 0, 8 * li + 1);
        ph.push_back(d);
        StepPhaseDesc at;
        at.kind = STEP_ATTN;
        at.at.q = b.qt;
        at.at.k = b.kt;
        at.at.v = b.vt;
        at.at.qkv_tag = 8 * li + 1;
        at.at.part = b.partt;
        at.at.part_tag = 8 * li + 2;
        at.at.out = out1(b.attt, R * m.lheads * hd, 8 * li + 3);
        at.at.rope = rope_args(li);
        at.at.nsplit = nsplit;
        at.at.ring_pages = ring;
        at.at.scale = 1.0f / sqrtf((float)hd);
        ph.push_back(at);
        StepPhaseDesc o;
        o.mv.nseg = 1;
        o.mv.seg[0].m = LW.o.dev;
        o.mv.seg[0].epi = EPI_ADD;
        o.mv.cols = LW.o.cols;
        o.mv.err = b.err.as<int>();
        o.xt = b.attt;
        o.x_tag = 8 * li + 3;
        o.out[0] = out1(b.xt, o_row0, 8 * li + 4);
        o.out[0].resid = b.xt;
        o.out[0].resid_tag = 8 * li;
        ph.push_back(o);
        StepPhaseDesc gu;
        gu.mv.nseg = 1;
        gu.mv.seg[0].m = LW.gate.dev;
        gu.mv.seg[0].m2 = LW.up.dev;
        gu.mv.seg[0].epi = EPI_SWIGLU;
        gu.mv.cols = (uint32_t)c.dim;
        gu.mv.norm_w = LW.ffn_norm;
        gu.mv.eps = c.eps;
        gu.mv.err = b.err.as<int>();
        gu.xt = b.xt;
        gu.x_tag = 8 * li + 4;
        gu.out[0] = out1(b.ht, (uint32_t)f0, 8 * li + 5);
        ph.push_back(gu);
        StepPhaseDesc dn;
        dn.mv.nseg = 1;
        dn.mv.seg[0].m = LW.down.dev;
        dn.mv.seg[0].epi = EPI_ADD;
        dn.mv.cols = LW.down.cols;
        dn.mv.err = b.err.as<int>();
        dn.xt = b.ht;
        dn.x_tag = 8 * li + 5;
        dn.out[0] = out1(b.xt, o_row0, 8 * (li + 1));
        dn.out[0].resid = b.xt;
        dn.out[0].resid_tag = 8 * li + 4;
        ph.push_back(dn);
    }
    {  // final RMSNorm + LM head into the logits (plain floats)
        StepPhaseDesc hd_;
        hd_.mv.nseg = 1;
        hd_.mv.seg[0].m = m.lm_head.dev;
        hd_.mv.cols = (uint32_t)c.dim;
        hd_.mv.norm_w = m.out_norm;
        hd_.mv.eps = c.eps;
        hd_.mv.err = b.err.as<int>();
        hd_.xt = b.xt;
        hd_.x_tag = 8 * L;
        hd_.out[0].plain[0] = b.logits.as<float>();
        hd_.out[0].ndst = 1;
        hd_.out[0].row0 = m.vocab0;
        ph.push_back(hd_);
    }
    StepKernel* k = nullptr;
    const cudaError_t e =
        step_kernel_create(ph.data(), (uint32_t)ph.size(), b.epoch.as<uint32_t>(), b.tag_period, b.err.as<int>(), &k);
    if (e != cudaSuccess) {
        cudaGetLastError();
        step_note = std::string("step kernel not used: ") + cudaGetErrorString(e);
        return;
    }
    step_k = k;
}

void Decoder::enqueue_head(bool pdl) {
    Model& m = *model;
    const Config& c = m.cfg;
    const uint32_t B = b.batch;
    const bool tp = m.tp_size > 1;
    const uint64_t V = c.vocab;
    // the LM head (this rank's vocabulary shard under tensor parallelism) into its
    // columns of the [batch][vocab] logits
    MatvecArgs a;
    a.nseg = 1;
    a.seg[0].m = m.lm_head.dev;
    a.seg[0].y = b.logits.as<float>() + m.vocab0;
    a.x = b.x.as<float>();
    a.cols = (uint32_t)c.dim;
    a.norm_w = m.out_norm;
    a.eps = c.eps;
    a.err = b.err.as<int>();
    const uint64_t ys[1] = {V};
    matvec_each(a, B, c.dim, ys, stream, pdl, "lm-head matvec");
    kernels += B;
    if (tp) {  // each rank's best of its shard, picked the same way on every rank
        cuda_check(launch_tp_argmax(b.tp, 2 * (uint32_t)c.layers, b.logits.as<float>(), (uint32_t)V, m.vocab0, m.lvocab,
                                    B, b.amax_v.as<float>(), b.amax_i.as<int32_t>(), b.amax_parts,
                                    b.argmax.as<int32_t>(), b.tokens.as<int32_t>(), b.pos.as<int32_t>(),
                                    b.hist.as<int32_t>(), b.max_ctx, b.epoch.as<uint32_t>(), b.err.as<int>(), stream,
                                    pdl),
                   "argmax");
    } else {
        cuda_check(launch_argmax(b.logits.as<float>(), (uint32_t)V, B, b.amax_v.as<float>(), b.amax_i.as<int32_t>(),
                                 b.amax_parts, b.argmax.as<int32_t>(), b.tokens.as<int32_t>(), b.pos.as<int32_t>(),
                                 b.hist.as<int32_t>(), b.max_ctx, stream, pdl),
                   "argmax");
    }
    kernels += 2;
}

// Tensor parallelism: the other ranks' vocabulary shards of the last step's logits,
// read from their buffers over NVLink (each rank wrote its shard before the step's
// pick, which every rank waited for).
void Decoder::gather_peer_logits() {
    Model& m = *model;
    const uint64_t V = m.cfg.vocab, T = (uint64_t)m.tp_size;
    for (uint64_t r = 0; r < T; ++r) {
        if ((int)r == m.tp_rank) continue;
        const uint64_t base = V / T, rem = V % T;
        const uint64_t lo = r * base + std::min<uint64_t>(r, rem), n = base + (r < rem ? 1 : 0);
        cuda_check(cudaMemcpy2DAsync(b.logits.as<float>() + lo, V * 4, b.peer_logits[r] + lo, V * 4, n * 4, b.batch,
                                     cudaMemcpyDeviceToDevice, stream),
                   "peer logits");
    }
}

void Decoder::enqueue_dense(bool pdl) {
    Model& m = *model;
    const Config& c = m.cfg;
    kernels = 0;
    if (step_k) {  // every layer and the LM head in one launch, then the argmax
        cuda_check(launch_embed_tagged(m.embed.dev, b.tokens.as<int32_t>(), b.xt, b.epoch.as<uint32_t>(), b.tag_period,
                                       b.err.as<int32_t>(), stream),
                   "embed");
        cuda_check(step_kernel_launch(step_k, stream), "step kernel");
        cuda_check(launch_argmax(b.logits.as<float>(), (uint32_t)c.vocab, 1, b.amax_v.as<float>(),
                                 b.amax_i.as<int32_t>(), b.amax_parts, b.argmax.as<int32_t>(), b.tokens.as<int32_t>(),
                                 b.pos.as<int32_t>(), b.hist.as<int32_t>(), b.max_ctx, stream, false,
                                 b.epoch.as<uint32_t>()),
                   "argmax");
        kernels_per_step = kernels = 4;
        return;
    }
    cuda_check(launch_embed(m.embed.dev, b.tokens.as<int32_t>(), b.batch, b.x.as<float>(), b.err.as<int32_t>(), stream,
                            pdl),
               "embed");
    kernels += 1;
    if (use_gemm) {
        enqueue_batched(pdl);
        kernels_per_step = kernels;
        return;
    }
    {
        for (uint32_t li = 0; li < c.layers; ++li) {
            enqueue_layer_attention(li, pdl);
            QMatDev next[3] = {m.lm_head.dev, QMatDev{}, QMatDev{}};
            if (li + 1 < c.layers) {
                next[0] = m.layers[li + 1].q.dev;
                next[1] = m.layers[li + 1].k.dev;
                next[2] = m.layers[li + 1].v.dev;
            }
            run_dense_ffn(m, li, b.x.as<float>(), m.layers[li].ffn_norm, b.x.as<float>(), true, b.batch,
                          b.h.as<float>(), b.y.as<float>(), b.err.as<int>(), next, stream, pdl,
                          m.tp_size > 1 ? &b.tp : nullptr, 2 * li + 1);
            kernels += 2 * b.batch + (m.tp_size > 1 ? 1 : 0);
        }
    }
    enqueue_head(pdl);
    kernels_per_step = kernels;
}

void Decoder::run_routed(const evl_ffn_backend& ffn) {
    Model& m = *model;
    const Config& c = m.cfg;
    if (b.batch != 1) raise(EVL_ERR_UNSUPPORTED, "FFN routing is available for single sessions");
    if (m.tp_size > 1) raise(EVL_ERR_UNSUPPORTED, "FFN routing with tensor parallelism is not supported");
    const bool pdl = false;
    float* x = b.x.as<float>();
    cuda_check(launch_embed(m.embed.dev, b.tokens.as<int32_t>(), 1, x, b.err.as<int32_t>(), stream, pdl), "embed");
    for (uint32_t li = 0; li < c.layers; ++li) {
        enqueue_layer_attention(li, pdl);
        const bool routed = ffn.ffn && (!ffn.routed || (li < ffn.routed_len && ffn.routed[li]));
        if (!routed) {
            run_dense_ffn(m, li, x, m.layers[li].ffn_norm, x, true, 1, b.h.as<float>(), b.y.as<float>(), b.err.as<int>(),
                          nullptr, stream, pdl);
            continue;
        }
        // Model::ffn_input (runtime.rs:801), then the backend on the host
        float* xn = b.xn.as<float>();
        cuda_check(launch_rmsnorm(x, m.layers[li].ffn_norm, xn, (uint32_t)c.dim, 1, c.eps, stream, pdl), "ffn norm");
        cuda_check(cudaMemcpyAsync(b.h_xn.p, xn, c.dim * 4, cudaMemcpyDeviceToHost, stream), "D2H ffn input");
        if (!b.routed_ev) cuda_check(cudaEventCreateWithFlags(&b.routed_ev, cudaEventDisableTiming), "event");
        cuda_check(cudaEventRecord(b.routed_ev, stream), "event");
        {  // while the host runs the backend, the device warms the next launches' weights
            L2Ranges r;
            auto put = [&](int i, const QMatrix& q) {
                r.base[i] = q.dev.q;
                r.bytes[i] = q.dev.q ? q.bytes() : 0;
            };
            if (li + 1 < c.layers) {
                const LayerWeights& N = m.layers[li + 1];
                if (N.delta) {
                    put(0, N.d.qkv), put(1, N.d.z), put(2, N.d.out);
                } else {
                    put(0, N.q), put(1, N.k), put(2, N.v), put(3, N.o);
                }
            } else {
                put(0, m.lm_head);
            }
            cuda_check(launch_l2_prefetch(r, stream), "L2 prefetch");
        }
        cuda_check(cudaEventSynchronize(b.routed_ev), "sync");  // the input only, not the prefetch
        const int rc = ffn.ffn(ffn.ctx, li, b.h_xn.as<float>(), c.dim, b.h_y.as<float>());
        if (rc == 0) {
            cuda_check(cudaMemcpyAsync(b.y.p, b.h_y.p, c.dim * 4, cudaMemcpyHostToDevice, stream), "H2D ffn output");
            cuda_check(launch_add(x, b.y.as<float>(), c.dim, stream, pdl), "residual add");
        } else {
            if (rc != EVL_FFN_DENSE && ffn.fallbacks) *ffn.fallbacks += 1;
            run_dense_ffn(m, li, xn, nullptr, x, true, 1, b.h.as<float>(), b.y.as<float>(), b.err.as<int>(), nullptr,
                          stream, pdl);
        }
    }
    enqueue_head(pdl);
}

void Decoder::launch_graph() {
    if (!graph) {
        if (!step_tried) build_step_kernel();  // allocates: before any capture
        for (int attempt = 0; attempt < 2 && !graph; ++attempt) {
            const bool pdl = attempt == 0;
            cudaGraph_t g = nullptr;
            cuda_check(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal), "begin capture");
            try {
                enqueue_dense(pdl);
            } catch (const Error& err) {
                cudaStreamEndCapture(stream, &g);
                if (g) cudaGraphDestroy(g);
                cudaGetLastError();
                if (!step_k) throw;
                step_note = "step kernel not captured: " + err.msg;  // retry with the launch sequence
                step_kernel_destroy(step_k);
                step_k = nullptr;
                --attempt;
                continue;
            } catch (...) {
                cudaStreamEndCapture(stream, &g);
                if (g) cudaGraphDestroy(g);
                throw;
            }
            cuda_check(cudaStreamEndCapture(stream, &g), "end capture");
            cudaError_t e = cudaGraphInstantiate(&graph, g, 0);
            cudaGraphDestroy(g);
            if (e != cudaSuccess) {
                cudaGetLastError();
                graph = nullptr;
                if (step_k) {  // retry with the per-kernel launch sequence
                    step_note = std::string("step kernel not captured: ") + cudaGetErrorString(e);
                    step_kernel_destroy(step_k);
                    step_k = nullptr;
                    --attempt;
                    continue;
                }
                if (attempt == 1) cuda_check(e, "graph instantiate");
            }
            graph_pdl = pdl;
        }
    }
    cuda_check(cudaGraphLaunch(graph, stream), "graph launch");
}

void Decoder::check_device_error() {
    const int e = *b.h_err.as<int>();
    if (e == DEV_OK) return;
    *b.h_err.as<int>() = 0;
    cudaMemsetAsync(b.err.p, 0, 4, stream);
    if (step_k) step_kernel_reset(step_k, stream);
    cudaStreamSynchronize(stream);
    switch (e) {
        case DEV_ERR_TOKEN: raise(EVL_ERR_INVALID_INPUT, "token ID outside the model vocabulary");
        case DEV_ERR_POSITION: raise(EVL_ERR_INVALID_INPUT, "position outside the session's KV cache");
        case DEV_ERR_WAIT_TIMEOUT: raise(EVL_ERR_TIMEOUT, "a device wait for KV pages timed out");
        default: raise(EVL_ERR_CUDA, "device error " + std::to_string(e));
    }
}

void Decoder::step(const uint32_t* tokens, const evl_ffn_backend* ffn, float* logits_out, uint32_t* argmax_out) {
    Model& m = *model;
    const Config& c = m.cfg;
    DeviceGuard g(m.device);
    for (uint32_t i = 0; i < b.batch; ++i) {
        if (tokens[i] >= c.vocab)
            raise(EVL_ERR_INVALID_INPUT, "token ID " + std::to_string(tokens[i]) + " is outside model vocabulary (" +
                                             std::to_string(c.vocab) + "); check that tokenizer and GGUF match");
        if (host_pos[i] >= b.max_ctx)
            raise(EVL_ERR_INVALID_INPUT, "session context is full (" + std::to_string(b.max_ctx) + " positions)");
    }
    std::memcpy(b.h_tokens.p, tokens, b.batch * 4);
    cuda_check(cudaMemcpyAsync(b.tokens.p, b.h_tokens.p, b.batch * 4, cudaMemcpyHostToDevice, stream), "H2D tokens");
    if (ffn && ffn->ffn) {
        run_routed(*ffn);
    } else {
        launch_graph();
    }
    if (logits_out && m.tp_size > 1 && !(ffn && ffn->ffn)) gather_peer_logits();
    if (logits_out)
        cuda_check(cudaMemcpyAsync(b.h_logits.p, b.logits.p, (size_t)b.batch * c.vocab * 4, cudaMemcpyDeviceToHost,
                                   stream),
                   "D2H logits");
    if (argmax_out)
        cuda_check(cudaMemcpyAsync(b.h_argmax.p, b.argmax.p, b.batch * 4, cudaMemcpyDeviceToHost, stream), "D2H argmax");
    cuda_check(cudaMemcpyAsync(b.h_err.p, b.err.p, 4, cudaMemcpyDeviceToHost, stream), "D2H error flag");
    cuda_check(cudaStreamSynchronize(stream), "step");
    check_device_error();
    for (auto& p : host_pos) ++p;
    if (logits_out) std::memcpy(logits_out, b.h_logits.p, (size_t)b.batch * c.vocab * 4);
    if (argmax_out) std::memcpy(argmax_out, b.h_argmax.p, b.batch * 4);
}

// Prompt processing in chunks of kPrefillRows tokens: each chunk is one batched step of
// a child decoder whose rows are the chunk's positions of this (single) sequence -- the
// same kernels as a batch, the products on the tensor cores with the prompt tokens as
// the N dimension, every row's K/V appended before any row attends, and row i attending
// positions [0, p0 + i] of this session's cache. Equal to n Session::step calls
// (src/runtime.rs:773-808, fed one token at a time by src/bin/evelyn-generate.rs:69-80)
// up to the products' summation order.
void Decoder::prefill(uint32_t seq, const uint32_t* tokens, size_t n, float* logits_out, uint32_t* argmax_out) {
    constexpr uint32_t kPrefillRows = 32;
    Model& m = *model;
    const Config& c = m.cfg;
    DeviceGuard g(m.device);
    if (seq >= b.batch)
        raise(EVL_ERR_INVALID_INPUT, "sequence " + std::to_string(seq) + " is outside the batch of " +
                                         std::to_string(b.batch));
    for (size_t i = 0; i < n; ++i)
        if (tokens[i] >= c.vocab)
            raise(EVL_ERR_INVALID_INPUT, "token ID " + std::to_string(tokens[i]) + " is outside model vocabulary (" +
                                             std::to_string(c.vocab) + "); check that tokenizer and GGUF match");
    if (host_pos[seq] + n > b.max_ctx)
        raise(EVL_ERR_INVALID_INPUT, "session context is full (" + std::to_string(b.max_ctx) + " positions)");
    if (n == 0) return;
    if (!pf && !pf_stepwise) {
        auto child = std::make_unique<Decoder>();
        child->init(&m, kPrefillRows, b.max_ctx, this);
        if (child->use_gemm) {
            pf = std::move(child);
        } else if (b.batch == 1) {
            pf_stepwise = true;  // (Qwen3.5 hybrid layers, unquantised matrices)
        } else {
            raise(EVL_ERR_UNSUPPORTED, "batch prefill needs the tensor-core products for this model");
        }
    }
    if (pf_stepwise) {  // the reference's own prompt loop: one step per token
        for (size_t i = 0; i < n; ++i)
            step(tokens + i, nullptr, logits_out ? logits_out + i * c.vocab : nullptr, argmax_out ? argmax_out + i : nullptr);
        return;
    }
    Decoder& P = *pf;
    const uint32_t C = P.b.batch, pps = b.pages_per_seq;
    const int32_t spare = (int32_t)(b.batch * pps);  // the page past every sequence's own
    std::vector<int32_t> pt((uint64_t)C * pps);
    for (size_t off = 0; off < n; off += C) {
        const uint32_t nr = (uint32_t)std::min<size_t>(C, n - off);
        int32_t* tok = P.b.h_tokens.as<int32_t>();
        std::vector<int32_t> pos(C);
        for (uint32_t i = 0; i < C; ++i) {
            tok[i] = i < nr ? (int32_t)tokens[off + i] : 0;
            pos[i] = i < nr ? (int32_t)(host_pos[seq] + off + i) : 0;
        }
        if (nr != pf_rows || seq != pf_seq) {  // padding rows append into the spare page and read only it
            for (uint32_t i = 0; i < C; ++i)
                for (uint32_t j = 0; j < pps; ++j) pt[(uint64_t)i * pps + j] = i < nr ? (int32_t)(seq * pps + j) : spare;
            cuda_check(cudaMemcpyAsync(P.b.page_table.p, pt.data(), pt.size() * 4, cudaMemcpyHostToDevice, P.stream),
                       "page table");
            pf_rows = nr;
            pf_seq = seq;
        }
        cuda_check(cudaMemcpyAsync(P.b.tokens.p, tok, C * 4, cudaMemcpyHostToDevice, P.stream), "H2D tokens");
        cuda_check(cudaMemcpyAsync(P.b.pos.p, pos.data(), C * 4, cudaMemcpyHostToDevice, P.stream), "H2D positions");
        P.launch_graph();
        if (m.tp_size > 1 && logits_out) P.gather_peer_logits();
        if (logits_out)
            cuda_check(cudaMemcpyAsync(logits_out + off * c.vocab, P.b.logits.p, (size_t)nr * c.vocab * 4,
                                       cudaMemcpyDeviceToHost, P.stream),
                       "D2H logits");
        if (argmax_out)
            cuda_check(cudaMemcpyAsync(argmax_out + off, P.b.argmax.p, nr * 4, cudaMemcpyDeviceToHost, P.stream),
                       "D2H argmax");
        // pos/tokens must not be rewritten before this chunk's graph has read them
        cuda_check(cudaStreamSynchronize(P.stream), "prefill chunk");
    }
    cuda_check(cudaMemcpyAsync(P.b.h_err.p, P.b.err.p, 4, cudaMemcpyDeviceToHost, P.stream), "D2H error flag");
    cuda_check(cudaStreamSynchronize(P.stream), "prefill");
    P.check_device_error();
    host_pos[seq] += n;
    const int32_t p = (int32_t)host_pos[seq];
    cuda_check(cudaMemcpy(b.pos.as<int32_t>() + seq, &p, 4, cudaMemcpyHostToDevice), "position");
}

// sample_token (src/server.rs:326-352) on the last step's logits, on the device: only
// the xorshift states and the picked tokens cross to and from the host.
void Decoder::sample(float temperature, uint64_t* states, uint32_t* tokens_out) {
    Model& m = *model;
    DeviceGuard g(m.device);
    const uint32_t B = b.batch;
    if (temperature <= FLT_EPSILON) {  // the greedy pick; the state is not touched
        cuda_check(cudaMemcpyAsync(b.h_argmax.p, b.argmax.p, B * 4, cudaMemcpyDeviceToHost, stream), "D2H argmax");
        cuda_check(cudaStreamSynchronize(stream), "sample");
        std::memcpy(tokens_out, b.h_argmax.p, B * 4);
        return;
    }
    if (!b.smp_rng.p) {
        b.smp_rng.alloc(B * 8);
        b.smp_out.alloc(B * 4);
        b.smp_m.alloc((uint64_t)B * b.amax_parts * 4);
        b.smp_s.alloc((uint64_t)B * b.amax_parts * 8);
        b.h_rng.alloc(B * 8);
    }
    if (m.tp_size > 1) gather_peer_logits();
    std::memcpy(b.h_rng.p, states, B * 8);
    cuda_check(cudaMemcpyAsync(b.smp_rng.p, b.h_rng.p, B * 8, cudaMemcpyHostToDevice, stream), "H2D rng");
    cuda_check(launch_sample(b.logits.as<float>(), (uint32_t)m.cfg.vocab, B, temperature, b.smp_rng.as<uint64_t>(),
                             b.argmax.as<int32_t>(), b.smp_m.as<float>(), b.smp_s.as<double>(), b.amax_parts,
                             b.smp_out.as<int32_t>(), stream),
               "sample");
    cuda_check(cudaMemcpyAsync(b.h_argmax.p, b.smp_out.p, B * 4, cudaMemcpyDeviceToHost, stream), "D2H token");
    cuda_check(cudaMemcpyAsync(b.h_rng.p, b.smp_rng.p, B * 8, cudaMemcpyDeviceToHost, stream), "D2H rng");
    cuda_check(cudaStreamSynchronize(stream), "sample");
    std::memcpy(tokens_out, b.h_argmax.p, B * 4);
    std::memcpy(states, b.h_rng.p, B * 8);
}

void Decoder::generate(uint32_t token, uint32_t n, uint32_t* tokens_out) {
    Model& m = *model;
    DeviceGuard g(m.device);
    if (b.batch != 1) raise(EVL_ERR_INVALID_INPUT, "generate drives a single sequence");
    if (token >= m.cfg.vocab)
        raise(EVL_ERR_INVALID_INPUT, "token ID " + std::to_string(token) + " is outside model vocabulary (" +
                                         std::to_string(m.cfg.vocab) + "); check that tokenizer and GGUF match");
    if (host_pos[0] + n > b.max_ctx)
        raise(EVL_ERR_INVALID_INPUT, "session context is full (" + std::to_string(b.max_ctx) + " positions)");
    if (n == 0) return;
    const uint64_t p0 = host_pos[0];
    *b.h_tokens.as<uint32_t>() = token;
    cuda_check(cudaMemcpyAsync(b.tokens.p, b.h_tokens.p, 4, cudaMemcpyHostToDevice, stream), "H2D token");
    for (uint32_t i = 0; i < n; ++i) launch_graph();
    std::vector<int32_t> hist(n);
    cuda_check(cudaMemcpyAsync(hist.data(), b.hist.as<int32_t>() + p0, n * 4, cudaMemcpyDeviceToHost, stream),
               "D2H tokens");
    cuda_check(cudaMemcpyAsync(b.h_err.p, b.err.p, 4, cudaMemcpyDeviceToHost, stream), "D2H error flag");
    cuda_check(cudaStreamSynchronize(stream), "generate");
    check_device_error();
    host_pos[0] += n;
    for (uint32_t i = 0; i < n; ++i) tokens_out[i] = (uint32_t)hist[i];
}

}  // namespace evl
