// model.cpp -- Model::load for the device (src/runtime.rs:199-406).
//
// Reads the same metadata keys with the same defaults (rope.freq_base 1e4,
// rope.dimension_count = head_dim, layer_norm_rms_epsilon 1e-6, head_count_kv from
// a number or the first positive array entry, key_length or dim/heads), the same
// tensor names (post_attention_norm preferred over ffn_norm, optional q/k norms,
// output.weight falling back to the tied token_embd.weight), and the same errors
// (InvalidData "missing {arch}.{key}", NotFound for absent tensors). It then
// uploads every matrix once, repacked for the GPU, keeping it quantised.
//
// Tensor parallelism (tp_size > 1): column split of attn_q/k/v by heads and of
// ffn_gate/up by output rows, row split of attn_output and ffn_down along their
// inputs on 256-value super-block boundaries (uneven shards when the block count
// does not divide), LM head split by vocabulary rows, norms replicated.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <thread>

#include "engine.hpp"

namespace evl {

namespace {

struct Planned {
    QMatrix* m;
    const uint8_t* raw;      // first byte of the first row of the shard
    size_t stride;           // bytes between rows in `raw`
    uint32_t col_byte0 = 0;  // byte offset of the shard's first column within a row
    uint32_t col_bytes = 0;  // bytes per row in the shard (0: whole row)
    // row selection (0: rows in order): row r of the matrix is source row
    // (r / run) * period + offset + r % run -- one half of each head's interleaved rows
    uint32_t run = 0, period = 0, offset = 0;
    // two tensors stacked as one matrix: rows from `split` on come from raw2
    const uint8_t* raw2 = nullptr;
    uint32_t split = 0;
};

uint32_t block_elems(uint32_t t) {
    switch (t) {
        case GGML_Q4_K:
        case GGML_Q5_K:
        case GGML_Q6_K: return 256;
        case GGML_Q8_0: return 32;
        default: return 1;
    }
}

// Even split of n items over p parts: part i gets [lo, hi).
void split_range(uint64_t n, int p, int i, uint64_t* lo, uint64_t* hi) {
    const uint64_t base = n / p, rem = n % p;
    *lo = i * base + std::min<uint64_t>(i, rem);
    *hi = *lo + base + (i < (int)rem ? 1 : 0);
}

}  // namespace

TpShard tp_shard_plan(const Config& c, int T, int R) {
    if (T < 1 || R < 0 || R >= T) raise(EVL_ERR_INVALID_INPUT, "tp_rank outside [0, tp_size)");
    if (c.kv_heads == 0 || c.kv_heads % T) raise(EVL_ERR_INVALID_INPUT, "tp_size must divide head_count_kv");
    TpShard s;
    const uint64_t hd = c.head_dim, lh = c.heads / T, lkv = c.kv_heads / T;
    s.q[0] = (uint64_t)R * lh * hd;
    s.q[1] = s.q[0] + lh * hd;
    s.kv[0] = (uint64_t)R * lkv * hd;
    s.kv[1] = s.kv[0] + lkv * hd;
    // the FFN is split on 256-value boundaries so ffn_down shards stay block aligned
    s.ffn[0] = 0;
    s.ffn[1] = c.ffn;
    if (T > 1) {
        if (c.ffn % 256) raise(EVL_ERR_UNSUPPORTED, "tensor parallelism needs feed_forward_length % 256 == 0");
        uint64_t b0, b1;
        split_range(c.ffn / 256, T, R, &b0, &b1);
        s.ffn[0] = b0 * 256;
        s.ffn[1] = b1 * 256;
    }
    s.vocab[0] = 0;
    s.vocab[1] = c.vocab;
    if (T > 1) split_range(c.vocab, T, R, &s.vocab[0], &s.vocab[1]);
    return s;
}

Model::~Model() {
    if (comm) nccl().CommDestroy(comm);
    if (stream) cudaStreamDestroy(stream);
}

std::unique_ptr<Model> load_model(const uint8_t* data, size_t len, const evl_model_options& o) {
    auto M = std::make_unique<Model>();
    Model& m = *M;
    if (o.device >= 0) {
        m.device = o.device;
    } else {
        cuda_check(cudaGetDevice(&m.device), "cudaGetDevice");
    }
    DeviceGuard guard(m.device);
    m.tp_size = o.tp_size > 0 ? o.tp_size : 1;
    m.tp_rank = o.tp_rank;
    if (m.tp_rank < 0 || m.tp_rank >= m.tp_size) raise(EVL_ERR_INVALID_INPUT, "tp_rank outside [0, tp_size)");
    m.kv_f32 = o.kv_f32 != 0;

    Gguf g;
    g.open(data, len);
    Config& c = m.cfg;
    std::string arch = g.architecture();
    if (arch.empty()) arch = "llama";
    auto need = [&](const std::string& k) -> uint64_t {
        uint64_t v;
        const GgufValue* val = g.meta(arch + "." + k);
        if (!val || !val->as_u64(&v)) raise(EVL_ERR_INVALID_DATA, "missing " + arch + "." + k);
        return v;
    };
    c.arch = arch;
    c.dim = need("embedding_length");
    c.heads = need("attention.head_count");
    if (const GgufValue* kv = g.meta(arch + ".attention.head_count_kv")) {
        uint64_t u;
        if (kv->as_u64(&u)) {
            c.kv_heads = u;
        } else {
            c.kv_heads = c.heads;
            if (kv->kind == GgufValue::ARRAY)
                for (const auto& e : kv->arr)
                    if (e.as_u64(&u) && u > 0) {
                        c.kv_heads = u;
                        break;
                    }
        }
    } else {
        c.kv_heads = c.heads;
    }
    uint64_t u64;
    const GgufValue* kl = g.meta(arch + ".attention.key_length");
    if (c.heads == 0) raise(EVL_ERR_INVALID_DATA, arch + ".attention.head_count is zero");
    c.head_dim = (kl && kl->as_u64(&u64)) ? u64 : c.dim / c.heads;
    if (arch == "qwen35") {  // runtime.rs:225-235
        c.has_ssm = true;
        c.ssm_conv_kernel = need("ssm.conv_kernel");
        c.ssm_inner = need("ssm.inner_size");
        c.ssm_state = need("ssm.state_size");
        c.ssm_groups = need("ssm.group_count");
        c.ssm_value_heads = need("ssm.time_step_rank");
    }
    c.layers = need("block_count");
    c.ffn = need("feed_forward_length");
    double f64;
    const GgufValue* rb = g.meta(arch + ".rope.freq_base");
    c.rope_base = (rb && rb->as_f64(&f64)) ? (float)f64 : 10000.0f;
    const GgufValue* rd = g.meta(arch + ".rope.dimension_count");
    c.rope_dim = (rd && rd->as_u64(&u64)) ? u64 : c.head_dim;
    const GgufValue* ri = g.meta(arch + ".rope.mrope_interleaved");
    c.rope_interleaved = ri && ri->kind == GgufValue::BOOL && ri->b;
    const GgufValue* ep = g.meta(arch + ".attention.layer_norm_rms_epsilon");
    c.eps = (ep && ep->as_f64(&f64)) ? (float)f64 : 1e-6f;
    const GgufValue* fa = g.meta(arch + ".full_attention_interval");
    c.full_attention_interval = (fa && fa->as_u64(&u64)) ? u64 : 4;  // runtime.rs:258
    c.vocab = g.has("token_embd.weight") && g.tensor("token_embd.weight").dims.size() > 1
                  ? g.tensor("token_embd.weight").dims[1]
                  : 0;
    const GgufValue* eos = g.meta("tokenizer.ggml.eos_token_id");
    c.eos = (eos && eos->as_u64(&u64) && u64 <= 0xffffffffu) ? (int64_t)u64 : -1;

    // ---- device-path constraints
    // (64 and 128 take the cluster attention, 256 the split kernels)
    if (c.head_dim != 64 && c.head_dim != 128 && c.head_dim != 256)
        raise(EVL_ERR_UNSUPPORTED,
              "head_dim " + std::to_string(c.head_dim) + " (device attention handles 64, 128 and 256)");
    if (c.kv_heads == 0 || c.heads % c.kv_heads)
        raise(EVL_ERR_INVALID_DATA, "head_count is not a multiple of head_count_kv");
    const uint64_t group = c.heads / c.kv_heads;
    if (group != 1 && group != 2 && group != 4 && group != 8)
        raise(EVL_ERR_UNSUPPORTED,
              "GQA group size " + std::to_string(group) + " (device attention handles 1, 2, 4, 8)");
    const int T = m.tp_size, R = m.tp_rank;
    if (c.has_ssm && T > 1)
        raise(EVL_ERR_UNSUPPORTED, "tensor parallelism over Qwen3.5 gated-delta layers is not supported");
    const TpShard sh = tp_shard_plan(c, T, R);
    m.lkv_heads = (uint32_t)(c.kv_heads / T);
    m.lheads = (uint32_t)(c.heads / T);
    const uint64_t hd = c.head_dim, qw = c.heads * hd, kw = c.kv_heads * hd;

    // ---- plan every matrix
    std::vector<Planned> plan;
    auto add_matrix = [&](QMatrix& q, const std::string& name, uint64_t want_rows, uint64_t want_cols, uint64_t r0,
                          uint64_t r1, uint64_t c0, uint64_t c1) {
        const GgufTensor& t = g.tensor(name);
        uint64_t cols, rows;
        if (t.dims.size() == 2) {
            cols = t.dims[0];
            rows = t.dims[1];
        } else if (t.dims.size() == 1) {
            cols = t.dims[0];
            rows = 1;
        } else {
            raise(EVL_ERR_INVALID_DATA, name + ": unsupported rank");
        }
        if ((want_rows && rows != want_rows) || (want_cols && cols != want_cols))
            raise(EVL_ERR_INVALID_DATA, name + ": shape [" + std::to_string(cols) + ", " + std::to_string(rows) +
                                            "] does not match the model metadata");
        if (r1 == 0) r1 = rows;
        if (c1 == 0) c1 = cols;
        const size_t nbytes_row = type_bytes(t.type, cols);
        size_t nb;
        const uint8_t* raw = g.raw(t, &nb);
        q.name = name;
        q.type = t.type;
        q.rows = (uint32_t)(r1 - r0);
        q.cols = (uint32_t)(c1 - c0);
        repack_sizes(q);
        Planned p;
        p.m = &q;
        p.raw = raw + r0 * nbytes_row;
        p.stride = nbytes_row;
        if (c0 != 0 || c1 != cols) {
            const uint32_t be = block_elems(t.type);
            if (c0 % be || c1 % be) raise(EVL_ERR_UNSUPPORTED, name + ": shard is not block aligned");
            p.col_byte0 = (uint32_t)type_bytes(t.type, c0);
            p.col_bytes = (uint32_t)type_bytes(t.type, c1 - c0);
        }
        plan.push_back(p);
        m.matrices[name] = &q;
    };
    // the query or the gate half of a gated attn_q (runtime.rs:687-693: per head
    // [query | gate], head_dim rows each), as a matrix of its own
    auto add_query_half = [&](QMatrix& q, const std::string& name, bool gate_half) {
        add_matrix(q, name, 2 * qw, c.dim, 0, 0, 0, 0);
        m.matrices.erase(name);
        q.name = name + (gate_half ? ":gate" : ":query");
        q.rows = (uint32_t)qw;
        repack_sizes(q);
        Planned& pl = plan.back();
        pl.run = (uint32_t)hd;
        pl.period = (uint32_t)(2 * hd);
        pl.offset = gate_half ? (uint32_t)hd : 0;
        m.matrices[q.name] = &q;
    };
    auto dims_of = [&](const std::string& name) {
        const GgufTensor& t = g.tensor(name);
        return std::make_pair(t.dims.size() > 0 ? t.dims[0] : 0, t.dims.size() > 1 ? t.dims[1] : 1);
    };

    const uint64_t f0 = sh.ffn[0], f1 = sh.ffn[1], v0 = sh.vocab[0], v1 = sh.vocab[1];
    m.lffn = (uint32_t)(f1 - f0);
    m.vocab0 = (uint32_t)v0;
    m.lvocab = (uint32_t)(v1 - v0);

    add_matrix(m.embed, "token_embd.weight", 0, c.dim, 0, 0, 0, 0);
    m.layers.resize(c.layers);
    const uint64_t hq0 = sh.q[0], hq1 = sh.q[1], hk0 = sh.kv[0], hk1 = sh.kv[1];
    uint64_t key_dim = 0, key_heads = 0, value_heads = 0, value_dim = 0, channels = 0;
    if (c.has_ssm) {
        key_dim = c.ssm_state;
        key_heads = c.ssm_groups;
        value_heads = c.ssm_value_heads;
    }
    for (uint64_t i = 0; i < c.layers; ++i) {
        const std::string p = "blk." + std::to_string(i) + ".";
        LayerWeights& L = m.layers[i];
        const bool has_delta = g.has(p + "attn_qkv.weight");
        if (arch == "qwen35" && c.full_attention_interval > 0 &&  // runtime.rs:278-290
            has_delta != ((i + 1) % c.full_attention_interval != 0))
            raise(EVL_ERR_INVALID_DATA, p + "attention type does not match qwen35.full_attention_interval=" +
                                            std::to_string(c.full_attention_interval));
        if (has_delta) {  // runtime.rs:298-356
            if (!c.has_ssm)
                raise(EVL_ERR_INVALID_DATA, "gated-delta tensors found without SSM architecture metadata");
            if (value_heads == 0 || c.ssm_inner % value_heads)
                raise(EVL_ERR_INVALID_DATA, "Qwen3.5 SSM inner size must divide evenly across value heads");
            value_dim = c.ssm_inner / value_heads;
            channels = 2 * key_dim * key_heads + value_dim * value_heads;
            const uint64_t vw = value_dim * value_heads;
            const std::string names[] = {"attn_qkv.weight", "attn_gate.weight", "ssm_conv1d.weight",
                                         "ssm_alpha.weight", "ssm_beta.weight", "ssm_a",
                                         "ssm_dt", "ssm_norm.weight", "ssm_out.weight"};
            for (const auto& n : names) g.tensor(p + n);  // NotFound in the reference's order
            auto elems = [&](const std::string& n) { return g.tensor(p + n).elements(); };
            const auto qkv = dims_of(p + "attn_qkv.weight"), z = dims_of(p + "attn_gate.weight"),
                       al = dims_of(p + "ssm_alpha.weight"), be = dims_of(p + "ssm_beta.weight"),
                       out = dims_of(p + "ssm_out.weight");
            if (qkv.second != channels || z.second != vw || elems("ssm_conv1d.weight") != c.ssm_conv_kernel * channels ||
                al.second != value_heads || be.second != value_heads || elems("ssm_a") != value_heads ||
                elems("ssm_dt") != value_heads || elems("ssm_norm.weight") != value_dim || out.first != vw ||
                out.second != c.dim || qkv.first != c.dim || z.first != c.dim || al.first != c.dim || be.first != c.dim)
                raise(EVL_ERR_INVALID_DATA, p + "gated-delta tensor shapes do not match Qwen3.5 metadata");
            if (c.ssm_conv_kernel == 0 || key_dim == 0 || key_heads == 0)
                raise(EVL_ERR_INVALID_DATA, p + "ssm.conv_kernel, ssm.state_size and ssm.group_count must be non-zero");
            if (gated_delta_smem((uint32_t)key_dim, (uint32_t)value_dim) > 48 * 1024)
                raise(EVL_ERR_UNSUPPORTED, p + "gated-delta key and value widths above 6144 values");
            L.delta = true;
            L.d.index = m.delta_layers++;
            m.delta_channels = (uint32_t)channels;
            m.delta_value_width = (uint32_t)vw;
            add_matrix(L.d.qkv, p + "attn_qkv.weight", channels, c.dim, 0, 0, 0, 0);
            add_matrix(L.d.z, p + "attn_gate.weight", vw, c.dim, 0, 0, 0, 0);
            // alpha and beta stacked, so they join the attn_qkv / attn_gate launch
            // (EVELYN_DELTA_STACK=0: two matrices and a launch of their own)
            const char* se = std::getenv("EVELYN_DELTA_STACK");
            if (g.tensor(p + "ssm_alpha.weight").type == g.tensor(p + "ssm_beta.weight").type &&
                !(se && se[0] == '0')) {
                add_matrix(L.d.ab, p + "ssm_alpha.weight", value_heads, c.dim, 0, 0, 0, 0);
                m.matrices.erase(p + "ssm_alpha.weight");
                L.d.ab.name = p + "ssm_alpha.weight+ssm_beta.weight";
                L.d.ab.rows = (uint32_t)(2 * value_heads);
                repack_sizes(L.d.ab);
                size_t nb2;
                plan.back().raw2 = g.raw(g.tensor(p + "ssm_beta.weight"), &nb2);
                plan.back().split = (uint32_t)value_heads;
                m.matrices[L.d.ab.name] = &L.d.ab;
            } else {
                add_matrix(L.d.alpha, p + "ssm_alpha.weight", value_heads, c.dim, 0, 0, 0, 0);
                add_matrix(L.d.beta, p + "ssm_beta.weight", value_heads, c.dim, 0, 0, 0, 0);
            }
            add_matrix(L.d.out, p + "ssm_out.weight", c.dim, vw, 0, 0, 0, 0);
            add_matrix(L.gate, p + "ffn_gate.weight", c.ffn, c.dim, f0, f1, 0, 0);
            add_matrix(L.up, p + "ffn_up.weight", c.ffn, c.dim, f0, f1, 0, 0);
            add_matrix(L.down, p + "ffn_down.weight", c.dim, c.ffn, 0, 0, T > 1 ? f0 : 0, T > 1 ? f1 : 0);
            continue;
        }
        if (arch == "qwen35") {  // the gated query (runtime.rs:371)
            L.gated = true;
            add_query_half(L.q, p + "attn_q.weight", false);
            add_query_half(L.qg, p + "attn_q.weight", true);
        } else {
            add_matrix(L.q, p + "attn_q.weight", qw, c.dim, hq0, hq1, 0, 0);
        }
        add_matrix(L.k, p + "attn_k.weight", kw, c.dim, hk0, hk1, 0, 0);
        add_matrix(L.v, p + "attn_v.weight", kw, c.dim, hk0, hk1, 0, 0);
        add_matrix(L.o, p + "attn_output.weight", c.dim, qw, 0, 0, T > 1 ? hq0 : 0, T > 1 ? hq1 : 0);
        add_matrix(L.gate, p + "ffn_gate.weight", c.ffn, c.dim, f0, f1, 0, 0);
        add_matrix(L.up, p + "ffn_up.weight", c.ffn, c.dim, f0, f1, 0, 0);
        add_matrix(L.down, p + "ffn_down.weight", c.dim, c.ffn, 0, 0, T > 1 ? f0 : 0, T > 1 ? f1 : 0);
    }
    // LM head: output.weight, else the tied embedding (runtime.rs:392-396). Tied, it is
    // planned as its own (vocabulary-sharded) copy and the embedding keeps the name.
    const std::string head_name = g.has("output.weight") ? "output.weight" : "token_embd.weight";
    add_matrix(m.lm_head, head_name, c.vocab, c.dim, v0, v1, 0, 0);
    if (head_name == "token_embd.weight") m.matrices["token_embd.weight"] = &m.embed;

    // ---- vectors (f32 on the device)
    struct VecPlan {
        std::string name;
        float** dst;
        uint64_t n;
    };
    std::vector<VecPlan> vplan;
    for (uint64_t i = 0; i < c.layers; ++i) {
        const std::string p = "blk." + std::to_string(i) + ".";
        LayerWeights& L = m.layers[i];
        vplan.push_back({p + "attn_norm.weight", &L.attn_norm, c.dim});
        const std::string fn = g.has(p + "post_attention_norm.weight") ? p + "post_attention_norm.weight"
                                                                         : p + "ffn_norm.weight";
        vplan.push_back({fn, &L.ffn_norm, c.dim});
        if (L.delta) {
            vplan.push_back({p + "ssm_conv1d.weight", &L.d.conv, channels * c.ssm_conv_kernel});
            vplan.push_back({p + "ssm_a", &L.d.a, value_heads});
            vplan.push_back({p + "ssm_dt", &L.d.dt, value_heads});
            vplan.push_back({p + "ssm_norm.weight", &L.d.norm, value_dim});
            continue;
        }
        if (g.has(p + "attn_q_norm.weight")) vplan.push_back({p + "attn_q_norm.weight", &L.q_norm, hd});
        if (g.has(p + "attn_k_norm.weight")) vplan.push_back({p + "attn_k_norm.weight", &L.k_norm, hd});
    }
    vplan.push_back({"output_norm.weight", &m.out_norm, c.dim});
    const uint32_t rdim = (uint32_t)(std::min<uint64_t>(c.rope_dim, hd) & ~1ull);
    const size_t rope_floats = std::max<uint32_t>((rdim / 2 + 63) / 64 * 64, 64);
    size_t vfloats = rope_floats;
    for (auto& v : vplan) {
        const GgufTensor& t = g.tensor(v.name);
        if (t.elements() != v.n) raise(EVL_ERR_INVALID_DATA, v.name + ": unexpected length");
        vfloats += (v.n + 63) / 64 * 64;
    }

    // ---- allocate and fill
    size_t total = 0;
    for (auto& p : plan) {
        p.m->offset = total;
        total += p.m->bytes();
    }
    m.weights.alloc(total);
    m.vectors.alloc(vfloats * 4);
    // the raw tensor bytes go to the device as they are and are repacked there
    // (launch_repack); a column shard of a tensor-parallel rank is gathered on the host
    // first, so only its own bytes cross
    size_t max_raw = 0, max_gather = 0;
    for (auto& p : plan) {
        place(*p.m, m.weights.as<uint8_t>());
        const size_t row = p.col_bytes ? p.col_bytes : p.stride;
        max_raw = std::max(max_raw, row * p.m->rows);
        if (p.col_bytes || p.run || p.raw2) max_gather = std::max(max_gather, row * p.m->rows);
    }
    std::vector<uint8_t> gather(max_gather);
    DeviceBuffer draw;
    draw.alloc(max_raw);
    for (auto& p : plan) {
        const uint8_t* src = p.raw;
        size_t stride = p.stride;
        if (p.col_bytes || p.run || p.raw2) {
            const size_t rb = p.col_bytes ? p.col_bytes : p.stride;
            for (uint32_t r = 0; r < p.m->rows; ++r) {
                const size_t sr = p.run ? (size_t)(r / p.run) * p.period + p.offset + r % p.run : r;
                const uint8_t* row = p.raw2 && r >= p.split ? p.raw2 + (sr - p.split) * p.stride : p.raw + sr * p.stride;
                std::memcpy(gather.data() + (size_t)r * rb, row + p.col_byte0, rb);
            }
            src = gather.data();
            stride = rb;
        }
        // (the legacy stream orders each copy after the previous repack that read the buffer)
        cuda_check(cudaMemcpy(draw.p, src, stride * p.m->rows, cudaMemcpyHostToDevice), "upload weights");
        cuda_check(launch_repack(p.m->dev, m.weights.as<uint8_t>() + p.m->offset, p.m->bytes(), draw.p, stride, 0),
                   "repack weights");
    }
    float* vbase = m.vectors.as<float>();
    m.rope_inv_freq = vbase;
    {
        std::vector<float> inv(rope_floats, 0.f);
        // src/runtime.rs:443 and :467: base.powf(-2i / rotary_dim), f32 powf
        for (uint32_t i = 0; i < rdim / 2; ++i) inv[i] = powf(c.rope_base, (-2.0f * (float)i) / (float)rdim);
        cuda_check(cudaMemcpy(vbase, inv.data(), inv.size() * 4, cudaMemcpyHostToDevice), "upload rope table");
    }
    size_t voff = rope_floats;
    DeviceBuffer tmp;
    for (auto& v : vplan) {
        const GgufTensor& t = g.tensor(v.name);
        size_t nb;
        const uint8_t* raw = g.raw(t, &nb);
        float* dst = vbase + voff;
        if (t.type == GGML_F32) {
            cuda_check(cudaMemcpy(dst, raw, nb, cudaMemcpyHostToDevice), "upload norm");
        } else {
            if (tmp.bytes < nb) tmp.alloc(nb);
            cuda_check(cudaMemcpy(tmp.p, raw, nb, cudaMemcpyHostToDevice), "upload norm");
            cuda_check(launch_dequant_raw(t.type, tmp.p, v.n, dst, 0), "dequantize norm");
        }
        *v.dst = dst;
        m.vecs[v.name] = {dst, (size_t)v.n};
        voff += (v.n + 63) / 64 * 64;
    }
    cuda_check(cudaDeviceSynchronize(), "load");

    // weight bytes one decode step streams on this rank
    uint64_t wb = 0;
    for (auto& L : m.layers)
        wb += L.q.bytes() + L.k.bytes() + L.v.bytes() + L.o.bytes() + L.gate.bytes() + L.up.bytes() + L.down.bytes() +
              L.qg.bytes() + L.d.qkv.bytes() + L.d.z.bytes() + L.d.alpha.bytes() + L.d.beta.bytes() + L.d.ab.bytes() +
              L.d.out.bytes();
    wb += m.lm_head.bytes();
    m.weight_bytes_per_step = wb;

    // ---- tensor-parallel communicator
    if (T > 1) {
        ncclUniqueId id;
        static_assert(sizeof(id.internal) == 128, "ncclUniqueId size");
        std::memcpy(id.internal, o.nccl_id, 128);
        nccl_check(nccl().CommInitRank(&m.comm, T, id, R), "ncclCommInitRank");
    }
    cuda_check(cudaStreamCreateWithFlags(&m.stream, cudaStreamNonBlocking), "cudaStreamCreate");
    const size_t sc = (size_t)c.dim * 3 + m.lffn + std::max<size_t>(c.dim, c.vocab) + 64;
    m.scratch.alloc(sc * 4 + 256);
    m.d_err = reinterpret_cast<int32_t*>(m.scratch.as<uint8_t>() + sc * 4);
    cuda_check(cudaMemset(m.d_err, 0, 4), "memset");
    return M;
}

void allreduce_sum(Model& m, float* buf, size_t n, cudaStream_t s) {
    nccl_check(nccl().AllReduce(buf, buf, n, ncclFloat32, ncclSum, m.comm, s), "ncclAllReduce");
}

bool build_gemm_weights(Model& m) {
    if (m.gemm_ready) return true;
    std::vector<QMatrix*> mats;
    for (auto& L : m.layers)
        for (QMatrix* q : {&L.q, &L.k, &L.v, &L.o, &L.gate, &L.up, &L.down}) mats.push_back(q);
    mats.push_back(&m.lm_head);
    uint64_t total = 0;
    std::vector<uint64_t> off;
    for (QMatrix* q : mats) {
        const uint64_t b = gemm_layout_bytes(q->type, q->rows, q->cols);
        if (!b) return false;
        off.push_back(total);
        total += (b + 255) / 256 * 256;
    }
    DeviceGuard g(m.device);
    m.gemm_weights.alloc(total);
    for (size_t i = 0; i < mats.size(); ++i) {
        QMatrix& q = *mats[i];
        q.gemm = gemm_view(q.type, q.rows, q.cols, m.gemm_weights.as<uint8_t>() + off[i]);
        cuda_check(launch_gemm_repack(q.dev, q.gemm, m.stream), "gemm repack");
    }
    cuda_check(cudaStreamSynchronize(m.stream), "gemm repack");
    m.gemm_ready = true;
    return true;
}

void run_dense_ffn(Model& m, size_t layer, const float* x, const float* norm_w, float* y, bool add, uint32_t batch,
                   float* h_buf, float* y_buf, int* err, const QMatDev* next, cudaStream_t s, bool pdl,
                   const TpPeers* peers, uint32_t slot) {
    const LayerWeights& L = m.layers[layer];
    const uint32_t dim = (uint32_t)m.cfg.dim;
    for (uint32_t b = 0; b < batch; ++b) {
        MatvecArgs a;
        a.nseg = 1;
        a.seg[0].m = L.gate.dev;
        a.seg[0].m2 = L.up.dev;
        a.seg[0].y = h_buf + (size_t)b * m.lffn;
        a.seg[0].epi = EPI_SWIGLU;
        a.x = x + (size_t)b * dim;
        a.cols = dim;
        a.norm_w = norm_w;
        a.eps = m.cfg.eps;
        a.err = err;
        if (b + 1 == batch) {
            a.prefetch[0] = L.down.dev;
            a.prefetch_bytes = prefetch_kb(96) << 10;
        }
        cuda_check(launch_qmatvec(a, s, pdl), "ffn gate/up");
    }
    const bool tp = m.tp_size > 1;
    for (uint32_t b = 0; b < batch; ++b) {
        MatvecArgs a;
        a.nseg = 1;
        a.seg[0].m = L.down.dev;
        a.seg[0].y = (tp ? y_buf : y) + (size_t)b * dim;
        a.seg[0].epi = (add && !tp) ? EPI_ADD : EPI_STORE;
        a.x = h_buf + (size_t)b * m.lffn;
        a.cols = m.lffn;
        a.err = err;
        if (next && b + 1 == batch) {
            for (int i = 0; i < 3; ++i) a.prefetch[i] = next[i];
            a.prefetch_bytes = prefetch_kb(96) << 10;
        }
        cuda_check(launch_qmatvec(a, s, pdl), "ffn down");
    }
    if (tp && peers && add) {  // partial sums through the peer inboxes, residual add fused
        cuda_check(launch_tp_allreduce_add(*peers, TP_DOWN, slot, y, y_buf, batch * dim, err, s, pdl), "ffn sum");
    } else if (tp) {
        allreduce_sum(m, y_buf, (size_t)batch * dim, s);
        if (add) {
            cuda_check(launch_add(y, y_buf, (size_t)batch * dim, s, false), "residual add");
        } else {
            cuda_check(cudaMemcpyAsync(y, y_buf, (size_t)batch * dim * 4, cudaMemcpyDeviceToDevice, s), "copy");
        }
    }
}

}  // namespace evl
