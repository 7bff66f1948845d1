// synth_gguf.cpp -- seeded synthetic Qwen3-family GGUF images and the block
// encoders (Q8_0, Q4_K, Q5_K, Q6_K, F16, BF16, F32) that produce them.
//
// The reference reads GGUF but never writes it (src/gguf.rs has dequantisers only),
// so these encoders are new. Any valid encoding is acceptable: parity is defined
// on what the reference's dequantisers (gguf.rs:338-430) return for the bytes
// written here. The metadata keys are the ones Model::load reads
// (src/runtime.rs:199-269); tensor names follow runtime.rs:274-396.
//
// Weights are N(0, stddev) from a counter-based generator keyed by
// (seed, tensor index, element index), so the image is identical however many
// threads build it. Norm weights are 1.0 (F32).

#include "synth_gguf.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

namespace {

thread_local std::string g_err;

constexpr uint32_t F32 = 0, F16 = 1, Q8_0 = 8, Q4_K = 12, Q5_K = 13, Q6_K = 14, BF16 = 30;

// ------------------------------------------------------------------ numbers
uint16_t f32_to_f16(float f) {  // IEEE binary16, round to nearest even
    uint32_t x;
    std::memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0));
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);  // rounds to inf
    if (ax < 0x38800000u) {                                      // subnormal or zero in f16
        if (ax < 0x33000000u) return (uint16_t)sign;
        uint32_t e = ax >> 23;
        uint32_t m = (ax & 0x7fffffu) | 0x800000u;
        uint32_t shift = 126 - e;  // value / 2^-24 = m * 2^(e - 126)
        uint32_t q = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1);
        uint32_t halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (q & 1))) ++q;
        return (uint16_t)(sign | q);
    }
    uint32_t r = ax - 0x38000000u;  // rebias exponent 127 -> 15
    uint32_t q = r >> 13;
    uint32_t rem = r & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1))) ++q;
    return (uint16_t)(sign | q);
}

float f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15) << 31, exp = (h >> 10) & 0x1f, frac = h & 0x3ff, bits;
    if (exp == 0 && frac == 0) {
        bits = sign;
    } else if (exp == 0) {
        int e = 127 - 15 + 1;
        while (!(frac & 0x400)) {
            frac <<= 1;
            --e;
        }
        bits = sign | ((uint32_t)e << 23) | ((frac & 0x3ff) << 13);
    } else if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (frac << 13);
    } else {
        bits = sign | ((exp + 112) << 23) | (frac << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

uint16_t f32_to_bf16(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40);
    x += 0x7fffu + ((x >> 16) & 1);
    return (uint16_t)(x >> 16);
}

inline int nearest(float v) { return (int)std::lround(v); }

// splitmix64 finaliser over a counter: deterministic per (seed, tensor, index)
inline uint64_t mix(uint64_t z) {
    z += 0x9E3779B97F4A7C15ULL;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
    return z ^ (z >> 31);
}

// Box-Muller pair for element pair (2k, 2k+1)
inline void normal_pair(uint64_t key, uint64_t k, float sd, float* a, float* b) {
    uint64_t r = mix(key ^ mix(k));
    double u1 = ((r >> 11) + 1.0) * (1.0 / 9007199254740993.0);  // (0, 1]
    uint64_t r2 = mix(r);
    double u2 = (r2 >> 11) * (1.0 / 9007199254740992.0);
    double rad = std::sqrt(-2.0 * std::log(u1));
    *a = (float)(sd * rad * std::cos(6.283185307179586 * u2));
    *b = (float)(sd * rad * std::sin(6.283185307179586 * u2));
}

void gen_normal(uint64_t key, size_t first, size_t n, float sd, float* out) {
    // first is even by construction (block aligned), n is even
    for (size_t i = 0; i < n; i += 2) normal_pair(key, (first + i) / 2, sd, &out[i], &out[i + 1]);
}

// ------------------------------------------------------------------ encoders
void enc_q8_0(const float* x, uint8_t* out) {  // one 32-value block -> 34 bytes
    float amax = 0;
    for (int i = 0; i < 32; ++i) amax = std::max(amax, std::fabs(x[i]));
    float d = amax / 127.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    uint16_t dh = f32_to_f16(d);
    std::memcpy(out, &dh, 2);
    for (int i = 0; i < 32; ++i) out[2 + i] = (uint8_t)(int8_t)std::max(-127, std::min(127, nearest(x[i] * id)));
}

// 6-bit scale/min packing, the inverse of get_scale_min_k4 (gguf.rs:327-336)
void pack_scale_min_k4(const int* ls, const int* lm, uint8_t* sc) {
    std::memset(sc, 0, 12);
    for (int j = 0; j < 8; ++j) {
        if (j < 4) {
            sc[j] = (uint8_t)(ls[j] & 63);
            sc[j + 4] = (uint8_t)(lm[j] & 63);
        } else {
            sc[j + 4] = (uint8_t)((ls[j] & 0xf) | ((lm[j] & 0xf) << 4));
            sc[j - 4] |= (uint8_t)((ls[j] >> 4) << 6);
            sc[j] |= (uint8_t)((lm[j] >> 4) << 6);
        }
    }
}

// Shared affine K-quant step for Q4_K (nmax 15) and Q5_K (nmax 31): 8 sub-blocks
// of 32, each value = d*s_j*q - dmin*m_j with 6-bit s_j, m_j.
void affine_k(const float* x, int nmax, uint16_t* dh, uint16_t* dminh, uint8_t* sc, int* q) {
    float scale[8], mins[8];
    for (int j = 0; j < 8; ++j) {
        float mn = x[32 * j], mx = x[32 * j];
        for (int i = 1; i < 32; ++i) {
            mn = std::min(mn, x[32 * j + i]);
            mx = std::max(mx, x[32 * j + i]);
        }
        if (mn > 0) mn = 0;
        scale[j] = (mx - mn) / (float)nmax;
        mins[j] = -mn;
    }
    float max_scale = 0, max_min = 0;
    for (int j = 0; j < 8; ++j) {
        max_scale = std::max(max_scale, scale[j]);
        max_min = std::max(max_min, mins[j]);
    }
    *dh = f32_to_f16(max_scale / 63.0f);
    *dminh = f32_to_f16(max_min / 63.0f);
    float d = f16_to_f32(*dh), dmin = f16_to_f32(*dminh);
    int ls[8], lm[8];
    for (int j = 0; j < 8; ++j) {
        ls[j] = d > 0 ? std::min(63, std::max(0, nearest(scale[j] / d))) : 0;
        lm[j] = dmin > 0 ? std::min(63, std::max(0, nearest(mins[j] / dmin))) : 0;
    }
    pack_scale_min_k4(ls, lm, sc);
    for (int j = 0; j < 8; ++j) {
        float dd = d * (float)ls[j], dm = dmin * (float)lm[j];
        for (int i = 0; i < 32; ++i) {
            int v = dd > 0 ? nearest((x[32 * j + i] + dm) / dd) : 0;
            q[32 * j + i] = std::max(0, std::min(nmax, v));
        }
    }
}

void enc_q4_k(const float* x, uint8_t* out) {  // 256 values -> 144 bytes
    uint16_t dh, dminh;
    int q[256];
    affine_k(x, 15, &dh, &dminh, out + 4, q);
    std::memcpy(out, &dh, 2);
    std::memcpy(out + 2, &dminh, 2);
    uint8_t* qs = out + 16;
    for (int b = 0; b < 4; ++b)
        for (int l = 0; l < 32; ++l) qs[32 * b + l] = (uint8_t)(q[64 * b + l] | (q[64 * b + 32 + l] << 4));
}

void enc_q5_k(const float* x, uint8_t* out) {  // 256 values -> 176 bytes
    uint16_t dh, dminh;
    int q[256];
    affine_k(x, 31, &dh, &dminh, out + 4, q);
    std::memcpy(out, &dh, 2);
    std::memcpy(out + 2, &dminh, 2);
    uint8_t* qh = out + 16;
    uint8_t* qs = out + 48;
    std::memset(qh, 0, 32);
    for (int b = 0; b < 4; ++b)
        for (int l = 0; l < 32; ++l) {
            int lo = q[64 * b + l], hi = q[64 * b + 32 + l];
            qs[32 * b + l] = (uint8_t)((lo & 0xf) | ((hi & 0xf) << 4));
            if (lo & 16) qh[l] |= (uint8_t)(1u << (2 * b));
            if (hi & 16) qh[l] |= (uint8_t)(1u << (2 * b + 1));
        }
}

void enc_q6_k(const float* x, uint8_t* out) {  // 256 values -> 210 bytes
    // 16 groups of 16 contiguous values; group g's scale sits at sc[g].
    float gs[16];
    float max_scale = 0;
    for (int g = 0; g < 16; ++g) {
        float amax = 0;
        for (int i = 0; i < 16; ++i) amax = std::max(amax, std::fabs(x[16 * g + i]));
        gs[g] = amax / 31.0f;
        max_scale = std::max(max_scale, gs[g]);
    }
    uint16_t dh = f32_to_f16(max_scale / 127.0f);
    float d = f16_to_f32(dh);
    int8_t sc[16];
    int L[256];
    for (int g = 0; g < 16; ++g) {
        sc[g] = (int8_t)(d > 0 ? std::min(127, std::max(0, nearest(gs[g] / d))) : 0);
        float dd = d * (float)sc[g];
        for (int i = 0; i < 16; ++i) {
            int v = dd > 0 ? nearest(x[16 * g + i] / dd) : 0;
            L[16 * g + i] = std::max(-32, std::min(31, v)) + 32;
        }
    }
    uint8_t* ql = out;
    uint8_t* qh = out + 128;
    for (int h = 0; h < 2; ++h)
        for (int l = 0; l < 32; ++l) {
            int q1 = L[128 * h + l], q2 = L[128 * h + l + 32], q3 = L[128 * h + l + 64], q4 = L[128 * h + l + 96];
            ql[64 * h + l] = (uint8_t)((q1 & 0xf) | ((q3 & 0xf) << 4));
            ql[64 * h + l + 32] = (uint8_t)((q2 & 0xf) | ((q4 & 0xf) << 4));
            qh[32 * h + l] = (uint8_t)((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
        }
    std::memcpy(out + 192, sc, 16);
    std::memcpy(out + 208, &dh, 2);
}

size_t block_elems(uint32_t t) {
    switch (t) {
        case Q8_0: return 32;
        case Q4_K:
        case Q5_K:
        case Q6_K: return 256;
        case F32:
        case F16:
        case BF16: return 2;  // handled element-wise; 2 keeps normal pairs aligned
        default: return 0;
    }
}
size_t block_bytes(uint32_t t) {
    switch (t) {
        case Q8_0: return 34;
        case Q4_K: return 144;
        case Q5_K: return 176;
        case Q6_K: return 210;
        case F32: return 8;
        case F16:
        case BF16: return 4;
        default: return 0;
    }
}

void encode_blocks(uint32_t t, const float* x, size_t nblocks, uint8_t* out) {
    size_t be = block_elems(t), bb = block_bytes(t);
    for (size_t b = 0; b < nblocks; ++b) {
        const float* xb = x + b * be;
        uint8_t* ob = out + b * bb;
        switch (t) {
            case Q8_0: enc_q8_0(xb, ob); break;
            case Q4_K: enc_q4_k(xb, ob); break;
            case Q5_K: enc_q5_k(xb, ob); break;
            case Q6_K: enc_q6_k(xb, ob); break;
            case F32: std::memcpy(ob, xb, 8); break;
            case F16:
                for (int i = 0; i < 2; ++i) {
                    uint16_t h = f32_to_f16(xb[i]);
                    std::memcpy(ob + 2 * i, &h, 2);
                }
                break;
            case BF16:
                for (int i = 0; i < 2; ++i) {
                    uint16_t h = f32_to_bf16(xb[i]);
                    std::memcpy(ob + 2 * i, &h, 2);
                }
                break;
        }
    }
}

template <class F> void parallel_for(size_t n, int threads, F&& fn) {
    if (threads <= 1 || n < 2) {
        for (size_t i = 0; i < n; ++i) fn(i);
        return;
    }
    std::vector<std::thread> ts;
    size_t per = (n + threads - 1) / threads;
    for (int t = 0; t < threads; ++t) {
        size_t a = t * per, b = std::min(n, a + per);
        if (a >= b) break;
        ts.emplace_back([=, &fn] {
            for (size_t i = a; i < b; ++i) fn(i);
        });
    }
    for (auto& th : ts) th.join();
}

// ------------------------------------------------------------------ GGUF writer
struct Tensor {
    std::string name;
    std::vector<uint64_t> dims;
    uint32_t type;
    bool ones;  // norm weight (all 1.0) instead of N(0, sd)
    float sd = 0.f;  // > 0: N(0, sd) instead of the spec's stddev; < 0: the decay rates below
    uint64_t offset = 0, nbytes = 0;
};

struct Buf {
    std::vector<uint8_t> b;
    template <class T> void put(T v) {
        size_t o = b.size();
        b.resize(o + sizeof(T));
        std::memcpy(b.data() + o, &v, sizeof(T));
    }
    void str(const std::string& s) {
        put<uint64_t>(s.size());
        b.insert(b.end(), s.begin(), s.end());
    }
    void kv_u32(const std::string& k, uint32_t v) { str(k); put<uint32_t>(4); put<uint32_t>(v); }
    void kv_f32(const std::string& k, float v) { str(k); put<uint32_t>(6); put<float>(v); }
    void kv_str(const std::string& k, const std::string& v) { str(k); put<uint32_t>(8); str(v); }
    void kv_bool(const std::string& k, bool v) { str(k); put<uint32_t>(7); put<uint8_t>(v ? 1 : 0); }
};

uint64_t tensor_bytes(uint32_t t, uint64_t n) {
    switch (t) {
        case F32: return n * 4;
        case F16:
        case BF16: return n * 2;
        case Q8_0: return n / 32 * 34;
        case Q4_K: return n / 256 * 144;
        case Q5_K: return n / 256 * 176;
        case Q6_K: return n / 256 * 210;
        default: return 0;
    }
}

bool valid_type(uint32_t t) { return block_elems(t) != 0; }

}  // namespace

extern "C" {

const char* evs_last_error(void) { return g_err.c_str(); }

int evs_encode(uint32_t type, const float* x, size_t n, uint8_t* out, size_t out_len) {
    if (!valid_type(type)) {
        g_err = "unsupported ggml type " + std::to_string(type);
        return 4;
    }
    size_t be = block_elems(type);
    if (type == F32 || type == F16 || type == BF16) be = 1;
    if (n % be != 0) {
        g_err = "element count is not a whole number of blocks";
        return 1;
    }
    if (out_len < tensor_bytes(type, n)) {
        g_err = "output buffer too small";
        return 1;
    }
    if (type == F32 || type == F16 || type == BF16) {
        for (size_t i = 0; i < n; ++i) {
            if (type == F32) {
                std::memcpy(out + 4 * i, &x[i], 4);
            } else {
                uint16_t h = type == F16 ? f32_to_f16(x[i]) : f32_to_bf16(x[i]);
                std::memcpy(out + 2 * i, &h, 2);
            }
        }
        return 0;
    }
    encode_blocks(type, x, n / be, out);
    return 0;
}

uint16_t evs_f32_to_f16(float f) { return f32_to_f16(f); }

int evs_build(const evs_model_spec* s, uint8_t** out, size_t* out_len) {
    *out = nullptr;
    *out_len = 0;
    const uint64_t hd = s->head_dim, qw = (uint64_t)s->heads * hd, kw = (uint64_t)s->kv_heads * hd;
    const std::string a = s->arch[0] ? s->arch : "qwen3";
    const bool q35 = a == "qwen35";
    uint32_t types[] = {s->type_attn_q, s->type_attn_k,    s->type_attn_v, s->type_attn_output,
                        s->type_ffn_gate, s->type_ffn_up,  s->type_ffn_down, s->type_embed,
                        s->type_output,   q35 ? s->type_ssm : F32};
    for (uint32_t t : types)
        if (!valid_type(t)) {
            g_err = "unsupported ggml type " + std::to_string(t);
            return 4;
        }
    if (q35 && (!s->ssm_value_heads || s->ssm_inner % s->ssm_value_heads || !s->ssm_conv_kernel)) {
        g_err = "qwen35 needs ssm_value_heads dividing ssm_inner and a conv kernel";
        return 2;
    }
    std::vector<Tensor> ts;
    auto add = [&](const std::string& n, std::vector<uint64_t> dims, uint32_t type, bool ones, float sd = 0.f) {
        ts.push_back(Tensor{n, dims, type, ones, sd});
    };
    const uint64_t kwd = (uint64_t)s->ssm_state * s->ssm_groups, vwd = s->ssm_inner;
    const uint64_t channels = 2 * kwd + vwd, vh = s->ssm_value_heads;
    add("token_embd.weight", {s->dim, s->vocab}, s->type_embed, false);
    for (uint32_t i = 0; i < s->layers; ++i) {
        std::string p = "blk." + std::to_string(i) + ".";
        add(p + "attn_norm.weight", {s->dim}, F32, true);
        const bool delta = q35 && s->full_attention_interval && (i + 1) % s->full_attention_interval != 0;
        if (delta) {  // runtime.rs:315-324 names and shapes
            add(p + "attn_qkv.weight", {s->dim, channels}, s->type_ssm, false);
            add(p + "attn_gate.weight", {s->dim, vwd}, s->type_ssm, false);
            add(p + "ssm_conv1d.weight", {s->ssm_conv_kernel, channels}, F32, false, 0.5f);
            add(p + "ssm_alpha.weight", {s->dim, vh}, s->type_ssm, false);
            add(p + "ssm_beta.weight", {s->dim, vh}, s->type_ssm, false);
            add(p + "ssm_a", {vh}, F32, false, -1.f);
            add(p + "ssm_dt", {vh}, F32, false, 0.5f);
            add(p + "ssm_norm.weight", {vwd / vh}, F32, true);
            add(p + "ssm_out.weight", {vwd, s->dim}, s->type_ssm, false);
        } else {
            add(p + "attn_q.weight", {s->dim, q35 ? 2 * qw : qw}, s->type_attn_q, false);
            add(p + "attn_k.weight", {s->dim, kw}, s->type_attn_k, false);
            add(p + "attn_v.weight", {s->dim, kw}, s->type_attn_v, false);
            add(p + "attn_output.weight", {qw, s->dim}, s->type_attn_output, false);
            if (s->qk_norm) {
                add(p + "attn_q_norm.weight", {hd}, F32, true);
                add(p + "attn_k_norm.weight", {hd}, F32, true);
            }
        }
        add(p + (q35 ? "post_attention_norm.weight" : "ffn_norm.weight"), {s->dim}, F32, true);
        add(p + "ffn_gate.weight", {s->dim, s->ffn}, s->type_ffn_gate, false);
        add(p + "ffn_up.weight", {s->dim, s->ffn}, s->type_ffn_up, false);
        add(p + "ffn_down.weight", {s->ffn, s->dim}, s->type_ffn_down, false);
    }
    add("output_norm.weight", {s->dim}, F32, true);
    if (!s->tied_output) add("output.weight", {s->dim, s->vocab}, s->type_output, false);

    const uint64_t align = 32;
    uint64_t off = 0;
    for (auto& t : ts) {
        uint64_t n = 1;
        for (auto d : t.dims) n *= d;
        // (norm weights and the small F32 vectors are written element by element)
        if ((!t.ones && t.sd == 0.f && n % block_elems(t.type) != 0) ||
            (t.type != F32 && t.type != F16 && t.type != BF16 && t.dims[0] % block_elems(t.type) != 0)) {
            g_err = t.name + ": row length is not a whole number of quant blocks";
            return 2;
        }
        t.offset = off;
        t.nbytes = tensor_bytes(t.type, n);
        off += (t.nbytes + align - 1) / align * align;
    }
    const uint64_t data_len = off;

    Buf h;
    h.b.insert(h.b.end(), {'G', 'G', 'U', 'F'});
    h.put<uint32_t>(3);
    h.put<uint64_t>(ts.size());
    const uint32_t n_kv = 13 + (q35 ? 6 : 0) + (s->rope_dim ? 1 : 0) + (s->mrope_interleaved ? 1 : 0);
    h.put<uint64_t>(n_kv);
    h.kv_str("general.architecture", a);
    h.kv_str("general.name", "evelyn-synthetic");
    h.kv_u32("general.alignment", (uint32_t)align);
    h.kv_u32(a + ".block_count", s->layers);
    h.kv_u32(a + ".context_length", 40960);
    h.kv_u32(a + ".embedding_length", s->dim);
    h.kv_u32(a + ".feed_forward_length", s->ffn);
    h.kv_u32(a + ".attention.head_count", s->heads);
    h.kv_u32(a + ".attention.head_count_kv", s->kv_heads);
    h.kv_u32(a + ".attention.key_length", s->head_dim);
    h.kv_f32(a + ".rope.freq_base", s->rope_base);
    h.kv_f32(a + ".attention.layer_norm_rms_epsilon", s->eps);
    h.kv_u32("tokenizer.ggml.eos_token_id", s->eos_token_id);
    if (q35) {  // runtime.rs:225-235, 258
        h.kv_u32(a + ".ssm.conv_kernel", s->ssm_conv_kernel);
        h.kv_u32(a + ".ssm.inner_size", s->ssm_inner);
        h.kv_u32(a + ".ssm.state_size", s->ssm_state);
        h.kv_u32(a + ".ssm.group_count", s->ssm_groups);
        h.kv_u32(a + ".ssm.time_step_rank", s->ssm_value_heads);
        h.kv_u32(a + ".full_attention_interval", s->full_attention_interval);
    }
    if (s->rope_dim) h.kv_u32(a + ".rope.dimension_count", s->rope_dim);
    if (s->mrope_interleaved) h.kv_bool(a + ".rope.mrope_interleaved", true);
    for (auto& t : ts) {
        h.str(t.name);
        h.put<uint32_t>((uint32_t)t.dims.size());
        for (auto d : t.dims) h.put<uint64_t>(d);
        h.put<uint32_t>(t.type);
        h.put<uint64_t>(t.offset);
    }
    const uint64_t data_start = (h.b.size() + align - 1) / align * align;
    const uint64_t total = data_start + data_len;
    uint8_t* img = (uint8_t*)std::malloc(total);
    if (!img) {
        g_err = "out of memory allocating " + std::to_string(total) + " bytes";
        return 5;
    }
    std::memset(img, 0, data_start);
    std::memcpy(img, h.b.data(), h.b.size());
    int threads = s->threads > 0 ? s->threads : (int)std::max(1u, std::thread::hardware_concurrency());
    const float sd = s->stddev > 0 ? s->stddev : 0.02f;

    for (size_t ti = 0; ti < ts.size(); ++ti) {
        const Tensor& t = ts[ti];
        uint8_t* dst = img + data_start + t.offset;
        uint64_t pad = (t.nbytes + align - 1) / align * align - t.nbytes;
        std::memset(dst + t.nbytes, 0, pad);
        uint64_t n = 1;
        for (auto d : t.dims) n *= d;
        if (t.ones) {
            for (uint64_t i = 0; i < n; ++i) {
                float one = 1.0f;
                std::memcpy(dst + 4 * i, &one, 4);
            }
            continue;
        }
        const uint64_t key = mix(s->seed * 0x100000001B3ULL + ti + 1);
        if (t.sd != 0.f) {  // small F32 vectors: N(0, sd), or (sd < 0) decay rates -(0.25 + |N(0, 1)|)
            std::vector<float> x(n + (n & 1));
            gen_normal(key, 0, x.size(), t.sd > 0 ? t.sd : 1.0f, x.data());
            for (uint64_t i = 0; i < n; ++i) {
                const float v = t.sd > 0 ? x[i] : -(0.25f + std::fabs(x[i]));
                std::memcpy(dst + 4 * i, &v, 4);
            }
            continue;
        }
        const size_t be = block_elems(t.type), bb = block_bytes(t.type);
        const size_t chunk_blocks = std::max<size_t>(1, 65536 / be);
        const size_t nblocks = n / be;
        const size_t nchunks = (nblocks + chunk_blocks - 1) / chunk_blocks;
        parallel_for(nchunks, threads, [&](size_t c) {
            size_t b0 = c * chunk_blocks, b1 = std::min(nblocks, b0 + chunk_blocks);
            std::vector<float> x((b1 - b0) * be);
            gen_normal(key, b0 * be, x.size(), sd, x.data());
            encode_blocks(t.type, x.data(), b1 - b0, dst + b0 * bb);
        });
    }
    *out = img;
    *out_len = total;
    return 0;
}

void evs_free(uint8_t* p) { std::free(p); }

int evs_write_file(const uint8_t* data, size_t len, const char* path) {
    FILE* f = std::fopen(path, "wb");
    if (!f) {
        g_err = std::string("cannot open ") + path;
        return 5;
    }
    size_t w = std::fwrite(data, 1, len, f);
    int rc = std::fclose(f);
    if (w != len || rc != 0) {
        g_err = std::string("short write to ") + path;
        return 5;
    }
    return 0;
}

}  // extern "C"
