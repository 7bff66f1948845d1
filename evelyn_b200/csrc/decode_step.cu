// decode_step.cu -- a whole single-sequence decode step (Session::step,
// src/runtime.rs:773-808, from the first layer's RMSNorm to the LM head) as ONE
// persistent kernel whose phases pass their vectors to one another as tagged words.
//
// Why: at batch 1 every weight byte is read once, so a step is a ~5 GB stream through
// 36 x 4 dequant-matvecs with attention in between. As separate launches, every kernel
// boundary costs the slowest CTA's tail, the dependent launch's wait for the whole
// previous grid, and the input staging, with most SMs' HBM streams stopped meanwhile.
// Here one CTA per SM lives for the whole step:
//   * its producer warp walks the weight tiles of every matvec phase of every layer in
//     order and keeps a shared-memory byte ring full across phase boundaries. It never
//     waits for activations, only for ring space, so HBM keeps streaming while the
//     consumers wait for their next input or run attention;
//   * its 16 consumer warps run the phases in order. Every vector a phase hands on
//     (x, q/k/v, the attention partials and output, h) is written as (tag, f32) words
//     in single 8-byte stores, and a reader waits until the words it needs carry this
//     step's tag for that vector. There is no grid barrier: a CTA starts a phase as
//     soon as the rows it reads exist. (Tags: see kernels.h, StepPhaseDesc.)
//   * the matvec phases use matvec_core.cuh's staging, dot products and reductions
//     (bit-identical rows to the standalone matvec); attention is a split-K pass per
//     (kv head, split) CTA over K/V pages copied into shared memory with TMA, merged
//     across splits through the tagged partials.
// With tensor parallelism every phase writes its rows to the same offsets of every
// rank's copy of the vector (all-gather layout), so the stores cross NVLink and no
// collective runs inside the step.
//
// No vector is overwritten while it is still being read: the writer of the next
// version of any vector depends, through the chain of phases, on an output of every
// CTA (on every rank) that reads the current version, produced after that read; and a
// CTA with no rows in a matvec phase does not read that phase's input.
//
// Every wait is bounded (2 s). A CTA that gives up raises the grid abort flag, which
// every other wait checks; the step reports DEV_ERR_WAIT_TIMEOUT and the CTA leaves
// once its TMA copies have landed.
#include <algorithm>
#include <atomic>
#include <cstring>
#include <vector>

#include "dequant.cuh"
#include "matvec_core.cuh"

namespace evl {

namespace {

using namespace mv;

constexpr uint32_t kSlots = kMaxStages;  // ring items in flight (< kRedBufs: see consume_items)
constexpr uint32_t kAlign = 128;         // ring items start on 128-byte boundaries
constexpr uint32_t kMaxG = 8;            // GQA group
constexpr uint32_t kMaxSplit = 32;       // splits per kv head (one lane each in the merge)
constexpr uint32_t kSmemOptin = 232448;  // sm_100 per-block shared memory (static + dynamic)

struct alignas(16) DPhase {
    uint32_t kind;
    uint32_t pad_[3];
    Plan p;
    const uint64_t* xt;
    uint32_t x_tag;
    TaggedOut out[kMaxSegs];
    StepAttn at;
};
static_assert(sizeof(DPhase) % 16 == 0, "phases are copied in 16-byte words");

struct Args {
    const DPhase* ph;
    uint32_t nph, cap, xs_bytes;
    const uint32_t* epoch;
    uint32_t period;
    int* abort_g;
    int* err;
};

// ---------------------------------------------------------------- tagged words
__device__ __forceinline__ void st_word(uint64_t* p, float v, uint32_t tag) {
    const uint64_t w = ((uint64_t)tag << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ uint64_t ld_word(const uint64_t* p) {
    uint64_t w;
    asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
// two words (16-byte aligned); each is one single-copy-atomic 8-byte access
__device__ __forceinline__ void ld_word2(const uint64_t* p, uint64_t& a, uint64_t& b) {
    asm volatile("ld.relaxed.sys.global.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ uint32_t tag_of(uint64_t w) { return (uint32_t)(w >> 32); }
__device__ __forceinline__ float val_of(uint64_t w) { return __uint_as_float((uint32_t)w); }

// The CTA's and the grid's abort flags; a wait gives up when either is set or after
// kWaitNs, raising both.
struct Waiter {
    volatile int* cta;
    int* grid;
};
__device__ __forceinline__ bool give_up(const Waiter& w, uint64_t& t0) {
    if (*w.cta || *reinterpret_cast<volatile int*>(w.grid)) return true;
    const uint64_t t = global_ns();
    if (!t0) {
        t0 = t;
        return false;
    }
    if (t - t0 > kWaitNs) {
        *w.cta = 1;
        atomicExch(w.grid, 1);
        return true;
    }
    return false;
}
// N words (N even, p 16-byte aligned) into v, waiting until each carries `tag`.
template <int N>
__device__ __forceinline__ bool ld_wait(const uint64_t* p, uint32_t tag, float (&v)[N], const Waiter& w) {
    uint64_t r[N];
#pragma unroll
    for (int i = 0; i < N; i += 2) ld_word2(p + i, r[i], r[i + 1]);
    uint64_t t0 = 0;
    bool ok = true;
    for (;;) {
        bool all = true;
#pragma unroll
        for (int i = 0; i < N; ++i) all &= tag_of(r[i]) == tag;
        if (all) break;
        if (give_up(w, t0)) {
            ok = false;
            break;
        }
#pragma unroll
        for (int i = 0; i < N; i += 2)
            if (tag_of(r[i]) != tag || tag_of(r[i + 1]) != tag) ld_word2(p + i, r[i], r[i + 1]);
    }
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = ok ? val_of(r[i]) : 0.f;
    return ok;
}
__device__ __forceinline__ bool ld_wait1(const uint64_t* p, uint32_t tag, float& v, const Waiter& w) {
    uint64_t r = ld_word(p), t0 = 0;
    while (tag_of(r) != tag) {
        if (give_up(w, t0)) {
            v = 0.f;
            return false;
        }
        r = ld_word(p);
    }
    v = val_of(r);
    return true;
}

// Barrier of the consumer threads that also ORs a flag across them: every consumer
// thread takes the same decision from the result.
__device__ __forceinline__ bool consumers_sync_any(bool v) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.or.pred q, %2, %3, p;\n selp.u32 %0, 1, 0, q;\n}"
        : "=r"(r)
        : "r"((uint32_t)v), "r"(kConsumerBarrier), "r"(kCW * 32)
        : "memory");
    return r != 0;
}

// ---------------------------------------------------------------- byte ring
// Items of different sizes go into one circular buffer of `cap` bytes, each at the
// cursor or, when it would pass the end, at 0. Producer and consumers place the same
// sequence of items, so both compute every item's offset the same way.
__device__ __forceinline__ uint32_t ring_place(uint32_t& off, uint32_t bytes, uint32_t cap) {
    const uint32_t sz = (bytes + kAlign - 1) & ~(kAlign - 1);
    if (off + sz > cap) off = 0;
    const uint32_t o = off;
    off += sz;
    return o;
}

// ---------------------------------------------------------------- matvec phases
// NE 8-value eighths of a tagged input, c, c + 512, ... (those below cols / 8), staged by
// one consumer thread: every word (and norm weight) is requested before any is waited
// for, so this costs one round trip. Returns false when the wait gave up.
template <int NE, bool NORM>
__device__ __forceinline__ bool stage_eighths(const Plan& p, const uint64_t* xt, uint32_t tag, uint8_t* xs, uint32_t c,
                                              const Waiter& wt, float& ss) {
    const MatvecArgs& a = p.a;
    const uint32_t ne = a.cols / 8, per = kCW * 32;
    float g[NORM ? NE : 1][8];
    if constexpr (NORM) {
#pragma unroll
        for (int k = 0; k < NE; ++k) {
            if (c + k * per >= ne) continue;
            const float4* gp = reinterpret_cast<const float4*>(a.norm_w + 8 * (c + k * per));
            const float4 t0 = gp[0], t1 = gp[1];
            g[k][0] = t0.x; g[k][1] = t0.y; g[k][2] = t0.z; g[k][3] = t0.w;
            g[k][4] = t1.x; g[k][5] = t1.y; g[k][6] = t1.z; g[k][7] = t1.w;
        }
    }
    // every word of the thread's eighths per round trip; all of them again until each
    // carries the tag
    uint64_t r[NE][8];
    uint64_t t0 = 0;
    bool ok = true;
    for (;;) {
#pragma unroll
        for (int k = 0; k < NE; ++k)
            if (c + k * per < ne)
#pragma unroll
                for (int i = 0; i < 8; i += 2) ld_word2(xt + 8 * (c + k * per) + i, r[k][i], r[k][i + 1]);
        bool all = true;
#pragma unroll
        for (int k = 0; k < NE; ++k)
            if (c + k * per < ne)
#pragma unroll
                for (int i = 0; i < 8; ++i) all &= tag_of(r[k][i]) == tag;
        if (all) break;
        if (give_up(wt, t0)) {
            ok = false;
            break;
        }
    }
    float vv[NE][8];  // the values, so the words' registers free up before the staging
#pragma unroll
    for (int k = 0; k < NE; ++k)
#pragma unroll
        for (int e = 0; e < 8; ++e) vv[k][e] = c + k * per < ne && ok ? val_of(r[k][e]) : 0.f;
#pragma unroll
    for (int k = 0; k < NE; ++k) {
        if ((c & ~31u) + k * per >= ne) continue;  // uniform over the warp
        const bool on = c + k * per < ne;           // uniform per block of four lanes
        float(&v)[8] = vv[k];
        if constexpr (NORM) {
#pragma unroll
            for (int e = 0; e < 8; ++e) ss += v[e] * v[e];
            if (on) {
#pragma unroll
                for (int e = 0; e < 8; ++e) v[e] = __fmul_rn(v[e], g[k][e]);
            }
        }
        stage_eighth(p, xs, c + k * per, on, v);
    }
    return ok;
}

// Input staging from a tagged vector (stage_input of matvec_core.cuh, with each load
// waiting for `tag`), in 8-value eighths: thread c takes eighths c, c + 512, ... Ends
// with a consumer
// barrier; `bad` is the OR over the consumers of a wait that gave up.
__device__ float stage_tagged(const Plan& p, const uint64_t* xt, uint32_t tag, uint8_t* xs, int warp, int lane,
                              float* red, const Waiter& wt, bool& bad) {
    const MatvecArgs& a = p.a;
    const uint32_t K = a.cols, per = kCW * 32;
    const uint32_t c = (uint32_t)(warp * 32 + lane);
    float ss = 0.f;
    bool ok = true;
    // one eighth per round trip with a fused norm (its weights share the registers), two
    // without
    if (a.norm_w) {
        for (uint32_t k = 0; k * per < K / 8; ++k) ok &= stage_eighths<1, true>(p, xt, tag, xs, c + k * per, wt, ss);
    } else {
        for (uint32_t k = 0; k * per < K / 8; k += 2) ok &= stage_eighths<2, false>(p, xt, tag, xs, c + k * per, wt, ss);
    }
    if (a.norm_w) {
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
    }
    if (c < kRedBufs) reinterpret_cast<unsigned*>(xs + p.off_red + kRedBufs * kRedBufBytes)[c] = 0u;
    bad = consumers_sync_any(!ok);
    if (!a.norm_w) return 1.f;
    ss = 0.f;
#pragma unroll
    for (int w = 0; w < kCW; ++w) ss += red[w];
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), a.eps)));
}

// Row slot i of row block rb: the eight super-block warps' partials added in warp
// order, scaled by the norm's 1/rms, the segment's epilogue, and the result written
// to every destination of the segment (finish_row of matvec_core.cuh, tagged).
__device__ __forceinline__ bool finish_tagged(const DPhase& P, const float* rd, uint32_t rb, uint32_t i, float inv,
                                              uint32_t tb, const Waiter& wt) {
    const Plan& p = P.p;
    const int si = seg_of(p, rb);
    const MatvecSeg& sg = p.a.seg[si];
    const TaggedOut& out = P.out[si];
    const uint32_t local = rb - p.rb_begin[si];
    auto sum = [&](uint32_t k) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kSbWarps; ++w) v += rd[w * kRB + k];
        return __fmul_rn(v, inv);
    };
    float v;
    uint32_t row;
    bool ok = true;
    if (sg.epi == EPI_SWIGLU) {
        row = local * kSlabRows + i;
        if (i >= kSlabRows || row >= sg.m.rows) return true;
        v = __fmul_rn(silu(sum(i)), sum(i + kSlabRows));
    } else {
        row = local * kRB + i;
        if (row >= sg.m.rows) return true;
        v = sum(i);
        if (sg.epi == EPI_ADD) {  // x += W x (src/runtime.rs:798-804)
            float res;
            ok = ld_wait1(out.resid + out.row0 + row, tb + out.resid_tag, res, wt);
            v = res + v;
        }
    }
    const uint32_t gr = out.row0 + row;
    for (uint32_t d = 0; d < out.ndst; ++d) {
        if (out.plain[d]) out.plain[d][gr] = v;
        else st_word(out.dst[d] + gr, v, tb + out.tag);
    }
    return ok;
}

// The fields of a matvec phase the consumers' inner loop needs, held in registers: the
// descriptor lives in shared memory, and every barrier or mbarrier operation (a
// "memory" clobber) would otherwise make the compiler load them again per item.
struct MvCtx {
    uint32_t ngroups, last_units, cap, rb1_, rb2_;
    uint32_t type[kMaxSegs], rb0[kMaxSegs], dual[kMaxSegs], rows2[kMaxSegs];
    const float* fscale;
    const float* xsum;
    const int* msum;
};
__device__ __forceinline__ MvCtx mv_ctx(const Plan& p, const uint8_t* xs, uint32_t cap) {
    MvCtx c;
    c.ngroups = p.ngroups;
    c.last_units = p.last_units;
    c.cap = cap;
    c.rb1_ = p.rb_begin[1];
    c.rb2_ = p.rb_begin[2];
#pragma unroll
    for (int s = 0; s < kMaxSegs; ++s) {
        const MatvecSeg& sg = p.a.seg[s];
        c.type[s] = sg.m.type;
        c.rb0[s] = p.rb_begin[s];
        c.dual[s] = sg.epi == EPI_SWIGLU;
        c.rows2[s] = c.dual[s] ? sg.m2.rows : sg.m.rows;
    }
    c.fscale = reinterpret_cast<const float*>(xs + p.off_fscale);
    c.xsum = reinterpret_cast<const float*>(xs + p.off_xsum);
    c.msum = reinterpret_cast<const int*>(xs + p.off_msum);
    return c;
}
__device__ __forceinline__ uint32_t ctx_seg(const MvCtx& c, uint32_t rb) { return rb >= c.rb2_ ? 2 : rb >= c.rb1_ ? 1 : 0; }
// bytes of item (rb, g): the panel of one or two 16-row slabs (item_slabs of matvec_core.cuh)
__device__ __forceinline__ uint32_t ctx_item_bytes(const MvCtx& c, uint32_t si, uint32_t rb, uint32_t g) {
    const uint32_t local = rb - c.rb0[si], U = g + 1 == c.ngroups ? c.last_units : kPanelUnits;
    const uint32_t sbk = c.dual[si] ? local : 2 * local + 1;
    return (sbk * kSlabRows < c.rows2[si] ? 2u : 1u) * U * unit16_bytes(c.type[si]);
}

// One consumer warp's part of a row block of type T out of the byte ring (consume_rows
// of matvec_core.cuh): for every panel, super-block `sbw` of slab `slab`. After an
// abort the warp keeps walking (and releasing) the items without computing, so every
// consumer warp reaches the same barriers.
template <uint32_t T>
__device__ __forceinline__ void rows_from_ring(const MvCtx& c, uint32_t si, uint8_t* base, uint64_t* full,
                                               uint64_t* empty, const uint8_t* xs, uint32_t& n, uint32_t& off,
                                               uint32_t rb, uint32_t slab, uint32_t sbw, const Lane& L, int lane,
                                               volatile int* abort_flag, float& acc0, float& acc1, bool& bad) {
    constexpr uint32_t u16 = T == GGML_Q4_K ? 576u : T == GGML_Q5_K ? 704u : T == GGML_Q6_K ? 840u : 1088u;
    const float wt = ((L.t & 1) ? 65536.f : 1.f) * ((T == GGML_Q4_K && L.part) ? 0.0625f : 1.f);
    for (uint32_t g = 0; g < c.ngroups; ++g, ++n) {
        const uint32_t o = ring_place(off, ctx_item_bytes(c, si, rb, g), c.cap);
        const uint32_t s = n % kSlots;
        if (!bad && !wait_or_abort(&full[s], (n / kSlots) & 1, abort_flag)) bad = true;
        if (!bad) {
            const uint32_t U = g + 1 == c.ngroups ? c.last_units : kPanelUnits, ub = 4 * sbw;
            const uint8_t* q = base + o + slab * U * u16 + ub * u16;
            const uint32_t u0 = g * kPanelUnits + ub;
            if (ub < U) {
                if constexpr (T == GGML_Q4_K) {
                    sb_q4k(q, u0, xs, c.fscale, c.xsum, L, lane, wt, acc0, acc1);
                } else if constexpr (T == GGML_Q5_K) {
                    sb_q5k(q, u0, xs, c.fscale, c.xsum, L, lane, wt, acc0, acc1);
                } else if constexpr (T == GGML_Q6_K) {
                    sb_q6k(q, u0, xs, c.fscale, c.msum, L, lane, wt, acc0, acc1);
                } else {
#pragma unroll
                    for (uint32_t i = 0; i < 4; ++i)
                        if (ub + i < U) unit_q8_0(q + i * 1088, u0 + i, xs, c.fscale, L, lane, wt, acc0, acc1);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
}

// Consumers: the dot products of row blocks [rb0, rb1) and their epilogues
// (consume_items of matvec_core.cuh, over the byte ring, tagged outputs). Returns the
// OR over the consumers of a failed wait.
__device__ bool consume_phase(const DPhase& P, uint8_t* base, uint64_t* full, uint64_t* empty, uint32_t cap,
                              uint8_t* xs, uint32_t rb0, uint32_t rb1, uint32_t& n, uint32_t& off, int warp, int lane,
                              volatile int* abort_flag, float inv, uint32_t tb, const Waiter& wt) {
    const Plan& p = P.p;
    const MvCtx c = mv_ctx(p, xs, cap);
    float* red = reinterpret_cast<float*>(xs + p.off_red);
    unsigned* cnt = reinterpret_cast<unsigned*>(xs + p.off_red + kRedBufs * kRedBufBytes);
    const Lane L = make_lane(lane);
    const uint32_t slab = (uint32_t)warp / kSbWarps, sbw = (uint32_t)warp % kSbWarps;
    const bool deferred = rb1 - rb0 <= kRedBufs;
    bool bad = false;
    for (uint32_t rb = rb0; rb < rb1; ++rb) {
        const uint32_t si = ctx_seg(c, rb);
        float acc0 = 0.f, acc1 = 0.f;
        switch (c.type[si]) {
            case GGML_Q4_K:
                rows_from_ring<GGML_Q4_K>(c, si, base, full, empty, xs, n, off, rb, slab, sbw, L, lane, abort_flag, acc0,
                                          acc1, bad);
                break;
            case GGML_Q5_K:
                rows_from_ring<GGML_Q5_K>(c, si, base, full, empty, xs, n, off, rb, slab, sbw, L, lane, abort_flag, acc0,
                                          acc1, bad);
                break;
            case GGML_Q6_K:
                rows_from_ring<GGML_Q6_K>(c, si, base, full, empty, xs, n, off, rb, slab, sbw, L, lane, abort_flag, acc0,
                                          acc1, bad);
                break;
            default:
                rows_from_ring<GGML_Q8_0>(c, si, base, full, empty, xs, n, off, rb, slab, sbw, L, lane, abort_flag, acc0,
                                          acc1, bad);
        }
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
        const uint32_t buf = (rb - rb0) % kRedBufs;
        float* rd = red + buf * (kSbWarps * kRB);
        if (L.t == 0) {
            rd[sbw * kRB + slab * kSlabRows + L.g8] = acc0;
            rd[sbw * kRB + slab * kSlabRows + L.g8 + 8] = acc1;
        }
        if (deferred) continue;
        __threadfence_block();
        __syncwarp();
        unsigned last = 0;
        if (lane == 0) last = atomicAdd(cnt + buf, 1u) == (unsigned)(kCW - 1);
        last = __shfl_sync(0xffffffffu, last, 0);
        if (!last) continue;
        __threadfence_block();
        if (lane == 0) cnt[buf] = 0u;
        if (!bad && !finish_tagged(P, rd, rb, (uint32_t)lane, inv, tb, wt)) bad = true;
    }
    if (deferred) {
        bad = consumers_sync_any(bad);
        const uint32_t cth = (uint32_t)(warp * 32 + lane);
        if (!bad && cth < (rb1 - rb0) * kRB)
            if (!finish_tagged(P, red + (cth / kRB) * (kSbWarps * kRB), rb0 + cth / kRB, cth % kRB, inv, tb, wt))
                bad = true;
    }
    return consumers_sync_any(bad);
}

// ---------------------------------------------------------------- attention phase
__device__ __forceinline__ const uint8_t* kv_tile(const KvCacheDev& kv, int32_t page, uint32_t layer, uint32_t which,
                                                  uint32_t head) {
    return (const uint8_t*)kv.pool + (uint64_t)page * kv.page_stride + (uint64_t)layer * kv.layer_stride +
           (uint64_t)head * kv.head_stride + (which ? kv.v_offset : 0);
}
// Positions per split: whole pages, nsplit splits at most (as attention.cu).
__host__ __device__ __forceinline__ uint32_t split_len(uint32_t t, uint32_t nsplit, uint32_t ps) {
    const uint32_t per = (t + nsplit - 1) / nsplit;
    return (per + ps - 1) / ps * ps;
}
__host__ __device__ __forceinline__ uint32_t attn_vec_bytes(uint32_t G, uint32_t hd) {
    return ((G + 2) * hd * 4 + kAlign - 1) & ~(kAlign - 1);
}
__host__ __device__ __forceinline__ uint32_t attn_ring_bytes(uint32_t ring_pages, uint32_t hd, uint32_t eb) {
    return ring_pages * 2 * 16 * hd * eb;
}
// Shared scratch of an attention item: the q/k/v vectors, then the page ring, whose
// bytes the per-warp partials [warps][G][hd + 2] reuse after the pass.
__host__ __device__ __forceinline__ uint32_t attn_scratch_bytes(uint32_t G, uint32_t hd, uint32_t eb,
                                                               uint32_t ring_pages) {
    return attn_vec_bytes(G, hd) + std::max<uint32_t>(attn_ring_bytes(ring_pages, hd, eb), kCW * G * (hd + 2) * 4);
}

struct AttnShared {
    float fac[kCW * kMaxG], mm[kMaxG], ml[kMaxG];
    unsigned live[kMaxG];
    float fac2[kMaxSplit * kMaxG], mm2[kMaxG], ml2[kMaxG];
    uint32_t use[2];  // completed uses of the two page-ring barriers (thread 0 advances)
};

// Merge weights of n <= 32 partials [n][G][stride] (o..., m, l) in shared memory: per
// head g the maximum M, fac[k][g] = exp(m_k - M) (-1 for an empty partial) and
// L = sum_k l_k fac[k][g]; warp g takes head g, lane k partial k.
template <int G>
__device__ __forceinline__ void warp_merge_weights(const float* part, uint32_t stride, int n, float* fac, float* mm,
                                                   float* ml, unsigned* live, int warp, int lane) {
    if (warp >= G) return;
    const float* pp = part + (lane * G + warp) * stride + stride - 2;
    const float m = lane < n ? pp[0] : -INFINITY;
    const float M = warp_max(m);
    const bool empty = m == -INFINITY;
    const float f = empty ? 0.f : expf(m - M);
    const float Lsum = warp_sum(empty ? 0.f : pp[1] * f);
    if (lane < n) fac[lane * G + warp] = empty ? -1.f : f;
    const unsigned msk = __ballot_sync(0xffffffffu, !empty);
    if (lane == 0) {
        mm[warp] = M;
        ml[warp] = Lsum;
        live[warp] = msk;
    }
}

// One attention item of layer A.rope.layer: kv head `kvh`, split `split` of the
// positions [0, pos]. Same arithmetic as attention_cluster.cu's scalar loop: per-head
// RMSNorm of q and k (src/runtime.rs:700-713), RoPE (:437-474) with accurate sincosf,
// K/V append (:721-722), online softmax of q.k / sqrt(hd) and the weighted sum of v
// (:723-766), then the split partials merged in split order. Returns false after a
// wait gave up (every consumer thread returns the same).
template <typename KV, int G, int HD>
__device__ __noinline__ bool attn_item(const StepAttn& A, uint32_t kvh, uint32_t split, uint8_t* xs, uint64_t* afull,
                          AttnShared& S, uint32_t tb, const Waiter& wt, int warp, int lane) {
    constexpr int DPL = HD / 32;
    const RopeArgs& r = A.rope;
    const uint32_t ps = r.kv.page_size, tile = ps * HD;
    const int tid = warp * 32 + lane;
    const int32_t pos = __ldcg(r.pos);
    const bool pos_ok = pos >= 0 && (uint32_t)pos / ps < r.max_pages;
    const uint32_t t_all = pos_ok ? (uint32_t)pos + 1 : 1;
    const uint32_t SL = split_len(t_all, A.nsplit, ps), t0 = split * SL;
    const uint32_t ns = (t_all + SL - 1) / SL;  // splits holding positions
    if (split >= ns) return true;               // uniform over the CTA
    const uint32_t t1 = min(t_all, t0 + SL);
    const bool last = t1 == t_all;
    const uint32_t npg = (t1 - t0 + ps - 1) / ps;
    const uint32_t H = A.ring_pages / 2, nch = (npg + H - 1) / H;
    float* vals = reinterpret_cast<float*>(xs);  // [G + 2][HD]: q heads, k, v (normed, rotated)
    KV* ring = reinterpret_cast<KV*>(xs + attn_vec_bytes(G, HD));
    float* wpart = reinterpret_cast<float*>(ring);  // after the pass: [warps][G][HD + 2]
    const int32_t* ptab = r.page_table;

    // the split's first two chunks of K/V pages: they do not depend on this step
    auto issue = [&](uint32_t c) {  // one warp; lane i copies page i of the chunk
        const uint32_t st = c & 1, p0 = c * H, p1 = min(npg, p0 + H);
        if (lane == 0) mbar_arrive_expect_tx(&afull[st], (p1 - p0) * 2 * tile * (uint32_t)sizeof(KV));
        __syncwarp();
        const uint32_t i = p0 + (uint32_t)lane;
        if (i < p1) {
            const int32_t page = __ldcg(ptab + t0 / ps + i);
            KV* slot = ring + (st * H + (i - p0)) * 2 * tile;
            tma_load_1d(slot, kv_tile(r.kv, page, r.layer, 0, kvh), tile * (uint32_t)sizeof(KV), &afull[st]);
            tma_load_1d(slot + tile, kv_tile(r.kv, page, r.layer, 1, kvh), tile * (uint32_t)sizeof(KV), &afull[st]);
        }
    };
    if (warp == kCW - 1 && pos_ok) {
        issue(0);
        if (nch > 1) issue(1);
    }

    // q heads, k, v of this kv head (warp w < G: q head kvh*G + w; G: k; G+1: v)
    bool ok = true;
    if (warp < G + 2) {
        const uint64_t* src = warp < G ? A.q + (uint64_t)(kvh * G + warp) * HD
                                       : (warp == G ? A.k : A.v) + (uint64_t)kvh * HD;
        float val[DPL];
        ok = ld_wait<DPL>(src + DPL * lane, tb + A.qkv_tag, val, wt);
        float* vv = vals + warp * HD;
        if (warp <= G) {
            const float* nw = warp < G ? r.q_norm : r.k_norm;
            if (nw) {  // rms_norm over the head (src/runtime.rs:193-196)
                float ss = 0.f;
#pragma unroll
                for (int e = 0; e < DPL; ++e) ss += val[e] * val[e];
                ss = warp_sum(ss);
                const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)HD), r.eps)));
#pragma unroll
                for (int e = 0; e < DPL; ++e) val[e] = __fmul_rn(__fmul_rn(val[e], inv), nw[DPL * lane + e]);
            }
#pragma unroll
            for (int e = 0; e < DPL; ++e) vv[DPL * lane + e] = val[e];
            __syncwarp();
            const uint32_t rd = min(r.rope_dim, (uint32_t)HD) & ~1u;
#pragma unroll
            for (int e = 0; e < DPL; ++e) {
                const uint32_t d = DPL * lane + e;
                if (d >= rd || !pos_ok) continue;
                uint32_t k, i0, i1;
                bool second;
                if (r.interleaved) {
                    k = d / 2;
                    i0 = d & ~1u;
                    i1 = i0 + 1;
                    second = d & 1;
                } else {
                    const uint32_t half = rd / 2;
                    second = d >= half;
                    k = second ? d - half : d;
                    i0 = k;
                    i1 = k + half;
                }
                float sn, cs;
                sincosf(__fmul_rn((float)pos, r.rope_inv_freq[k]), &sn, &cs);
                const float x0 = vv[i0], x1 = vv[i1];
                val[e] = second ? __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs))
                                : __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
            }
            __syncwarp();
        }
#pragma unroll
        for (int e = 0; e < DPL; ++e) vv[DPL * lane + e] = val[e];
        if (warp >= G && last && pos_ok && ok) {  // KV append at pos (src/runtime.rs:721-722)
            const int32_t page = __ldcg(ptab + (uint32_t)pos / ps);
            KV* dst = (KV*)kv_tile(r.kv, page, r.layer, warp == G ? 0 : 1, kvh) + ((uint32_t)pos % ps) * HD;
#pragma unroll
            for (int e = 0; e < DPL; ++e) {
                if constexpr (sizeof(KV) == 2) dst[DPL * lane + e] = __float2half_rn(val[e]);
                else dst[DPL * lane + e] = val[e];
            }
        }
    }
    if (!pos_ok) {  // outside the cache (the host checks first): zeros, and the step reports it
        if (tid == 0) atomicExch(r.err, DEV_ERR_POSITION);
        for (uint32_t i = tid; i < (uint32_t)(G * HD); i += kCW * 32)
            for (uint32_t d = 0; d < A.out.ndst; ++d)
                st_word(A.out.dst[d] + A.out.row0 + kvh * G * HD + i, 0.f, tb + A.out.tag);
        return !consumers_sync_any(!ok);
    }
    if (consumers_sync_any(!ok)) {
        // the first chunks' copies land before the ring bytes can be reused
        if (tid == 0) {
            for (uint32_t c = 0; c < min(nch, 2u); ++c) mbar_wait(&afull[c & 1], S.use[c & 1] & 1);
            S.use[0] += nch > 0 ? 1 : 0;
            S.use[1] += nch > 1 ? 1 : 0;
        }
        consumers_sync_any(false);
        return false;
    }

    // online softmax over the split's positions, chunk by chunk out of shared memory:
    // one position per warp at a time, lanes over the head dimensions
    float qr[G][DPL], m[G], l[G], o[G][DPL];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int e = 0; e < DPL; ++e) {
            qr[g][e] = vals[g * HD + DPL * lane + e];
            o[g][e] = 0.f;
        }
    }
    const uint32_t pnew = last ? ((uint32_t)pos - t0) / ps : 0xffffffffu;  // page of the new position
    bool bad = false;
    for (uint32_t c = 0; c < nch; ++c) {
        const uint32_t st = c & 1, p0 = c * H, p1 = min(npg, p0 + H);
        const uint32_t par = (S.use[st] + (c >> 1)) & 1;
        if (!bad && !mbar_wait(&afull[st], par)) bad = true;
        if (!bad && pnew >= p0 && pnew < p1 && (warp == 0 || warp == 1)) {
            // the new position's k, v into the split's copy of its page
            KV* tl = ring + ((st * H + pnew - p0) * 2 + warp) * tile + ((uint32_t)pos % ps) * HD;
#pragma unroll
            for (int e = 0; e < DPL; ++e) {
                const float v = vals[(G + warp) * HD + DPL * lane + e];
                if constexpr (sizeof(KV) == 2) tl[DPL * lane + e] = __float2half_rn(v);
                else tl[DPL * lane + e] = v;
            }
        }
        bad = consumers_sync_any(bad);
        if (!bad) {
            const uint32_t tc0 = t0 + p0 * ps, tc1 = min(t1, t0 + p1 * ps);
            for (uint32_t t = tc0 + (uint32_t)warp; t < tc1; t += kCW) {
                const uint32_t li = t - tc0;
                const KV* kp = ring + (st * H + li / ps) * 2 * tile + (li % ps) * HD + DPL * lane;
                float kf[DPL], vf[DPL];
#pragma unroll
                for (int e = 0; e < DPL; ++e) {
                    if constexpr (sizeof(KV) == 2) {
                        kf[e] = __half2float(kp[e]);
                        vf[e] = __half2float(kp[tile + e]);
                    } else {
                        kf[e] = kp[e];
                        vf[e] = kp[tile + e];
                    }
                }
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    float sc = qr[g][0] * kf[0];
#pragma unroll
                    for (int e = 1; e < DPL; ++e) sc = fmaf(qr[g][e], kf[e], sc);
                    sc = warp_sum(sc) * A.scale;
                    const float mn = fmaxf(m[g], sc);
                    const float alpha = expf(m[g] - mn);  // exp(-inf) = 0 on the first position
                    const float w = expf(sc - mn);
                    l[g] = l[g] * alpha + w;
#pragma unroll
                    for (int e = 0; e < DPL; ++e) o[g][e] = fmaf(w, vf[e], o[g][e] * alpha);
                    m[g] = mn;
                }
            }
        }
        bad = consumers_sync_any(bad);  // the stage is read: refill it
        if (!bad && warp == kCW - 1 && c + 2 < nch) issue(c + 2);
    }
    if (tid == 0) {  // the barriers' completed uses (chunks per stage)
        S.use[0] += (nch + 1) / 2;
        S.use[1] += nch / 2;
    }
    if (bad) {
        consumers_sync_any(false);
        return false;
    }
    // this CTA's partial: the warps' (m, l, o) merged in warp order
#pragma unroll
    for (int g = 0; g < G; ++g) {
        float* wp = wpart + (warp * G + g) * (HD + 2);
#pragma unroll
        for (int e = 0; e < DPL; ++e) wp[DPL * lane + e] = o[g][e];
        if (lane == 0) {
            wp[HD] = m[g];
            wp[HD + 1] = l[g];
        }
    }
    consumers_sync_any(false);
    warp_merge_weights<G>(wpart, HD + 2, kCW, S.fac, S.mm, S.ml, S.live, warp, lane);
    consumers_sync_any(false);
    uint64_t* mypart = A.part + ((uint64_t)kvh * A.nsplit + split) * G * (HD + 2);
    for (uint32_t i = tid; i < (uint32_t)(G * HD); i += kCW * 32) {
        const uint32_t g = i / HD, d = i % HD;
        float O = 0.f;
        for (unsigned msk = S.live[g]; msk; msk &= msk - 1) {
            const int w = __ffs(msk) - 1;
            O += wpart[(w * G + g) * (HD + 2) + d] * S.fac[w * G + g];
        }
        st_word(mypart + g * (HD + 2) + d, O, tb + A.part_tag);
        if (d == 0) {
            st_word(mypart + g * (HD + 2) + HD, S.mm[g], tb + A.part_tag);
            st_word(mypart + g * (HD + 2) + HD + 1, S.ml[g], tb + A.part_tag);
        }
    }
    // the merge of the ns splits: this CTA takes values [i0, i1) of the G x HD outputs
    const uint64_t* kpart = A.part + (uint64_t)kvh * A.nsplit * G * (HD + 2);
    ok = true;
    if (warp < G) {  // warp g, lane k: (m, l) of split k, head g
        float ml2[2] = {-INFINITY, 0.f};
        if ((uint32_t)lane < ns) ok = ld_wait<2>(kpart + ((uint64_t)lane * G + warp) * (HD + 2) + HD, tb + A.part_tag, ml2, wt);
        const float M = warp_max(ml2[0]);
        const float f = (uint32_t)lane < ns ? expf(ml2[0] - M) : 0.f;
        const float Ls = warp_sum((uint32_t)lane < ns ? ml2[1] * f : 0.f);
        if ((uint32_t)lane < ns) S.fac2[lane * G + warp] = f;
        if (lane == 0) {
            S.mm2[warp] = M;
            S.ml2[warp] = Ls;
        }
    }
    if (consumers_sync_any(!ok)) return false;
    const uint32_t per = (G * HD + ns - 1) / ns, i0 = split * per, i1 = min((uint32_t)(G * HD), i0 + per);
    // warp w takes outputs i0 + 4w .. +3, then 64 further on, ...; lane k loads split k's
    // partial of each (one round trip for all of them), and the warp adds them in a
    // fixed butterfly order
    for (uint32_t ib = i0 + 4 * (uint32_t)warp; ib < i1; ib += 4 * kCW) {
        uint64_t w4[4];
        uint32_t live = 0;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t i = ib + j;
            w4[j] = 0;
            if (i < i1 && (uint32_t)lane < ns) {
                w4[j] = ld_word(kpart + ((uint64_t)lane * G + i / HD) * (HD + 2) + i % HD);
                live |= 1u << j;
            }
        }
        uint64_t t0w = 0;
        for (;;) {
            bool all = true;
#pragma unroll
            for (int j = 0; j < 4; ++j) all &= !((live >> j) & 1) || tag_of(w4[j]) == tb + A.part_tag;
            if (all) break;
            if (give_up(wt, t0w)) {
                ok = false;
                break;
            }
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (((live >> j) & 1) && tag_of(w4[j]) != tb + A.part_tag)
                    w4[j] = ld_word(kpart + ((uint64_t)lane * G + (ib + j) / HD) * (HD + 2) + (ib + j) % HD);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t i = ib + j;
            if (i >= i1) break;  // uniform over the warp
            const uint32_t g = i / HD;
            const float O = warp_sum((live >> j) & 1 ? val_of(w4[j]) * S.fac2[lane * G + g] : 0.f);
            if (lane == 0) {
                const float res = O / S.ml2[g];
                for (uint32_t dd = 0; dd < A.out.ndst; ++dd)
                    st_word(A.out.dst[dd] + A.out.row0 + kvh * G * HD + i, res, tb + A.out.tag);
            }
        }
    }
    return !consumers_sync_any(!ok);
}

template <int HD>
__device__ bool attn_dispatch(const StepAttn& A, uint32_t kvh, uint32_t split, uint8_t* xs, uint64_t* afull,
                              AttnShared& S, uint32_t tb, const Waiter& wt, int warp, int lane) {
    const bool f16 = A.rope.kv.elem_bytes == 2;
#define EVL_ATTN(G_)                                                                                           \
    return f16 ? attn_item<__half, G_, HD>(A, kvh, split, xs, afull, S, tb, wt, warp, lane)                 \
               : attn_item<float, G_, HD>(A, kvh, split, xs, afull, S, tb, wt, warp, lane)
    switch (A.rope.heads / A.rope.kv_heads) {
        case 1: EVL_ATTN(1);
        case 2: EVL_ATTN(2);
        case 4: EVL_ATTN(4);
        default: EVL_ATTN(8);
    }
#undef EVL_ATTN
}

// ---------------------------------------------------------------- the kernel
__global__ void __launch_bounds__(kThreads, 1) decode_step_kernel(const __grid_constant__ Args A) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
    uint8_t* xs = base + A.cap;
    __shared__ __align__(8) uint64_t full[kSlots], empty[kSlots], afull[2];
    __shared__ __align__(16) DPhase P;
    __shared__ float red[kCW];
    __shared__ volatile int abort_flag;
    __shared__ uint32_t tb_sh;
    __shared__ AttnShared S;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    if (tid == 0) {
        abort_flag = 0;
        for (uint32_t s = 0; s < kSlots; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kCW);
        }
        mbar_init(&afull[0], 1);
        mbar_init(&afull[1], 1);
        S.use[0] = S.use[1] = 0;
        fence_barrier_init();
        tb_sh = *reinterpret_cast<const volatile uint32_t*>(A.epoch) * A.period + 1u;
    }
    __syncthreads();

    if (warp == kCW) {  // producer: every matvec phase's tiles in order, into the byte ring
        if (lane != 0) return;
        const uint64_t pol = l2_evict_first();
        uint32_t n = 0, off = 0, oldest = 0, st[kSlots], en[kSlots];
        for (uint32_t ph = 0; ph < A.nph && !abort_flag; ++ph) {
            const DPhase& D = A.ph[ph];
            if (D.kind != STEP_MATVEC) continue;
            const Plan& p = D.p;
            uint32_t rb0, rb1;
            cta_rows(p, blockIdx.x, gridDim.x, rb0, rb1);
            for (uint32_t rb = rb0; rb < rb1 && !abort_flag; ++rb)
                for (uint32_t g = 0; g < p.ngroups && !abort_flag; ++g) {
                    const uint8_t *a, *b;
                    uint32_t sb;
                    const uint32_t nsl = item_slabs(p, rb, g, a, b, sb);
                    const uint32_t bytes = nsl * sb;
                    uint32_t cur = off;
                    const uint32_t o = ring_place(cur, bytes, A.cap);
                    // free the slot and the ring bytes the item lands on (oldest first)
                    for (;;) {
                        bool clash = n - oldest >= kSlots;
                        for (uint32_t i = oldest; i < n && !clash; ++i)
                            clash = st[i % kSlots] < cur && o < en[i % kSlots];
                        if (!clash) break;
                        if (!wait_or_abort(&empty[oldest % kSlots], (oldest / kSlots) & 1, &abort_flag)) break;
                        ++oldest;
                    }
                    if (abort_flag) break;
                    off = cur;
                    st[n % kSlots] = o;
                    en[n % kSlots] = cur;
                    uint64_t* bar = &full[n % kSlots];
                    mbar_arrive_expect_tx(bar, bytes);
                    tma_load_1d_hint(base + o, a, sb, bar, pol);
                    if (nsl == 2) tma_load_1d_hint(base + o + sb, b, sb, bar, pol);
                    ++n;
                }
        }
        if (abort_flag)  // copies in flight land before the CTA leaves
            for (uint32_t i = oldest; i < n; ++i) mbar_wait(&full[i % kSlots], (i / kSlots) & 1);
        return;
    }

    // consumers
    const Waiter wt{&abort_flag, A.abort_g};
    const uint32_t tb = tb_sh;
    uint32_t n = 0, off = 0;  // ring items consumed, ring cursor
    bool bad = false;
    for (uint32_t ph = 0; ph < A.nph && !bad; ++ph) {
        // this thread's shared-memory writes of the last phase before any TMA copy that
        // the next one issues into the same bytes
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        consumers_sync_any(false);  // every consumer is done with the previous descriptor
        {
            const uint4* src = reinterpret_cast<const uint4*>(A.ph + ph);
            uint4* dst = reinterpret_cast<uint4*>(&P);
            for (uint32_t i = tid; i < sizeof(DPhase) / 16; i += kCW * 32) dst[i] = src[i];
        }
        consumers_sync_any(false);
        if (P.kind == STEP_MATVEC) {
            uint32_t rb0, rb1;
            cta_rows(P.p, blockIdx.x, gridDim.x, rb0, rb1);
            if (rb0 == rb1) continue;  // no rows: this CTA does not read the phase's input
            const float inv = stage_tagged(P.p, P.xt, tb + P.x_tag, xs, warp, lane, red, wt, bad);
            if (bad) break;
            bad = consume_phase(P, base, full, empty, A.cap, xs, rb0, rb1, n, off, warp, lane, &abort_flag, inv, tb, wt);
        } else {
            const StepAttn& at = P.at;
            const uint32_t item = blockIdx.x;
            if (item >= at.rope.kv_heads * at.nsplit) continue;
            const uint32_t kvh = item / at.nsplit, split = item % at.nsplit;
            const bool ok = at.rope.head_dim == 128
                                ? attn_dispatch<128>(at, kvh, split, xs, afull, S, tb, wt, warp, lane)
                                : attn_dispatch<64>(at, kvh, split, xs, afull, S, tb, wt, warp, lane);
            bad = !ok;
        }
    }
    if (bad) {
        abort_flag = 1;  // stops this CTA's producer
        if (tid == 0) {
            atomicExch(A.err, DEV_ERR_WAIT_TIMEOUT);
            atomicExch(A.abort_g, 1);
        }
    }
}

// grid (ceil(cols / 256)): the embedding row of tokens[0] as tagged words, slot 0
__global__ void embed_tagged_kernel(QMatDev m, const int32_t* __restrict__ tokens, uint64_t* xt, const uint32_t* epoch,
                                    uint32_t period, int32_t* err) {
    const uint32_t c = blockIdx.x * blockDim.x + threadIdx.x;
    const int32_t tok = tokens[0];
    if (tok < 0 || (uint32_t)tok >= m.rows) {
        if (c == 0) atomicExch(err, DEV_ERR_TOKEN);
        return;
    }
    if (c < m.cols) st_word(xt + c, dq_repacked_value(m, (uint32_t)tok, c), *epoch * period + 1u);
}

std::atomic<int> g_attr_done[64];

}  // namespace

struct StepKernel {
    Args args{};
    DPhase* d_phases = nullptr;
    int* d_abort = nullptr;
    uint32_t smem = 0, grid = 0;
};

uint32_t step_attn_splits(uint32_t kv_heads, uint32_t max_pages, int sms) {
    if (!kv_heads) return 1;
    uint32_t s = std::min<uint32_t>(kMaxSplit, (uint32_t)sms / kv_heads);
    s = std::min<uint32_t>(s, std::max<uint32_t>(1, max_pages));
    return std::max<uint32_t>(1, s);
}

cudaError_t step_kernel_create(const StepPhaseDesc* phases, uint32_t n, const uint32_t* epoch, uint32_t period,
                               int* err, StepKernel** out) {
    *out = nullptr;
    if (!phases || !n || !epoch || !err) return cudaErrorInvalidValue;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    int sms = 0, coop = 0;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev)) != cudaSuccess) return e;
    if (!coop) return cudaErrorNotSupported;
    std::vector<DPhase> ph(n);
    uint32_t xs = 0, max_item = 0;
    for (uint32_t i = 0; i < n; ++i) {
        const StepPhaseDesc& d = phases[i];
        DPhase& D = ph[i];
        std::memset(static_cast<void*>(&D), 0, sizeof(D));
        D.kind = d.kind;
        if (d.kind == STEP_MATVEC) {
            if (!d.xt || (reinterpret_cast<uintptr_t>(d.xt) & 15)) return cudaErrorInvalidValue;
            MatvecArgs a = d.mv;
            a.x = reinterpret_cast<const float*>(d.xt);  // unused: the plan's checks want a vector
            for (int s = 0; s < a.nseg; ++s) {
                const TaggedOut& o = d.out[s];
                if (!o.ndst || o.ndst > (uint32_t)kMaxPeers) return cudaErrorInvalidValue;
                for (uint32_t k = 0; k < o.ndst; ++k)
                    if (!o.dst[k] && !o.plain[k]) return cudaErrorInvalidValue;
                if (a.seg[s].epi == EPI_ADD && !o.resid) return cudaErrorInvalidValue;
                a.seg[s].y = reinterpret_cast<float*>(o.dst[0] ? (void*)o.dst[0] : (void*)o.plain[0]);
            }
            a.prefetch_bytes = 0;
            for (auto& q : a.prefetch) q = QMatDev{};
            e = plan_matvec(a, D.p);
            if (e != cudaSuccess) return e;
            D.p.pf_cap = 0;
            D.xt = d.xt;
            D.x_tag = d.x_tag;
            for (int s = 0; s < kMaxSegs; ++s) D.out[s] = d.out[s];
            xs = std::max(xs, D.p.xbytes);
            max_item = std::max(max_item, D.p.item_bytes);
        } else if (d.kind == STEP_ATTN) {
            const StepAttn& at = d.at;
            const RopeArgs& r = at.rope;
            if (r.batch != 1 || (r.head_dim != 64 && r.head_dim != 128) || !r.kv_heads || r.heads % r.kv_heads)
                return cudaErrorInvalidValue;
            const uint32_t G = r.heads / r.kv_heads;
            if (G != 1 && G != 2 && G != 4 && G != 8) return cudaErrorInvalidValue;
            if (r.kv.page_size != 16 || (r.kv.elem_bytes != 2 && r.kv.elem_bytes != 4)) return cudaErrorInvalidValue;
            if (!at.nsplit || at.nsplit > kMaxSplit || at.ring_pages < 2 || (at.ring_pages & 1) ||
                at.ring_pages > 64)
                return cudaErrorInvalidValue;
            if (!at.q || !at.k || !at.v || !at.part || !r.pos || !r.page_table || !at.out.ndst ||
                at.out.ndst > (uint32_t)kMaxPeers)
                return cudaErrorInvalidValue;
            if (r.kv_heads * at.nsplit > (uint32_t)sms) return cudaErrorInvalidValue;
            D.at = at;
            xs = std::max(xs, attn_scratch_bytes(G, r.head_dim, r.kv.elem_bytes, at.ring_pages));
        } else {
            return cudaErrorInvalidValue;
        }
    }
    cudaFuncAttributes fa{};
    if ((e = cudaFuncGetAttributes(&fa, decode_step_kernel)) != cudaSuccess) return e;
    xs = (xs + kAlign - 1) & ~(kAlign - 1);
    // all the shared memory a block may have: static + dynamic <= kSmemOptin
    const uint32_t dyn = (kSmemOptin - (uint32_t)fa.sharedSizeBytes - 1024u) & ~(kAlign - 1);
    if (!g_attr_done[dev]) {
        e = cudaFuncSetAttribute(decode_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dyn);
        if (e != cudaSuccess) return e;
        g_attr_done[dev] = 1;
    }
    if (dyn <= xs + 128) return cudaErrorInvalidValue;
    const uint32_t cap = (dyn - xs - 128) & ~(kAlign - 1);
    if (cap < 2 * ((max_item + kAlign - 1) & ~(kAlign - 1))) return cudaErrorInvalidValue;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_step_kernel, kThreads, dyn);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorCooperativeLaunchTooLarge;
    StepKernel* k = new StepKernel();
    k->smem = dyn;
    k->grid = (uint32_t)sms;
    if ((e = cudaMalloc(&k->d_phases, ph.size() * sizeof(DPhase))) != cudaSuccess ||
        (e = cudaMemcpy(k->d_phases, ph.data(), ph.size() * sizeof(DPhase), cudaMemcpyHostToDevice)) !=
            cudaSuccess ||
        (e = cudaMalloc(&k->d_abort, 16)) != cudaSuccess || (e = cudaMemset(k->d_abort, 0, 16)) != cudaSuccess) {
        step_kernel_destroy(k);
        return e;
    }
    k->args.ph = k->d_phases;
    k->args.nph = n;
    k->args.cap = cap;
    k->args.xs_bytes = xs;
    k->args.epoch = epoch;
    k->args.period = period;
    k->args.abort_g = k->d_abort;
    k->args.err = err;
    *out = k;
    return cudaSuccess;
}

cudaError_t step_kernel_launch(const StepKernel* k, cudaStream_t s) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(k->grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = k->smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, decode_step_kernel, k->args);
}

cudaError_t step_kernel_reset(const StepKernel* k, cudaStream_t s) { return cudaMemsetAsync(k->d_abort, 0, 16, s); }

void step_kernel_destroy(StepKernel* k) {
    if (!k) return;
    if (k->d_phases) cudaFree(k->d_phases);
    if (k->d_abort) cudaFree(k->d_abort);
    delete k;
}

cudaError_t launch_embed_tagged(const QMatDev& embed, const int32_t* tokens, uint64_t* xt, const uint32_t* epoch,
                                uint32_t period, int32_t* err, cudaStream_t s) {
    embed_tagged_kernel<<<(embed.cols + 255) / 256, 256, 0, s>>>(embed, tokens, xt, epoch, period, err);
    return cudaGetLastError();
}

}  // namespace evl
