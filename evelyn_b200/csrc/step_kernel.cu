// step_kernel.cu -- the layer stack of one single-sequence decode step
// (Session::step, src/runtime.rs:773-808, between the embedding and the final norm)
// as ONE persistent, cooperative kernel.
//
// Why: at batch 1 every weight byte is read once, so the step is a stream of ~5 GB
// through 36 x 4 matvecs with small dependent kernels in between. As separate
// launches each boundary costs a pipeline drain and refill (the next matvec's CTA can
// only start streaming when the previous CTA has left its SM) plus the input
// staging. Here one CTA per SM lives for the whole step:
//   * the producer warp walks the weight tiles of every matvec phase of every layer
//     in order and keeps the shared-memory ring full across phase boundaries -- it
//     never waits for activations, only for free ring slots, so HBM keeps streaming
//     while the consumers do attention or wait at a barrier;
//   * the 16 consumer warps run the phases in order, separated by grid barriers
//     (the inputs of every phase are complete vectors written by all CTAs):
//       QKV matvec (attn RMSNorm fused) | QK-norm + RoPE + KV append + split-K GQA
//       attention, the last split of each kv head merging its heads | o matvec +
//       residual | gate/up SwiGLU matvec (ffn RMSNorm fused) | down matvec + residual;
//   * besides the ring, the producer keeps an L2 prefetch cursor a few items ahead,
//     so a phase's first tiles are on chip by the time its consumers get there.
// The matvec phases use the same plan, staging and dot-product code as the
// standalone matvec (matvec_core.cuh), so results match it bit for bit; attention
// and the merge restate attention.cu's arithmetic with plain (L2) loads.
//
// Grid barriers need every CTA resident: the kernel is launched cooperatively with
// one CTA per SM. Every wait is bounded (2 s); a CTA that gives up raises a global
// abort flag that the others see at their next barrier, sets the device error flag
// and leaves after its TMA copies have landed.
#include <algorithm>
#include <atomic>
#include <vector>

#include "matvec_core.cuh"

namespace evl {

namespace {

using namespace mv;

enum : uint32_t { PH_MATVEC = 0, PH_ATTN = 1 };

constexpr uint32_t kPrefetchLead = 8;  // items the L2 prefetch cursor runs ahead of the copies

struct AttnPhase {
    RopeArgs rope;  // q/k/v buffers, norms, rope table, KV cache, page table, position
    AttnArgs at;    // heads, nsplit, partials, output, scale
};

struct StepPhase {
    uint32_t kind;
    Plan mv;
    AttnPhase att;
};

struct StepArgs {
    const StepPhase* phases;
    uint32_t nphases;
    uint32_t stages, slot_bytes;
    unsigned long long* bar_count;  // grid barrier arrivals, never reset between launches
    unsigned int* epoch;            // launches so far (bumped by CTA 0 at its end)
    int* abort_g;                   // set by a CTA that gave up; every barrier checks it
    unsigned int* kv_done;          // per kv head: splits finished (reset by the merging CTA)
    int* err;
};

constexpr uint32_t kAttnWarps = kCW;

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Grid barrier among the consumer warps of all CTAs (the producers keep streaming):
// one release-add per CTA on a counter that only grows, then acquire-polls until it
// reaches `target` (this launch's base + barrier index x CTAs). Returns false when
// some CTA aborted or the wait timed out.
__device__ bool grid_sync(const StepArgs& A, unsigned long long target, int tc, volatile int* cta_abort, int* ok_sh) {
    named_sync(kConsumerBarrier, kCW * 32);
    if (tc == 0) {
        bool ok = !*cta_abort;
        asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(A.bar_count) : "memory");
        const uint64_t t0 = global_ns();
        while (ld_acquire_u64(A.bar_count) < target) {
            if (*reinterpret_cast<volatile int*>(A.abort_g)) {
                ok = false;
                break;
            }
            if (global_ns() - t0 > kWaitNs) {
                atomicExch(A.abort_g, 1);
                ok = false;
                break;
            }
        }
        if (*reinterpret_cast<volatile int*>(A.abort_g)) ok = false;
        *ok_sh = ok ? 1 : 0;
    }
    named_sync(kConsumerBarrier, kCW * 32);
    return *reinterpret_cast<volatile int*>(ok_sh) != 0;
}

__device__ __forceinline__ const uint8_t* kv_tile(const KvCacheDev& kv, int32_t page, uint32_t layer, uint32_t which,
                                                  uint32_t head) {
    return (const uint8_t*)kv.pool + (uint64_t)page * kv.page_stride + (uint64_t)layer * kv.layer_stride +
           (uint64_t)head * kv.head_stride + (which ? kv.v_offset : 0);
}

// Positions per split (attention.cu's split_len): whole pages, nsplit splits at most.
__device__ __forceinline__ uint32_t split_len(uint32_t t, uint32_t nsplit, uint32_t ps) {
    const uint32_t per = (t + nsplit - 1) / nsplit;
    return (per + ps - 1) / ps * ps;
}

template <int N>
__device__ __forceinline__ void load_row(const __half* p, float (&o)[N]) {
    if constexpr (N == 4) {
        const uint2 r = __ldcg(reinterpret_cast<const uint2*>(p));
        const float2 x = __half22float2(*reinterpret_cast<const __half2*>(&r.x));
        const float2 y = __half22float2(*reinterpret_cast<const __half2*>(&r.y));
        o[0] = x.x; o[1] = x.y; o[2] = y.x; o[3] = y.y;
    } else {
        const unsigned r = __ldcg(reinterpret_cast<const unsigned*>(p));
        const float2 x = __half22float2(*reinterpret_cast<const __half2*>(&r));
        o[0] = x.x; o[1] = x.y;
    }
}
template <int N>
__device__ __forceinline__ void load_row(const float* p, float (&o)[N]) {
    if constexpr (N == 4) {
        const float4 r = __ldcg(reinterpret_cast<const float4*>(p));
        o[0] = r.x; o[1] = r.y; o[2] = r.z; o[3] = r.w;
    } else {
        const float2 r = __ldcg(reinterpret_cast<const float2*>(p));
        o[0] = r.x; o[1] = r.y;
    }
}

// RMSNorm (src/runtime.rs:193-196) + RoPE (:437-474) of `nvec` head vectors staged in
// vals[nvec][HD] (shared): vectors j < nq use the norm weight wq, the rest wk (null:
// no norm). `tmp` holds the normed values; the rotated result is written back to
// vals. Same arithmetic as qk_norm_rope_append_kernel. Called by all consumer
// threads; ends with a consumer barrier.
template <int HD>
__device__ void norm_rope(const RopeArgs& r, int32_t pos, float* vals, float* tmp, uint32_t nvec, uint32_t nq,
                          const float* wq, const float* wk, float* red, int warp, int lane, int tc) {
    constexpr int NW = HD / 32;  // per vector: warp sums over 32-value slices, summed in order
    for (uint32_t i = warp; i < nvec * NW; i += kCW) {
        const uint32_t j = i / NW, w = i % NW;
        const float v = vals[j * HD + w * 32 + lane];
        const float ss = warp_sum(v * v);
        if (lane == 0) red[i] = ss;
    }
    named_sync(kConsumerBarrier, kCW * 32);
    for (uint32_t i = tc; i < nvec * HD; i += kCW * 32) {
        const uint32_t j = i / HD, d = i % HD;
        const float* nw = j < nq ? wq : wk;
        float v = vals[i];
        if (nw) {
            float ss = 0.f;
            for (int w = 0; w < NW; ++w) ss += red[j * NW + w];
            const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)HD), r.eps)));
            v = __fmul_rn(__fmul_rn(v, inv), nw[d]);
        }
        tmp[i] = v;
    }
    named_sync(kConsumerBarrier, kCW * 32);
    const uint32_t rd = min(r.rope_dim, (uint32_t)HD) & ~1u;
    for (uint32_t i = tc; i < nvec * HD; i += kCW * 32) {
        const uint32_t j = i / HD, d = i % HD;
        const float* vv = tmp + j * HD;
        float o = vv[d];
        if (d < rd) {
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
            const float theta = __fmul_rn((float)pos, r.rope_inv_freq[k]);
            float sn, cs;
            sincosf(theta, &sn, &cs);
            const float x0 = vv[i0], x1 = vv[i1];
            o = second ? __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs)) : __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
        }
        vals[i] = o;
    }
    named_sync(kConsumerBarrier, kCW * 32);
}

// One attention item: kv head `kvh`, split `split` (attention.cu's split kernel with
// plain loads), then -- in the CTA that finishes the last of the kv head's splits --
// the merge of its G heads (attention_combine_kernel's arithmetic). Shared scratch:
// see attn_scratch_bytes.
template <typename KV, int G, int HD>
__device__ void attn_item(const AttnPhase& P, unsigned int* kv_done, int32_t pos, uint32_t kvh, uint32_t split,
                          float* scr, int* flag_sh, int warp, int lane, int tc) {
    constexpr int DPL = HD / 32;
    constexpr int CH = G >= 8 ? 1 : 2;  // positions per warp whose K/V loads are in flight together
    const RopeArgs& r = P.rope;
    const AttnArgs& a = P.at;
    const uint32_t ps = a.kv.page_size, t_all = (uint32_t)pos + 1;
    const uint32_t S = split_len(t_all, a.nsplit, ps), t0 = split * S;
    if (t0 >= t_all) return;  // empty split (uniform over the CTA)
    const uint32_t t1 = min(t_all, t0 + S);
    const uint32_t ns = (t_all + S - 1) / S;  // non-empty splits of every kv head
    const bool last = t1 == t_all;  // this split holds the new position: it appends k, v
    float* vals = scr;                      // [G+1][HD] q heads (and k), normed + rotated in place
    float* tmp = vals + (G + 1) * HD;       // [G+1][HD]
    float* red = tmp + (G + 1) * HD;        // [(G+1) * HD/32]
    float* wm = red + (G + 1) * (HD / 32);  // [warps][G]
    float* wl = wm + kAttnWarps * G;        // [warps][G]
    float* wo = wl + kAttnWarps * G;        // [warps][G][HD]
    const uint32_t nvec = G + (last ? 1 : 0);
    for (uint32_t i = tc; i < nvec * HD; i += kCW * 32) {
        const uint32_t j = i / HD, d = i % HD;
        vals[i] = j < (uint32_t)G ? __ldcg(r.q + (uint64_t)(kvh * G + j) * HD + d) : __ldcg(r.k + (uint64_t)kvh * HD + d);
    }
    named_sync(kConsumerBarrier, kCW * 32);
    norm_rope<HD>(r, pos, vals, tmp, nvec, G, r.q_norm, r.k_norm, red, warp, lane, tc);
    const int32_t* pt = r.page_table;
    if (last) {  // KV append (src/runtime.rs:721-722) at position pos
        const int32_t page = __ldcg(pt + (uint32_t)pos / ps);
        const uint32_t slot = (uint32_t)pos % ps;
        KV* kt = (KV*)kv_tile(a.kv, page, r.layer, 0, kvh);
        KV* vt = (KV*)kv_tile(a.kv, page, r.layer, 1, kvh);
        for (uint32_t d = tc; d < (uint32_t)HD; d += kCW * 32) {
            const float kk = vals[G * HD + d], vv = __ldcg(r.v + (uint64_t)kvh * HD + d);
            if constexpr (sizeof(KV) == 2) {
                kt[slot * HD + d] = __float2half_rn(kk);
                vt[slot * HD + d] = __float2half_rn(vv);
            } else {
                kt[slot * HD + d] = kk;
                vt[slot * HD + d] = vv;
            }
        }
        named_sync(kConsumerBarrier, kCW * 32);  // the appended row is visible to this CTA
    }
    const float* qv = vals + DPL * lane;  // q of head g at qv[g * HD + e], read from shared memory
    float m[G], l[G], o[G][DPL];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int e = 0; e < DPL; ++e) o[g][e] = 0.f;
    }
    for (uint32_t tb = t0 + warp; tb < t1; tb += CH * kAttnWarps) {
        float kf[CH][DPL], vf[CH][DPL];
#pragma unroll
        for (int c = 0; c < CH; ++c) {  // issue the chunk's loads first
            const uint32_t t = tb + c * kAttnWarps;
            if (t < t1) {
                const int32_t page = __ldcg(pt + t / ps);
                const uint64_t off = (uint64_t)(t % ps) * HD + DPL * lane;
                load_row<DPL>(reinterpret_cast<const KV*>(kv_tile(a.kv, page, r.layer, 0, kvh)) + off, kf[c]);
                load_row<DPL>(reinterpret_cast<const KV*>(kv_tile(a.kv, page, r.layer, 1, kvh)) + off, vf[c]);
            }
        }
#pragma unroll
        for (int c = 0; c < CH; ++c) {
            if (tb + c * kAttnWarps >= t1) break;  // uniform over the warp
#pragma unroll
            for (int g = 0; g < G; ++g) {
                float sc = qv[g * HD] * kf[c][0];
#pragma unroll
                for (int e = 1; e < DPL; ++e) sc = fmaf(qv[g * HD + e], kf[c][e], sc);
                sc = warp_sum(sc) * a.scale;
                const float mn = fmaxf(m[g], sc);
                const float alpha = expf(m[g] - mn);  // exp(-inf) = 0 on the first position
                const float w = expf(sc - mn);
                l[g] = l[g] * alpha + w;
#pragma unroll
                for (int e = 0; e < DPL; ++e) o[g][e] = fmaf(w, vf[c][e], o[g][e] * alpha);
                m[g] = mn;
            }
        }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
        if (lane == 0) {
            wm[warp * G + g] = m[g];
            wl[warp * G + g] = l[g];
        }
#pragma unroll
        for (int e = 0; e < DPL; ++e) wo[(warp * G + g) * HD + DPL * lane + e] = o[g][e];
    }
    named_sync(kConsumerBarrier, kCW * 32);
    for (uint32_t i = tc; i < (uint32_t)(G * HD); i += kCW * 32) {
        const uint32_t g = i / HD, dd = i % HD;
        float M = -INFINITY;
        for (uint32_t w = 0; w < kAttnWarps; ++w) M = fmaxf(M, wm[w * G + g]);
        float L = 0.f, O = 0.f;
        for (uint32_t w = 0; w < kAttnWarps; ++w) {
            if (wm[w * G + g] == -INFINITY) continue;
            const float f = expf(wm[w * G + g] - M);
            L += wl[w * G + g] * f;
            O += wo[(w * G + g) * HD + dd] * f;
        }
        const uint32_t head = kvh * G + g;
        float* part = a.part + ((uint64_t)head * a.nsplit + split) * (HD + 2);
        part[dd] = O;
        if (dd == 0) {
            part[HD] = M;
            part[HD + 1] = L;
        }
    }
    // the CTA that completes the kv head's last split merges its heads
    named_sync(kConsumerBarrier, kCW * 32);
    if (tc == 0) {
        __threadfence();  // this split's partials before the count
        const unsigned done = atomicAdd(kv_done + kvh, 1u) + 1u;
        *flag_sh = done == ns;
        if (done == ns) {
            __threadfence();
            atomicExch(kv_done + kvh, 0u);  // ready for the next layer
        }
    }
    named_sync(kConsumerBarrier, kCW * 32);
    if (*reinterpret_cast<volatile int*>(flag_sh)) {
        for (uint32_t i = tc; i < (uint32_t)(G * HD); i += kCW * 32) {
            const uint32_t head = kvh * G + i / HD, d = i % HD;
            const float* part = a.part + (uint64_t)head * a.nsplit * (HD + 2);
            float M = -INFINITY;
            for (uint32_t sp = 0; sp < ns; ++sp) M = fmaxf(M, __ldcg(part + sp * (HD + 2) + HD));
            float L = 0.f, O = 0.f;
            for (uint32_t sp = 0; sp < ns; ++sp) {
                const float* p = part + sp * (HD + 2);
                const float f = expf(__ldcg(p + HD) - M);
                L += __ldcg(p + HD + 1) * f;
                O += __ldcg(p + d) * f;
            }
            a.out[(uint64_t)head * HD + d] = O / L;
        }
    }
    named_sync(kConsumerBarrier, kCW * 32);  // scratch reused by the next item
}

// Not inlined: each (KV, G, HD) instantiation gets its own register allocation instead
// of all of them sharing the kernel body's.
template <typename KV, int G, int HD>
__device__ __noinline__ void attn_phase_t(const AttnPhase& P, unsigned int* kv_done, int32_t pos, float* scr,
                                          int* flag_sh, int warp, int lane, int tc) {
    const uint32_t items = P.at.kv_heads * P.at.nsplit;
    for (uint32_t it = blockIdx.x; it < items; it += gridDim.x)
        attn_item<KV, G, HD>(P, kv_done, pos, it / P.at.nsplit, it % P.at.nsplit, scr, flag_sh, warp, lane, tc);
}

template <int HD>
__device__ void attn_phase_hd(const AttnPhase& P, unsigned int* kv_done, int32_t pos, float* scr, int* flag_sh,
                              int warp, int lane, int tc) {
    const bool f16 = P.at.kv.elem_bytes == 2;
#define EVL_ATTN(G_) (f16 ? attn_phase_t<__half, G_, HD>(P, kv_done, pos, scr, flag_sh, warp, lane, tc) \
                          : attn_phase_t<float, G_, HD>(P, kv_done, pos, scr, flag_sh, warp, lane, tc))
    switch (P.at.heads / P.at.kv_heads) {
        case 1: EVL_ATTN(1); break;
        case 2: EVL_ATTN(2); break;
        case 4: EVL_ATTN(4); break;
        default: EVL_ATTN(8); break;
    }
#undef EVL_ATTN
}

// Producer cursor over this CTA's items of every matvec phase: (phase, row block, group).
struct Cursor {
    uint32_t ph, rb, rb1, g;
};

__device__ bool cursor_first(const StepArgs& A, uint32_t ph0, Cursor& c) {
    for (uint32_t ph = ph0; ph < A.nphases; ++ph) {
        const StepPhase& P = A.phases[ph];
        if (P.kind != PH_MATVEC) continue;
        uint32_t rb0, rb1;
        cta_rows(P.mv, blockIdx.x, gridDim.x, rb0, rb1);
        if (rb0 < rb1) {
            c = Cursor{ph, rb0, rb1, 0};
            return true;
        }
    }
    return false;
}

__device__ bool cursor_next(const StepArgs& A, Cursor& c) {
    if (++c.g < A.phases[c.ph].mv.ngroups) return true;
    c.g = 0;
    if (++c.rb < c.rb1) return true;
    return cursor_first(A, c.ph + 1, c);
}

__device__ void prefetch_item(const StepArgs& A, const Cursor& c) {
    const uint8_t *a, *b;
    uint32_t sb;
    const uint32_t n = item_slabs(A.phases[c.ph].mv, c.rb, c.g, a, b, sb);
    prefetch_l2_bulk(a, sb);
    if (n == 2) prefetch_l2_bulk(b, sb);
}

__global__ void __launch_bounds__(kThreads, 1) step_kernel(const __grid_constant__ StepArgs A) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t full[kMaxStages], empty[kMaxStages];
    __shared__ float red[kCW];
    __shared__ volatile int abort_flag;
    __shared__ int ok_sh, flag_sh;
    __shared__ unsigned long long bar_base;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const Ring ring{smem, full, empty, A.stages, A.slot_bytes};
    uint8_t* xs = smem + A.stages * A.slot_bytes;  // staged input, or attention scratch

    if (tid == 0) {
        abort_flag = 0;
        for (uint32_t s = 0; s < A.stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kCW);
        }
        fence_barrier_init();
        // this launch's barrier counter base: every earlier launch added
        // (nphases - 1) arrivals per CTA
        bar_base = (unsigned long long)*reinterpret_cast<volatile unsigned*>(A.epoch) * (A.nphases - 1) * gridDim.x;
    }
    __syncthreads();

    if (warp == kCW) {  // producer: every matvec phase's tiles, in phase order
        if (lane != 0) return;
        Cursor c, f;
        bool cv = cursor_first(A, 0, c), fv = cv;
        f = c;
        for (uint32_t k = 0; k < kPrefetchLead && fv; ++k) {  // warm L2 ahead of the first copies
            prefetch_item(A, f);
            fv = cursor_next(A, f);
        }
        RingPos rp;
        while (cv) {
            if (rp.n >= A.stages && !wait_or_abort(&empty[rp.s], rp.par ^ 1, &abort_flag)) break;
            if (abort_flag) break;
            issue_item(A.phases[c.ph].mv, ring, c.rb, c.g, rp.s);
            rp.advance(A.stages);
            cv = cursor_next(A, c);
            if (fv) {
                prefetch_item(A, f);
                fv = cursor_next(A, f);
            }
        }
        if (abort_flag) drain_ring(ring, rp.n);
        return;
    }

    // consumers
    const int tc = tid;
    RingPos rp;
    bool ok = true;
    for (uint32_t ph = 0; ph < A.nphases && ok; ++ph) {
        const StepPhase& P = A.phases[ph];
        NormRegs nr;
        if (P.kind == PH_MATVEC) load_norm_regs(P.mv, warp, lane, nr);  // static: before the barrier
        if (ph > 0 && !grid_sync(A, bar_base + (unsigned long long)ph * gridDim.x, tc, &abort_flag, &ok_sh)) {
            ok = false;
            break;
        }
        if (P.kind == PH_MATVEC) {
            uint32_t rb0, rb1;
            cta_rows(P.mv, blockIdx.x, gridDim.x, rb0, rb1);
            prefetch_rows(P.mv, xs, rb0, rb1, (uint32_t)tc);
            const float inv = stage_input(P.mv, xs, warp, lane, red, nr);
            if (!consume_items(P.mv, ring, xs, rb0, rb1, rp, warp, lane, &abort_flag, inv)) ok = false;
        } else {
            const int32_t pos = __ldcg(P.att.rope.pos);
            if (pos < 0 || (uint32_t)pos / P.att.at.kv.page_size >= P.att.at.max_pages) {
                if (blockIdx.x == 0 && tc == 0) atomicExch(A.err, DEV_ERR_POSITION);
                continue;  // every CTA skips alike; the host reports the error after the step
            }
            float* scr = reinterpret_cast<float*>(xs);
            if (P.att.at.head_dim == 128) attn_phase_hd<128>(P.att, A.kv_done, pos, scr, &flag_sh, warp, lane, tc);
            else attn_phase_hd<64>(P.att, A.kv_done, pos, scr, &flag_sh, warp, lane, tc);
        }
    }
    if (!ok) {
        if (tc == 0) {
            atomicExch(A.err, DEV_ERR_WAIT_TIMEOUT);
            atomicExch(A.abort_g, 1);
        }
        abort_flag = 1;  // stops this CTA's producer
    } else if (blockIdx.x == 0 && tc == 0) {
        // every CTA read the epoch before the first barrier, which CTA 0 has passed
        atomicAdd(A.epoch, 1u);
    }
}

// Shared scratch one attention item needs (see attn_item).
size_t attn_scratch_bytes(uint32_t G, uint32_t hd) {
    return 4ull * (2 * (G + 1) * hd + (G + 1) * (hd / 32) + 2 * kAttnWarps * G + (size_t)kAttnWarps * G * hd);
}

std::atomic<int> g_attr_done[64];

}  // namespace

struct StepKernel {
    StepArgs args{};
    StepPhase* d_phases = nullptr;
    void* d_sync = nullptr;  // barrier counter (u64), epoch, abort flag, per-kv-head split counts
    size_t sync_bytes = 0;
    uint32_t smem = 0, grid = 0;
    int device = 0;
};

cudaError_t step_kernel_create(const StepLayer* layers, uint32_t nlayers, int* err, StepKernel** out) {
    *out = nullptr;
    if (!layers || !nlayers || !err) return cudaErrorInvalidValue;
    std::vector<StepPhase> ph;
    uint32_t slot = 0, xbytes = 0, kv_heads = 0;
    for (uint32_t li = 0; li < nlayers; ++li) {
        const StepLayer& L = layers[li];
        const AttnArgs& at = L.attn;
        if (at.batch != 1 || L.rope.batch != 1) return cudaErrorInvalidValue;
        if (at.head_dim != 64 && at.head_dim != 128) return cudaErrorInvalidValue;
        const uint32_t G = at.kv_heads ? at.heads / at.kv_heads : 0;
        if (!at.kv_heads || at.heads % at.kv_heads || (G != 1 && G != 2 && G != 4 && G != 8)) return cudaErrorInvalidValue;
        if (L.rope.pos != at.pos || !at.pos || !at.part || !at.out || !at.nsplit) return cudaErrorInvalidValue;
        xbytes = std::max<uint32_t>(xbytes, (uint32_t)((attn_scratch_bytes(G, at.head_dim) + 127) & ~size_t(127)));
        kv_heads = std::max(kv_heads, at.kv_heads);
        const MatvecArgs* mvs[4] = {&L.qkv, &L.o, &L.gateup, &L.down};
        for (int k = 0; k < 4; ++k) {
            StepPhase p{};
            p.kind = PH_MATVEC;
            cudaError_t e = plan_matvec(*mvs[k], p.mv);
            if (e != cudaSuccess) return e;
            p.mv.pf_cap = 0;  // the producer runs ahead across phases instead
            slot = std::max(slot, p.mv.item_bytes);
            xbytes = std::max(xbytes, p.mv.xbytes);
            ph.push_back(p);
            if (k == 0) {  // attention (with the split merge) between QKV and o
                StepPhase a{};
                a.kind = PH_ATTN;
                a.att.rope = L.rope;
                a.att.at = L.attn;
                ph.push_back(a);
            }
        }
    }
    if (xbytes + 2 * slot > kSmemBudget) return cudaErrorInvalidValue;
    const uint32_t stages = std::min<uint32_t>(kMaxStages, (kSmemBudget - xbytes) / slot);
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    int sms = 0, coop = 0;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev)) != cudaSuccess) return e;
    if (!coop) return cudaErrorNotSupported;
    if (dev >= 0 && dev < 64 && !g_attr_done[dev]) {
        e = cudaFuncSetAttribute(step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBudget);
        if (e != cudaSuccess) return e;
        g_attr_done[dev] = 1;
    }
    const uint32_t smem = stages * slot + xbytes;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, step_kernel, kThreads, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorCooperativeLaunchTooLarge;
    StepKernel* k = new StepKernel();
    k->device = dev;
    k->smem = smem;
    k->grid = (uint32_t)sms;  // one CTA per SM: all resident, as the grid barriers need
    if ((e = cudaMalloc(&k->d_phases, ph.size() * sizeof(StepPhase))) != cudaSuccess ||
        (e = cudaMemcpy(k->d_phases, ph.data(), ph.size() * sizeof(StepPhase), cudaMemcpyHostToDevice)) !=
            cudaSuccess ||
        (e = cudaMalloc(&k->d_sync, k->sync_bytes = 16 + 4 * (size_t)kv_heads)) != cudaSuccess ||
        (e = cudaMemset(k->d_sync, 0, k->sync_bytes)) != cudaSuccess) {
        step_kernel_destroy(k);
        return e;
    }
    k->args.phases = k->d_phases;
    k->args.nphases = (uint32_t)ph.size();
    k->args.stages = stages;
    k->args.slot_bytes = slot;
    uint8_t* sync = static_cast<uint8_t*>(k->d_sync);
    k->args.bar_count = reinterpret_cast<unsigned long long*>(sync);
    k->args.epoch = reinterpret_cast<unsigned int*>(sync + 8);
    k->args.abort_g = reinterpret_cast<int*>(sync + 12);
    k->args.kv_done = reinterpret_cast<unsigned int*>(sync + 16);
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
    return cudaLaunchKernelEx(&cfg, step_kernel, k->args);
}

cudaError_t step_kernel_reset(const StepKernel* k, cudaStream_t s) {
    return cudaMemsetAsync(k->d_sync, 0, k->sync_bytes, s);
}

void step_kernel_destroy(StepKernel* k) {
    if (!k) return;
    if (k->d_phases) cudaFree(k->d_phases);
    if (k->d_sync) cudaFree(k->d_sync);
    delete k;
}

}  // namespace evl
