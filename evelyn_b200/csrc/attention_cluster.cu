// attention_cluster.cu -- single-sequence decode attention in one launch: QK-norm,
// RoPE, KV append, split-K GQA attention and the split merge.
//
// Same arithmetic as attention.cu (full_attention, src/runtime.rs:663-768): per-head
// RMSNorm of q and k (:700-713), NeoX or adjacent-pair RoPE (:437-474) with accurate
// sincosf of pos * base^(-2i/rot_dim), K/V append (:721-722) in f16 (or f32) pages,
// max-subtracted softmax of q.k / sqrt(hd) and the weighted sum of v (:723-766).
//
// Layout of the launch: one thread-block cluster of C CTAs per (sequence, kv head);
// CTA `rank` of the cluster owns positions [rank*S, (rank+1)*S) (S whole pages). One
// sequence uses C = 8; a batch the largest C (down to 1, no merge) that keeps about
// two CTAs per SM. Everything that does not come from the QKV matvec is done before
// griddepcontrol.wait: the position and page table are read, the first chunks of the
// split's K and V page tiles are copied into a shared-memory ring with TMA, and the
// norm weights and RoPE sin/cos for the position are loaded. (The position, the page
// table and the cached K/V rows were written by earlier steps or by the host before
// this step's first kernel; the launch before this one has passed its own
// griddepcontrol.wait, so every kernel before it has completed.) After the wait, one
// warp per q head, k and v loads its vector, normalises and rotates it in registers,
// the split that holds the new position appends k and v (to HBM and to its shared
// copy), and the warps run an online softmax over the split's positions entirely out
// of shared memory: on the tensor cores one 16-position page per warp (f16 pages), or
// a batch of 32 / G positions per warp (the scalar loop). The ring streams any number of chunks; a
// warp group per ring stage. The C partials (m, l, o) of a kv head meet through
// distributed shared memory: cluster rank 0 merges them in rank order.
#include <cooperative_groups.h>
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>

#include "common.cuh"
#include "kernels.h"

namespace evl {

namespace {

namespace cg = cooperative_groups;

constexpr int kAW = 16;  // warps per CTA
constexpr uint32_t kMaxSplits = 8;  // CTAs per cluster (portable cluster size)
constexpr uint32_t kMaxRingPages = 24;
constexpr uint32_t kMaxStages = 4;  // ring stages (2 or 4: a warp group per stage)
static_assert(kMaxRingPages <= 32, "one warp copies up to a ring of pages, one per lane");
constexpr uint32_t kSmemCap = 225 * 1024;  // dynamic shared memory (static use stays under 2 KB)

struct ClusterAttn {
    KvTmap tmap;          // the KV pool as [rows][head_dim] f16 (tensor-core path)
    RopeArgs r;
    AttnArgs a;
    uint32_t ring_pages;  // page tiles (K and V) the shared ring holds
    uint32_t stages;      // ring stages (chunks of ring_pages / stages pages)
};

__device__ __forceinline__ const uint8_t* kv_tile(const KvCacheDev& kv, int32_t page, uint32_t layer, uint32_t which,
                                                  uint32_t head) {
    return (const uint8_t*)kv.pool + kv.k_offset + (uint64_t)page * kv.page_stride + (uint64_t)layer * kv.layer_stride +
           (uint64_t)head * kv.head_stride + (which ? kv.v_offset : 0);
}

// Positions per split (attention.cu's split_len): whole pages, nsplit splits at most.
__host__ __device__ __forceinline__ uint32_t split_len(uint32_t t, uint32_t nsplit, uint32_t ps) {
    const uint32_t per = (t + nsplit - 1) / nsplit;
    return (per + ps - 1) / ps * ps;
}

template <int N>
__device__ __forceinline__ void load_kv(const __half* p, float (&o)[N]) {
    if constexpr (N == 4) {
        const uint2 r = *reinterpret_cast<const uint2*>(p);
        const float2 x = __half22float2(*reinterpret_cast<const __half2*>(&r.x));
        const float2 y = __half22float2(*reinterpret_cast<const __half2*>(&r.y));
        o[0] = x.x; o[1] = x.y; o[2] = y.x; o[3] = y.y;
    } else {
        const unsigned r = *reinterpret_cast<const unsigned*>(p);
        const float2 x = __half22float2(*reinterpret_cast<const __half2*>(&r));
        o[0] = x.x; o[1] = x.y;
    }
}
template <int N>
__device__ __forceinline__ void load_kv(const float* p, float (&o)[N]) {  // p: 4 N-byte aligned
    if constexpr (N == 4) {
        const float4 r = *reinterpret_cast<const float4*>(p);
        o[0] = r.x; o[1] = r.y; o[2] = r.z; o[3] = r.w;
    } else if constexpr (N == 2) {
        const float2 r = *reinterpret_cast<const float2*>(p);
        o[0] = r.x; o[1] = r.y;
    } else {
#pragma unroll
        for (int e = 0; e < N; ++e) o[e] = p[e];
    }
}
template <typename KV>
__device__ __forceinline__ KV to_kv(float v) {
    if constexpr (sizeof(KV) == 2) return __float2half_rn(v);
    else return v;
}

// ---- tensor-core path (f16 KV, 16-token pages): page tiles arrive by TMA tensor copies
// in boxes of 16 rows x 64 values (128 B) with the 128-byte swizzle, so that ldmatrix
// reads 8 rows of one 16-byte column without bank conflicts.
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, int32_t x, int32_t y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_addr(dst)),
        "l"(tmap), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}
// byte offset of 16-byte column c (values 8c..8c+7) of row r in a swizzled page tile
__device__ __forceinline__ uint32_t swz(uint32_t r, uint32_t c) {
    return (c >> 3) * 2048u + r * 128u + (((c & 7u) ^ (r & 7u)) << 4);
}
__device__ __forceinline__ void named_sync(uint32_t id, uint32_t n) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
// D (16 x 8) += A (16 x 16 f16, row) * B (16 x 8 f16, col), f32 accumulators
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&h);
}
// f32 pair -> f16 hi pair and f16 residual pair (v = hi + lo to ~22 bits)
__device__ __forceinline__ void split_h2(float a, float b, uint32_t& hi, uint32_t& lo) {
    const __half ha = __float2half_rn(a), hb = __float2half_rn(b);
    hi = pack_h2(__half2float(ha), __half2float(hb));
    lo = pack_h2(a - __half2float(ha), b - __half2float(hb));
}

// Merge weights of n <= 32 partials [n][G][stride] (o..., m, l): per head g the
// maximum M of the partials' m, fac[k][g] = exp(m_k - M) (-1 for an empty partial,
// m = -inf) and L = sum_k l_k fac[k][g]. Warp g (< G) takes head g, lane k partial k;
// the maximum and the sum meet by butterfly shuffles.
template <int G>
__device__ __forceinline__ void merge_weights(const float* part, uint32_t stride, int n, float* fac, float* mm, float* ml,
                                              unsigned* live, int warp, int lane) {
    if (warp >= G) return;
    const float* pp = part + (lane * G + warp) * stride + stride - 2;
    const float m = lane < n ? pp[0] : -INFINITY;
    float M = m;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
    const bool empty = m == -INFINITY;  // also every lane >= n
    const float f = empty ? 0.f : expf(m - M);
    float L = empty ? 0.f : pp[1] * f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
    if (lane < n) fac[lane * G + warp] = empty ? -1.f : f;
    const unsigned msk = __ballot_sync(0xffffffffu, !empty);  // the partials that hold positions
    if (lane == 0) {
        mm[warp] = M;
        ml[warp] = L;
        live[warp] = msk;
    }
}

// The warp partials (written after every warp is done with the ring) reuse the ring's
// bytes when it is large enough, so a larger ring fits.
__host__ __device__ __forceinline__ bool wpart_in_ring(uint32_t ring_pages, uint32_t ps, uint32_t hd, uint32_t eb,
                                                       uint32_t G) {
    return (size_t)ring_pages * 2 * ps * hd * eb >= 4ull * kAW * G * (hd + 2);
}
// Shared-memory bytes of one CTA (ring, q, per-warp vectors, warp partials, CTA partial).
__host__ __device__ __forceinline__ size_t cluster_smem(uint32_t ring_pages, uint32_t ps, uint32_t hd, uint32_t eb,
                                                       uint32_t G) {
    return 1024 + (size_t)ring_pages * 2 * ps * hd * eb + 4ull * G * hd + 4ull * (G + 2) * hd +
           (wpart_in_ring(ring_pages, ps, hd, eb, G) ? 0 : 4ull * kAW * G * (hd + 2)) +
           4ull * kMaxSplits * G * (hd + 2) + 2ull * 32 * hd;  // + q fragments (hd/16 x 32 x 16 B)
}

template <typename KV, int G, int HD, bool MM>
__global__ void __launch_bounds__(kAW * 32, 1) attn_cluster_kernel(const __grid_constant__ ClusterAttn F) {
    constexpr int DPL = HD / 32;
    static_assert(G <= kAW && kAW <= 32 && kMaxSplits <= 32, "one warp per head merges up to 32 partials");
    static_assert(G + 2 < kAW, "the last warp is free to issue the first page copies");
    extern __shared__ __align__(128) uint8_t smem_raw[];
    // the ring starts on a 1024-byte boundary (the swizzle atom of the tensor copies)
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ __align__(8) uint64_t full[kMaxStages];  // the stages of the page ring
    __shared__ int bad_sh, grp_bad[kMaxStages];
    cg::cluster_group cl = cg::this_cluster();
    const RopeArgs& r = F.r;
    const AttnArgs& a = F.a;
    // CTA (sequence sq, kv head kvh, split rank): clusters of C consecutive CTAs
    const uint32_t C = cl.num_blocks(), rank = cl.block_rank();
    const uint32_t sq = blockIdx.x / (a.kv_heads * C), kvh = (blockIdx.x / C) % a.kv_heads;
    const int32_t* ptab = a.page_table + (uint64_t)sq * a.max_pages;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t ps = a.kv.page_size, tile = ps * HD;  // elements of one K (or V) page tile
    const uint32_t lps = 31u - __clz(ps);                // ps is a power of two
    KV* ring = reinterpret_cast<KV*>(smem);                                   // [ring][K|V][ps][HD]
    float* qs = reinterpret_cast<float*>(smem + (size_t)F.ring_pages * 2 * tile * sizeof(KV));  // [G][HD]
    float* vec = qs + G * HD;                                                 // [G+2][HD] per-warp vectors
    const bool wr = wpart_in_ring(F.ring_pages, ps, HD, sizeof(KV), G);
    float* wpart = wr ? reinterpret_cast<float*>(smem) : vec + (G + 2) * HD;  // [warps][G][HD+2]
    float* cpart = vec + (G + 2) * HD + (wr ? 0 : kAW * G * (HD + 2));  // rank 0: [split][G][HD+2] (o, m, l)
    uint4* qfrag = reinterpret_cast<uint4*>(cpart + kMaxSplits * G * (HD + 2));  // [HD/16][lanes]: q hi/lo fragments
    __shared__ float fac[kAW * G], mrg_m[G], mrg_l[G];  // merge weights, maxima and sums
    __shared__ unsigned live[G];                         // per head: the partials holding positions

    if (tid == 0) {
        for (uint32_t i = 0; i < F.stages; ++i) mbar_init(&full[i], 1);
        fence_barrier_init();
        bad_sh = 0;
        for (uint32_t i = 0; i < kMaxStages; ++i) grp_bad[i] = 0;
    }
    __syncthreads();
    pdl_launch_dependents();  // the next kernel's weight streaming may start on idle SMs

    // ---- before the wait: position, pages, static vectors
    // (a.pos null: one caller-given position; r.k null: q is ready and k, v are already in
    // the pages -- the standalone decode attention -- so nothing is normed, rotated or
    // appended)
    const int32_t pos = a.pos ? __ldcg(a.pos + sq) : a.pos_value;
    const bool app = r.k != nullptr;
    const bool pos_ok = pos >= 0 && (uint32_t)pos / ps < a.max_pages;
    const uint32_t t_all = pos_ok ? (uint32_t)pos + 1 : 0;
    const uint32_t S = pos_ok ? split_len(t_all, C, ps) : 0;
    const uint32_t t0 = rank * S, t1 = pos_ok ? min(t_all, t0 + S) : 0;
    const uint32_t npg = t0 < t1 ? (t1 - t0 + ps - 1) / ps : 0;
    const bool valid = pos_ok;  // the same in every thread
    const bool last = valid && npg > 0 && t1 == t_all;  // this split holds the new position
    // The split's pages stream through the ring in chunks of H pages, chunk c into stage
    // c % NS: chunks 0 .. NS-1 are issued now, chunk c + NS once every warp is done with
    // chunk c (NS = 2 for one sequence's few pages per split; a batch's long splits keep
    // NS - 1 chunks in flight behind the one being read).
    const uint32_t NS = F.stages, H = F.ring_pages / NS, nch = (npg + H - 1) / H;
    // One warp issues chunks [c0, c1) (at most the ring's pages, <= 32): lane 0 sets
    // each chunk's byte count, lane i reads the page id of the range's page i and
    // copies it (the page ids arrive in one round trip, not one each).
    auto issue = [&](uint32_t c0, uint32_t c1) {
        const uint32_t p0 = c0 * H, p1 = min(npg, c1 * H);
        if (lane == 0)
            for (uint32_t c = c0; c < c1; ++c)
                mbar_arrive_expect_tx(&full[c % NS], (min(npg, (c + 1) * H) - c * H) * 2 * tile * (uint32_t)sizeof(KV));
        __syncwarp();
        const uint32_t i = p0 + (uint32_t)lane;
        if (i < p1) {
            const uint32_t half = (i / H) % NS;
            const int32_t page = __ldcg(ptab + t0 / ps + i);
            KV* slot = ring + (half * H + i % H) * 2 * tile;
            if constexpr (MM) {  // row coordinates of the K and V tiles in the pool's [rows][HD] view
                const uint8_t* pool = (const uint8_t*)a.kv.pool;
                const int32_t yk = (int32_t)((kv_tile(a.kv, page, r.layer, 0, kvh) - pool) / (HD * 2));
                const int32_t yv = (int32_t)((kv_tile(a.kv, page, r.layer, 1, kvh) - pool) / (HD * 2));
#pragma unroll
                for (int bx = 0; bx < HD / 64; ++bx) {
                    tma_load_2d(reinterpret_cast<uint8_t*>(slot) + bx * 2048, &F.tmap, 64 * bx, yk, &full[half]);
                    tma_load_2d(reinterpret_cast<uint8_t*>(slot + tile) + bx * 2048, &F.tmap, 64 * bx, yv, &full[half]);
                }
            } else {
                tma_load_1d(slot, kv_tile(a.kv, page, r.layer, 0, kvh), tile * sizeof(KV), &full[half]);
                tma_load_1d(slot + tile, kv_tile(a.kv, page, r.layer, 1, kvh), tile * sizeof(KV), &full[half]);
            }
        }
    };
    if (warp == kAW - 1) {  // a warp with no q, k or v vector to prepare
        if (!valid) {
            if (lane == 0) atomicExch(a.err, DEV_ERR_POSITION);
        } else if (nch > 0) {
            issue(0, min(NS, nch));  // the first NS chunks in one round trip
        }
    }
    // warp w < G: q head kvh*G + w; w == G: k; w == G+1: v. Lane dims d = DPL*lane + e.
    const bool vw = warp < (app ? G + 2 : G), normed = warp <= G;
    float nw[DPL], sn[DPL], cs[DPL];
    uint32_t i0[DPL], i1[DPL];
    bool rot[DPL], second[DPL];
    const uint32_t rd = min(r.rope_dim, (uint32_t)HD) & ~1u;
    if (vw && normed) {
        const float* w = warp < G ? r.q_norm : r.k_norm;
#pragma unroll
        for (int e = 0; e < DPL; ++e) {
            const uint32_t d = DPL * lane + e;
            nw[e] = w ? w[d] : 1.f;
            rot[e] = d < rd && pos_ok;
            uint32_t k = 0;
            if (r.interleaved) {
                k = d / 2;
                i0[e] = d & ~1u;
                i1[e] = i0[e] + 1;
                second[e] = d & 1;
            } else {
                const uint32_t half = rd / 2;
                second[e] = d >= half;
                k = second[e] ? d - half : d;
                i0[e] = k;
                i1[e] = k + half;
            }
            sn[e] = 0.f;
            cs[e] = 1.f;
            if (rot[e]) sincosf(__fmul_rn((float)pos, r.rope_inv_freq[k]), &sn[e], &cs[e]);
        }
    }

    // the page the new position's k and v go to (the page table is not written by the
    // previous kernel), so the append does no dependent load after the wait
    const int32_t apage = vw && warp >= G && last ? __ldcg(ptab + (uint32_t)pos / ps) : 0;

    pdl_wait();

    // ---- q, k, v of this kv head: norm + rope in registers
    float val[DPL];
    if (vw) {
        const float* src = warp < G ? r.q + ((uint64_t)sq * a.heads + kvh * G + warp) * HD
                                    : (warp == G ? r.k : r.v) + ((uint64_t)sq * a.kv_heads + kvh) * HD;
#pragma unroll
        for (int e = 0; e < DPL; ++e) val[e] = __ldcg(src + DPL * lane + e);
        if (normed) {
            const float* w = warp < G ? r.q_norm : r.k_norm;
            if (w) {  // rms_norm over the head (src/runtime.rs:193-196)
                float ss = 0.f;
#pragma unroll
                for (int e = 0; e < DPL; ++e) ss += val[e] * val[e];
                ss = warp_sum(ss);
                const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)HD), r.eps)));
#pragma unroll
                for (int e = 0; e < DPL; ++e) val[e] = __fmul_rn(__fmul_rn(val[e], inv), nw[e]);
            }
            float* vv = vec + warp * HD;
#pragma unroll
            for (int e = 0; e < DPL; ++e) vv[DPL * lane + e] = val[e];
            __syncwarp();
#pragma unroll
            for (int e = 0; e < DPL; ++e) {
                if (!rot[e]) continue;
                const float x0 = vv[i0[e]], x1 = vv[i1[e]];
                val[e] = second[e] ? __fadd_rn(__fmul_rn(x0, sn[e]), __fmul_rn(x1, cs[e]))
                                   : __fsub_rn(__fmul_rn(x0, cs[e]), __fmul_rn(x1, sn[e]));
            }
        }
        if (warp < G) {
#pragma unroll
            for (int e = 0; e < DPL; ++e) qs[warp * HD + DPL * lane + e] = val[e];
        } else if (last) {  // KV append at pos (src/runtime.rs:721-722)
            KV* dst = (KV*)kv_tile(a.kv, apage, r.layer, warp == G ? 0 : 1, kvh) + ((uint32_t)pos % ps) * HD;
#pragma unroll
            for (int e = 0; e < DPL; ++e) {
                dst[DPL * lane + e] = to_kv<KV>(val[e]);
                vec[warp * HD + DPL * lane + e] = val[e];  // for the split's own copy (same lane reads it)
            }
        }
    }
    __syncthreads();  // q in shared memory

    // ---- online softmax over this split's positions, chunk by chunk, entirely out of
    // shared memory. Scalar path: one position per warp at a time, lanes over the head
    // dimensions. Tensor-core path: one 16-position page per warp at a time on
    // mma.sync m16n8k16 with the positions as the M dimension and the G <= 8 heads as
    // N: S^T = K Q^T (A = the K page from ldmatrix, B = q), then O^T += V^T P^T (A = the
    // V page from ldmatrix.trans, B = the softmax weights, moved into B-fragment order
    // by shuffles). q and the weights are split into f16 hi + lo, so the products carry
    // ~22 bits like the f32 reference. Lane (g, t) holds positions g, g+8 (and head
    // dims 16i + g, +8 of O^T) of heads 2t, 2t+1.
    // scalar path: q and o over this lane's dimensions; the running maximum and sum of
    // head lane / (32 / G), the same in every lane of that head
    float qr[G][DPL], o[G][DPL], mrun = -INFINITY, lrun = 0.f;
    const uint32_t g8 = (uint32_t)lane >> 2, t4 = (uint32_t)lane & 3;
    float mrow[2] = {-INFINITY, -INFINITY}, lrow[2] = {0.f, 0.f}, oacc[MM ? HD / 16 : 1][4];
    const bool hv0 = 2 * t4 < (uint32_t)G, hv1 = 2 * t4 + 1 < (uint32_t)G;  // real heads of this lane
    if constexpr (MM) {
        // the B fragments of q for every k step, the same for all warps: built once
        // (lane (g, t): head g, dims 16 ks + 2t, +1, +8, +9; heads >= G are zero)
        if (tid < (HD / 16) * 32) {
            const uint32_t ks = tid >> 5, fg = (tid & 31) >> 2, ft = tid & 3;
            uint4 f = make_uint4(0u, 0u, 0u, 0u);
            if (fg < (uint32_t)G) {
                const float* qg = qs + fg * HD + 16 * ks + 2 * ft;
                split_h2(qg[0], qg[1], f.x, f.z);
                split_h2(qg[8], qg[9], f.y, f.w);
            }
            qfrag[tid] = f;  // x, y: hi (b0, b1); z, w: lo
        }
        __syncthreads();
#pragma unroll
        for (int i = 0; i < HD / 16; ++i) oacc[i][0] = oacc[i][1] = oacc[i][2] = oacc[i][3] = 0.f;
    } else {
#pragma unroll
        for (int g = 0; g < G; ++g) {
#pragma unroll
            for (int e = 0; e < DPL; ++e) {
                qr[g][e] = qs[g * HD + DPL * lane + e];
                o[g][e] = 0.f;
            }
        }
    }
    const uint32_t pnew = last && app ? ((uint32_t)pos - t0) / ps : 0xffffffffu;  // page of the new position
    // Chunk c sits in stage c % NS. With 2 stages, warp group grp (half the warps) reads
    // the chunks of stage grp; with 4 stages, two groups of 8 warps read chunks grp,
    // grp + 2, ..., alternating between their two stages, so a group's next chunk is
    // already in flight while it reads the current one (double buffering: the copy
    // latency hides behind the reading of long splits). A group syncs on its own named
    // barrier and refills the stage it has just read, so groups never wait on one another.
    const uint32_t NG = NS >= 4 ? NS / 2 : NS, GW = kAW / NG, grp = (uint32_t)warp / GW, gw = (uint32_t)warp % GW;
    uint32_t cw = grp;  // the next chunk of this group not yet waited for
    for (uint32_t c = grp; valid && c < nch; c += NG) {
        const uint32_t half = c % NS, p0 = c * H, p1 = min(npg, p0 + H);
        cw = c;
        if (!mbar_wait(&full[half], (c / NS) & 1)) {
            atomicExch(a.err, DEV_ERR_WAIT_TIMEOUT);
            bad_sh = 1;
            grp_bad[grp] = 1;
        }
        // the new position's k (group warp 0) and v (group warp 1) into the split's copy
        if (pnew >= p0 && pnew < p1 && gw < 2) {
            const float* src = vec + (G + gw) * HD + DPL * lane;
            KV* tl = ring + ((half * H + pnew - p0) * 2 + gw) * tile;
            const uint32_t rr = (uint32_t)pos % ps;
            if constexpr (MM) {  // swizzled tile: this lane's DPL values are contiguous in one 16-byte column
                const uint32_t d0 = DPL * lane;
                __half* dst = reinterpret_cast<__half*>(reinterpret_cast<uint8_t*>(tl) + swz(rr, d0 / 8) + (d0 % 8) * 2);
#pragma unroll
                for (int e = 0; e < DPL; ++e) dst[e] = __float2half_rn(src[e]);
            } else {
#pragma unroll
                for (int e = 0; e < DPL; ++e) tl[rr * HD + DPL * lane + e] = to_kv<KV>(src[e]);
            }
        }
        named_sync(1 + grp, GW * 32);
        if (grp_bad[grp]) break;  // uniform over the group after its barrier
        const uint32_t tc0 = t0 + p0 * ps, tc1 = min(t1, t0 + p1 * ps);
        if constexpr (MM) {
            for (uint32_t pg = gw; pg < p1 - p0; pg += GW) {
                const uint32_t tu = tc0 + pg * 16;  // first position of the page (live: tu < tc1)
                const uint32_t kb = smem_addr(ring + (half * H + pg) * 2 * tile), vb = kb + tile * 2;
                // S^T: four independent accumulators (q hi / lo x even / odd k step)
                float sa[4][4] = {};
#pragma unroll 2
                for (int ks = 0; ks < HD / 16; ++ks) {
                    uint32_t a0, a1, a2, a3;
                    ldsm_x4(kb + swz(lane & 15, 2 * ks + (lane >> 4)), a0, a1, a2, a3);
                    const uint4 f = qfrag[ks * 32 + lane];
                    mma16816(sa[2 * (ks & 1)], a0, a1, a2, a3, f.x, f.y);
                    mma16816(sa[2 * (ks & 1) + 1], a0, a1, a2, a3, f.z, f.w);
                }
                float sc[4];  // positions g8, g8, g8+8, g8+8 x heads 2t, 2t+1, 2t, 2t+1
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const float v = (sa[0][r] + sa[2][r]) + (sa[1][r] + sa[3][r]);
                    const bool live = (r & 1 ? hv1 : hv0) && tu + g8 + 8 * (r >> 1) < tc1;
                    sc[r] = live ? v * a.scale : -INFINITY;
                }
                float mx[2] = {fmaxf(sc[0], sc[2]), fmaxf(sc[1], sc[3])};
#pragma unroll
                for (int o2 = 4; o2 < 32; o2 <<= 1) {
                    mx[0] = fmaxf(mx[0], __shfl_xor_sync(0xffffffffu, mx[0], o2));
                    mx[1] = fmaxf(mx[1], __shfl_xor_sync(0xffffffffu, mx[1], o2));
                }
                float alpha[2], pw[4];
#pragma unroll
                for (int jh = 0; jh < 2; ++jh) {
                    const bool hv = jh ? hv1 : hv0;
                    const float mn = fmaxf(mrow[jh], mx[jh]);  // finite for a real head: position tu is live
                    alpha[jh] = hv ? expf(mrow[jh] - mn) : 1.f;  // exp(-inf) = 0 on the first page
                    pw[jh] = hv ? expf(sc[jh] - mn) : 0.f;
                    pw[jh + 2] = hv ? expf(sc[jh + 2] - mn) : 0.f;
                    lrow[jh] = lrow[jh] * alpha[jh] + pw[jh] + pw[jh + 2];  // this lane's two positions
                    if (hv) mrow[jh] = mn;
                }
                // P^T as the B fragment: lane (g, t) takes positions 2t, 2t+1 (b0) and
                // 2t+8, 2t+9 (b1) of head g from lanes 8t + g/2 and 8t + 4 + g/2
                const int s1 = 8 * t4 + (g8 >> 1), s2 = s1 + 4;
                const bool odd = g8 & 1;
                const float x0 = __shfl_sync(0xffffffffu, pw[0], s1), x1 = __shfl_sync(0xffffffffu, pw[1], s1);
                const float x2 = __shfl_sync(0xffffffffu, pw[2], s1), x3 = __shfl_sync(0xffffffffu, pw[3], s1);
                const float y0 = __shfl_sync(0xffffffffu, pw[0], s2), y1 = __shfl_sync(0xffffffffu, pw[1], s2);
                const float y2 = __shfl_sync(0xffffffffu, pw[2], s2), y3 = __shfl_sync(0xffffffffu, pw[3], s2);
                uint32_t bh0, bl0, bh1, bl1;
                split_h2(odd ? x1 : x0, odd ? y1 : y0, bh0, bl0);  // positions 2t, 2t+1
                split_h2(odd ? x3 : x2, odd ? y3 : y2, bh1, bl1);  // positions 2t+8, 2t+9
#pragma unroll
                for (int i = 0; i < HD / 16; ++i) {  // O^T rows 16i .. 16i+15 (head dims)
                    uint32_t a0, a1, a2, a3;
                    ldsm_x4_t(vb + swz((lane & 7) + 8 * (lane >> 4), 2 * i + ((lane >> 3) & 1)), a0, a1, a2, a3);
                    oacc[i][0] *= alpha[0];
                    oacc[i][1] *= alpha[1];
                    oacc[i][2] *= alpha[0];
                    oacc[i][3] *= alpha[1];
                    mma16816(oacc[i], a0, a1, a2, a3, bh0, bh1);
                    mma16816(oacc[i], a0, a1, a2, a3, bl0, bl1);
                }
            }
        } else {
            // a batch of P = 32 / G consecutive positions per warp: the G x P dot
            // products are summed over the lanes' head dimensions by one reduce-scatter,
            // after which lane j = g * P + p holds the score of head g at position p, so
            // the softmax bookkeeping (maximum, two exps, sum) runs once per lane and
            // batch; the weights return to the dimension lanes by shuffles for the V sum
            constexpr int P = 32 / G;
            // row li of the chunk: K at li * HD + (li / ps) * tile past the chunk's first
            // K tile (page tiles K, V alternate), V one tile further
            const KV* kc = ring + half * H * 2 * tile + DPL * lane;
            const uint32_t nb = (tc1 - tc0 + P - 1) / P;
            for (uint32_t bt = gw; bt < nb; bt += GW) {
                const uint32_t tb = tc0 + bt * P;  // live: tb < tc1
                float dot[32];
#pragma unroll
                for (int p = 0; p < P; ++p) {
                    float kf[DPL];
                    const uint32_t li = bt * P + p;
                    if (tb + p < tc1) {
                        load_kv<DPL>(kc + li * HD + (li >> lps) * tile, kf);
                    } else {
#pragma unroll
                        for (int e = 0; e < DPL; ++e) kf[e] = 0.f;
                    }
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        float sc = qr[g][0] * kf[0];
#pragma unroll
                        for (int e = 1; e < DPL; ++e) sc = fmaf(qr[g][e], kf[e], sc);
                        dot[g * P + p] = sc;
                    }
                }
                // reduce-scatter: at offset o2 a lane keeps the half of its sums whose index
                // bit o2 matches its own lane bit and adds its partner's copy of that half
#pragma unroll
                for (int o2 = 16; o2 >= 1; o2 >>= 1) {
                    const bool up = (lane & o2) != 0;
#pragma unroll
                    for (int i = 0; i < o2; ++i) {
                        const float send = up ? dot[i] : dot[i + o2];
                        const float keep = up ? dot[i + o2] : dot[i];
                        dot[i] = keep + __shfl_xor_sync(0xffffffffu, send, o2);
                    }
                }
                const float sc = tb + (uint32_t)lane % P < tc1 ? dot[0] * a.scale : -INFINITY;
                float bm = sc;
#pragma unroll
                for (int o2 = 1; o2 < P; o2 <<= 1) bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, o2));
                const float mn = fmaxf(mrun, bm);     // finite: position tb is live
                const float alpha = expf(mrun - mn);  // exp(-inf) = 0 on the first batch
                const float w = expf(sc - mn);
                float ws = w;
#pragma unroll
                for (int o2 = 1; o2 < P; o2 <<= 1) ws += __shfl_xor_sync(0xffffffffu, ws, o2);
                lrun = lrun * alpha + ws;
                mrun = mn;
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const float ag = __shfl_sync(0xffffffffu, alpha, g * P);
#pragma unroll
                    for (int e = 0; e < DPL; ++e) o[g][e] *= ag;
                }
#pragma unroll
                for (int p = 0; p < P; ++p) {
                    if (tb + p >= tc1) break;  // uniform over the warp
                    const uint32_t li = bt * P + p;
                    float vf[DPL];
                    load_kv<DPL>(kc + tile + li * HD + (li >> lps) * tile, vf);
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        const float wg = __shfl_sync(0xffffffffu, w, g * P + p);
#pragma unroll
                        for (int e = 0; e < DPL; ++e) o[g][e] = fmaf(wg, vf[e], o[g][e]);
                    }
                }
            }
        }
        named_sync(1 + grp, GW * 32);  // the group is done with its stage of the ring
        cw = c + NG;
        if (gw == 0 && c + NS < nch) issue(c + NS, c + NS + 1);
    }
    // a wait of this group gave up: the copies of its chunk cw and (double buffering) of
    // its next chunk may still land; let them before leaving
    if (grp_bad[grp]) {
        if (cw < nch) mbar_wait(&full[cw % NS], (cw / NS) & 1);
        if (NS > NG && cw + NG < nch) mbar_wait(&full[(cw + NG) % NS], ((cw + NG) / NS) & 1);
    }
    __syncthreads();
    if constexpr (MM) {
#pragma unroll
        for (int o2 = 4; o2 < 32; o2 <<= 1) {  // the lane partial sums of a head over its 8 row lanes
            lrow[0] += __shfl_xor_sync(0xffffffffu, lrow[0], o2);
            lrow[1] += __shfl_xor_sync(0xffffffffu, lrow[1], o2);
        }
#pragma unroll
        for (int jh = 0; jh < 2; ++jh) {
            if (!(jh ? hv1 : hv0)) continue;
            float* wp = wpart + (warp * G + 2 * t4 + jh) * (HD + 2);
#pragma unroll
            for (int i = 0; i < HD / 16; ++i) {
                wp[16 * i + g8] = oacc[i][jh];
                wp[16 * i + g8 + 8] = oacc[i][2 + jh];
            }
            if (g8 == 0) {
                wp[HD] = mrow[jh];
                wp[HD + 1] = lrow[jh];
            }
        }
    } else {
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float* wp = wpart + (warp * G + g) * (HD + 2);
#pragma unroll
            for (int e = 0; e < DPL; ++e) wp[DPL * lane + e] = o[g][e];
            const float mg = __shfl_sync(0xffffffffu, mrun, g * (32 / G));
            const float lg = __shfl_sync(0xffffffffu, lrun, g * (32 / G));
            if (lane == 0) {
                wp[HD] = mg;
                wp[HD + 1] = lg;
            }
        }
    }
    __syncthreads();
    // ---- this CTA's partial: the warps merged in order (attention_combine_kernel's
    // arithmetic). The weight exp(m_w - M) of a (warp, head) is the same for every
    // dimension, so G threads compute them once; the partial goes straight into rank
    // 0's shared memory (slot `rank`), which then merges the splits from its own copy.
    merge_weights<G>(wpart, HD + 2, kAW, fac, mrg_m, mrg_l, live, warp, lane);
    __syncthreads();
    float* dst = cl.map_shared_rank(cpart, 0) + rank * G * (HD + 2);
    for (uint32_t i = tid; i < (uint32_t)(G * HD); i += kAW * 32) {
        const uint32_t g = i / HD, d = i % HD;
        float O = 0.f;
        for (unsigned msk = live[g]; msk; msk &= msk - 1) {  // the warps that read positions, in order
            const int w = __ffs(msk) - 1;
            O += wpart[(w * G + g) * (HD + 2) + d] * fac[w * G + g];
        }
        dst[g * (HD + 2) + d] = O;
        if (d == 0) {
            dst[g * (HD + 2) + HD] = mrg_m[g];
            dst[g * (HD + 2) + HD + 1] = mrg_l[g];
        }
    }
    cl.sync();  // every CTA's partial is in rank 0's shared memory
    if (rank != 0) return;
    merge_weights<G>(cpart, HD + 2, (int)C, fac, mrg_m, mrg_l, live, warp, lane);
    __syncthreads();
    for (uint32_t i = tid; i < (uint32_t)(G * HD); i += kAW * 32) {
        const uint32_t g = i / HD, d = i % HD;
        float O = 0.f;
        for (unsigned msk = live[g]; msk; msk &= msk - 1) {
            const int c = __ffs(msk) - 1;
            O += cpart[(c * G + g) * (HD + 2) + d] * fac[c * G + g];
        }
        if (valid && !bad_sh) {
            const uint64_t o = ((uint64_t)sq * a.heads + kvh * G + g) * HD + d;
            const float r = O / mrg_l[g];
            a.out[o] = a.gate ? __fmul_rn(r, sigmoid_ref(a.gate[o])) : r;
        }
    }
}

template <typename KV, int G, int HD, bool MM>
cudaError_t launch_t(const ClusterAttn& F, cudaStream_t s, bool pdl) {
    const size_t smem = cluster_smem(F.ring_pages, F.a.kv.page_size, HD, sizeof(KV), G);
    static std::atomic<int> attr_done[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_done[dev]) {
        cudaError_t e = cudaFuncSetAttribute(attn_cluster_kernel<KV, G, HD, MM>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemCap);
        if (e != cudaSuccess) return e;
        attr_done[dev] = 1;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(F.a.kv_heads * F.a.nsplit * F.a.batch);
    cfg.blockDim = dim3(kAW * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = F.a.nsplit;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, attn_cluster_kernel<KV, G, HD, MM>, F);
}

template <typename KV, int HD, bool MM>
cudaError_t launch_hd(const ClusterAttn& F, uint32_t G, cudaStream_t s, bool pdl) {
    switch (G) {
        case 1: return launch_t<KV, 1, HD, MM>(F, s, pdl);
        case 2: return launch_t<KV, 2, HD, MM>(F, s, pdl);
        case 4: return launch_t<KV, 4, HD, MM>(F, s, pdl);
        default: return launch_t<KV, 8, HD, MM>(F, s, pdl);
    }
}

}  // namespace

uint32_t attention_cluster_pages(uint32_t max_pages, uint32_t nsplit, uint32_t page_size, uint32_t head_dim,
                                 uint32_t elem_bytes, uint32_t group, uint32_t cap) {
    if (!nsplit || nsplit > 8 || (nsplit & (nsplit - 1)) || !page_size) return 0;
    if (head_dim != 64 && head_dim != 128) return 0;
    if (group != 1 && group != 2 && group != 4 && group != 8) return 0;
    if (elem_bytes != 2 && elem_bytes != 4) return 0;
    if (page_size & (page_size - 1)) return 0;  // the loops address rows by shifts
    // a split holds at most ceil(ceil(t / nsplit) / page) pages; longer splits stream
    // through the ring, which holds an even number of pages (two halves)
    uint32_t ring = std::min<uint32_t>(std::min<uint32_t>(kMaxRingPages, std::max<uint32_t>(cap, 2) & ~1u),
                                       ((max_pages + nsplit - 1) / nsplit + 2) & ~1u);
    while (ring > 2 && cluster_smem(ring, page_size, head_dim, elem_bytes, group) > kSmemCap) ring -= 2;
    return cluster_smem(ring, page_size, head_dim, elem_bytes, group) <= kSmemCap ? ring : 0;
}

bool make_kv_tmap(const void* pool, uint64_t bytes, uint32_t head_dim, KvTmap* out) {
    static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
    static std::atomic<int> tried{0};
    if (!tried.exchange(1)) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    if (!encode || !pool || (head_dim != 64 && head_dim != 128) || (reinterpret_cast<uintptr_t>(pool) & 127))
        return false;
    // the pool as [rows][head_dim] f16 rows; a box is 16 rows x 64 values (128 B), swizzled
    const cuuint64_t dims[2] = {head_dim, bytes / (2ull * head_dim)};
    const cuuint64_t strides[1] = {2ull * head_dim};
    const cuuint32_t box[2] = {64, 16};
    const cuuint32_t estr[2] = {1, 1};
    static_assert(sizeof(KvTmap) == sizeof(CUtensorMap), "tensor map size");
    return encode(reinterpret_cast<CUtensorMap*>(out), CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(pool), dims,
                  strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t launch_attention_cluster(const RopeArgs& r, const AttnArgs& a, uint32_t ring_pages, uint32_t stages,
                                     cudaStream_t s, bool pdl, const KvTmap* tmap) {
    const bool standalone = !a.pos && !r.pos && !r.k && !r.v && a.batch == 1;  // q ready, k and v in the pages
    if (!a.batch || r.batch != a.batch || !a.out || (!standalone && (!a.pos || r.pos != a.pos)) || ring_pages < 2 ||
        (ring_pages & 1) ||
        a.nsplit < 1 || a.nsplit > kMaxSplits || stages < 2 || stages > kMaxStages || kAW % stages ||
        ring_pages % stages)
        return cudaErrorInvalidValue;
    const uint32_t G = a.kv_heads ? a.heads / a.kv_heads : 0;
    if (!a.kv_heads || a.heads % a.kv_heads ||
        attention_cluster_pages(1, a.nsplit, a.kv.page_size, a.head_dim, a.kv.elem_bytes, G, 2) == 0)
        return cudaErrorInvalidValue;
    if (cluster_smem(ring_pages, a.kv.page_size, a.head_dim, a.kv.elem_bytes, G) > kSmemCap)
        return cudaErrorInvalidValue;
    ClusterAttn F;
    F.r = r;
    F.a = a;
    F.ring_pages = ring_pages;
    F.stages = stages;
    const bool f16 = a.kv.elem_bytes == 2;
    // tensor cores for f16 pages of 16 rows whose tiles the tensor map addresses (row
    // strides and offsets multiples of one head_dim row)
    const uint64_t row = 2ull * a.head_dim;
    const bool mm = tmap && f16 && a.kv.page_size == 16 && a.kv.page_stride % row == 0 && a.kv.layer_stride % row == 0 &&
                    a.kv.head_stride % row == 0 && a.kv.v_offset % (int64_t)row == 0;
    if (mm) {
        F.tmap = *tmap;
        return a.head_dim == 128 ? launch_hd<__half, 128, true>(F, G, s, pdl) : launch_hd<__half, 64, true>(F, G, s, pdl);
    }
    if (a.head_dim == 128)
        return f16 ? launch_hd<__half, 128, false>(F, G, s, pdl) : launch_hd<float, 128, false>(F, G, s, pdl);
    return f16 ? launch_hd<__half, 64, false>(F, G, s, pdl) : launch_hd<float, 64, false>(F, G, s, pdl);
}

}  // namespace evl
