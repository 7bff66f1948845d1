// attention.cu -- QK-norm + RoPE + KV append, and GQA decode attention over a paged KV cache.
//
// Restates full_attention (src/runtime.rs:663-768) for the non-gated Qwen3/Llama path:
//   * per-head RMSNorm of q and k with shared [head_dim] weights (:700-713),
//   * rotary embedding, split-half NeoX (:437-450) or adjacent pairs (:455-474),
//     theta = pos * base^(-2i/rot_dim) with the base powers computed on the host
//     by powf exactly as the reference does, and accurate sincosf here,
//   * K/V append (:721-722) -- here into 16-position pages of f16 (or f32) rows,
//   * scores q.k * 1/sqrt(hd), max-subtracted softmax, sum w/sum * v (:723-766),
//     with GQA kv_head = head / (heads/kv_heads) (:729).
// The attention is split over the sequence ("flash decoding"): CTA (kv_head, split,
// seq) stages its KV pages in shared memory with TMA bulk copies, serves all
// `group` query heads of the kv head from one read of K/V, keeps an online
// softmax, and writes (o, m, l) partials; a small kernel merges the splits.
// The grid is fixed (nsplit splits); the split length follows the position on the
// device, so one captured CUDA graph serves every step.
#include "common.cuh"
#include "kernels.h"

namespace evl {

namespace {

__device__ __forceinline__ uint8_t* kv_tile(const KvCacheDev& kv, int32_t page, uint32_t layer, uint32_t which,
                                            uint32_t head) {
    return (uint8_t*)kv.pool + kv.k_offset + (uint64_t)page * kv.page_stride + (uint64_t)layer * kv.layer_stride +
           (uint64_t)head * kv.head_stride + (which ? kv.v_offset : 0);
}

// grid (heads + kv_heads, batch), block = head_dim threads (<= 256, multiple of 32)
__global__ void qk_norm_rope_append_kernel(const __grid_constant__ RopeArgs a) {
    const uint32_t hidx = blockIdx.x, b = blockIdx.y, d = threadIdx.x, hd = a.head_dim;
    const bool is_q = hidx < a.heads;
    const uint32_t head = is_q ? hidx : hidx - a.heads;
    __shared__ float vals[256];
    __shared__ float red[8];
    pdl_wait();
    const int32_t pos = a.pos[b];
    const float* src =
        is_q ? a.q + (uint64_t)b * a.heads * hd + head * hd : a.k + (uint64_t)b * a.kv_heads * hd + head * hd;
    float v = src[d];
    const float* nw = is_q ? a.q_norm : a.k_norm;
    if (nw) {  // rms_norm(x, w, eps) over the head (src/runtime.rs:193-196)
        float ss = warp_sum(v * v);
        if ((d & 31) == 0) red[d >> 5] = ss;
        __syncthreads();
        ss = 0.f;
        for (uint32_t w = 0; w < hd / 32; ++w) ss += red[w];
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)hd), a.eps)));
        v = __fmul_rn(__fmul_rn(v, inv), nw[d]);
    }
    vals[d] = v;
    __syncthreads();
    const uint32_t rd = min(a.rope_dim, hd) & ~1u;
    float out = v;
    if (d < rd) {
        uint32_t i, i0, i1;
        bool second;
        if (a.interleaved) {
            i = d / 2;
            i0 = d & ~1u;
            i1 = i0 + 1;
            second = d & 1;
        } else {
            const uint32_t half = rd / 2;
            second = d >= half;
            i = second ? d - half : d;
            i0 = i;
            i1 = i + half;
        }
        const float theta = __fmul_rn((float)pos, a.rope_inv_freq[i]);
        float sn, cs;
        sincosf(theta, &sn, &cs);
        const float x0 = vals[i0], x1 = vals[i1];
        out = second ? __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs)) : __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
    }
    if (is_q) {
        a.q[(uint64_t)b * a.heads * hd + head * hd + d] = out;
    } else {
        const uint32_t pidx = (uint32_t)pos / a.kv.page_size, slot = (uint32_t)pos % a.kv.page_size;
        if (pos < 0 || pidx >= a.max_pages) {
            if (d == 0) atomicExch(a.err, DEV_ERR_POSITION);
            return;
        }
        const int32_t page = a.page_table[(uint64_t)b * a.max_pages + pidx];
        uint8_t* kt = kv_tile(a.kv, page, a.layer, 0, head);
        uint8_t* vt = kv_tile(a.kv, page, a.layer, 1, head);
        const float vv = a.v[(uint64_t)b * a.kv_heads * hd + head * hd + d];
        const uint64_t idx = (uint64_t)slot * hd + d;
        if (a.kv.elem_bytes == 2) {
            reinterpret_cast<__half*>(kt)[idx] = __float2half_rn(out);
            reinterpret_cast<__half*>(vt)[idx] = __float2half_rn(vv);
        } else {
            reinterpret_cast<float*>(kt)[idx] = out;
            reinterpret_cast<float*>(vt)[idx] = vv;
        }
    }
    pdl_launch_dependents();
}

constexpr int kAttnThreads = 128;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kChunkPages = 4;  // pages staged per pipeline stage
// pages per stage for an element type and head size: 4, or 2 for rows of 1 KB (head_dim
// 256 in f32), which keeps the two double-buffered K and V stages within 128 KB
template <typename KV, int HD>
constexpr int chunk_pages() { return HD * (int)sizeof(KV) >= 1024 ? 2 : kChunkPages; }

// N consecutive cache values (N = 2, 4 or 8) as floats
template <int N>
__device__ __forceinline__ void load_vals(const __half* p, float (&o)[N]) {
    static_assert(N == 2 || N == 4 || N == 8, "2, 4 or 8 values per lane");
    if constexpr (N == 8) {
        const uint4 r = *reinterpret_cast<const uint4*>(p);
        const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float2 x = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
            o[2 * i] = x.x;
            o[2 * i + 1] = x.y;
        }
    } else if constexpr (N == 4) {
        const uint2 r = *reinterpret_cast<const uint2*>(p);
        const float2 x = __half22float2(*reinterpret_cast<const __half2*>(&r.x));
        const float2 y = __half22float2(*reinterpret_cast<const __half2*>(&r.y));
        o[0] = x.x; o[1] = x.y; o[2] = y.x; o[3] = y.y;
    } else {
        const float2 x = __half22float2(*reinterpret_cast<const __half2*>(p));
        o[0] = x.x; o[1] = x.y;
    }
}
template <int N>
__device__ __forceinline__ void load_vals(const float* p, float (&o)[N]) {
    static_assert(N == 2 || N == 4 || N == 8, "2, 4 or 8 values per lane");
    if constexpr (N == 8) {
        const float4 r0 = *reinterpret_cast<const float4*>(p), r1 = *reinterpret_cast<const float4*>(p + 4);
        o[0] = r0.x; o[1] = r0.y; o[2] = r0.z; o[3] = r0.w;
        o[4] = r1.x; o[5] = r1.y; o[6] = r1.z; o[7] = r1.w;
    } else if constexpr (N == 4) {
        const float4 r = *reinterpret_cast<const float4*>(p);
        o[0] = r.x; o[1] = r.y; o[2] = r.z; o[3] = r.w;
    } else {
        const float2 r = *reinterpret_cast<const float2*>(p);
        o[0] = r.x; o[1] = r.y;
    }
}

// Positions per split for t attended positions: whole pages, nsplit splits at most.
__device__ __forceinline__ uint32_t split_len(uint32_t t, uint32_t nsplit, uint32_t ps) {
    const uint32_t per = (t + nsplit - 1) / nsplit;
    return (per + ps - 1) / ps * ps;
}

// grid (kv_heads, nsplit, batch); HD/32 dims per lane.
template <typename KV, int G, int HD>
__global__ void __launch_bounds__(kAttnThreads) attention_split_kernel(const __grid_constant__ AttnArgs a) {
    constexpr int DPL = HD / 32;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t bar[2];
    __shared__ float wm[kAttnWarps][G], wl[kAttnWarps][G];
    __shared__ float wo[kAttnWarps][G][HD];

    const uint32_t kvh = blockIdx.x, split = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int CP = chunk_pages<KV, HD>();
    const uint32_t ps = a.kv.page_size;
    const uint32_t tile_bytes = ps * HD * sizeof(KV);  // one (k|v, head) page tile
    const uint32_t stage_bytes = 2 * CP * tile_bytes;
    KV* stage[2] = {reinterpret_cast<KV*>(smem_raw), reinterpret_cast<KV*>(smem_raw + stage_bytes)};

    if (tid == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        fence_barrier_init();
    }
    __syncthreads();
    pdl_wait();
    const uint32_t t_all = (uint32_t)(a.pos ? a.pos[b] : a.pos_value) + 1;
    const uint32_t S = split_len(t_all, a.nsplit, ps);
    const uint32_t t0 = split * S;
    if (t0 >= t_all) return;  // empty split
    const uint32_t t1 = min(t_all, t0 + S);
    const int32_t* pt = a.page_table + (uint64_t)b * a.max_pages;
    const uint32_t chunk_tokens = CP * ps;
    const uint32_t nchunks = (t1 - t0 + chunk_tokens - 1) / chunk_tokens;

    auto issue = [&](uint32_t c, int s) {  // thread 0 only
        const uint32_t c0 = t0 + c * chunk_tokens;
        const uint32_t p0 = c0 / ps, p1 = (min(t1, c0 + chunk_tokens) + ps - 1) / ps;
        mbar_arrive_expect_tx(&bar[s], (p1 - p0) * 2 * tile_bytes);
        for (uint32_t p = p0; p < p1; ++p) {
            const int32_t page = pt[p];
            uint8_t* kd = reinterpret_cast<uint8_t*>(stage[s]) + (p - p0) * tile_bytes;
            uint8_t* vd = kd + CP * tile_bytes;
            tma_load_1d(kd, kv_tile(a.kv, page, a.layer, 0, kvh), tile_bytes, &bar[s]);
            tma_load_1d(vd, kv_tile(a.kv, page, a.layer, 1, kvh), tile_bytes, &bar[s]);
        }
    };
    if (tid == 0) {
        issue(0, 0);
        if (nchunks > 1) issue(1, 1);
    }
    // queries of this kv head's group (normed + rotated), DPL dims per lane
    const float* qb = a.q + (uint64_t)b * a.heads * HD + (uint64_t)kvh * G * HD;
    float qr[G][DPL];
#pragma unroll
    for (int g = 0; g < G; ++g) load_vals<DPL>(qb + g * HD + DPL * lane, qr[g]);
    float m[G], l[G], o[G][DPL];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int e = 0; e < DPL; ++e) o[g][e] = 0.f;
    }
    bool ok = true;
    for (uint32_t c = 0; c < nchunks; ++c) {
        const int s = c & 1;
        const bool got = mbar_wait(&bar[s], (c >> 1) & 1);
        if (__syncthreads_or(!got)) {  // uniform decision: every thread leaves together
            ok = false;
            break;
        }
        const uint32_t c0 = t0 + c * chunk_tokens, c1 = min(t1, c0 + chunk_tokens);
        const uint32_t base = (c0 / ps) * ps;  // first position held by the stage
        const KV* ks = stage[s];
        const KV* vs = stage[s] + CP * ps * HD;
        for (uint32_t t = c0 + warp; t < c1; t += kAttnWarps) {
            const uint32_t r = t - base;
            float kf[DPL], vf[DPL];
            load_vals<DPL>(ks + (uint64_t)r * HD + DPL * lane, kf);
            load_vals<DPL>(vs + (uint64_t)r * HD + DPL * lane, vf);
#pragma unroll
            for (int g = 0; g < G; ++g) {
                float sc = qr[g][0] * kf[0];
#pragma unroll
                for (int e = 1; e < DPL; ++e) sc = fmaf(qr[g][e], kf[e], sc);
                sc = warp_sum(sc) * a.scale;
                const float mn = fmaxf(m[g], sc);
                const float alpha = expf(m[g] - mn);  // exp(-inf) = 0 on the first position
                const float w = expf(sc - mn);
                l[g] = l[g] * alpha + w;
#pragma unroll
                for (int e = 0; e < DPL; ++e) o[g][e] = fmaf(w, vf[e], o[g][e] * alpha);
                m[g] = mn;
            }
        }
        __syncthreads();  // every warp is done with stage s before it is refilled
        if (tid == 0 && c + 2 < nchunks) issue(c + 2, s);
    }
    if (!ok) {  // a TMA copy never completed: report, give the copies in flight a
                // last bounded chance to land, and leave
        if (tid == 0) {
            atomicExch(a.err, DEV_ERR_WAIT_TIMEOUT);
            for (uint32_t c = 0; c < 2 && c < nchunks; ++c) mbar_wait(&bar[c], 0);
        }
        __syncthreads();
        return;
    }
    // merge the warps' online-softmax states
#pragma unroll
    for (int g = 0; g < G; ++g) {
        if (lane == 0) {
            wm[warp][g] = m[g];
            wl[warp][g] = l[g];
        }
#pragma unroll
        for (int e = 0; e < DPL; ++e) wo[warp][g][DPL * lane + e] = o[g][e];
    }
    __syncthreads();
    for (int i = tid; i < G * HD; i += kAttnThreads) {
        const int g = i / HD, dd = i % HD;
        float M = -INFINITY;
        for (int w = 0; w < kAttnWarps; ++w) M = fmaxf(M, wm[w][g]);
        float L = 0.f, O = 0.f;
        for (int w = 0; w < kAttnWarps; ++w) {
            if (wm[w][g] == -INFINITY) continue;
            const float f = expf(wm[w][g] - M);
            L += wl[w][g] * f;
            O += wo[w][g][dd] * f;
        }
        const uint32_t head = kvh * G + g;
        float* part = a.part + (((uint64_t)b * a.heads + head) * a.nsplit + split) * (HD + 2);
        part[dd] = O;
        if (dd == 0) {
            part[HD] = M;
            part[HD + 1] = L;
        }
    }
    pdl_launch_dependents();
}

// grid (heads, batch), block HD: merge the split partials of one head.
template <int HD>
__global__ void attention_combine_kernel(const __grid_constant__ AttnArgs a) {
    const uint32_t head = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
    pdl_wait();
    const uint32_t t = (uint32_t)(a.pos ? a.pos[b] : a.pos_value) + 1;
    const uint32_t S = split_len(t, a.nsplit, a.kv.page_size);
    const uint32_t ns = (t + S - 1) / S;
    const float* part = a.part + ((uint64_t)b * a.heads + head) * a.nsplit * (HD + 2);
    float M = -INFINITY;
    for (uint32_t s = 0; s < ns; ++s) M = fmaxf(M, part[s * (HD + 2) + HD]);
    float L = 0.f, O = 0.f;
    for (uint32_t s = 0; s < ns; ++s) {
        const float* p = part + s * (HD + 2);
        const float f = expf(p[HD] - M);
        L += p[HD + 1] * f;
        O += p[d] * f;
    }
    const uint64_t o = (uint64_t)b * a.heads * HD + head * HD + d;
    a.out[o] = a.gate ? __fmul_rn(O / L, sigmoid_ref(a.gate[o])) : O / L;
    pdl_launch_dependents();
}

cudaLaunchConfig_t make_cfg(dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl, cudaLaunchAttribute* attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cfg;
}

template <typename KV, int G, int HD>
cudaError_t launch_split(const AttnArgs& a, cudaStream_t s, bool pdl) {
    const uint32_t tile = a.kv.page_size * HD * sizeof(KV);
    const size_t smem = 2 * 2 * chunk_pages<KV, HD>() * (size_t)tile;
    cudaError_t e = cudaFuncSetAttribute(attention_split_kernel<KV, G, HD>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    cudaLaunchAttribute at[1];
    auto cfg = make_cfg(dim3(a.kv_heads, a.nsplit, a.batch), dim3(kAttnThreads), smem, s, pdl, at);
    e = cudaLaunchKernelEx(&cfg, attention_split_kernel<KV, G, HD>, a);
    if (e != cudaSuccess) return e;
    auto cfg2 = make_cfg(dim3(a.heads, a.batch), dim3(HD), 0, s, pdl, at);
    return cudaLaunchKernelEx(&cfg2, attention_combine_kernel<HD>, a);
}

template <int HD>
cudaError_t launch_hd(const AttnArgs& a, cudaStream_t s, bool pdl) {
    const bool f16 = a.kv.elem_bytes == 2;
    switch (a.heads / a.kv_heads) {
        case 1: return f16 ? launch_split<__half, 1, HD>(a, s, pdl) : launch_split<float, 1, HD>(a, s, pdl);
        case 2: return f16 ? launch_split<__half, 2, HD>(a, s, pdl) : launch_split<float, 2, HD>(a, s, pdl);
        case 4: return f16 ? launch_split<__half, 4, HD>(a, s, pdl) : launch_split<float, 4, HD>(a, s, pdl);
        case 8: return f16 ? launch_split<__half, 8, HD>(a, s, pdl) : launch_split<float, 8, HD>(a, s, pdl);
        default: return cudaErrorInvalidValue;
    }
}

}  // namespace

cudaError_t launch_qk_norm_rope_append(const RopeArgs& a, cudaStream_t s, bool pdl) {
    if (a.head_dim > 256 || a.head_dim % 32 != 0 || !a.err) return cudaErrorInvalidValue;
    cudaLaunchAttribute at[1];
    auto cfg = make_cfg(dim3(a.heads + a.kv_heads, a.batch), dim3(a.head_dim), 0, s, pdl, at);
    return cudaLaunchKernelEx(&cfg, qk_norm_rope_append_kernel, a);
}

cudaError_t launch_attention(const AttnArgs& a, cudaStream_t s, bool pdl) {
    if (!a.err || a.nsplit == 0 || a.kv_heads == 0 || a.heads % a.kv_heads) return cudaErrorInvalidValue;
    if (a.head_dim == 128) return launch_hd<128>(a, s, pdl);
    if (a.head_dim == 64) return launch_hd<64>(a, s, pdl);
    if (a.head_dim == 256) return launch_hd<256>(a, s, pdl);  // Qwen3.5's full-attention heads
    return cudaErrorInvalidValue;
}

}  // namespace evl
