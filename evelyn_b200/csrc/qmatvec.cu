// qmatvec.cu -- dequant-fused matrix-vector products for Q4_K, Q6_K and Q8_0.
//
// Replaces QMatrix::matvec (src/runtime.rs:72-88), which dequantises every row into
// a fresh Vec<f32> and sums sequentially. Here the quantised blocks stream from HBM
// with 128-bit non-allocating loads (the unit-interleaved layout of common.cuh), are
// unpacked in registers with integer byte permutes (2^23 magic-number conversion:
// exact for 0..255), and meet the input vector, which every CTA stages once in
// shared memory in the unit order of the matrix type (64 values + 4 pad floats per
// unit, so the 32 lanes of a warp hit distinct banks). Each warp owns NR rows at a
// time and reuses each x register NR times; f32 pairs go through the sm_100 packed
// FFMA2/FADD2 pipes. The block scales are applied once per 32 (Q4_K, Q8_0) or 16
// (Q6_K) values per row, the Q4_K minimum term through per-32 sums of x.
//
// Optional fused prologue: RMSNorm of the input (src/runtime.rs:193-196) with the
// reference's evaluation order v*inv*g.  Epilogues: store, residual add
// (src/runtime.rs:798-804), and SwiGLU silu(g)*u over paired gate/up rows
// (src/runtime.rs:409-418, src/activation.rs:50).
#include "common.cuh"
#include "kernels.h"

namespace evl {

namespace {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kUnitStride = 68;  // floats per unit in shared memory
constexpr float kMagic = 8388608.0f;

__device__ __forceinline__ uint32_t word(const uint4& v, int t) {
    return t == 0 ? v.x : t == 1 ? v.y : t == 2 ? v.z : v.w;
}

__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }

// 4 bytes of w (each 0..255) as exact floats minus `bias`, multiplied into acc.
__device__ __forceinline__ void fma_bytes(uint32_t w, float bias, float4 x, float2& acc) {
    const float2 nb = f2(-bias, -bias);
    float2 a = __fadd2_rn(f2(byte_magic(w, 0x7650), byte_magic(w, 0x7651)), nb);
    float2 b = __fadd2_rn(f2(byte_magic(w, 0x7652), byte_magic(w, 0x7653)), nb);
    acc = __ffma2_rn(a, f2(x.x, x.y), acc);
    acc = __ffma2_rn(b, f2(x.z, x.w), acc);
}

struct RowPtrs {
    const uint8_t* q;
    const uint8_t* aux;
    const uint16_t* d;
};

// ---------------------------------------------------------------- Q4_K
template <int NR>
__device__ __forceinline__ void dot_q4k(const RowPtrs (&rp)[NR], uint32_t nunits, const float* __restrict__ xs,
                                        const float* __restrict__ xsum, int lane, float (&acc)[NR]) {
    for (uint32_t u = lane; u < nunits; u += 32) {
        const uint64_t o0 = chunk_offset(nunits, 2, u, 0), o1 = chunk_offset(nunits, 2, u, 1);
        uint4 w0[NR], w1[NR], hd[NR];
#pragma unroll
        for (int i = 0; i < NR; ++i) {
            w0[i] = ldg_nc(rp[i].q + o0);
            w1[i] = ldg_nc(rp[i].q + o1);
            hd[i] = ldg_nc_keep(rp[i].aux + (u >> 2) * 16);
        }
        const float* xu = xs + u * kUnitStride;
        float2 p1[NR], p2[NR];
#pragma unroll
        for (int i = 0; i < NR; ++i) p1[i] = p2[i] = f2(0.f, 0.f);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const float4 xl = *reinterpret_cast<const float4*>(xu + 16 * c + 4 * t);
                const float4 xh = *reinterpret_cast<const float4*>(xu + 32 + 16 * c + 4 * t);
#pragma unroll
                for (int i = 0; i < NR; ++i) {
                    const uint32_t wd = word(c == 0 ? w0[i] : w1[i], t);
                    fma_bytes(wd & 0x0F0F0F0Fu, kMagic, xl, p1[i]);
                    fma_bytes((wd >> 4) & 0x0F0F0F0Fu, kMagic, xh, p2[i]);
                }
            }
        }
        const float X1 = xsum[2 * u], X2 = xsum[2 * u + 1];
        const uint32_t j = u & 3, k = (2 * j) & 3, sh = 8 * k;
        const bool high = j >= 2;
#pragma unroll
        for (int i = 0; i < NR; ++i) {
            const float d = h2f(hd[i].x & 0xffff), dmin = h2f(hd[i].x >> 16);
            const uint32_t w0s = hd[i].y >> sh, w1s = hd[i].z >> sh, w2s = hd[i].w >> sh;
            // get_scale_min_k4 (src/gguf.rs:327-336) for sub-blocks 2j and 2j+1:
            // bytes k and k+1 of each scale word
            uint32_t s1, m1, s2, m2;
            if (!high) {
                s1 = w0s & 63; m1 = w1s & 63;
                s2 = (w0s >> 8) & 63; m2 = (w1s >> 8) & 63;
            } else {
                s1 = (w2s & 15) | (((w0s >> 6) & 3) << 4);
                m1 = ((w2s >> 4) & 15) | (((w1s >> 6) & 3) << 4);
                s2 = ((w2s >> 8) & 15) | (((w0s >> 14) & 3) << 4);
                m2 = ((w2s >> 12) & 15) | (((w1s >> 14) & 3) << 4);
            }
            const float dot = (float)s1 * (p1[i].x + p1[i].y) + (float)s2 * (p2[i].x + p2[i].y);
            const float mn = (float)m1 * X1 + (float)m2 * X2;
            acc[i] += d * dot - dmin * mn;
        }
    }
}

// ---------------------------------------------------------------- Q6_K
template <int NR>
__device__ __forceinline__ void dot_q6k(const RowPtrs (&rp)[NR], uint32_t nunits, const float* __restrict__ xs,
                                        int lane, float (&acc)[NR]) {
    for (uint32_t u = lane; u < nunits; u += 32) {
        const uint64_t o0 = chunk_offset(nunits, 3, u, 0), o1 = chunk_offset(nunits, 3, u, 1),
                       o2 = chunk_offset(nunits, 3, u, 2);
        uint4 lo[NR], hi[NR], qh[NR];
        uint32_t scw[NR];
        uint16_t dd[NR];
#pragma unroll
        for (int i = 0; i < NR; ++i) {
            lo[i] = ldg_nc(rp[i].q + o0);
            hi[i] = ldg_nc(rp[i].q + o1);
            qh[i] = ldg_nc(rp[i].q + o2);
            scw[i] = __ldg(reinterpret_cast<const uint32_t*>(rp[i].aux) + u);
            dd[i] = __ldg(rp[i].d + (u >> 2));
        }
        const float* xu = xs + u * kUnitStride;
        float2 p[NR][4];
#pragma unroll
        for (int i = 0; i < NR; ++i)
#pragma unroll
            for (int k = 0; k < 4; ++k) p[i][k] = f2(0.f, 0.f);
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const float4 x0 = *reinterpret_cast<const float4*>(xu + 0 + 4 * t);
            const float4 x1 = *reinterpret_cast<const float4*>(xu + 16 + 4 * t);
            const float4 x2 = *reinterpret_cast<const float4*>(xu + 32 + 4 * t);
            const float4 x3 = *reinterpret_cast<const float4*>(xu + 48 + 4 * t);
#pragma unroll
            for (int i = 0; i < NR; ++i) {
                const uint32_t L = word(lo[i], t), H = word(hi[i], t), Q = word(qh[i], t);
                const uint32_t q0 = (L & 0x0F0F0F0Fu) | ((Q << 4) & 0x30303030u);
                const uint32_t q1 = (H & 0x0F0F0F0Fu) | ((Q << 2) & 0x30303030u);
                const uint32_t q2 = ((L >> 4) & 0x0F0F0F0Fu) | (Q & 0x30303030u);
                const uint32_t q3 = ((H >> 4) & 0x0F0F0F0Fu) | ((Q >> 2) & 0x30303030u);
                fma_bytes(q0, kMagic + 32.f, x0, p[i][0]);
                fma_bytes(q1, kMagic + 32.f, x1, p[i][1]);
                fma_bytes(q2, kMagic + 32.f, x2, p[i][2]);
                fma_bytes(q3, kMagic + 32.f, x3, p[i][3]);
            }
        }
#pragma unroll
        for (int i = 0; i < NR; ++i) {
            const float d = h2f(dd[i]);
            float s = 0.f;
#pragma unroll
            for (int k = 0; k < 4; ++k) s += (float)(int8_t)((scw[i] >> (8 * k)) & 0xff) * (p[i][k].x + p[i][k].y);
            acc[i] += d * s;
        }
    }
}

// ---------------------------------------------------------------- Q8_0
template <int NR>
__device__ __forceinline__ void dot_q8_0(const RowPtrs (&rp)[NR], uint32_t nunits, const float* __restrict__ xs,
                                         int lane, float (&acc)[NR]) {
    for (uint32_t u = lane; u < nunits; u += 32) {
        uint4 w[NR][4];
        uint32_t dw[NR];
#pragma unroll
        for (int i = 0; i < NR; ++i) {
#pragma unroll
            for (int c = 0; c < 4; ++c) w[i][c] = ldg_nc(rp[i].q + chunk_offset(nunits, 4, u, c));
            dw[i] = __ldg(reinterpret_cast<const uint32_t*>(rp[i].aux) + u);
        }
        const float* xu = xs + u * kUnitStride;
        float2 p0[NR], p1[NR];
#pragma unroll
        for (int i = 0; i < NR; ++i) p0[i] = p1[i] = f2(0.f, 0.f);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const float4 xv = *reinterpret_cast<const float4*>(xu + 16 * c + 4 * t);
#pragma unroll
                for (int i = 0; i < NR; ++i) {
                    const uint32_t wd = word(w[i][c], t) ^ 0x80808080u;  // int8 -> q + 128
                    fma_bytes(wd, kMagic + 128.f, xv, c < 2 ? p0[i] : p1[i]);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < NR; ++i)
            acc[i] += h2f(dw[i] & 0xffff) * (p0[i].x + p0[i].y) + h2f(dw[i] >> 16) * (p1[i].x + p1[i].y);
    }
}

__device__ __forceinline__ RowPtrs row_ptrs(const QMatDev& m, uint32_t r) {
    const uint32_t ch = chunks_per_unit(m.type);
    RowPtrs p;
    p.q = m.q + (uint64_t)r * m.nunits * ch * 16;
    p.d = nullptr;
    switch (m.type) {
        case GGML_Q4_K: p.aux = m.aux + (uint64_t)r * (m.cols / 256) * 16; break;
        case GGML_Q6_K:
            p.aux = m.aux + (uint64_t)r * m.nunits * 4;
            p.d = m.d + (uint64_t)r * (m.cols / 256);
            break;
        default: p.aux = m.aux + (uint64_t)r * m.nunits * 4; break;
    }
    return p;
}

__device__ __forceinline__ float silu(float z) { return __fdiv_rn(z, __fadd_rn(1.0f, expf(-z))); }

template <int NR>
__global__ void __launch_bounds__(kThreads) qmatvec_kernel(const __grid_constant__ MatvecArgs a, uint32_t need_layouts,
                                                           uint32_t total_rg, uint32_t rg_begin1, uint32_t rg_begin2) {
    extern __shared__ __align__(16) float smem[];
    const uint32_t nunits = a.cols / 64;
    float* xs_nat = smem;
    float* xs_q6 = smem + ((need_layouts & 1) ? nunits * kUnitStride : 0);
    float* xsum = xs_q6 + ((need_layouts & 2) ? nunits * kUnitStride : 0);
    __shared__ float red[kWarps];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    pdl_wait();
    float inv = 1.f;
    if (a.norm_w) {
        float ss = 0.f;
        for (uint32_t i = tid; i < a.cols; i += kThreads) {
            float v = a.x[i];
            ss += v * v;
        }
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        ss = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) ss += red[w];
        inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)a.cols), a.eps)));
    }
    for (uint32_t i = tid; i < a.cols; i += kThreads) {
        float v = a.x[i];
        if (a.norm_w) v = __fmul_rn(__fmul_rn(v, inv), a.norm_w[i]);
        if (a.x_out && blockIdx.x == 0) a.x_out[i] = v;
        if (need_layouts & 1) xs_nat[(i >> 6) * kUnitStride + (i & 63)] = v;
        if (need_layouts & 2) {
            const uint32_t r = i & 255, h = r >> 7, k = (r >> 5) & 3, b = (r >> 4) & 1, l = r & 15;
            const uint32_t u = (i >> 8) * 4 + h * 2 + b;
            xs_q6[u * kUnitStride + k * 16 + l] = v;
        }
    }
    __syncthreads();
    if (need_layouts & 4) {  // per-32 sums for the Q4_K minimum term
        for (uint32_t s = tid; s < a.cols / 32; s += kThreads) {
            const float* p = xs_nat + (s >> 1) * kUnitStride + (s & 1) * 32;
            float acc = 0.f;
#pragma unroll 8
            for (int e = 0; e < 32; ++e) acc += p[e];
            xsum[s] = acc;
        }
        __syncthreads();
    }
    pdl_launch_dependents();

    const uint32_t stride = gridDim.x * kWarps;
    for (uint32_t rg = blockIdx.x * kWarps + warp; rg < total_rg; rg += stride) {
        const int si = rg >= rg_begin2 ? 2 : rg >= rg_begin1 ? 1 : 0;
        const MatvecSeg& sg = a.seg[si];
        const uint32_t local = rg - (si == 2 ? rg_begin2 : si == 1 ? rg_begin1 : 0);
        const bool dual = sg.epi == EPI_SWIGLU;
        const int rpg = dual ? NR / 2 : NR;  // output rows per group
        const uint32_t r0 = local * rpg;
        RowPtrs rp[NR];
#pragma unroll
        for (int i = 0; i < NR; ++i) {
            const bool second = dual && i >= NR / 2;
            const QMatDev& m = second ? sg.m2 : sg.m;
            const uint32_t r = min(r0 + (second ? i - NR / 2 : i), m.rows - 1);
            rp[i] = row_ptrs(m, r);
        }
        float acc[NR];
#pragma unroll
        for (int i = 0; i < NR; ++i) acc[i] = 0.f;
        switch (sg.m.type) {
            case GGML_Q4_K: dot_q4k<NR>(rp, nunits, xs_nat, xsum, lane, acc); break;
            case GGML_Q6_K: dot_q6k<NR>(rp, nunits, xs_q6, lane, acc); break;
            case GGML_Q8_0: dot_q8_0<NR>(rp, nunits, xs_nat, lane, acc); break;
            default: break;
        }
#pragma unroll
        for (int i = 0; i < NR; ++i) acc[i] = warp_sum(acc[i]);
        if (lane == 0) {
            if (dual) {
#pragma unroll
                for (int i = 0; i < NR / 2; ++i) {
                    const uint32_t r = r0 + i;
                    if (r < sg.m.rows) sg.y[r] = __fmul_rn(silu(acc[i]), acc[i + NR / 2]);
                }
            } else {
#pragma unroll
                for (int i = 0; i < NR; ++i) {
                    const uint32_t r = r0 + i;
                    if (r < sg.m.rows) {
                        if (sg.epi == EPI_ADD) sg.y[r] += acc[i];
                        else sg.y[r] = acc[i];
                    }
                }
            }
        }
    }
}

template <int NR>
cudaError_t launch_nr(const MatvecArgs& a, cudaStream_t s, bool pdl) {
    uint32_t need = 0, rg[kMaxSegs] = {0, 0, 0};
    for (int i = 0; i < a.nseg; ++i) {
        const uint32_t t = a.seg[i].m.type;
        need |= (t == GGML_Q6_K) ? 2u : 1u;
        if (t == GGML_Q4_K) need |= 4u;
        const int rpg = a.seg[i].epi == EPI_SWIGLU ? NR / 2 : NR;
        rg[i] = (a.seg[i].m.rows + rpg - 1) / rpg;
    }
    const uint32_t b1 = rg[0], b2 = rg[0] + rg[1], total = rg[0] + rg[1] + rg[2];
    const uint32_t nunits = a.cols / 64;
    size_t smem = 0;
    if (need & 1) smem += (size_t)nunits * kUnitStride * 4;
    if (need & 2) smem += (size_t)nunits * kUnitStride * 4;
    if (need & 4) smem += (size_t)(a.cols / 32) * 4;
    cudaError_t e = cudaFuncSetAttribute(qmatvec_kernel<NR>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
    const uint32_t grid = (total + kWarps - 1) / kWarps;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, qmatvec_kernel<NR>, a, need, total, b1, b2);
}

}  // namespace

cudaError_t launch_qmatvec(const MatvecArgs& a, cudaStream_t s, bool pdl) {
    if (a.nseg < 1 || a.nseg > kMaxSegs || a.cols % 64 != 0 || a.cols == 0) return cudaErrorInvalidValue;
    uint32_t rows = 0;
    bool dual = false;
    for (int i = 0; i < a.nseg; ++i) {
        rows += a.seg[i].m.rows;
        dual |= a.seg[i].epi == EPI_SWIGLU;
        const uint32_t t = a.seg[i].m.type;
        if (t != GGML_Q4_K && t != GGML_Q6_K && t != GGML_Q8_0) return cudaErrorInvalidValue;
        if (a.seg[i].m.cols != a.cols || a.seg[i].m.rows == 0) return cudaErrorInvalidValue;
    }
    // Rows per warp: enough warps to cover the SMs several times over, and
    // as many rows per warp as that allows (each x register is reused NR times).
    if (dual) return rows >= 148 * 16 * 2 ? launch_nr<4>(a, s, pdl) : launch_nr<2>(a, s, pdl);
    if (rows >= 148 * 16 * 4) return launch_nr<4>(a, s, pdl);
    if (rows >= 148 * 16 * 2) return launch_nr<2>(a, s, pdl);
    return launch_nr<1>(a, s, pdl);
}

}  // namespace evl
