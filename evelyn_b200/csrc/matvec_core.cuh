// matvec_core.cuh -- the dequant-fused matrix-vector machinery shared by the
// standalone matvec kernel (qmatvec.cu) and the persistent step kernel
// (step_kernel.cu): plan, input staging, per-unit dot products, TMA producer and
// consumer loops.
//
// Replaces QMatrix::matvec (src/runtime.rs:72-88), which dequantises every row into
// a fresh Vec<f32> and sums sequentially in f32.
//
// Shape of the kernel (one persistent CTA per SM, warp-specialised):
//   * a producer warp streams the CTA's contiguous range of 32-row blocks, one
//     32-unit column tile at a time, from HBM into a ring of shared-memory stages
//     with TMA bulk copies (cp.async.bulk + mbarrier complete_tx). It needs nothing
//     from the previous kernel, so it starts before griddepcontrol.wait and keeps the
//     ring full across the kernel boundary; after its last copy it prefetches the
//     next matrix's first tiles into L2;
//   * sixteen consumer warps stage the input vector once per CTA as 24-bit block
//     fixed point -- per 32-value block x = 2^-s * m, |m| <= 2^22, m split into three
//     signed 8-bit limbs -- then run the dot products on the raw quant bytes with
//     integer dp4a (4 products per instruction), two rows per warp per stage, one
//     64-value unit per lane. Block scales (d*s_j, dmin*m_j, Q6_K int8 scales, the
//     2^-s of x) are applied in f32 once per 32 (Q4_K, Q8_0) or 16 (Q6_K) values.
// The integer products are exact, so the only rounding against the reference's
// f32 loop is the 2^-22-relative quantisation of x and the order of the f32 sums.
//
// Optional fused prologue: RMSNorm of the input (src/runtime.rs:193-196) in the
// reference's v*inv*g order. Epilogues: store, residual add (src/runtime.rs:798-804),
// and SwiGLU silu(g)*u over paired gate/up rows (src/runtime.rs:409-418,
// src/activation.rs:50).
#pragma once
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace evl {
namespace mv {

namespace {

constexpr int kCW = 16;               // consumer warps
constexpr int kThreads = 32 * (kCW + 1);
constexpr int kNR = 2;                 // row slots per consumer warp
constexpr int kRB = kCW * kNR;         // 32 row slots per stage
constexpr int kLimbStride = 208;       // bytes of limbs per unit: 3 x 64 + 16 pad (bank spread)
constexpr int kMaxStages = 8;
constexpr uint32_t kSmemBudget = 225 * 1024;
constexpr uint32_t kConsumerBarrier = 1;  // named barrier of the consumer threads
static_assert(kRB == 2 * kSlabRows && kNR % 2 == 0, "a stage is two 16-row slabs; SwiGLU pairs split kNR");

// need bits
constexpr uint32_t NEED_NAT = 1, NEED_Q6 = 2, NEED_XSUM = 4, NEED_MSUM = 8;

// One matvec launch (or one phase of the step kernel), prepared on the host.
struct Plan {
    MatvecArgs a;
    uint32_t rb_begin[kMaxSegs + 1];  // first row-block of each segment (+ total)
    uint32_t nunits, ngroups;
    uint32_t item_bytes;  // largest stage (32 rows x one 32-unit group) of any segment
    uint32_t need;
    uint32_t off_nat, off_q6, off_fscale, off_xsum, off_msum;  // offsets in the staged-input area
    uint32_t xbytes;                                           // size of the staged-input area
    const uint8_t* pf_base;  // next matrix to prefetch into L2 (optional)
    uint32_t pf_row_bytes, pf_rows;
    int* err;
};

// The ring of shared-memory stages the producer fills and the consumers drain.
struct Ring {
    uint8_t* base;
    uint64_t* full;
    uint64_t* empty;
    uint32_t stages, slot_bytes;
};

__device__ __forceinline__ int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

__device__ __forceinline__ void named_sync(uint32_t id, uint32_t n) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// Bounded wait that also gives up as soon as another thread of the CTA has aborted.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (*abort_flag) return false;
        if (global_ns() - t0 > kWaitNs) {
            *abort_flag = 1;
            return false;
        }
    }
    return true;
}

__device__ __forceinline__ float silu(float z) { return __fdiv_rn(z, __fadd_rn(1.0f, expf(-z))); }

__device__ __forceinline__ int seg_of(const Plan& p, uint32_t rb) {
    return rb >= p.rb_begin[2] ? 2 : rb >= p.rb_begin[1] ? 1 : 0;
}


// ---------------------------------------------------------------- per-unit dot products
// Each returns, per row slot, the f32 contribution of one 64-value unit.

// Q4_K: low nibbles of the 32 qs bytes are values 0..31 of the unit (sub-block A),
// high nibbles values 32..63 (sub-block B).
__device__ __forceinline__ void unit_q4k(const uint8_t* const (&tiles)[kNR], uint32_t U, uint32_t lane, uint32_t u,
                                         const uint8_t* limbs, const float* fscale, const float* xsum,
                                         float (&acc)[kNR]) {
    int SA[kNR][3], SB[kNR][3];
#pragma unroll
    for (int i = 0; i < kNR; ++i)
#pragma unroll
        for (int k = 0; k < 3; ++k) SA[i][k] = SB[i][k] = 0;
#pragma unroll
    for (int half = 0; half < 2; ++half) {  // qs chunk `half`: words t = 4*half .. 4*half+3
        int4 la[3], lb[3];
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            la[k] = *reinterpret_cast<const int4*>(limbs + k * 64 + 16 * half);
            lb[k] = *reinterpret_cast<const int4*>(limbs + k * 64 + 32 + 16 * half);
        }
#pragma unroll
        for (int i = 0; i < kNR; ++i) {
            const int4 w = *reinterpret_cast<const int4*>(tiles[i] + half * U * 16 + lane * 16);
            const int wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const int lo = wv[t] & 0x0F0F0F0F, hi = (wv[t] >> 4) & 0x0F0F0F0F;
                const int a0 = t == 0 ? la[0].x : t == 1 ? la[0].y : t == 2 ? la[0].z : la[0].w;
                const int a1 = t == 0 ? la[1].x : t == 1 ? la[1].y : t == 2 ? la[1].z : la[1].w;
                const int a2 = t == 0 ? la[2].x : t == 1 ? la[2].y : t == 2 ? la[2].z : la[2].w;
                const int b0 = t == 0 ? lb[0].x : t == 1 ? lb[0].y : t == 2 ? lb[0].z : lb[0].w;
                const int b1 = t == 0 ? lb[1].x : t == 1 ? lb[1].y : t == 2 ? lb[1].z : lb[1].w;
                const int b2 = t == 0 ? lb[2].x : t == 1 ? lb[2].y : t == 2 ? lb[2].z : lb[2].w;
                SA[i][0] = dp4a(lo, a0, SA[i][0]);
                SA[i][1] = dp4a(lo, a1, SA[i][1]);
                SA[i][2] = dp4a(lo, a2, SA[i][2]);
                SB[i][0] = dp4a(hi, b0, SB[i][0]);
                SB[i][1] = dp4a(hi, b1, SB[i][1]);
                SB[i][2] = dp4a(hi, b2, SB[i][2]);
            }
        }
    }
    const float fa = fscale[2 * u], fb = fscale[2 * u + 1];
    const float XA = xsum[2 * u], XB = xsum[2 * u + 1];
    const uint32_t j = u & 3, sh = 8 * ((2 * j) & 3);
    const bool high = j >= 2;
#pragma unroll
    for (int i = 0; i < kNR; ++i) {
        const uint4 hd = *reinterpret_cast<const uint4*>(tiles[i] + U * 32 + (lane / 4) * 16);
        const float d = h2f(hd.x & 0xffff), dmin = h2f(hd.x >> 16);
        const uint32_t w0s = hd.y >> sh, w1s = hd.z >> sh, w2s = hd.w >> sh;
        // get_scale_min_k4 (src/gguf.rs:327-336) for sub-blocks 2j, 2j+1
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
        const float va = fmaf((float)SA[i][2], 65536.f, (float)(SA[i][0] + 256 * SA[i][1])) * fa;
        const float vb = fmaf((float)SB[i][2], 65536.f, (float)(SB[i][0] + 256 * SB[i][1])) * fb;
        acc[i] += d * ((float)s1 * va + (float)s2 * vb) - dmin * ((float)m1 * XA + (float)m2 * XB);
    }
}

// Q6_K: unit (super-block, half h, l0) holds values 128h + 32k + l0 + l for k = 0..3,
// l < 16; its limbs are stored [limb][l/4][k][l%4].
__device__ __forceinline__ void unit_q6k(const uint8_t* const (&tiles)[kNR], uint32_t U, uint32_t lane, uint32_t u,
                                         const uint8_t* limbs, const float* fscale, const int* msum,
                                         float (&acc)[kNR]) {
    int S[kNR][4][3];
#pragma unroll
    for (int i = 0; i < kNR; ++i)
#pragma unroll
        for (int k = 0; k < 4; ++k) S[i][k][0] = S[i][k][1] = S[i][k][2] = 0;
    // the three 16-byte chunks of each row, as whole vector loads (a lane's chunk is
    // 16 contiguous bytes; word-sized loads at a 16-byte lane stride would conflict)
    uint4 Lc[kNR], Hc[kNR], Qc[kNR];
#pragma unroll
    for (int i = 0; i < kNR; ++i) {
        Lc[i] = *reinterpret_cast<const uint4*>(tiles[i] + lane * 16);
        Hc[i] = *reinterpret_cast<const uint4*>(tiles[i] + U * 16 + lane * 16);
        Qc[i] = *reinterpret_cast<const uint4*>(tiles[i] + 2 * U * 16 + lane * 16);
    }
#pragma unroll
    for (int t = 0; t < 4; ++t) {
        int4 lv[3];
#pragma unroll
        for (int c = 0; c < 3; ++c) lv[c] = *reinterpret_cast<const int4*>(limbs + c * 64 + 16 * t);
#pragma unroll
        for (int i = 0; i < kNR; ++i) {
            const uint32_t L = t == 0 ? Lc[i].x : t == 1 ? Lc[i].y : t == 2 ? Lc[i].z : Lc[i].w;
            const uint32_t H = t == 0 ? Hc[i].x : t == 1 ? Hc[i].y : t == 2 ? Hc[i].z : Hc[i].w;
            const uint32_t Q = t == 0 ? Qc[i].x : t == 1 ? Qc[i].y : t == 2 ? Qc[i].z : Qc[i].w;
            const int q0 = (int)((L & 0x0F0F0F0Fu) | ((Q << 4) & 0x30303030u));
            const int q1 = (int)((H & 0x0F0F0F0Fu) | ((Q << 2) & 0x30303030u));
            const int q2 = (int)(((L >> 4) & 0x0F0F0F0Fu) | (Q & 0x30303030u));
            const int q3 = (int)(((H >> 4) & 0x0F0F0F0Fu) | ((Q >> 2) & 0x30303030u));
#pragma unroll
            for (int c = 0; c < 3; ++c) {
                S[i][0][c] = dp4a(q0, lv[c].x, S[i][0][c]);
                S[i][1][c] = dp4a(q1, lv[c].y, S[i][1][c]);
                S[i][2][c] = dp4a(q2, lv[c].z, S[i][2][c]);
                S[i][3][c] = dp4a(q3, lv[c].w, S[i][3][c]);
            }
        }
    }
    // x-block of run k: 8*(u/4) + 4*h + k with h = (u/2) & 1
    const uint32_t jb = 8 * (u >> 2) + 4 * ((u >> 1) & 1);
    const int* ms = msum + u * 12;  // [k][limb] sums of the limbs (the -32 bias)
#pragma unroll
    for (int i = 0; i < kNR; ++i) {
        const uint32_t scw = *reinterpret_cast<const uint32_t*>(tiles[i] + U * 48 + lane * 4);
        const uint32_t dh = *reinterpret_cast<const uint16_t*>(tiles[i] + U * 48 + pad16(U * 4) + (lane / 4) * 2);
        float s = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int a = S[i][k][0] - 32 * ms[3 * k], b = S[i][k][1] - 32 * ms[3 * k + 1],
                      c = S[i][k][2] - 32 * ms[3 * k + 2];
            const float v = fmaf((float)c, 65536.f, (float)(a + 256 * b)) * fscale[jb + k];
            s = fmaf((float)(int8_t)((scw >> (8 * k)) & 0xff), v, s);
        }
        acc[i] = fmaf(h2f(dh), s, acc[i]);
    }
}

// Q8_0: two 32-value blocks per unit.
__device__ __forceinline__ void unit_q8_0(const uint8_t* const (&tiles)[kNR], uint32_t U, uint32_t lane, uint32_t u,
                                          const uint8_t* limbs, const float* fscale, float (&acc)[kNR]) {
    int S[kNR][2][3];
#pragma unroll
    for (int i = 0; i < kNR; ++i)
#pragma unroll
        for (int b = 0; b < 2; ++b) S[i][b][0] = S[i][b][1] = S[i][b][2] = 0;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        int4 lv[3];
#pragma unroll
        for (int k = 0; k < 3; ++k) lv[k] = *reinterpret_cast<const int4*>(limbs + k * 64 + 16 * c);
#pragma unroll
        for (int i = 0; i < kNR; ++i) {
            const int4 w = *reinterpret_cast<const int4*>(tiles[i] + c * U * 16 + lane * 16);
#pragma unroll
            for (int k = 0; k < 3; ++k) {
                int s = S[i][c >> 1][k];
                s = dp4a(w.x, lv[k].x, s);
                s = dp4a(w.y, lv[k].y, s);
                s = dp4a(w.z, lv[k].z, s);
                s = dp4a(w.w, lv[k].w, s);
                S[i][c >> 1][k] = s;
            }
        }
    }
    const float f0 = fscale[2 * u], f1 = fscale[2 * u + 1];
#pragma unroll
    for (int i = 0; i < kNR; ++i) {
        const uint32_t dw = *reinterpret_cast<const uint32_t*>(tiles[i] + U * 64 + lane * 4);
        const float v0 = fmaf((float)S[i][0][2], 65536.f, (float)(S[i][0][0] + 256 * S[i][0][1])) * f0;
        const float v1 = fmaf((float)S[i][1][2], 65536.f, (float)(S[i][1][0] + 256 * S[i][1][1])) * f1;
        acc[i] += h2f(dw & 0xffff) * v0 + h2f(dw >> 16) * v1;
    }
}

// ---------------------------------------------------------------- input staging
// x (optionally RMS-normalised, src/runtime.rs:193-196) -> per 32-value block j a scale
// 2^-s and |m| <= 2^22 with x = 2^-s * m, m = l0 + 2^8 l1 + 2^16 l2 in three int8 limbs,
// written in the layouts the unit functions read. Each consumer thread stages one
// 16-value half of a block from registers: the two halves of a block sit in adjacent
// lanes and meet with one shuffle for the block maximum and sum.

// x is read through L2 (ld.global.cg): inside the persistent step kernel it was written
// by other CTAs in the previous phase, and L1 is not coherent across SMs.

// limb bytes of four staged values: t = m + 0x8080 makes bytes 0 and 1 of t the
// limbs l0, l1 biased by 128, and t >> 16 = l2
__device__ __forceinline__ void pack_limbs(int m0, int m1, int m2, int m3, uint32_t& w0, uint32_t& w1, uint32_t& w2) {
    const uint32_t t0 = (uint32_t)(m0 + 0x8080), t1 = (uint32_t)(m1 + 0x8080), t2 = (uint32_t)(m2 + 0x8080),
                   t3 = (uint32_t)(m3 + 0x8080);
    const uint32_t a01 = __byte_perm(t0, t1, 0x5140), a23 = __byte_perm(t2, t3, 0x5140);  // b0 b0' b1 b1'
    w0 = __byte_perm(a01, a23, 0x5410) ^ 0x80808080u;  // byte 0 of each
    w1 = __byte_perm(a01, a23, 0x7632) ^ 0x80808080u;  // byte 1 of each
    w2 = __byte_perm(__byte_perm(t0, t1, 0x0062), __byte_perm(t2, t3, 0x0062), 0x5410);  // byte 2 of each
}

__device__ void stage_input(const Plan& p, uint8_t* xs, int warp, int lane, float* red) {
    const MatvecArgs& a = p.a;
    const uint32_t K = a.cols, nhalf = K / 16;
    const uint32_t c = (uint32_t)(warp * 32 + lane);  // consumer thread 0 .. kCW*32-1
    float inv = 1.f;
    if (a.norm_w) {
        float ss = 0.f;
        for (uint32_t hb = c; hb < nhalf; hb += kCW * 32) {
            const float4* xp = reinterpret_cast<const float4*>(a.x + 16 * hb);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float4 v = __ldcg(xp + q);
                ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
            }
        }
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        named_sync(kConsumerBarrier, kCW * 32);
        ss = 0.f;
#pragma unroll
        for (int w = 0; w < kCW; ++w) ss += red[w];
        inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), a.eps)));
    }
    uint8_t* nat = xs + p.off_nat;
    uint8_t* q6 = xs + p.off_q6;
    float* fscale = reinterpret_cast<float*>(xs + p.off_fscale);
    float* xsum = reinterpret_cast<float*>(xs + p.off_xsum);
    int* msum = reinterpret_cast<int*>(xs + p.off_msum);
    // nhalf is a multiple of 4, so a warp's 32 lanes cover whole blocks or none
    for (uint32_t hb0 = (uint32_t)warp * 32; hb0 < nhalf; hb0 += kCW * 32) {
        const uint32_t hb = hb0 + lane;
        const bool on = hb < nhalf;  // uniform per lane pair
        float v[16];
        if (on) {
            const float4* xp = reinterpret_cast<const float4*>(a.x + 16 * hb);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float4 t = __ldcg(xp + q);
                v[4 * q] = t.x; v[4 * q + 1] = t.y; v[4 * q + 2] = t.z; v[4 * q + 3] = t.w;
            }
            if (a.norm_w) {
                const float4* gp = reinterpret_cast<const float4*>(a.norm_w + 16 * hb);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float4 g = gp[q];
                    v[4 * q] = __fmul_rn(__fmul_rn(v[4 * q], inv), g.x);
                    v[4 * q + 1] = __fmul_rn(__fmul_rn(v[4 * q + 1], inv), g.y);
                    v[4 * q + 2] = __fmul_rn(__fmul_rn(v[4 * q + 2], inv), g.z);
                    v[4 * q + 3] = __fmul_rn(__fmul_rn(v[4 * q + 3], inv), g.w);
                }
            }
            if (a.x_out && blockIdx.x == 0) {
                float4* op = reinterpret_cast<float4*>(a.x_out + 16 * hb);
#pragma unroll
                for (int q = 0; q < 4; ++q) op[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
            }
        } else {
#pragma unroll
            for (int e = 0; e < 16; ++e) v[e] = 0.f;
        }
        // |x| bit patterns order like the values; the biased exponent E of the block
        // maximum puts it in [2^(E-127), 2^(E-126)), i.e. frexp's e = E - 126, and
        // s = 22 - e keeps |m| <= 2^22
        uint32_t abits = 0;
#pragma unroll
        for (int e = 0; e < 16; ++e) abits = max(abits, __float_as_uint(v[e]) & 0x7fffffffu);
        abits = max(abits, __shfl_xor_sync(0xffffffffu, abits, 1));
        const int s = abits ? min(max(148 - (int)(abits >> 23), -100), 120) : 0;
        // 2^s and 2^-s are normal floats for s in [-100, 120]: the scaling is exact
        const float up = __uint_as_float((uint32_t)(s + 127) << 23);
        int m[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) m[e] = __float2int_rn(__fmul_rn(v[e], up));
        uint32_t L0[4], L1[4], L2[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) pack_limbs(m[4 * q], m[4 * q + 1], m[4 * q + 2], m[4 * q + 3], L0[q], L1[q], L2[q]);
        const uint32_t j = hb >> 1, h = hb & 1;
        const float fs = __uint_as_float((uint32_t)(127 - s) << 23);
        if (p.need & NEED_XSUM) {  // sum of the staged (quantised) block: exact in int32
            int sm = 0;
#pragma unroll
            for (int e = 0; e < 16; ++e) sm += m[e];
            sm += __shfl_xor_sync(0xffffffffu, sm, 1);
            if (on && h == 0) xsum[j] = __fmul_rn((float)sm, fs);
        }
        if (!on) continue;
        if (h == 0) fscale[j] = fs;
        if (p.need & NEED_NAT) {  // unit j/2: [limb][64 values], block j&1 at +32, half at +16
            uint8_t* b = nat + (j >> 1) * kLimbStride + (j & 1) * 32 + h * 16;
            *reinterpret_cast<uint4*>(b) = make_uint4(L0[0], L0[1], L0[2], L0[3]);
            *reinterpret_cast<uint4*>(b + 64) = make_uint4(L1[0], L1[1], L1[2], L1[3]);
            *reinterpret_cast<uint4*>(b + 128) = make_uint4(L2[0], L2[1], L2[2], L2[3]);
        }
        if (p.need & NEED_Q6) {  // the half is run k of unit u: value l at (l/4)*16 + k*4 + l%4
            const uint32_t i = 16 * hb, r8 = i & 255, hh = r8 >> 7, k = (r8 >> 5) & 3;
            const uint32_t u = (i >> 8) * 4 + hh * 2 + h;
            uint8_t* b = q6 + u * kLimbStride + k * 4;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                *reinterpret_cast<uint32_t*>(b + q * 16) = L0[q];
                *reinterpret_cast<uint32_t*>(b + 64 + q * 16) = L1[q];
                *reinterpret_cast<uint32_t*>(b + 128 + q * 16) = L2[q];
            }
            if (p.need & NEED_MSUM) {  // per run: sums of each limb (the -32 bias)
                int s0 = 0, s1 = 0, s2 = 0;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    s0 = dp4a((int)L0[q], 0x01010101, s0);
                    s1 = dp4a((int)L1[q], 0x01010101, s1);
                    s2 = dp4a((int)L2[q], 0x01010101, s2);
                }
                int* ms = msum + u * 12 + 3 * k;
                ms[0] = s0;
                ms[1] = s1;
                ms[2] = s2;
            }
        }
    }
    named_sync(kConsumerBarrier, kCW * 32);
}


// This CTA's row blocks [rb0, rb1) of a plan. Every CTA takes a contiguous range.
__device__ __forceinline__ void cta_rows(const Plan& p, uint32_t cta, uint32_t ncta, uint32_t& rb0, uint32_t& rb1) {
    const uint32_t total = p.rb_begin[kMaxSegs];
    rb0 = (uint32_t)(((uint64_t)total * cta) / ncta);
    rb1 = (uint32_t)(((uint64_t)total * (cta + 1)) / ncta);
}

// Global addresses of item (rb, g): the one or two 16-row slabs of column group g that
// one stage holds -- rows [32*local, +32), or gate and up rows [16*local, +16) for the
// SwiGLU pair. Returns the number of slabs (1 when the second is past the end).
__device__ __forceinline__ uint32_t item_slabs(const Plan& p, uint32_t rb, uint32_t g, const uint8_t*& a,
                                               const uint8_t*& b, uint32_t& slab_bytes) {
    const int si = seg_of(p, rb);
    const MatvecSeg& sg = p.a.seg[si];
    const uint32_t local = rb - p.rb_begin[si];
    const uint32_t T = sg.m.type;
    slab_bytes = kSlabRows * tile_bytes(T, group_units(p.nunits, g));
    const bool dual = sg.epi == EPI_SWIGLU;
    const QMatDev& mb = dual ? sg.m2 : sg.m;
    const uint32_t sa = dual ? local : 2 * local, sbk = dual ? local : 2 * local + 1;
    a = sg.m.q + (uint64_t)sa * kSlabRows * sg.m.row_bytes + slab_group_offset(T, g);
    b = mb.q + (uint64_t)sbk * kSlabRows * mb.row_bytes + slab_group_offset(T, g);
    return sbk * kSlabRows < mb.rows ? 2 : 1;
}

// Producer: copy item (rb, g) into ring slot s, completing on full[s].
__device__ __forceinline__ void issue_item(const Plan& p, const Ring& r, uint32_t rb, uint32_t g, uint32_t s) {
    const uint8_t *a, *b;
    uint32_t sb;
    const uint32_t n = item_slabs(p, rb, g, a, b, sb);
    uint8_t* slot = r.base + s * r.slot_bytes;
    mbar_arrive_expect_tx(&r.full[s], n * sb);
    tma_load_1d(slot, a, sb, &r.full[s]);
    if (n == 2) tma_load_1d(slot + sb, b, sb, &r.full[s]);
}

// Producer (one thread): stream row blocks [rb0, rb1) of `p`, one 32-unit column group
// per stage, continuing the ring sequence at `item`. Returns false after an abort.
__device__ bool produce_items(const Plan& p, const Ring& r, uint32_t rb0, uint32_t rb1, uint32_t& item,
                              volatile int* abort_flag) {
    for (uint32_t rb = rb0; rb < rb1; ++rb) {
        for (uint32_t g = 0; g < p.ngroups; ++g, ++item) {
            const uint32_t s = item % r.stages, n = item / r.stages;
            if (n > 0 && !wait_or_abort(&r.empty[s], (n - 1) & 1, abort_flag)) return false;
            if (*abort_flag) return false;
            issue_item(p, r, rb, g, s);
        }
    }
    return true;
}

// Producer, after its last copy of a plan: warm L2 with the first slabs of the next
// matrix this CTA index will read (at most 96 KB).
__device__ void prefetch_next(const Plan& p, uint32_t cta, uint32_t ncta) {
    if (!p.pf_base || !p.pf_rows) return;
    const uint32_t slabs = (p.pf_rows + kSlabRows - 1) / kSlabRows;
    const uint32_t pr0 = (uint32_t)(((uint64_t)slabs * cta) / ncta);
    const uint32_t pr1 = (uint32_t)(((uint64_t)slabs * (cta + 1)) / ncta);
    uint64_t bytes = (uint64_t)(pr1 - pr0) * kSlabRows * p.pf_row_bytes;
    if (bytes > (96u << 10)) bytes = 96u << 10;
    const uint8_t* base = p.pf_base + (uint64_t)pr0 * kSlabRows * p.pf_row_bytes;
    for (uint64_t o = 0; o < bytes; o += 16384)
        prefetch_l2_bulk(base + o, (uint32_t)((bytes - o) < 16384 ? (bytes - o) & ~15ull : 16384));
}

// Producer: after an abort, give the copies in flight a bounded chance to land.
__device__ void drain_ring(const Ring& r, uint32_t item) {
    for (uint32_t s = 0; s < r.stages && s < item; ++s) mbar_wait(&r.full[s], ((item - 1 - s) / r.stages) & 1);
}

// Consumers (all kCW warps): dot products of row blocks [rb0, rb1) against the staged
// input `xs`, epilogue per row block. Returns false after an abort.
__device__ bool consume_items(const Plan& p, const Ring& r, const uint8_t* xs, uint32_t rb0, uint32_t rb1,
                              uint32_t& item, int warp, int lane, volatile int* abort_flag) {
    const uint8_t* nat = xs + p.off_nat;
    const uint8_t* q6 = xs + p.off_q6;
    const float* fscale = reinterpret_cast<const float*>(xs + p.off_fscale);
    const float* xsum = reinterpret_cast<const float*>(xs + p.off_xsum);
    const int* msum = reinterpret_cast<const int*>(xs + p.off_msum);
    for (uint32_t rb = rb0; rb < rb1; ++rb) {
        const int si = seg_of(p, rb);
        const MatvecSeg& sg = p.a.seg[si];
        const uint32_t local = rb - p.rb_begin[si];
        const uint32_t T = sg.m.type;
        const bool dual = sg.epi == EPI_SWIGLU;
        uint32_t slots[kNR];
#pragma unroll
        for (int i = 0; i < kNR; ++i)
            slots[i] = dual ? (uint32_t)((i < kNR / 2 ? 0 : kRB / 2) + (kNR / 2) * warp + i % (kNR / 2))
                            : (uint32_t)(kNR * warp + i);
        float acc[kNR];
#pragma unroll
        for (int i = 0; i < kNR; ++i) acc[i] = 0.f;
        for (uint32_t g = 0; g < p.ngroups; ++g, ++item) {
            const uint32_t s = item % r.stages, n = item / r.stages;
            if (!wait_or_abort(&r.full[s], n & 1, abort_flag)) return false;
            const uint32_t U = group_units(p.nunits, g), tb = tile_bytes(T, U);
            const uint8_t* slot = r.base + s * r.slot_bytes;
            if ((uint32_t)lane < U) {
                const uint32_t u = g * 32 + lane;
                const uint8_t* tiles[kNR];
#pragma unroll
                for (int i = 0; i < kNR; ++i) tiles[i] = slot + slots[i] * tb;
                // rows past the end were not copied: their slots hold stale bytes whose
                // (finite) results are discarded below
                if (T == GGML_Q4_K) {
                    unit_q4k(tiles, U, lane, u, nat + u * kLimbStride, fscale, xsum, acc);
                } else if (T == GGML_Q6_K) {
                    unit_q6k(tiles, U, lane, u, q6 + u * kLimbStride, fscale, msum, acc);
                } else {
                    unit_q8_0(tiles, U, lane, u, nat + u * kLimbStride, fscale, acc);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&r.empty[s]);
        }
#pragma unroll
        for (int i = 0; i < kNR; ++i) acc[i] = warp_sum(acc[i]);
        if (lane == 0) {
            if (dual) {
#pragma unroll
                for (int i = 0; i < kNR / 2; ++i) {
                    const uint32_t row = local * (kRB / 2) + (kNR / 2) * warp + i;
                    if (row < sg.m.rows) sg.y[row] = __fmul_rn(silu(acc[i]), acc[i + kNR / 2]);
                }
            } else {
#pragma unroll
                for (int i = 0; i < kNR; ++i) {
                    const uint32_t row = local * kRB + kNR * warp + i;
                    if (row < sg.m.rows) {
                        if (sg.epi == EPI_ADD) sg.y[row] = __ldcg(sg.y + row) + acc[i];
                        else sg.y[row] = acc[i];
                    }
                }
            }
        }
    }
    return true;
}

// Host: check `a` and fill the launch-independent part of a plan (segments, row
// blocks, staged-input layout, stage size). cudaErrorInvalidValue /
// cudaErrorMisalignedAddress when `a` is not a supported matvec.
__host__ cudaError_t plan_matvec(const MatvecArgs& a, Plan& p) {
    if (a.nseg < 1 || a.nseg > kMaxSegs || a.cols % 64 != 0 || a.cols == 0 || !a.err) return cudaErrorInvalidValue;
    // the staging reads x, norm_w and writes x_out as float4
    auto misaligned = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) != 0; };
    if (!a.x || misaligned(a.x) || misaligned(a.norm_w) || misaligned(a.x_out)) return cudaErrorMisalignedAddress;
    p = Plan{};
    p.a = a;
    p.err = a.err;
    p.nunits = a.cols / 64;
    p.ngroups = (p.nunits + 31) / 32;
    uint32_t slot = 0;
    p.rb_begin[0] = 0;
    for (int i = 0; i < kMaxSegs; ++i) {
        uint32_t rbs = 0;
        if (i < a.nseg) {
            const MatvecSeg& sg = a.seg[i];
            const uint32_t t = sg.m.type;
            if (t != GGML_Q4_K && t != GGML_Q6_K && t != GGML_Q8_0) return cudaErrorInvalidValue;
            if (sg.m.cols != a.cols || sg.m.rows == 0 || !sg.y) return cudaErrorInvalidValue;
            if (sg.epi == EPI_SWIGLU && (sg.m2.type != t || sg.m2.rows != sg.m.rows || sg.m2.cols != a.cols))
                return cudaErrorInvalidValue;
            p.need |= t == GGML_Q6_K ? NEED_Q6 | NEED_MSUM : NEED_NAT;
            if (t == GGML_Q4_K) p.need |= NEED_XSUM;
            slot = std::max(slot, kRB * tile_bytes(t, 32));
            const uint32_t per = sg.epi == EPI_SWIGLU ? kRB / 2 : kRB;
            rbs = (sg.m.rows + per - 1) / per;
        }
        p.rb_begin[i + 1] = p.rb_begin[i] + rbs;
    }
    const uint32_t K = a.cols, nb = K / 32;
    uint32_t off = 0;
    p.off_nat = off;
    if (p.need & NEED_NAT) off += p.nunits * kLimbStride;
    p.off_q6 = off;
    if (p.need & NEED_Q6) off += p.nunits * kLimbStride;
    p.off_fscale = off;
    off += nb * 4;
    p.off_xsum = off;
    if (p.need & NEED_XSUM) off += nb * 4;
    p.off_msum = off;
    if (p.need & NEED_MSUM) off += p.nunits * 48;
    p.xbytes = (off + 127) & ~127u;
    p.item_bytes = slot;
    if (p.xbytes + 2 * slot > kSmemBudget) return cudaErrorInvalidValue;
    p.pf_base = a.prefetch.q;
    p.pf_row_bytes = a.prefetch.row_bytes;
    p.pf_rows = a.prefetch.q ? a.prefetch.rows : 0;
    return cudaSuccess;
}

}  // namespace
}  // namespace mv
}  // namespace evl
