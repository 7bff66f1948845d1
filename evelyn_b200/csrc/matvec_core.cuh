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
//     32-unit panel of both 16-row slabs at a time, from HBM into a ring of shared-
//     memory stages with TMA bulk copies (cp.async.bulk + mbarrier complete_tx). It
//     needs nothing from the previous kernel, so it starts before griddepcontrol.wait
//     and keeps the ring full across the kernel boundary; after its last copy it
//     prefetches the next matrix's first slabs into L2;
//   * sixteen consumer warps stage the input vector once per CTA as 24-bit block
//     fixed point -- per 32-value block x = 2^-s * m, |m| <= 2^22, m split into three
//     signed 8-bit limbs -- laid out as the B fragments of mma.sync m16n8k32. Consumer
//     warp (slab, k) of a stage takes the 16 rows of one slab over one super-block (4
//     units) and runs the dot products on the tensor cores: A = the raw quant bytes of
//     16 rows (Q4_K nibbles masked in place, Q6_K 6-bit values, Q8_0 int8), B = the
//     limbs of x; each k32 step holds 16 values of two sub-blocks, B columns 0-2 the
//     limbs of the first and 4-6 those of the second, so every lane of a quad ends with
//     one sub-block's limb sums of rows g and g+8. Block scales (d*s_j, dmin*m_j, Q6_K
//     int8 scales, the 2^-s of x) are applied to those exact integer sums in f32; the
//     eight warps of a slab meet in shared memory at the end of each row block.
#pragma once
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace evl {
namespace mv {

namespace {

constexpr int kCW = 16;               // consumer warps
constexpr int kThreads = 32 * (kCW + 1);
constexpr int kRB = 2 * kSlabRows;     // rows per row block (two slabs)
constexpr int kSbWarps = kCW / 2;      // consumer warps per slab of a stage
constexpr int kXUnit = 192;            // staged B-fragment bytes of one unit
constexpr int kMaxStages = 8;
constexpr uint32_t kSmemBudget = 225 * 1024;
constexpr uint32_t kConsumerBarrier = 1;  // named barrier of the consumer threads
constexpr uint32_t kRedBufs = kMaxStages + 1;            // row-block partial buffers (> stages)
constexpr uint32_t kRedBufBytes = kSbWarps * kRB * 4;
constexpr uint32_t kRedBytes = kRedBufs * kRedBufBytes + 16 * kRedBufs;  // + arrival counters
constexpr uint32_t kRowBuf = 256;  // residual rows a CTA keeps in shared memory
constexpr uint32_t kMaxCtas = 1024;     // grid bound of the row-block partition's 32-bit arithmetic
constexpr uint32_t kMaxEighths = 3;     // staging: up to three 8-value eighths per consumer thread
static_assert(kSbWarps * 4 == kPanelUnits, "each consumer warp of a slab takes one super-block of a panel");

// need bits
constexpr uint32_t NEED_XSUM = 1, NEED_MSUM = 2;

// One matvec launch (or one phase of the step kernel), prepared on the host.
struct Plan {
    MatvecArgs a;
    uint32_t rb_begin[kMaxSegs + 1];  // first row-block of each segment (+ total)
    uint32_t rb_w[kMaxSegs];          // weight of one row block of each segment (bytes >> a shift)
    uint32_t total_w;                 // of all row blocks, < 2^31 / (2 * kMaxCtas)
    uint32_t nunits, ngroups, last_units;  // units per row, panels per row, units of the last panel
    uint32_t item_bytes;  // largest stage (two slabs x one 32-unit panel) of any segment
    uint32_t need;
    uint32_t off_fscale, off_xsum, off_msum, off_red;  // offsets in the staged-input area (B fragments at 0)
    uint32_t off_rows;                                 // residual rows of this CTA (kRowBuf floats)
    uint32_t xbytes;                                   // size of the staged-input area
    const uint8_t* pf_base[3];  // next matrices to prefetch into L2 (optional)
    uint32_t pf_row_bytes[3], pf_rows[3], pf_cap;
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


// ---------------------------------------------------------------- MMA dot products
// D (16 x 8, s32) += A (16 x 32, u8 / s8, row) * B (32 x 8, s8, col): rows g8, g8+8 of
// A in a0/a2 (k < 16) and a1/a3 (k >= 16); B k 4t..4t+3 in b0, 16+4t.. in b1, column g8.
__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_s8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Per-lane constants of the fragment layout. A k32 step of unit u, half h covers the
// 16-value quarters 2h' = h (k < 16, "part 0") and 2 + h (k >= 16, "part 1") of the
// unit; B column c < 3 holds limb c of part 0, 4 <= c < 7 limb c - 4 of part 1, the
// rest zero. So the D columns 2t, 2t+1 of lane t are (limb 0, limb 1) of part t/2 for
// even t and (limb 2, zero) for odd t, and v = d[2t] + 256 d[2t+1] is exact.
struct Lane {
    uint32_t g8, t, part;  // part: which of the two sub-blocks of a step this lane's D holds
    uint32_t boff;         // this lane's B words inside a unit's staged fragments
    bool bload;            // B column g8 is a limb column
    uint32_t mlo, mhi;     // b0 / b1 select: part-0 columns feed b0, part-1 columns b1
};
__device__ __forceinline__ Lane make_lane(int lane) {
    Lane L;
    L.g8 = (uint32_t)lane >> 2;
    L.t = (uint32_t)lane & 3;
    L.part = L.t >> 1;
    L.bload = (L.g8 & 3) < 3;
    L.boff = ((L.g8 >> 2) * 3 + (L.g8 & 3)) * 32 + L.t * 8;
    L.mlo = L.g8 < 4 ? 0xffffffffu : 0u;
    L.mhi = ~L.mlo;
    return L;
}
// the staged B words (halves 0 and 1) of unit u for this lane
__device__ __forceinline__ uint2 load_b(const uint8_t* xb, uint32_t u, const Lane& L) {
    return L.bload ? *reinterpret_cast<const uint2*>(xb + u * kXUnit + L.boff) : make_uint2(0u, 0u);
}
// byte k of w as an exact float (unsigned), or of w ^ 0x80808080 minus 128 (signed)
__device__ __forceinline__ float ubyte_f(uint32_t w, uint32_t k) {
    return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7650u | k)) - 8388608.f;
}
__device__ __forceinline__ float sbyte_f(uint32_t wx, uint32_t k) {
    return __uint_as_float(__byte_perm(wx, 0x4B000000u, 0x7650u | k)) - 8388736.f;
}

// Q4_K: one super-block (4 units from u0) of 16 rows. The qs byte holds value l of
// sub-block 2j in its low nibble and of 2j+1 in its high nibble: the low nibbles are
// masked in place (part 0), the high ones kept at 16x (part 1, wt carries the 1/16).
// acc += d*s_j*(q . x) per sub-block, minus dmin*m_j*sum(x) of sub-blocks 2t, 2t+1.
__device__ __forceinline__ void q4k_row_scales(uint4 h, const Lane& L, float wt, const float* X, float (&c)[4],
                                               float& acc) {
    const float d = h2f(h.x & 0xffff), dmin = h2f(h.x >> 16);
    const uint32_t scl = h.y & 0x3F3F3F3Fu;                                  // s_0..3
    const uint32_t sch = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);   // s_4..7
    const uint32_t mnl = h.z & 0x3F3F3F3Fu;                                  // m_0..3
    const uint32_t mnh = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);  // m_4..7
    const float dw = d * wt;
    c[0] = dw * ubyte_f(scl, L.part);
    c[1] = dw * ubyte_f(scl, 2 + L.part);
    c[2] = dw * ubyte_f(sch, L.part);
    c[3] = dw * ubyte_f(sch, 2 + L.part);
    const uint32_t mw = L.t < 2 ? mnl : mnh, k0 = (2 * L.t) & 3;
    acc -= dmin * fmaf(ubyte_f(mw, k0), X[2 * L.t], ubyte_f(mw, k0 + 1) * X[2 * L.t + 1]);
}

__device__ __forceinline__ void sb_q4k(const uint8_t* sb, uint32_t u0, const uint8_t* xb, const float* fs,
                                       const float* xsum, const Lane& L, int lane, float wt, float& acc0,
                                       float& acc1) {
    float c0[4], c1[4];
    q4k_row_scales(*reinterpret_cast<const uint4*>(sb + 2048 + L.g8 * 16), L, wt, xsum + 2 * u0, c0, acc0);
    q4k_row_scales(*reinterpret_cast<const uint4*>(sb + 2048 + (L.g8 + 8) * 16), L, wt, xsum + 2 * u0, c1, acc1);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t u = u0 + j;
        const uint4 A = *reinterpret_cast<const uint4*>(sb + j * 512 + lane * 16);
        const uint2 B = load_b(xb, u, L);
        int d[4] = {0, 0, 0, 0};
        mma_u8s8(d, A.x & 0x0F0F0F0Fu, A.y & 0x0F0F0F0Fu, A.x & 0xF0F0F0F0u, A.y & 0xF0F0F0F0u, B.x & L.mlo,
                 B.x & L.mhi);
        mma_u8s8(d, A.z & 0x0F0F0F0Fu, A.w & 0x0F0F0F0Fu, A.z & 0xF0F0F0F0u, A.w & 0xF0F0F0F0u, B.y & L.mlo,
                 B.y & L.mhi);
        const float f = fs[2 * u + L.part];
        acc0 = fmaf(c0[j] * f, (float)(d[0] + 256 * d[1]), acc0);
        acc1 = fmaf(c1[j] * f, (float)(d[2] + 256 * d[3]), acc1);
    }
}

// Q5_K: one super-block (4 units from u0) of 16 rows, as Q4_K with the fifth bit of every
// value from the lane's qh words (bit 2j of qh byte l for value l of sub-block 2j, bit
// 2j + 1 for sub-block 2j + 1, gguf.rs:373-396); the high nibbles are shifted down
// to 0..31 as well, so the lane weight has no 1/16.
__device__ __forceinline__ uint32_t q5_lo(uint32_t a, uint32_t h, uint32_t bit) {
    return (a & 0x0F0F0F0Fu) | (((h >> bit) & 0x01010101u) << 4);
}
__device__ __forceinline__ uint32_t q5_hi(uint32_t a, uint32_t h, uint32_t bit) {
    return ((a >> 4) & 0x0F0F0F0Fu) | (((h >> bit) & 0x01010101u) << 4);
}
__device__ __forceinline__ void sb_q5k(const uint8_t* sb, uint32_t u0, const uint8_t* xb, const float* fs,
                                       const float* xsum, const Lane& L, int lane, float wt, float& acc0,
                                       float& acc1) {
    float c0[4], c1[4];
    q4k_row_scales(*reinterpret_cast<const uint4*>(sb + 2560 + L.g8 * 16), L, wt, xsum + 2 * u0, c0, acc0);
    q4k_row_scales(*reinterpret_cast<const uint4*>(sb + 2560 + (L.g8 + 8) * 16), L, wt, xsum + 2 * u0, c1, acc1);
    const uint4 H = *reinterpret_cast<const uint4*>(sb + 2048 + lane * 16);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t u = u0 + j;
        const uint4 A = *reinterpret_cast<const uint4*>(sb + j * 512 + lane * 16);
        const uint2 B = load_b(xb, u, L);
        int d[4] = {0, 0, 0, 0};
        mma_u8s8(d, q5_lo(A.x, H.x, 2 * j), q5_lo(A.y, H.y, 2 * j), q5_hi(A.x, H.x, 2 * j + 1),
                 q5_hi(A.y, H.y, 2 * j + 1), B.x & L.mlo, B.x & L.mhi);
        mma_u8s8(d, q5_lo(A.z, H.z, 2 * j), q5_lo(A.w, H.w, 2 * j), q5_hi(A.z, H.z, 2 * j + 1),
                 q5_hi(A.w, H.w, 2 * j + 1), B.y & L.mlo, B.y & L.mhi);
        const float f = fs[2 * u + L.part];
        acc0 = fmaf(c0[j] * f, (float)(d[0] + 256 * d[1]), acc0);
        acc1 = fmaf(c1[j] * f, (float)(d[2] + 256 * d[3]), acc1);
    }
}

// Q6_K: one super-block of 16 rows. Step (unit j = 2H + jj, half h) holds the values
// 128H + 32kq + 16h + l', kq = 2jj (part 0) and 2jj + 1 (part 1), i.e. sub-blocks
// 4j + h and 4j + 2 + h; q = 6-bit value (u8), the -32 offset is taken off the integer
// sums with the staged limb sums of each part.
__device__ __forceinline__ void sb_q6k(const uint8_t* sb, uint32_t u0, const uint8_t* xb, const float* fs,
                                       const int* ms, const Lane& L, int lane, float wt, float& acc0, float& acc1) {
    const uint4 S0 = *reinterpret_cast<const uint4*>(sb + 3072 + L.g8 * 16);
    const uint4 S1 = *reinterpret_cast<const uint4*>(sb + 3072 + (L.g8 + 8) * 16);
    const float dA = h2f(*reinterpret_cast<const uint16_t*>(sb + 3328 + L.g8 * 2)) * wt;
    const float dB = h2f(*reinterpret_cast<const uint16_t*>(sb + 3328 + (L.g8 + 8) * 2)) * wt;
    const uint32_t sA[4] = {S0.x ^ 0x80808080u, S0.y ^ 0x80808080u, S0.z ^ 0x80808080u, S0.w ^ 0x80808080u};
    const uint32_t sB[4] = {S1.x ^ 0x80808080u, S1.y ^ 0x80808080u, S1.z ^ 0x80808080u, S1.w ^ 0x80808080u};
#pragma unroll
    for (int H = 0; H < 2; ++H) {
        const uint8_t* lp = sb + H * 1536 + lane * 48;
        const uint4 P0 = *reinterpret_cast<const uint4*>(lp);
        const uint4 P1 = *reinterpret_cast<const uint4*>(lp + 16);
        const uint4 P2 = *reinterpret_cast<const uint4*>(lp + 32);
#pragma unroll
        for (int jj = 0; jj < 2; ++jj) {
            const int j = 2 * H + jj;
            const uint32_t u = u0 + j;
            const uint2 B = load_b(xb, u, L);
            const int2 M = *reinterpret_cast<const int2*>(ms + u * 8 + L.t * 2);
            const float f = fs[2 * u + L.part];
            const float fA = dA * f, fB = dB * f;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint32_t l0a = h ? P0.y : P0.x, l0b = h ? P0.w : P0.z;  // rows g8, g8 + 8
                const uint32_t l1a = h ? P1.y : P1.x, l1b = h ? P1.w : P1.z;
                const uint32_t qa = h ? P2.y : P2.x, qb = h ? P2.w : P2.z;
                uint32_t a0, a1, a2, a3;
                if (jj == 0) {
                    a0 = (l0a & 0x0F0F0F0Fu) | ((qa << 4) & 0x30303030u);
                    a1 = (l0b & 0x0F0F0F0Fu) | ((qb << 4) & 0x30303030u);
                    a2 = (l1a & 0x0F0F0F0Fu) | ((qa << 2) & 0x30303030u);
                    a3 = (l1b & 0x0F0F0F0Fu) | ((qb << 2) & 0x30303030u);
                } else {
                    a0 = ((l0a >> 4) & 0x0F0F0F0Fu) | (qa & 0x30303030u);
                    a1 = ((l0b >> 4) & 0x0F0F0F0Fu) | (qb & 0x30303030u);
                    a2 = ((l1a >> 4) & 0x0F0F0F0Fu) | ((qa >> 2) & 0x30303030u);
                    a3 = ((l1b >> 4) & 0x0F0F0F0Fu) | ((qb >> 2) & 0x30303030u);
                }
                const uint32_t bw = h ? B.y : B.x;
                int d[4] = {0, 0, 0, 0};
                mma_u8s8(d, a0, a1, a2, a3, bw & L.mlo, bw & L.mhi);
                const int bias = 32 * (h ? M.y : M.x);
                const uint32_t k = h + 2 * L.part;  // scale byte of sub-block 4j + k in word j
                acc0 = fmaf(fA * sbyte_f(sA[j], k), (float)(d[0] + 256 * d[1] - bias), acc0);
                acc1 = fmaf(fB * sbyte_f(sB[j], k), (float)(d[2] + 256 * d[3] - bias), acc1);
            }
        }
    }
}

// Q8_0: one unit (blocks 2u = part 0, 2u + 1 = part 1) of 16 rows.
__device__ __forceinline__ void unit_q8_0(const uint8_t* ub, uint32_t u, const uint8_t* xb, const float* fs,
                                          const Lane& L, int lane, float wt, float& acc0, float& acc1) {
    const uint4 A0 = *reinterpret_cast<const uint4*>(ub + lane * 16);
    const uint4 A1 = *reinterpret_cast<const uint4*>(ub + 512 + lane * 16);
    const uint32_t dw0 = *reinterpret_cast<const uint32_t*>(ub + 1024 + L.g8 * 4);
    const uint32_t dw1 = *reinterpret_cast<const uint32_t*>(ub + 1024 + (L.g8 + 8) * 4);
    const uint2 B = load_b(xb, u, L);
    int d[4] = {0, 0, 0, 0};
    mma_s8s8(d, A0.x, A0.y, A0.z, A0.w, B.x & L.mlo, B.x & L.mhi);
    mma_s8s8(d, A1.x, A1.y, A1.z, A1.w, B.y & L.mlo, B.y & L.mhi);
    const float f = fs[2 * u + L.part] * wt;
    const float d0 = h2f(L.part ? dw0 >> 16 : dw0 & 0xffff), d1 = h2f(L.part ? dw1 >> 16 : dw1 & 0xffff);
    acc0 = fmaf(d0 * f, (float)(d[0] + 256 * d[1]), acc0);
    acc1 = fmaf(d1 * f, (float)(d[2] + 256 * d[3]), acc1);
}

// ---------------------------------------------------------------- input staging
// x (optionally RMS-normalised, src/runtime.rs:193-196) -> per 32-value block j a scale
// 2^-s and |m| <= 2^22 with x = 2^-s * m, m = l0 + 2^8 l1 + 2^16 l2 in three int8 limbs,
// written as the B fragments of the MMA steps: unit u's 192 bytes hold, for part p
// (values 64u + 32p + 16h + [0, 16) in half h) and limb l, the words of lanes
// t = 0..3 (values 4t..4t+3 of the quarter) for halves h = 0, 1 at
// ((3p + l) * 4 + t) * 8 + 4h. Each consumer thread stages one 16-value quarter from
// registers: the two quarters of a block sit in adjacent lanes and meet with one
// shuffle for the block maximum and sum.

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

// One 16-value quarter hb of the input (times the norm weight), held in v: block
// scale, limbs, sums, and the writes of the staged layouts. All lanes of the warp call
// it (the block maximum and sum meet by shuffle); `on` is uniform per lane pair.
__device__ __forceinline__ void stage_quarter(const Plan& p, uint8_t* xs, uint32_t hb, bool on, const float (&v)[16]) {
    // |x| bit patterns order like the values; the biased exponent E of the block
    // maximum puts it in [2^(E-127), 2^(E-126)), i.e. frexp's e = E - 126, and
    // s = 22 - e keeps |m| <= 2^22
    uint32_t abits = 0;
#pragma unroll
    for (int e = 0; e < 16; ++e) abits = max(abits, __float_as_uint(v[e]) & 0x7fffffffu);
    abits = max(abits, __shfl_xor_sync(0xffffffffu, abits, 1));
    const int s = abits ? min(max(148 - (int)(abits >> 23), -100), 120) : 0;
    // 2^s and 2^-s are normal floats for s in [-100, 120]: the scaling is exact, and
    // |v * 2^s| <= 2^22, so adding 1.5 * 2^23 in the same FMA leaves the integer
    // rounded to nearest even in the low mantissa bits (= __float2int_rn(v * 2^s))
    const float up = __uint_as_float((uint32_t)(s + 127) << 23);
    int m[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) m[e] = __float_as_int(__fmaf_rn(v[e], up, 12582912.0f)) - 0x4B400000;
    uint32_t L0[4], L1[4], L2[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) pack_limbs(m[4 * q], m[4 * q + 1], m[4 * q + 2], m[4 * q + 3], L0[q], L1[q], L2[q]);
    const uint32_t j = hb >> 1, h = hb & 1, u = hb >> 2, part = (hb >> 1) & 1;
    const float fs = __uint_as_float((uint32_t)(127 - s) << 23);
    if (p.need & NEED_XSUM) {  // sum of the staged (quantised) block: exact in int32
        int sm = 0;
#pragma unroll
        for (int e = 0; e < 16; ++e) sm += m[e];
        sm += __shfl_xor_sync(0xffffffffu, sm, 1);
        if (on && h == 0) reinterpret_cast<float*>(xs + p.off_xsum)[j] = __fmul_rn((float)sm, fs);
    }
    if (!on) return;
    if (h == 0) reinterpret_cast<float*>(xs + p.off_fscale)[j] = fs;
    uint8_t* b = xs + u * kXUnit + part * 96 + h * 4;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        *reinterpret_cast<uint32_t*>(b + e * 8) = L0[e];
        *reinterpret_cast<uint32_t*>(b + 32 + e * 8) = L1[e];
        *reinterpret_cast<uint32_t*>(b + 64 + e * 8) = L2[e];
    }
    if (p.need & NEED_MSUM) {  // per quarter: limb sums for the Q6_K -32 offset, as the lanes combine them
        int s0 = 0, s1 = 0, s2 = 0;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            s0 = dp4a((int)L0[q], 0x01010101, s0);
            s1 = dp4a((int)L1[q], 0x01010101, s1);
            s2 = dp4a((int)L2[q], 0x01010101, s2);
        }
        int* ms = reinterpret_cast<int*>(xs + p.off_msum) + u * 8 + part * 4 + h;  // [u][t = 2 part + (limb 2)][h]
        ms[0] = s0 + 256 * s1;
        ms[2] = s2;
    }
}

// The same for one 8-value eighth he of the input (rows of up to 4096 values take one
// eighth per consumer thread: twice the threads of quarters, half the chain each). The
// four eighths of a block sit in lanes 4k..4k+3 and meet by shuffles; eighth e8 = he & 1
// of quarter he >> 1 holds the B words of lanes t = 2 e8, 2 e8 + 1.
__device__ __forceinline__ void stage_eighth(const Plan& p, uint8_t* xs, uint32_t he, bool on, const float (&v)[8]) {
    uint32_t abits = 0;
#pragma unroll
    for (int e = 0; e < 8; ++e) abits = max(abits, __float_as_uint(v[e]) & 0x7fffffffu);
    abits = max(abits, __shfl_xor_sync(0xffffffffu, abits, 1));
    abits = max(abits, __shfl_xor_sync(0xffffffffu, abits, 2));
    const int s = abits ? min(max(148 - (int)(abits >> 23), -100), 120) : 0;  // as stage_quarter
    const float up = __uint_as_float((uint32_t)(s + 127) << 23);
    int m[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) m[e] = __float_as_int(__fmaf_rn(v[e], up, 12582912.0f)) - 0x4B400000;
    uint32_t L0[2], L1[2], L2[2];
#pragma unroll
    for (int q = 0; q < 2; ++q) pack_limbs(m[4 * q], m[4 * q + 1], m[4 * q + 2], m[4 * q + 3], L0[q], L1[q], L2[q]);
    const uint32_t hb = he >> 1, e8 = he & 1, j = hb >> 1, h = hb & 1, u = hb >> 2, part = (hb >> 1) & 1;
    const float fs = __uint_as_float((uint32_t)(127 - s) << 23);
    if (p.need & NEED_XSUM) {  // sum of the staged (quantised) block: exact in int32
        int sm = 0;
#pragma unroll
        for (int e = 0; e < 8; ++e) sm += m[e];
        sm += __shfl_xor_sync(0xffffffffu, sm, 1);
        sm += __shfl_xor_sync(0xffffffffu, sm, 2);
        if (on && (he & 3) == 0) reinterpret_cast<float*>(xs + p.off_xsum)[j] = __fmul_rn((float)sm, fs);
    }
    int s0 = 0, s1 = 0, s2 = 0;  // the quarter's limb sums (both eighths) for the Q6_K -32 offset
    if (p.need & NEED_MSUM) {
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            s0 = dp4a((int)L0[q], 0x01010101, s0);
            s1 = dp4a((int)L1[q], 0x01010101, s1);
            s2 = dp4a((int)L2[q], 0x01010101, s2);
        }
        s0 += __shfl_xor_sync(0xffffffffu, s0, 1);
        s1 += __shfl_xor_sync(0xffffffffu, s1, 1);
        s2 += __shfl_xor_sync(0xffffffffu, s2, 1);
    }
    if (!on) return;
    if ((he & 3) == 0) reinterpret_cast<float*>(xs + p.off_fscale)[j] = fs;
    uint8_t* b = xs + u * kXUnit + part * 96 + h * 4 + e8 * 16;
#pragma unroll
    for (int q = 0; q < 2; ++q) {
        *reinterpret_cast<uint32_t*>(b + q * 8) = L0[q];
        *reinterpret_cast<uint32_t*>(b + 32 + q * 8) = L1[q];
        *reinterpret_cast<uint32_t*>(b + 64 + q * 8) = L2[q];
    }
    if ((p.need & NEED_MSUM) && e8 == 0) {
        int* ms = reinterpret_cast<int*>(xs + p.off_msum) + u * 8 + part * 4 + h;  // [u][t = 2 part + (limb 2)][h]
        ms[0] = s0 + 256 * s1;
        ms[2] = s2;
    }
}

__device__ __forceinline__ void load_eighth(const float* x, uint32_t he, bool on, float (&v)[8]) {
    if (on) {
        const float4* xp = reinterpret_cast<const float4*>(x + 8 * he);
        const float4 t0 = __ldcg(xp), t1 = __ldcg(xp + 1);
        v[0] = t0.x; v[1] = t0.y; v[2] = t0.z; v[3] = t0.w; v[4] = t1.x; v[5] = t1.y; v[6] = t1.z; v[7] = t1.w;
    } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = 0.f;
    }
}

__device__ __forceinline__ void load_quarter(const float* x, uint32_t hb, bool on, float (&v)[16]) {
    if (on) {
        const float4* xp = reinterpret_cast<const float4*>(x + 16 * hb);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float4 t = __ldcg(xp + q);
            v[4 * q] = t.x; v[4 * q + 1] = t.y; v[4 * q + 2] = t.z; v[4 * q + 3] = t.w;
        }
    } else {
#pragma unroll
        for (int e = 0; e < 16; ++e) v[e] = 0.f;
    }
}
__device__ __forceinline__ void load_weights(const float* w, uint32_t hb, bool on, float (&g)[16]) {
    if (on) {
        const float4* gp = reinterpret_cast<const float4*>(w + 16 * hb);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float4 t = gp[q];
            g[4 * q] = t.x; g[4 * q + 1] = t.y; g[4 * q + 2] = t.z; g[4 * q + 3] = t.w;
        }
    }
}
__device__ __forceinline__ float sum_sq(const float (&v)[16]) {
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 16; ++e) ss += v[e] * v[e];
    return ss;
}
__device__ __forceinline__ void mul_weights(float (&v)[16], const float (&g)[16]) {
#pragma unroll
    for (int e = 0; e < 16; ++e) v[e] = __fmul_rn(v[e], g[e]);
}

// The norm weights of this consumer thread's quarters, read before
// griddepcontrol.wait (they do not depend on the previous kernel); rows of up to 1024
// quarters (16384 values) only, longer rows read them while staging.
struct NormRegs {
    float g0[16], g1[16];
};
__device__ __forceinline__ void load_norm_regs(const Plan& p, int warp, int lane, NormRegs& n) {
    const MatvecArgs& a = p.a;
    const uint32_t nq = a.cols / 16, per = kCW * 32, c = (uint32_t)(warp * 32 + lane);
    if (!a.norm_w || nq > 2 * per) return;
    if (a.cols / 8 <= kMaxEighths * per) {  // eighths c, c + per, c + 2 per: g0[0..7], g0[8..15], g1[0..7]
#pragma unroll
        for (uint32_t k = 0; k < kMaxEighths; ++k) {
            if (c + k * per >= a.cols / 8) continue;
            const float4* gp = reinterpret_cast<const float4*>(a.norm_w + 8 * (c + k * per));
            const float4 t0 = gp[0], t1 = gp[1];
            float* g = k == 2 ? n.g1 : n.g0 + 8 * k;
            g[0] = t0.x; g[1] = t0.y; g[2] = t0.z; g[3] = t0.w; g[4] = t1.x; g[5] = t1.y; g[6] = t1.z; g[7] = t1.w;
        }
        return;
    }
    load_weights(a.norm_w, c, c < nq, n.g0);
    if (nq > per) load_weights(a.norm_w, c + per, c + per < nq, n.g1);
}

// Called by the consumer threads after griddepcontrol.wait, in one pass over the row.
// With a fused RMSNorm (src/runtime.rs:193-196) the staged values are x * w and the
// returned 1/rms(x) scales each dot product in the row epilogue, so staging needs no
// barrier between the sum of squares and the writes; without a norm it returns 1.
__device__ float stage_input(const Plan& p, uint8_t* xs, int warp, int lane, float* red, const NormRegs& nr) {
    const MatvecArgs& a = p.a;
    const uint32_t K = a.cols, nq = K / 16, per = kCW * 32;
    const uint32_t c = (uint32_t)(warp * 32 + lane);  // consumer thread 0 .. kCW*32-1
    float ss = 0.f;
    if (K / 8 <= kMaxEighths * per) {  // 8-value eighths c, c + per, c + 2 per (independent chains)
        float v[kMaxEighths][8];
#pragma unroll
        for (uint32_t k = 0; k < kMaxEighths; ++k)
            if (k * per < K / 8) load_eighth(a.x, c + k * per, c + k * per < K / 8, v[k]);  // uniform test first
#pragma unroll
        for (uint32_t k = 0; k < kMaxEighths; ++k) {
            if (k * per >= K / 8) continue;
            const bool on = c + k * per < K / 8;  // uniform per block of four lanes
            if (a.norm_w) {
                const float* g = k == 2 ? nr.g1 : nr.g0 + 8 * k;
#pragma unroll
                for (int e = 0; e < 8; ++e) ss += v[k][e] * v[k][e];
                if (on) {
#pragma unroll
                    for (int e = 0; e < 8; ++e) v[k][e] = __fmul_rn(v[k][e], g[e]);
                }
            }
            stage_eighth(p, xs, c + k * per, on, v[k]);
        }
    } else if (nq <= 2 * per) {
        // nq is a multiple of 4, so a warp's 32 lanes cover whole blocks or none
        const uint32_t q0 = c, q1 = c + per;
        const bool on0 = q0 < nq, on1 = q1 < nq, two = nq > per;
        float v0[16], v1[16];
        load_quarter(a.x, q0, on0, v0);
        if (two) load_quarter(a.x, q1, on1, v1);
        if (a.norm_w) {
            ss = sum_sq(v0) + (two ? sum_sq(v1) : 0.f);
            if (on0) mul_weights(v0, nr.g0);
            if (two && on1) mul_weights(v1, nr.g1);
        }
        stage_quarter(p, xs, q0, on0, v0);
        if (two) stage_quarter(p, xs, q1, on1, v1);
    } else {
        for (uint32_t hb0 = (uint32_t)warp * 32; hb0 < nq; hb0 += per) {
            const uint32_t hb = hb0 + lane;
            const bool on = hb < nq;  // uniform per lane pair
            float v[16], g[16];
            load_quarter(a.x, hb, on, v);
            if (a.norm_w) {
                load_weights(a.norm_w, hb, on, g);
                ss += sum_sq(v);
                if (on) mul_weights(v, g);
            }
            stage_quarter(p, xs, hb, on, v);
        }
    }
    if (a.norm_w) {
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
    }
    if (c < kRedBufs) reinterpret_cast<unsigned*>(xs + p.off_red + kRedBufs * kRedBufBytes)[c] = 0u;
    named_sync(kConsumerBarrier, kCW * 32);
    if (!a.norm_w) return 1.f;
    ss = 0.f;
#pragma unroll
    for (int w = 0; w < kCW; ++w) ss += red[w];
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), a.eps)));
}


// The residual y of a single-segment EPI_ADD plan whose CTA rows fit kRowBuf, read
// into shared memory after griddepcontrol.wait (it was written by an earlier kernel)
// alongside the input staging, so the row epilogue does no dependent global load.
// Consumer thread c; visible after the staging's closing barrier.
__device__ __forceinline__ bool rows_cached(const Plan& p, uint32_t rb0, uint32_t rb1) {
    return p.a.nseg == 1 && p.a.seg[0].epi == EPI_ADD && (rb1 - rb0) * kRB <= kRowBuf;
}
__device__ __forceinline__ void prefetch_rows(const Plan& p, uint8_t* xs, uint32_t rb0, uint32_t rb1, uint32_t c) {
    if (!rows_cached(p, rb0, rb1) || c >= (rb1 - rb0) * kRB) return;
    const MatvecSeg& sg = p.a.seg[0];
    const uint32_t row = rb0 * kRB + c;
    reinterpret_cast<float*>(xs + p.off_rows)[c] = row < sg.m.rows ? __ldcg(sg.y + row) : 0.f;
}

// The first row block whose byte midpoint lies at or past c / n of the plan's weight
// bytes: row block k goes to the CTA whose equal share of the bytes holds its
// midpoint, so segments of heavier types (a Q6_K block is 1.46 Q4_K blocks) spread
// over more CTAs instead of doubling up on some.
__host__ __device__ __forceinline__ uint32_t rb_boundary(const Plan& p, uint32_t c, uint32_t n) {
    if (c >= n) return p.rb_begin[kMaxSegs];
    // 32-bit: total_w * 2 * n < 2^31 (the host picks the weight unit)
    const uint32_t t2 = 2u * c * p.total_w;  // (2 W_before + (2k + 1) w) n >= t2
    uint32_t wb = 0;
    for (int s = 0; s < kMaxSegs; ++s) {
        const uint32_t nrb = p.rb_begin[s + 1] - p.rb_begin[s], w = p.rb_w[s];
        if (nrb && (2 * wb + (2 * nrb - 1) * w) * n >= t2) {
            const uint32_t base = (2 * wb + w) * n;
            const uint32_t k = base >= t2 ? 0 : (t2 - base + 2 * w * n - 1) / (2 * w * n);
            return p.rb_begin[s] + k;
        }
        wb += nrb * w;
    }
    return p.rb_begin[kMaxSegs];
}
// This CTA's row blocks [rb0, rb1) of a plan: a contiguous range of about 1/ncta of
// the weight bytes.
__device__ __forceinline__ void cta_rows(const Plan& p, uint32_t cta, uint32_t ncta, uint32_t& rb0, uint32_t& rb1) {
    rb0 = rb_boundary(p, cta, ncta);
    rb1 = rb_boundary(p, cta + 1, ncta);
}

// Global addresses of item (rb, g): panel g of the one or two 16-row slabs one stage
// holds -- rows [32*local, +32), or gate and up rows [16*local, +16) for the SwiGLU
// pair. Returns the number of slabs (1 when the second is past the end).
__device__ __forceinline__ uint32_t item_slabs(const Plan& p, uint32_t rb, uint32_t g, const uint8_t*& a,
                                               const uint8_t*& b, uint32_t& slab_bytes) {
    const int si = seg_of(p, rb);
    const MatvecSeg& sg = p.a.seg[si];
    const uint32_t local = rb - p.rb_begin[si];
    const uint32_t T = sg.m.type;
    slab_bytes = panel_bytes(T, group_units(p.nunits, g));
    const bool dual = sg.epi == EPI_SWIGLU;
    const QMatDev& mb = dual ? sg.m2 : sg.m;
    const uint32_t sa = dual ? local : 2 * local, sbk = dual ? local : 2 * local + 1;
    a = sg.m.q + (uint64_t)sa * kSlabRows * sg.m.row_bytes + panel_offset(T, g);
    b = mb.q + (uint64_t)sbk * kSlabRows * mb.row_bytes + panel_offset(T, g);
    return sbk * kSlabRows < mb.rows ? 2 : 1;
}

// Producer: copy item (rb, g) into ring slot s, completing on full[s].
__device__ __forceinline__ void issue_item(const Plan& p, const Ring& r, uint32_t rb, uint32_t g, uint32_t s) {
    const uint8_t *a, *b;
    uint32_t sb;
    const uint32_t n = item_slabs(p, rb, g, a, b, sb);
    uint8_t* slot = r.base + s * r.slot_bytes;
    const uint64_t pol = l2_evict_first();
    mbar_arrive_expect_tx(&r.full[s], n * sb);
    tma_load_1d_hint(slot, a, sb, &r.full[s], pol);
    if (n == 2) tma_load_1d_hint(slot + sb, b, sb, &r.full[s], pol);
}

// Position in the ring sequence: items issued (or consumed) so far, the slot, and the
// parity of the slot's current lap.
struct RingPos {
    uint32_t n = 0, s = 0, par = 0;
    __device__ __forceinline__ void advance(uint32_t stages) {
        ++n;
        if (++s == stages) {
            s = 0;
            par ^= 1;
        }
    }
};

// Producer (one thread): stream row blocks [rb0, rb1) of `p`, one 32-unit panel of the
// row block's slabs per stage, continuing the ring sequence at `rp`. Returns false
// after an abort.
// Items are numbered n = (rb - rb0) * ngroups + g; a call issues items [rp.n, stop).
__device__ bool produce_items(const Plan& p, const Ring& r, uint32_t rb0, uint32_t rb1, RingPos& rp,
                              volatile int* abort_flag, uint32_t stop = 0xffffffffu) {
    const uint32_t end = min((rb1 - rb0) * p.ngroups, stop);
    uint32_t rb = rb0 + rp.n / p.ngroups, g = rp.n % p.ngroups;
    for (; rp.n < end; rp.advance(r.stages)) {
        // a slot's lap L >= 1 waits for the consumers' release of lap L - 1
        if (rp.n >= r.stages && !wait_or_abort(&r.empty[rp.s], rp.par ^ 1, abort_flag)) return false;
        if (*abort_flag) return false;
        issue_item(p, r, rb, g, rp.s);
        if (++g == p.ngroups) {
            g = 0;
            ++rb;
        }
    }
    return true;
}

// Producer, after its last copy of a plan: warm L2 with this CTA index's share of the
// next matrices, in order, at most pf_cap bytes in all. The next kernels' CTAs start
// only as this one's leave; meanwhile HBM keeps streaming their first tiles.
__device__ void prefetch_next(const Plan& p, uint32_t cta, uint32_t ncta) {
    uint64_t left = p.pf_cap;
    for (int i = 0; i < 3 && left; ++i) {
        if (!p.pf_base[i] || !p.pf_rows[i]) continue;
        const uint32_t slabs = (p.pf_rows[i] + kSlabRows - 1) / kSlabRows;
        const uint32_t pr0 = (uint32_t)(((uint64_t)slabs * cta) / ncta);
        const uint32_t pr1 = (uint32_t)(((uint64_t)slabs * (cta + 1)) / ncta);
        uint64_t bytes = (uint64_t)(pr1 - pr0) * kSlabRows * p.pf_row_bytes[i];
        if (bytes > left) bytes = left;
        left -= bytes;
        const uint8_t* base = p.pf_base[i] + (uint64_t)pr0 * kSlabRows * p.pf_row_bytes[i];
        for (uint64_t o = 0; o < bytes; o += 16384)
            prefetch_l2_bulk(base + o, (uint32_t)((bytes - o) < 16384 ? (bytes - o) & ~15ull : 16384));
    }
}

// Producer: after an abort, give the copies in flight a bounded chance to land.
__device__ void drain_ring(const Ring& r, uint32_t item) {
    for (uint32_t s = 0; s < r.stages && s < item; ++s) mbar_wait(&r.full[s], ((item - 1 - s) / r.stages) & 1);
}

// One consumer warp's part of a row block of type T: for every panel, super-block
// `sbw` of slab `slab` (or the Q8_0 units of it). Returns false after an abort.
template <uint32_t T>
__device__ __forceinline__ bool consume_rows(const Plan& p, const Ring& r, const uint8_t* xs, RingPos& rp,
                                             uint32_t slab, uint32_t sbw, const Lane& L, int lane,
                                             volatile int* abort_flag, float& acc0, float& acc1) {
    constexpr uint32_t u16 = T == GGML_Q4_K ? 576u : T == GGML_Q5_K ? 704u : T == GGML_Q6_K ? 840u : 1088u;
    const uint8_t* xb = xs;
    const float* fscale = reinterpret_cast<const float*>(xs + p.off_fscale);
    // limb weight of this lane's D columns (and the 16x of Q4_K high nibbles)
    const float wt = ((L.t & 1) ? 65536.f : 1.f) * ((T == GGML_Q4_K && L.part) ? 0.0625f : 1.f);
    for (uint32_t g = 0; g < p.ngroups; ++g, rp.advance(r.stages)) {
        if (!wait_or_abort(&r.full[rp.s], rp.par, abort_flag)) return false;
        const uint32_t U = g + 1 == p.ngroups ? p.last_units : kPanelUnits, ub = 4 * sbw;
        // rows past the end were not copied: their slots hold stale bytes whose
        // (finite) results are discarded by the epilogue
        const uint8_t* q = r.base + rp.s * r.slot_bytes + slab * U * u16 + ub * u16;
        const uint32_t u0 = g * kPanelUnits + ub;
        if (ub < U) {
            if constexpr (T == GGML_Q4_K) {
                sb_q4k(q, u0, xb, fscale, reinterpret_cast<const float*>(xs + p.off_xsum), L, lane, wt, acc0, acc1);
            } else if constexpr (T == GGML_Q5_K) {
                sb_q5k(q, u0, xb, fscale, reinterpret_cast<const float*>(xs + p.off_xsum), L, lane, wt, acc0, acc1);
            } else if constexpr (T == GGML_Q6_K) {
                sb_q6k(q, u0, xb, fscale, reinterpret_cast<const int*>(xs + p.off_msum), L, lane, wt, acc0, acc1);
            } else {
#pragma unroll
                for (uint32_t i = 0; i < 4; ++i)
                    if (ub + i < U) unit_q8_0(q + i * 1088, u0 + i, xb, fscale, L, lane, wt, acc0, acc1);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&r.empty[rp.s]);
    }
    return true;
}

// Row slot i (0 .. kRB-1) of row block rb (CTA range from rb0): the eight super-block
// warps' partials in `rd` added in warp order, scaled by the norm's 1/rms `inv`, and
// the segment's epilogue (store, residual add, or SiLU(gate) * up for slots < 16).
__device__ __forceinline__ void finish_row(const Plan& p, const uint8_t* xs, const float* rd, uint32_t rb, uint32_t rb0,
                                           uint32_t i, float inv, bool cached) {
    const int si = seg_of(p, rb);
    const MatvecSeg& sg = p.a.seg[si];
    const uint32_t local = rb - p.rb_begin[si];
    auto sum = [&](uint32_t k) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kSbWarps; ++w) v += rd[w * kRB + k];
        return __fmul_rn(v, inv);
    };
    if (sg.epi == EPI_SWIGLU) {
        const uint32_t row = local * kSlabRows + i;
        if (i < kSlabRows && row < sg.m.rows) sg.y[row] = __fmul_rn(silu(sum(i)), sum(i + kSlabRows));
    } else {
        const uint32_t row = local * kRB + i;
        if (row < sg.m.rows) {
            const float v = sum(i);
            if (sg.epi == EPI_ADD)
                sg.y[row] = (cached ? reinterpret_cast<const float*>(xs + p.off_rows)[(rb - rb0) * kRB + i]
                                    : __ldcg(sg.y + row)) + v;
            else sg.y[row] = v;
        }
    }
}

// Consumers (all kCW warps): dot products of row blocks [rb0, rb1) against the staged
// input `xs`; warp (slab w / 8, super-block w % 8) of every stage. At the end of a row
// block each warp parks its partial sums of the block's rows in a shared buffer.
// When the CTA's row blocks fit the kRedBufs buffers, every block has its own and the
// rows are finished after the last block by all consumer threads at once. Otherwise
// the buffers rotate and the last warp to arrive at a block adds its partials and runs
// the epilogue, with no CTA-wide barrier. (A warp is at most `stages` items, so at
// most `stages` row blocks, ahead of the slowest one, and stages < kRedBufs, so a
// buffer is reused only after its last reader is done.) `inv` is staging's 1/rms.
// Returns false after an abort (every consumer warp returns at the same stage).
__device__ bool consume_items(const Plan& p, const Ring& r, uint8_t* xs, uint32_t rb0, uint32_t rb1, RingPos& rp,
                              int warp, int lane, volatile int* abort_flag, float inv) {
    float* red = reinterpret_cast<float*>(xs + p.off_red);
    unsigned* cnt = reinterpret_cast<unsigned*>(xs + p.off_red + kRedBufs * kRedBufBytes);
    const Lane L = make_lane(lane);
    const uint32_t slab = (uint32_t)warp / kSbWarps, sbw = (uint32_t)warp % kSbWarps;
    const bool cached = rows_cached(p, rb0, rb1);
    const bool deferred = rb1 - rb0 <= kRedBufs;
    for (uint32_t rb = rb0; rb < rb1; ++rb) {
        const MatvecSeg& sg = p.a.seg[seg_of(p, rb)];
        float acc0 = 0.f, acc1 = 0.f;  // rows g8 and g8 + 8 of this warp's slab
        bool ok;
        switch (sg.m.type) {
            case GGML_Q4_K: ok = consume_rows<GGML_Q4_K>(p, r, xs, rp, slab, sbw, L, lane, abort_flag, acc0, acc1); break;
            case GGML_Q5_K: ok = consume_rows<GGML_Q5_K>(p, r, xs, rp, slab, sbw, L, lane, abort_flag, acc0, acc1); break;
            case GGML_Q6_K: ok = consume_rows<GGML_Q6_K>(p, r, xs, rp, slab, sbw, L, lane, abort_flag, acc0, acc1); break;
            default: ok = consume_rows<GGML_Q8_0>(p, r, xs, rp, slab, sbw, L, lane, abort_flag, acc0, acc1);
        }
        if (!ok) return false;
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
        finish_row(p, xs, rd, rb, rb0, (uint32_t)lane, inv, cached);  // lane = row slot of the block
    }
    if (deferred) {
        named_sync(kConsumerBarrier, kCW * 32);
        const uint32_t c = (uint32_t)(warp * 32 + lane);
        if (c < (rb1 - rb0) * kRB)
            finish_row(p, xs, red + (c / kRB) * (kSbWarps * kRB), rb0 + c / kRB, rb0, c % kRB, inv, cached);
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
    if (!a.x || misaligned(a.x) || misaligned(a.norm_w)) return cudaErrorMisalignedAddress;
    p = Plan{};
    p.a = a;
    p.err = a.err;
    p.nunits = a.cols / 64;
    p.ngroups = (p.nunits + 31) / 32;
    p.last_units = group_units(p.nunits, p.ngroups - 1);
    uint32_t slot = 0;
    p.rb_begin[0] = 0;
    for (int i = 0; i < kMaxSegs; ++i) {
        uint32_t rbs = 0;
        if (i < a.nseg) {
            const MatvecSeg& sg = a.seg[i];
            const uint32_t t = sg.m.type;
            if (t != GGML_Q4_K && t != GGML_Q5_K && t != GGML_Q6_K && t != GGML_Q8_0) return cudaErrorInvalidValue;
            if (sg.m.cols != a.cols || sg.m.rows == 0 || sg.m.row_bytes == 0 || !sg.y) return cudaErrorInvalidValue;
            if (sg.epi == EPI_SWIGLU && (sg.m2.type != t || sg.m2.rows != sg.m.rows || sg.m2.cols != a.cols))
                return cudaErrorInvalidValue;
            if (t == GGML_Q6_K) p.need |= NEED_MSUM;
            if (t == GGML_Q4_K || t == GGML_Q5_K) p.need |= NEED_XSUM;
            slot = std::max(slot, 2 * panel_bytes(t, kPanelUnits));
            const uint32_t per = sg.epi == EPI_SWIGLU ? kRB / 2 : kRB;
            rbs = (sg.m.rows + per - 1) / per;
        }
        p.rb_begin[i + 1] = p.rb_begin[i] + rbs;
    }
    // row-block weights in units of 2^sh bytes, small enough for 32-bit boundaries
    for (uint32_t sh = 0; sh < 40; ++sh) {
        uint64_t tot = 0;
        for (int i = 0; i < a.nseg; ++i) {
            p.rb_w[i] = (uint32_t)std::max<uint64_t>(1, ((uint64_t)kRB * a.seg[i].m.row_bytes) >> sh);
            tot += (uint64_t)(p.rb_begin[i + 1] - p.rb_begin[i]) * p.rb_w[i];
        }
        if (tot * 2 * kMaxCtas < (1ull << 31)) {
            p.total_w = (uint32_t)tot;
            break;
        }
        if (sh == 39) return cudaErrorInvalidValue;
    }
    const uint32_t K = a.cols, nb = K / 32;
    uint32_t off = p.nunits * kXUnit;  // B fragments
    p.off_fscale = off;
    off += nb * 4;
    p.off_xsum = off;
    if (p.need & NEED_XSUM) off += nb * 4;
    p.off_msum = off;
    if (p.need & NEED_MSUM) off += p.nunits * 32;
    p.off_red = (off + 15) & ~15u;
    off = p.off_red + kRedBytes;
    p.off_rows = off;
    off += kRowBuf * 4;
    p.xbytes = (off + 127) & ~127u;
    p.item_bytes = slot;
    if (p.xbytes + 2 * slot > kSmemBudget) return cudaErrorInvalidValue;
    for (int i = 0; i < 3; ++i) {
        p.pf_base[i] = a.prefetch[i].q;
        p.pf_row_bytes[i] = a.prefetch[i].row_bytes;
        p.pf_rows[i] = a.prefetch[i].q ? a.prefetch[i].rows : 0;
    }
    p.pf_cap = a.prefetch_bytes;
    return cudaSuccess;
}

}  // namespace
}  // namespace mv
}  // namespace evl
