// qgemm.cu -- batched decode products Y[s][r] = sum_k W[r][k] X[s][k] for up to 32
// sequences on the 5th-generation tensor cores (tcgen05), for Batch steps (the
// reference runs one Session::step per sequence, src/runtime.rs:773-808, each doing
// QMatrix::matvec, :72-88).
//
// Weights: a second, GEMM-shaped copy of every matrix, made on the device from the
// matvec layout (gemm_repack_kernel): per 128-row M tile and 256-value K chunk one
// contiguous block holding the original quant bytes of those rows, split by field
// (Q4_K: d|dmin, scales, qs; Q6_K: ql, qh, scales, d; Q8_0: d x 8, qs) with 16-byte
// chunks XOR-swizzled by row so a warp reading 32 rows at once hits 32 banks.
//
// Inputs: x of every sequence (optionally RMS-normalised, src/runtime.rs:193-196)
// becomes f16 hi + lo parts, x * 2^e = hi + lo exactly to ~22 bits, laid out as the
// MMA's B operand (K-major canonical core matrices, N = 2 x sequences padded to 8),
// one 34 KB block per K chunk (gemm_stage_x_kernel).
//
// Kernel (one CTA per SM, items = (M tile, K range)):
//   warp 0    TMA producer: weight block + x block of each chunk into a 3-stage ring;
//   warp 1    TMEM owner and MMA issuer (one thread): tcgen05.mma kind::f16 with A in
//             tensor memory, B from shared memory, f32 accumulators in tensor memory;
//   warps 2-9 dequantisation and epilogue, one row (TMEM lane) per thread: the quant
//             values times their integer sub-block scale are exact in f16 (Q4_K
//             q*s <= 945; Q6_K q*sc as two planes q*(sc & 15) and q*16*(sc >> 4);
//             Q8_0 q), written to tensor memory with tcgen05.st; the f16/f32 scales
//             (Q4_K d, dmin; Q6_K d; Q8_0 d per 32) are applied when the accumulators of
//             one scale span are read back (tcgen05.ld). The Q4_K -dmin*m term is one
//             more MMA per chunk against per-sub-block sums of x.
// The tensor cores multiply exact integers by the 22-bit x parts and accumulate in
// f32, so the result differs from the reference's sequential f32 sum only by
// rounding order and the 2^-22-relative split of x.
// Split K ranges write partial sums; gemm_reduce_kernel adds them in a fixed order
// and applies the epilogue (store, residual add, SwiGLU).
// Every wait is bounded; on a timeout the CTA raises the error flag, lets its copies
// and MMAs land, frees its tensor memory and leaves.
#include <algorithm>
#include <atomic>
#include <cooperative_groups.h>
#include <cstdlib>

#include "common.cuh"
#include "dequant.cuh"
#include "kernels.h"

namespace evl {

namespace {

constexpr uint32_t kMT = 128;          // rows per M tile (TMEM lanes)
constexpr uint32_t kChunk = 256;       // values per K chunk
constexpr uint32_t kMathWarps = 16;   // four groups of four (one warp per TMEM lane quadrant)
constexpr uint32_t kGroups = kMathWarps / 4;
constexpr uint32_t kGemmThreads = 64 + 32 * kMathWarps;  // producer, MMA, math warps
constexpr uint32_t kMaxStages = 4;     // weight + x stages in shared memory (as many as fit)
constexpr uint32_t kASlots = 7;        // A operand slots in TMEM, 32 columns each
constexpr uint32_t kTmemCols = 512;
// TMEM column map: A slots [0, 224), min-term A 2 x 8 [224, 240), accumulator slots
// 4 x 64 [256, 512) (per slot: the product at +0, the Q4_K min term at +32)
constexpr uint32_t kColA = 0, kColD = 256;
constexpr uint32_t kDSlots = 4, kDCols = 64;
constexpr uint32_t kLag = 2;  // accumulator spans between an MMA and its read-back

__host__ __device__ inline uint32_t gemm_block_bytes(uint32_t type) {
    switch (type) {
        case GGML_Q4_K: return kMT * 144;  // 512 d|dmin + 1536 scales + 16384 qs
        case GGML_Q6_K: return kMT * 210;  // 16384 ql + 8192 qh + 2048 scales + 256 d
        case GGML_Q8_0: return kMT * 272;  // 2048 d + 32768 qs
        default: return 0;
    }
}
// staged x per K chunk: 16 B tiles of N x 16 f16 (hi rows, then lo rows), then the f32
// sums of x over each 32-value sub-block, [8][nsp] (the Q4_K min term)
__host__ __device__ inline uint32_t gemm_xchunk_bytes(uint32_t nsp) { return 16u * (2 * nsp) * 32u + 8u * nsp * 4u; }

// position of value kk (0..15) of a 16-value K step inside the MMA's K order: the
// dequantisers pack values (4a, 4a+2) and (4a+1, 4a+3) into one 32-bit column each
__device__ __forceinline__ uint32_t kslot(uint32_t kk) {
    const uint32_t r = kk & 3;
    return (kk & ~3u) | (r == 1 ? 2u : r == 2 ? 1u : r);
}
// byte offset of element (n, slot) in a K-major canonical tile (8x16 B core matrices,
// K-adjacent cores 128 B apart, 8-row groups 256 B apart)
__device__ __forceinline__ uint32_t bt_off(uint32_t n, uint32_t slot) {
    return (n >> 3) * 256u + (slot >> 3) * 128u + (n & 7u) * 16u + (slot & 7u) * 2u;
}

// ------------------------------------------------------------------ PTX wrappers (tcgen05)
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// D[128 x N] (+)= A[128 x 16] (TMEM) x B[N x 16]^T (shared memory descriptor)
__device__ __forceinline__ void mma_tmem_a(uint32_t d, uint32_t a, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}" ::"r"(d),
        "r"(a), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
}
// arrive on `bar` once every tcgen05 operation this thread issued so far has completed
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_st16(uint32_t t, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            t),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}
__device__ __forceinline__ void tmem_ld8(uint32_t t, uint32_t (&v)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
                 : "r"(t)
                 : "memory");
}
__device__ __forceinline__ void tmem_ld4(uint32_t t, uint32_t (&v)[8]) {  // columns 0..3 of v
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3])
                 : "r"(t)
                 : "memory");
}
// shared-memory matrix descriptor: K-major, no swizzle, LBO 128 B, SBO 256 B
__device__ __forceinline__ uint64_t bdesc(const void* p) {
    const uint64_t a = (smem_addr(p) & 0x3FFFFu) >> 4;
    return a | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(256 >> 4) << 32) | (1ull << 46);
}
// instruction descriptor: kind::f16, f16 A and B (K-major), f32 D, M = 128, N
__host__ __device__ inline uint32_t mma_idesc(uint32_t n) {
    return (1u << 4) | ((n >> 3) << 17) | ((kMT >> 4) << 24);
}

// two 10-bit unsigned integers in the low 10 bits of each half -> exact f16 pair,
// times (s, s) minus (bias, bias): (1024 + v) * s - 1024 * s = v * s, one rounding of
// an exact value (all terms < 65504)
// Exact conversions on the FMA and ALU pipes instead of the conversion unit: an
// integer 0 <= k < 1024 sits in the mantissa of half 1024 + k (0x6400 | k), and
// 0 <= k < 2^23 in that of float 2^23 + k.
__device__ __forceinline__ uint32_t small_int_h2(uint32_t k) {  // half2(k, k)
    const uint32_t h = 0x64006400u | (k * 0x00010001u);
    const uint32_t c = 0x64006400u;  // half2(1024, 1024)
    __half2 r = __hsub2(*reinterpret_cast<const __half2*>(&h), *reinterpret_cast<const __half2*>(&c));
    return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ uint32_t hmul2_bits(uint32_t a, uint32_t b) {
    __half2 r = __hmul2(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ float small_int_f(uint32_t k) { return __uint_as_float(0x4B000000u | k) - 8388608.f; }

__device__ __forceinline__ uint32_t magic_fma(uint32_t v2, uint32_t s2, uint32_t b2) {
    const uint32_t h = v2 | 0x64006400u;
    __half2 r = __hfma2(*reinterpret_cast<const __half2*>(&h), *reinterpret_cast<const __half2*>(&s2),
                        *reinterpret_cast<const __half2*>(&b2));
    return *reinterpret_cast<uint32_t*>(&r);
}

// ------------------------------------------------------------------ device repack
// One thread per (row, K chunk): copies the chunk's original block bytes out of the
// matvec layout (block_byte_address) into the GEMM block.
__device__ __forceinline__ uint32_t ld_word(const QMatDev& m, uint32_t r, uint32_t b, uint32_t o) {
    const uint8_t* p = m.q + block_byte_address(m, r, b, o);
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}
// 16 GGUF bytes o..o+15 of block b (four payload words)
__device__ __forceinline__ uint4 ld_piece(const QMatDev& m, uint32_t r, uint32_t b, uint32_t o) {
    return make_uint4(ld_word(m, r, b, o), ld_word(m, r, b, o + 4), ld_word(m, r, b, o + 8), ld_word(m, r, b, o + 12));
}

__global__ void gemm_repack_kernel(const QMatDev src, QGemmDev dst) {
    const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const uint64_t rows_pad = (uint64_t)dst.mtiles * kMT;
    if (idx >= rows_pad * dst.nchunks) return;
    const uint32_t r = (uint32_t)(idx % rows_pad), c = (uint32_t)(idx / rows_pad);
    const uint32_t t = r % kMT, mt = r / kMT, T = src.type;
    uint8_t* blk = const_cast<uint8_t*>(dst.q) + ((uint64_t)mt * dst.nchunks + c) * dst.block_bytes;
    const bool live = r < src.rows;
    const uint4 zero = make_uint4(0, 0, 0, 0);
    if (T == GGML_Q4_K) {
        uint8_t head[16];
        uint4 qs[8];
        if (live) {
            const uint8_t* h = src.q + block_byte_address(src, r, c, 0);
            for (int i = 0; i < 16; ++i) head[i] = h[i];
            for (uint32_t q = 0; q < 8; ++q) qs[q] = ld_piece(src, r, c, 16 + 16 * q);
        } else {
            for (int i = 0; i < 16; ++i) head[i] = 0;
            for (int q = 0; q < 8; ++q) qs[q] = zero;
        }
        for (int i = 0; i < 4; ++i) blk[t * 4 + i] = head[i];
        for (int i = 0; i < 12; ++i) blk[512 + t * 12 + i] = head[4 + i];
        for (uint32_t q = 0; q < 8; ++q) *reinterpret_cast<uint4*>(blk + 2048 + t * 128 + ((q ^ (t & 7)) * 16)) = qs[q];
    } else if (T == GGML_Q6_K) {
        // ql pieces i (bytes 16i..16i+15 of ql[128]), qh pieces k (of qh[64])
        for (uint32_t i = 0; i < 8; ++i)
            *reinterpret_cast<uint4*>(blk + t * 128 + ((i ^ (t & 7)) * 16)) = live ? ld_piece(src, r, c, 16 * i) : zero;
        for (uint32_t k = 0; k < 4; ++k)
            *reinterpret_cast<uint4*>(blk + 16384 + t * 64 + ((k ^ ((t >> 1) & 3)) * 16)) =
                live ? ld_piece(src, r, c, 128 + 16 * k) : zero;
        const uint8_t* sc = src.q + block_byte_address(src, r, c, 192);
        for (uint32_t i = 0; i < 16; ++i) blk[24576 + t * 16 + i] = live ? sc[i] : (uint8_t)0;
        const uint8_t* dp = src.q + block_byte_address(src, r, c, 208);
        *reinterpret_cast<uint16_t*>(blk + 26624 + t * 2) = live ? (uint16_t)(dp[0] | (dp[1] << 8)) : (uint16_t)0;
    } else {  // Q8_0: units 4c..4c+3, two 32-value blocks each
        for (uint32_t j = 0; j < 4; ++j) {
            const uint32_t b0 = 2 * (4 * c + j);
            uint32_t dw = 0;
            uint4 q[4] = {zero, zero, zero, zero};
            if (live) {
                const uint8_t* d0 = src.q + block_byte_address(src, r, b0, 0);
                const uint8_t* d1 = src.q + block_byte_address(src, r, b0 + 1, 0);
                dw = (uint32_t)d0[0] | ((uint32_t)d0[1] << 8) | ((uint32_t)d1[0] << 16) | ((uint32_t)d1[1] << 24);
                for (uint32_t k = 0; k < 4; ++k) q[k] = ld_piece(src, r, b0 + (k >> 1), 2 + 16 * (k & 1));
            }
            *reinterpret_cast<uint32_t*>(blk + t * 16 + j * 4) = dw;  // d of blocks 2j, 2j+1
            for (uint32_t k = 0; k < 4; ++k) {
                const uint32_t ci = 4 * j + k;  // 16-byte piece of the chunk's 256 qs bytes
                *reinterpret_cast<uint4*>(blk + 2048 + t * 256 + (((ci & 8) | ((ci & 7) ^ (t & 7))) * 16)) = q[k];
            }
        }
    }
}

// ------------------------------------------------------------------ x staging
// Two launches: per sequence (CTA s < nsp) the RMS scale and the power of two that
// brings max|x| just under 2^14 (stats[2s] = inv, stats[2s+1] = 2^e, xinv[s] = 2^-e);
// then one CTA per (sequence, K chunk) writes that chunk's hi/lo f16 B rows s and
// nsp + s and the Q4_K min-term sums. Sequences >= nseq are zero rows.
__device__ __forceinline__ float staged_val(const GemmX& a, const float* x, uint32_t i, float inv) {
    float v = x[i];
    if (a.norm_w) v = __fmul_rn(__fmul_rn(v, inv), a.norm_w[i]);
    return v;
}

constexpr uint32_t kStatsThreads = 1024, kStatsPer = 16;  // rows of up to 16384 values in registers

// One CTA per sequence: x (and the norm weights, loaded before the dependency wait)
// read once into registers, then two block reductions (sum of squares, maximum).
// Longer rows take the loop below.
__global__ void __launch_bounds__(kStatsThreads) gemm_stage_stats_kernel(const GemmX a) {
    const uint32_t s = blockIdx.x, K = a.cols, tid = threadIdx.x, nt = blockDim.x;
    __shared__ float red[32];
    const bool inreg = K <= nt * kStatsPer;
    float v[kStatsPer], g[kStatsPer];
    if (inreg && a.norm_w) {
#pragma unroll
        for (uint32_t i = 0; i < kStatsPer; ++i) g[i] = tid + i * nt < K ? a.norm_w[tid + i * nt] : 0.f;
    }
    pdl_wait();
    const bool live = s < a.nseq;
    if (!live && !inreg) return;  // the whole CTA (padding rows are staged by gemm_stage_x_kernel)
    const float* x = a.x + (uint64_t)(live ? s : 0) * a.x_stride;
    auto block_sum = [&](float t) {
        t = warp_sum(t);
        __syncthreads();
        if ((tid & 31) == 0) red[tid >> 5] = t;
        __syncthreads();
        float r = 0.f;
        for (uint32_t w = 0; w < nt / 32; ++w) r += red[w];
        return r;
    };
    auto block_max = [&](float t) {
        t = warp_max(t);
        __syncthreads();
        if ((tid & 31) == 0) red[tid >> 5] = t;
        __syncthreads();
        float r = 0.f;
        for (uint32_t w = 0; w < nt / 32; ++w) r = fmaxf(r, red[w]);
        return r;
    };
    float inv = 1.f, mx = 0.f;
    if (inreg) {
#pragma unroll
        for (uint32_t i = 0; i < kStatsPer; ++i) v[i] = live && tid + i * nt < K ? x[tid + i * nt] : 0.f;
        if (a.norm_w) {
            float ss = 0.f;
#pragma unroll
            for (uint32_t i = 0; i < kStatsPer; ++i) ss += v[i] * v[i];
            const float t = block_sum(ss);
            inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)K), a.eps)));
#pragma unroll
            for (uint32_t i = 0; i < kStatsPer; ++i) v[i] = __fmul_rn(__fmul_rn(v[i], inv), g[i]);  // staged_val
        }
#pragma unroll
        for (uint32_t i = 0; i < kStatsPer; ++i) mx = fmaxf(mx, fabsf(v[i]));
    } else {
        if (a.norm_w) {
            float ss = 0.f;
            for (uint32_t i = tid; i < K; i += nt) ss += x[i] * x[i];
            const float t = block_sum(ss);
            inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)K), a.eps)));
        }
        for (uint32_t i = tid; i < K; i += nt) mx = fmaxf(mx, fabsf(staged_val(a, x, i, inv)));
    }
    const float t = block_max(mx);
    int e = 0;
    if (t > 0.f) frexpf(t, &e);  // t in [2^(e-1), 2^e)
    const int sc = max(-100, min(100, 14 - e));  // |x| * 2^sc < 2^14
    if (tid == 0 && live) {
        a.stats[2 * s] = inv;
        a.stats[2 * s + 1] = ldexpf(1.0f, sc);
        a.xinv[s] = ldexpf(1.0f, -sc);
    }
    if (!inreg) return;
    // rows held in registers are staged here as well (gemm_stage_x_kernel's layout:
    // value k of chunk c as f16 hi/lo B rows s and nsp + s, the Q4_K min-term sums);
    // padding sequences s >= nseq stage zeros
    const float up = ldexpf(1.0f, sc);
    const uint32_t nsp = a.nsp, N = 2 * nsp;
#pragma unroll
    for (uint32_t i = 0; i < kStatsPer; ++i) {
        const uint32_t k = tid + i * nt;
        if (i * nt >= K) break;  // uniform
        const float val = k < K ? __fmul_rn(v[i], up) : 0.f;
        const __half hi = __float2half_rn(val);
        const __half lo = __float2half_rn(val - __half2float(hi));
        uint8_t* chunk = a.bx + (uint64_t)(k / kChunk) * gemm_xchunk_bytes(nsp);
        const uint32_t kc = k % kChunk;
        uint8_t* tile = chunk + (kc / 16) * (N * 32u);
        const uint32_t sl = kslot(kc % 16);
        if (k < K) {
            *reinterpret_cast<__half*>(tile + bt_off(s, sl)) = hi;
            *reinterpret_cast<__half*>(tile + bt_off(nsp + s, sl)) = lo;
        }
        const float sm = warp_sum(val);  // the warp's 32 values are one sub-block
        if (k < K && (k & 31) == 0) reinterpret_cast<float*>(chunk + 16 * (N * 32u))[(kc / 32) * nsp + s] = sm;
    }
    pdl_launch_dependents();
}

// The same statistics and staging with a row split over a cluster of kStageSplit CTAs
// (rows of K % (kStageSplit * 256) == 0 values, at most kStatsThreads * kStatsPer per
// CTA): CTA rank r reads and stages values [r K / S, (r + 1) K / S) of its sequence. The
// row's sum of squares and maximum meet over distributed shared memory, every CTA
// storing its block total into slot `rank` of every CTA of the cluster and adding the
// slots in rank order.
constexpr uint32_t kStageSplit = 4;
__global__ void __launch_bounds__(kStatsThreads) gemm_stage_cluster_kernel(const GemmX a) {
    namespace cg = cooperative_groups;
    cg::cluster_group cl = cg::this_cluster();
    const uint32_t rank = blockIdx.x % kStageSplit, s = blockIdx.x / kStageSplit;
    const uint32_t K = a.cols, Kp = K / kStageSplit, k0 = rank * Kp, tid = threadIdx.x, nt = blockDim.x;
    __shared__ float red[32];
    __shared__ float xch[2][kStageSplit];  // per rank: sum of squares, maximum
    auto block_reduce = [&](float t, bool is_max) {
        t = is_max ? warp_max(t) : warp_sum(t);
        __syncthreads();
        if ((tid & 31) == 0) red[tid >> 5] = t;
        __syncthreads();
        float r = 0.f;
        for (uint32_t w = 0; w < nt / 32; ++w) r = is_max ? fmaxf(r, red[w]) : r + red[w];
        return r;
    };
    float v[kStatsPer], g[kStatsPer];
    if (a.norm_w) {
#pragma unroll
        for (uint32_t i = 0; i < kStatsPer; ++i) g[i] = tid + i * nt < Kp ? a.norm_w[k0 + tid + i * nt] : 0.f;
    }
    pdl_wait();
    const bool live = s < a.nseq;  // padding sequences stage zeros
    const float* x = a.x + (uint64_t)(live ? s : 0) * a.x_stride;
#pragma unroll
    for (uint32_t i = 0; i < kStatsPer; ++i) v[i] = live && tid + i * nt < Kp ? x[k0 + tid + i * nt] : 0.f;
    float inv = 1.f;
    if (a.norm_w) {
        float ss = 0.f;
#pragma unroll
        for (uint32_t i = 0; i < kStatsPer; ++i) ss += v[i] * v[i];
        const float t = block_reduce(ss, false);
        if (tid < kStageSplit) *cl.map_shared_rank(&xch[0][rank], tid) = t;
        cl.sync();
        float tot = 0.f;
        for (uint32_t r = 0; r < kStageSplit; ++r) tot += xch[0][r];
        inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)K), a.eps)));
#pragma unroll
        for (uint32_t i = 0; i < kStatsPer; ++i) v[i] = __fmul_rn(__fmul_rn(v[i], inv), g[i]);  // staged_val
    }
    float mx = 0.f;
#pragma unroll
    for (uint32_t i = 0; i < kStatsPer; ++i) mx = fmaxf(mx, fabsf(v[i]));
    const float tm = block_reduce(mx, true);
    if (tid < kStageSplit) *cl.map_shared_rank(&xch[1][rank], tid) = tm;
    cl.sync();
    float T = 0.f;
    for (uint32_t r = 0; r < kStageSplit; ++r) T = fmaxf(T, xch[1][r]);
    int e = 0;
    if (T > 0.f) frexpf(T, &e);  // T in [2^(e-1), 2^e)
    const int sc = max(-100, min(100, 14 - e));  // |x| * 2^sc < 2^14
    if (rank == 0 && tid == 0 && live) {
        a.stats[2 * s] = inv;
        a.stats[2 * s + 1] = ldexpf(1.0f, sc);
        a.xinv[s] = ldexpf(1.0f, -sc);
    }
    const float up = ldexpf(1.0f, sc);
    const uint32_t nsp = a.nsp, N = 2 * nsp;
#pragma unroll
    for (uint32_t i = 0; i < kStatsPer; ++i) {
        if (i * nt >= Kp) break;  // uniform
        const bool in = tid + i * nt < Kp;
        const uint32_t k = k0 + tid + i * nt;
        const float val = in ? __fmul_rn(v[i], up) : 0.f;
        const __half hi = __float2half_rn(val);
        const __half lo = __float2half_rn(val - __half2float(hi));
        uint8_t* chunk = a.bx + (uint64_t)(k / kChunk) * gemm_xchunk_bytes(nsp);
        const uint32_t kc = k % kChunk;
        uint8_t* tile = chunk + (kc / 16) * (N * 32u);
        const uint32_t sl = kslot(kc % 16);
        if (in) {
            *reinterpret_cast<__half*>(tile + bt_off(s, sl)) = hi;
            *reinterpret_cast<__half*>(tile + bt_off(nsp + s, sl)) = lo;
        }
        const float sm = warp_sum(val);  // the warp's 32 values are one sub-block
        if (in && (k & 31) == 0) reinterpret_cast<float*>(chunk + 16 * (N * 32u))[(kc / 32) * nsp + s] = sm;
    }
    pdl_launch_dependents();
}

// grid (nsp, K / 256), 256 threads: thread k stages value k of the chunk
__global__ void gemm_stage_x_kernel(const GemmX a) {
    const uint32_t s = blockIdx.x, c = blockIdx.y, k = threadIdx.x, nsp = a.nsp, N = 2 * nsp;
    pdl_wait();
    const bool live = s < a.nseq;
    float v = 0.f;
    if (live) {
        const float* x = a.x + (uint64_t)s * a.x_stride;
        v = __fmul_rn(staged_val(a, x, c * kChunk + k, a.stats[2 * s]), a.stats[2 * s + 1]);
    }
    const __half hi = __float2half_rn(v);
    const __half lo = __float2half_rn(v - __half2float(hi));
    uint8_t* chunk = a.bx + (uint64_t)c * gemm_xchunk_bytes(nsp);
    uint8_t* tile = chunk + (k / 16) * (N * 32u);
    const uint32_t sl = kslot(k % 16);
    *reinterpret_cast<__half*>(tile + bt_off(s, sl)) = hi;
    *reinterpret_cast<__half*>(tile + bt_off(nsp + s, sl)) = lo;
    // per 32-value sub-block sums (warp w = sub-block w)
    const float sm = warp_sum(v);
    if ((k & 31) == 0) reinterpret_cast<float*>(chunk + 16 * (N * 32u))[(k / 32) * nsp + s] = sm;
    pdl_launch_dependents();
}

// ------------------------------------------------------------------ the GEMM
struct GemmPlan {
    GemmArgs a;
    uint32_t nsp, N, ksplit, items, xchunk, stages;
    uint32_t sub_per_chunk;  // A slots per chunk: Q4_K 4 (64 values), Q6_K 8 (32 x 2 planes), Q8_0 8
    uint32_t eu_per_chunk;   // accumulator spans per chunk: Q4_K, Q6_K 1; Q8_0 8
};

__device__ __forceinline__ bool bwait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
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

__device__ __forceinline__ void item_range(const GemmPlan& P, uint32_t item, uint32_t& mt, uint32_t& c0, uint32_t& c1,
                                           uint32_t& kr) {
    const uint32_t nch = P.a.w.nchunks;
    mt = item / P.ksplit;
    kr = item % P.ksplit;
    c0 = (uint32_t)(((uint64_t)nch * kr) / P.ksplit);
    c1 = (uint32_t)(((uint64_t)nch * (kr + 1)) / P.ksplit);
}

// T is the weight type: the sub-chunk loops unroll and the per-chunk scales stay in registers.
template <uint32_t T>
__global__ void __launch_bounds__(kGemmThreads, 1) qgemm_kernel(const __grid_constant__ GemmPlan P) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t st_full[kMaxStages], st_empty[kMaxStages];
    __shared__ __align__(8) uint64_t a_full[kASlots], a_empty[kASlots];
    __shared__ __align__(8) uint64_t d_full[kDSlots], d_empty[kDSlots];
    __shared__ __align__(8) uint64_t fin_bar;
    __shared__ uint32_t tmem_base;
    __shared__ volatile int abort_flag;
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const GemmArgs& A = P.a;
    const uint32_t wbytes = A.w.block_bytes, stage_bytes = wbytes + P.xchunk, kStages = P.stages;
    constexpr uint32_t SP = T == GGML_Q4_K ? 4 : 8;  // A slots per chunk
    const uint32_t item0 = (uint32_t)(((uint64_t)P.items * blockIdx.x) / gridDim.x);
    const uint32_t item1 = (uint32_t)(((uint64_t)P.items * (blockIdx.x + 1)) / gridDim.x);

    if (tid == 0) {
        abort_flag = 0;
        for (uint32_t i = 0; i < kStages; ++i) {
            mbar_init(&st_full[i], 1);
            mbar_init(&st_empty[i], kMathWarps + 1);
        }
        for (uint32_t i = 0; i < kASlots; ++i) {
            mbar_init(&a_full[i], 4);  // the four quadrant warps of one math group
            mbar_init(&a_empty[i], 1);
        }
        for (uint32_t i = 0; i < kDSlots; ++i) {
            mbar_init(&d_full[i], 1);
            mbar_init(&d_empty[i], kMathWarps);
        }
        mbar_init(&fin_bar, 1);
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(&tmem_base, kTmemCols);
        tmem_relinquish();
    }
    tc_before();
    __syncthreads();
    tc_after();
    const uint32_t tm = tmem_base;
    pdl_wait();  // the staged x (and xinv) come from the previous launch

    if (warp == 0) {
        // ---------------------------------------------------------------- producer
        if (lane == 0) {
            uint32_t n = 0;
            for (uint32_t it = item0; it < item1 && !abort_flag; ++it) {
                uint32_t mt, c0, c1, kr;
                item_range(P, it, mt, c0, c1, kr);
                for (uint32_t c = c0; c < c1; ++c, ++n) {
                    const uint32_t s = n % kStages, ph = n / kStages;
                    if (ph > 0 && !bwait(&st_empty[s], (ph - 1) & 1, &abort_flag)) break;
                    uint8_t* dst = smem + s * stage_bytes;
                    mbar_arrive_expect_tx(&st_full[s], stage_bytes);
                    tma_load_1d_hint(dst, A.w.q + ((uint64_t)mt * A.w.nchunks + c) * wbytes, wbytes, &st_full[s],
                                     l2_evict_first());
                    tma_load_1d(dst + wbytes, A.bx + (uint64_t)c * P.xchunk, P.xchunk, &st_full[s]);
                }
                if (abort_flag) break;
            }
            if (abort_flag)  // copies in flight land before the CTA leaves
                for (uint32_t s = 0; s < kStages && s < n; ++s) mbar_wait(&st_full[s], ((n - 1 - s) / kStages) & 1);
        }
    } else if (warp == 1) {
        // ---------------------------------------------------------------- MMA issuer
        if (lane == 0) {
            const uint32_t idesc = mma_idesc(2 * P.nsp);  // N = x hi rows then lo rows, one MMA per K step
            uint32_t n = 0, g = 0, e = 0;
            bool ok = true;
            for (uint32_t it = item0; it < item1 && ok; ++it) {
                uint32_t mt, c0, c1, kr;
                item_range(P, it, mt, c0, c1, kr);
                for (uint32_t c = c0; c < c1 && ok; ++c, ++n) {
                    const uint32_t s = n % kStages;
                    if (!bwait(&st_full[s], (n / kStages) & 1, &abort_flag)) { ok = false; break; }
                    const uint8_t* bx = smem + s * stage_bytes + wbytes;
                    const uint32_t tile_b = P.N * 32;
#pragma unroll
                    for (uint32_t q = 0; q < SP && ok; ++q, ++g) {
                        const uint32_t as = g % kASlots;
                        const uint32_t eu_first = (T == GGML_Q8_0) || q == 0;
                        const uint32_t ds = e % kDSlots;
                        if (eu_first && e >= kDSlots &&
                            !bwait(&d_empty[ds], ((e / kDSlots) - 1) & 1, &abort_flag)) { ok = false; break; }
                        if (!bwait(&a_full[as], (g / kASlots) & 1, &abort_flag)) { ok = false; break; }
                        tc_after();
                        const uint32_t acol = tm + kColA + as * 32, dcol = tm + kColD + ds * kDCols;
                        // A columns 8i..8i+7 against B tile `bt` (x hi rows, then x lo rows)
                        auto mma1 = [&](uint32_t i, uint32_t bt, bool first) {
                            mma_tmem_a(dcol, acol + 8 * i, bdesc(bx + bt * tile_b), idesc, !first);
                        };
                        if (T == GGML_Q4_K) {  // 64 values: B tiles 4q..4q+3
                            for (uint32_t i = 0; i < 4; ++i) mma1(i, 4 * q + i, (q | i) == 0);
                        } else if (T == GGML_Q6_K) {  // 32 values x two planes: B tiles 2q, 2q+1
                            for (uint32_t i = 0; i < 4; ++i) mma1(i, 2 * q + (i & 1), (q | i) == 0);
                        } else {  // Q8_0 block q: B tiles 2q, 2q+1
                            for (uint32_t i = 0; i < 2; ++i) mma1(i, 2 * q + i, i == 0);
                        }
                        mma_commit(&a_empty[as]);
                        const bool eu_last = (T == GGML_Q8_0) || q + 1 == SP;
                        if (eu_last) {
                            mma_commit(&d_full[ds]);
                            ++e;
                        }
                    }
                    if (ok) mma_commit(&st_empty[s]);
                }
            }
            if (!ok) {
                abort_flag = 1;
                if (A.err) atomicExch(A.err, DEV_ERR_WAIT_TIMEOUT);
            }
            // every MMA issued has completed before the tensor memory is freed
            mma_commit(&fin_bar);
            mbar_wait(&fin_bar, 0);
        }
    } else {
        // ---------------------------------------------------------------- math warps
        const uint32_t mw = warp - 2, grp = mw / 4, qd = warp & 3;  // group 0..kGroups-1, TMEM lane quadrant
        const uint32_t t = qd * 32 + lane;                            // row within the M tile
        const uint32_t lane_addr = (qd * 32u) << 16;
        const uint32_t half = P.nsp / kGroups;                         // sequences per group in the epilogue (4 or 8)
        float acc[8];
        uint32_t n = 0, g = 0, e = 0;
        bool ok = true;
        // scales of the accumulator spans not yet read back (two in flight)
        float eu_d[kDSlots] = {0.f, 0.f, 0.f, 0.f};
        auto epilogue = [&](uint32_t eu) -> bool {  // read span eu back and scale it into acc
            const uint32_t ds = eu % kDSlots;
            if (!bwait(&d_full[ds], (eu / kDSlots) & 1, &abort_flag)) return false;
            tc_after();
            uint32_t dv[8], lv[8];  // this group's sequences: x hi columns, x lo columns
            const uint32_t dcol = tm + lane_addr + kColD + ds * kDCols + grp * half;
            if (half == 8) {
                tmem_ld8(dcol, dv);
                tmem_ld8(dcol + P.nsp, lv);
            } else {
                tmem_ld4(dcol, dv);
                tmem_ld4(dcol + P.nsp, lv);
#pragma unroll
                for (int i = 4; i < 8; ++i) dv[i] = lv[i] = 0u;
            }
            tmem_ld_wait();
            tc_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&d_empty[ds]);
            const float d = eu_d[ds];
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] = fmaf(d, __uint_as_float(dv[i]) + __uint_as_float(lv[i]), acc[i]);
            return true;
        };
        for (uint32_t it = item0; it < item1 && ok; ++it) {
            uint32_t mt, c0, c1, kr;
            item_range(P, it, mt, c0, c1, kr);
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] = 0.f;
            uint32_t first_eu = e;
            for (uint32_t c = c0; c < c1 && ok; ++c, ++n) {
                const uint32_t s = n % kStages;
                if (!bwait(&st_full[s], (n / kStages) & 1, &abort_flag)) { ok = false; break; }
                const uint8_t* wb = smem + s * stage_bytes;
                // this row's scales for the chunk
                float q4_m[8], d = 0.f, dmin = 0.f;
                uint32_t q4_sb[8];
                float q8_d[8];
                uint32_t q6_sc[4];
                if (T == GGML_Q4_K) {
                    const uint32_t dm = *reinterpret_cast<const uint32_t*>(wb + t * 4);
                    d = f16_exact(dm & 0xffff);
                    dmin = f16_exact(dm >> 16);
                    // the 12 scale bytes as three words (gguf.rs's get_scale_min_k4 on four
                    // sub-blocks at once): s_0..3, s_4..7, m_0..3, m_4..7 one per byte
                    const uint32_t* sw = reinterpret_cast<const uint32_t*>(wb + 512 + t * 12);
                    const uint32_t w0 = sw[0], w1 = sw[1], w2 = sw[2];
                    const uint32_t sb[2] = {w0 & 0x3F3F3F3Fu, (w2 & 0x0F0F0F0Fu) | ((w0 >> 2) & 0x30303030u)};
                    const uint32_t mb[2] = {w1 & 0x3F3F3F3Fu, ((w2 >> 4) & 0x0F0F0F0Fu) | ((w1 >> 2) & 0x30303030u)};
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        q4_sb[j] = (sb[j >> 2] >> (8 * (j & 3))) & 0xffu;
                        q4_m[j] = small_int_f((mb[j >> 2] >> (8 * (j & 3))) & 0xffu);
                    }
                    // -dmin * sum_j m_j * sum(x of sub-block j), this group's sequences
                    // (4 or 8 consecutive floats per sub-block: 16-byte loads; same FMA order)
                    const float* xs = reinterpret_cast<const float*>(wb + wbytes + 16u * (P.N * 32u)) + grp * half;
                    float mt[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const float4 a0 = *reinterpret_cast<const float4*>(xs + j * P.nsp);
                        mt[0] = fmaf(q4_m[j], a0.x, mt[0]);
                        mt[1] = fmaf(q4_m[j], a0.y, mt[1]);
                        mt[2] = fmaf(q4_m[j], a0.z, mt[2]);
                        mt[3] = fmaf(q4_m[j], a0.w, mt[3]);
                        if (half == 8) {
                            const float4 a1 = *reinterpret_cast<const float4*>(xs + j * P.nsp + 4);
                            mt[4] = fmaf(q4_m[j], a1.x, mt[4]);
                            mt[5] = fmaf(q4_m[j], a1.y, mt[5]);
                            mt[6] = fmaf(q4_m[j], a1.z, mt[6]);
                            mt[7] = fmaf(q4_m[j], a1.w, mt[7]);
                        }
                    }
#pragma unroll
                    for (uint32_t i = 0; i < 8; ++i) {
                        if (i >= half) break;
                        acc[i] = fmaf(-dmin, mt[i], acc[i]);
                    }
                } else if (T == GGML_Q6_K) {
                    const uint4 sc4 = *reinterpret_cast<const uint4*>(wb + 24576 + t * 16);
                    q6_sc[0] = sc4.x; q6_sc[1] = sc4.y; q6_sc[2] = sc4.z; q6_sc[3] = sc4.w;
                    d = f16_exact(*reinterpret_cast<const uint16_t*>(wb + 26624 + t * 2));
                } else {
                    const uint4 dd = *reinterpret_cast<const uint4*>(wb + t * 16);
                    const uint32_t w4[4] = {dd.x, dd.y, dd.z, dd.w};
                    for (int j = 0; j < 4; ++j) {
                        q8_d[2 * j] = f16_exact(w4[j] & 0xffff);
                        q8_d[2 * j + 1] = f16_exact(w4[j] >> 16);
                    }
                }
#pragma unroll
                for (uint32_t q = 0; q < SP && ok; ++q, ++g) {
                    if (g % kGroups == grp) {  // this group dequantises sub-chunk g
                        const uint32_t as = g % kASlots;
                        if (g >= kASlots && !bwait(&a_empty[as], ((g / kASlots) - 1) & 1, &abort_flag)) {
                            ok = false;
                            break;
                        }
                        tc_after();
                        uint32_t v[32];
                        if (T == GGML_Q4_K) {  // unit q: qs bytes 32q..32q+31, sub-blocks 2q (low), 2q+1 (high)
                            // half2 (s, s) and (-1024 s, -1024 s), exact (s <= 63)
                            const uint32_t s2l = small_int_h2(q4_sb[2 * q]), b2l = hmul2_bits(s2l, 0xE400E400u);
                            const uint32_t s2h = small_int_h2(q4_sb[2 * q + 1]), b2h = hmul2_bits(s2h, 0xE400E400u);
                            for (uint32_t hc = 0; hc < 2; ++hc) {
                                const uint32_t ci = 2 * q + hc;
                                const uint4 w = *reinterpret_cast<const uint4*>(wb + 2048 + t * 128 + ((ci ^ (t & 7)) * 16));
                                const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                                for (int a = 0; a < 4; ++a) {
                                    const uint32_t col = 2 * (4 * hc + a);  // value group 16hc + 4a
                                    v[col] = magic_fma(ws[a] & 0x000F000Fu, s2l, b2l);
                                    v[col + 1] = magic_fma((ws[a] >> 8) & 0x000F000Fu, s2l, b2l);
                                    v[16 + col] = magic_fma((ws[a] >> 4) & 0x000F000Fu, s2h, b2h);
                                    v[16 + col + 1] = magic_fma((ws[a] >> 12) & 0x000F000Fu, s2h, b2h);
                                }
                            }
                            tmem_st16(tm + lane_addr + kColA + as * 32, *reinterpret_cast<uint32_t(*)[16]>(&v[0]));
                            tmem_st16(tm + lane_addr + kColA + as * 32 + 16, *reinterpret_cast<uint32_t(*)[16]>(&v[16]));
                        } else if (T == GGML_Q6_K) {  // values 32q..32q+31: half hh = q/4, run kq = q%4
                            const uint32_t hh = q >> 2, kq = q & 3;
                            const uint32_t lci0 = 4 * hh + 2 * (kq & 1), hci0 = 2 * hh;  // 16-byte pieces
                            const uint32_t sw = (t & 7), swq = ((t >> 1) & 3);
                            const uint4 L0 = *reinterpret_cast<const uint4*>(wb + t * 128 + (((lci0) ^ sw) * 16));
                            const uint4 L1 = *reinterpret_cast<const uint4*>(wb + t * 128 + (((lci0 + 1) ^ sw) * 16));
                            const uint4 H0 = *reinterpret_cast<const uint4*>(wb + 16384 + t * 64 + (((hci0) ^ swq) * 16));
                            const uint4 H1 = *reinterpret_cast<const uint4*>(wb + 16384 + t * 64 + (((hci0 + 1) ^ swq) * 16));
                            const uint32_t lw[8] = {L0.x, L0.y, L0.z, L0.w, L1.x, L1.y, L1.z, L1.w};
                            const uint32_t hw[8] = {H0.x, H0.y, H0.z, H0.w, H1.x, H1.y, H1.z, H1.w};
                            // run scales sc[8hh + l/16 + 2kq] for l < 16 and l >= 16
                            const uint32_t sidx0 = 8 * hh + 2 * kq, sidx1 = sidx0 + 1;
                            const int sc0 = (int8_t)(q6_sc[sidx0 >> 2] >> (8 * (sidx0 & 3)));
                            const int sc1 = (int8_t)(q6_sc[sidx1 >> 2] >> (8 * (sidx1 & 3)));
                            const uint32_t bias_b = 0x64206420u;  // half2(1056, 1056)
                            const __half2 bias = *reinterpret_cast<const __half2*>(&bias_b);
                            // per run: half2 of sc & 15 and of 16 (sc >> 4), exact, for the two planes
                            uint32_t p1b[2], p2b[2];
#pragma unroll
                            for (int h = 0; h < 2; ++h) {
                                const int sc = h ? sc1 : sc0;
                                const int shi = sc >> 4, slo = sc - 16 * shi;     // shi in [-8, 7], slo in [0, 15]
                                p1b[h] = small_int_h2((uint32_t)slo);
                                const uint32_t sh8 = small_int_h2((uint32_t)(shi + 8));  // shi + 8, then - 8 and x 16
                                const uint32_t m8 = 0xC800C800u;                       // half2(-8, -8)
                                __half2 t = __hadd2(*reinterpret_cast<const __half2*>(&sh8), *reinterpret_cast<const __half2*>(&m8));
                                const uint32_t c16 = 0x4C004C00u;                      // half2(16, 16)
                                t = __hmul2(t, *reinterpret_cast<const __half2*>(&c16));
                                p2b[h] = *reinterpret_cast<uint32_t*>(&t);
                            }
#pragma unroll
                            for (int a = 0; a < 8; ++a) {  // bytes 4a..4a+3 of the 32-value run pair
                                const __half2 p1 = *reinterpret_cast<const __half2*>(&p1b[a < 4 ? 0 : 1]);
                                const __half2 p2 = *reinterpret_cast<const __half2*>(&p2b[a < 4 ? 0 : 1]);
                                const uint32_t nib = (kq < 2) ? (lw[a] & 0x0F0F0F0Fu) : ((lw[a] >> 4) & 0x0F0F0F0Fu);
                                const uint32_t qv = nib | (((hw[a] >> (2 * kq)) & 0x03030303u) << 4);  // 0..63 per byte
                                const uint32_t e0 = (qv & 0x00FF00FFu) | 0x64006400u, e1 = ((qv >> 8) & 0x00FF00FFu) | 0x64006400u;
                                const __half2 q0 = __hsub2(*reinterpret_cast<const __half2*>(&e0), bias);  // q - 32
                                const __half2 q1 = __hsub2(*reinterpret_cast<const __half2*>(&e1), bias);
                                __half2 r;
                                r = __hmul2(q0, p1); v[2 * a] = *reinterpret_cast<uint32_t*>(&r);
                                r = __hmul2(q1, p1); v[2 * a + 1] = *reinterpret_cast<uint32_t*>(&r);
                                r = __hmul2(q0, p2); v[16 + 2 * a] = *reinterpret_cast<uint32_t*>(&r);
                                r = __hmul2(q1, p2); v[16 + 2 * a + 1] = *reinterpret_cast<uint32_t*>(&r);
                            }
                            tmem_st16(tm + lane_addr + kColA + as * 32, *reinterpret_cast<uint32_t(*)[16]>(&v[0]));
                            tmem_st16(tm + lane_addr + kColA + as * 32 + 16, *reinterpret_cast<uint32_t(*)[16]>(&v[16]));
                        } else {  // Q8_0 block q: qs bytes 32q..32q+31
                            const uint32_t bias_b = 0x64806480u;  // half2(1152, 1152)
                            const __half2 bias = *reinterpret_cast<const __half2*>(&bias_b);
                            for (uint32_t hc = 0; hc < 2; ++hc) {
                                const uint32_t ci = 2 * q + hc;
                                const uint4 w = *reinterpret_cast<const uint4*>(
                                    wb + 2048 + t * 256 + (((ci & 8) | ((ci & 7) ^ (t & 7))) * 16));
                                const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                                for (int a = 0; a < 4; ++a) {
                                    const uint32_t u = ws[a] ^ 0x80808080u;  // q + 128, per byte
                                    const uint32_t e0 = (u & 0x00FF00FFu) | 0x64006400u, e1 = ((u >> 8) & 0x00FF00FFu) | 0x64006400u;
                                    __half2 r;
                                    r = __hsub2(*reinterpret_cast<const __half2*>(&e0), bias);
                                    v[2 * (4 * hc + a)] = *reinterpret_cast<uint32_t*>(&r);
                                    r = __hsub2(*reinterpret_cast<const __half2*>(&e1), bias);
                                    v[2 * (4 * hc + a) + 1] = *reinterpret_cast<uint32_t*>(&r);
                                }
                            }
                            tmem_st16(tm + lane_addr + kColA + as * 32, *reinterpret_cast<uint32_t(*)[16]>(&v[0]));
                        }
                        tmem_st_wait();
                        tc_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&a_full[as]);
                    }
                    const bool eu_last = (T == GGML_Q8_0) || q + 1 == SP;
                    if (eu_last) {
                        const uint32_t ds = e % kDSlots;
                        eu_d[ds] = (T == GGML_Q8_0) ? q8_d[q] : d;
                        // read back the previous span (one span of lag keeps the MMAs busy)
                        if (e >= first_eu + kLag && !epilogue(e - kLag)) { ok = false; break; }
                        ++e;
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&st_empty[s]);  // done with this stage's weights
            }
            if (!ok) break;
            for (uint32_t k = kLag; k >= 1 && ok; --k)  // drain the spans still in flight
                if (e >= first_eu + k && !epilogue(e - k)) ok = false;
            if (!ok) break;
            // partial sums of this item: part[kr][seq][row]
            const uint32_t row = mt * kMT + t;
#pragma unroll
            for (uint32_t i = 0; i < 8; ++i) {
                const uint32_t sq = grp * half + i;
                if (i < half && sq < A.nseq)
                    A.part[((uint64_t)kr * A.nseq + sq) * A.rows_pad + row] = acc[i] * A.xinv[sq];
            }
        }
        if (!ok) {
            abort_flag = 1;
            if (lane == 0 && A.err) atomicExch(A.err, DEV_ERR_WAIT_TIMEOUT);
        }
    }
    tc_before();
    __syncthreads();
    tc_after();
    if (warp == 1) tmem_dealloc(tm, kTmemCols);
}

// ------------------------------------------------------------------ reduce + epilogue
struct GemmReduceN {
    GemmReduce r[3];
    uint64_t end[3];  // cumulative element counts
    uint32_t n;
};

__device__ __forceinline__ void reduce_one(const GemmReduce& a, uint64_t i) {
    const uint32_t s = (uint32_t)(i / a.rows), r = (uint32_t)(i % a.rows);
    float sum = 0.f, sum2 = 0.f;
    for (uint32_t k = 0; k < a.ksplit; ++k) sum += a.part[((uint64_t)k * a.nseq + s) * a.rows_pad + r];
    if (a.part2)
        for (uint32_t k = 0; k < a.ksplit2; ++k) sum2 += a.part2[((uint64_t)k * a.nseq + s) * a.rows_pad2 + r];
    float* y = a.y + (uint64_t)s * a.y_stride + r;
    if (a.epi == EPI_SWIGLU) *y = __fmul_rn(__fdiv_rn(sum, __fadd_rn(1.0f, expf(-sum))), sum2);
    else if (a.epi == EPI_ADD) *y += sum;
    else *y = sum;
}

__global__ void gemm_reduce_n_kernel(const GemmReduceN a) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    pdl_wait();
    if (i < a.end[0]) reduce_one(a.r[0], i);
    else if (a.n > 1 && i < a.end[1]) reduce_one(a.r[1], i - a.end[0]);
    else if (a.n > 2 && i < a.end[2]) reduce_one(a.r[2], i - a.end[1]);
    pdl_launch_dependents();
}

__global__ void gemm_reduce_kernel(const GemmReduce a) {
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (uint64_t)a.nseq * a.rows) return;
    const uint32_t s = (uint32_t)(i / a.rows), r = (uint32_t)(i % a.rows);
    pdl_wait();
    float sum = 0.f, sum2 = 0.f;
    for (uint32_t k = 0; k < a.ksplit; ++k) sum += a.part[((uint64_t)k * a.nseq + s) * a.rows_pad + r];
    if (a.part2)
        for (uint32_t k = 0; k < a.ksplit2; ++k) sum2 += a.part2[((uint64_t)k * a.nseq + s) * a.rows_pad2 + r];
    float* y = a.y + (uint64_t)s * a.y_stride + r;
    if (a.epi == EPI_SWIGLU) *y = __fmul_rn(__fdiv_rn(sum, __fadd_rn(1.0f, expf(-sum))), sum2);
    else if (a.epi == EPI_ADD) *y += sum;
    else *y = sum;
    pdl_launch_dependents();
}

std::atomic<int> g_gemm_attr[64];

cudaLaunchConfig_t cfg_of(dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl, cudaLaunchAttribute* at) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    return cfg;
}

}  // namespace

uint64_t gemm_layout_bytes(uint32_t type, uint32_t rows, uint32_t cols) {
    const uint32_t bb = gemm_block_bytes(type);
    if (!bb || !rows || cols % kChunk) return 0;
    return (uint64_t)((rows + kMT - 1) / kMT) * (cols / kChunk) * bb;
}

QGemmDev gemm_view(uint32_t type, uint32_t rows, uint32_t cols, const uint8_t* q) {
    QGemmDev g;
    g.type = type;
    g.rows = rows;
    g.cols = cols;
    g.mtiles = (rows + kMT - 1) / kMT;
    g.nchunks = cols / kChunk;
    g.block_bytes = gemm_block_bytes(type);
    g.q = q;
    return g;
}

cudaError_t launch_gemm_repack(const QMatDev& src, const QGemmDev& dst, cudaStream_t s) {
    if (src.type != dst.type || !gemm_block_bytes(src.type) || src.cols != dst.cols || src.cols % kChunk)
        return cudaErrorInvalidValue;
    const uint64_t n = (uint64_t)dst.mtiles * kMT * dst.nchunks;
    gemm_repack_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(src, dst);
    return cudaGetLastError();
}

uint64_t gemm_x_bytes(uint32_t nseq, uint32_t cols) {
    const uint32_t nsp = (nseq + 15) / 16 * 16;
    return (uint64_t)(cols / kChunk) * gemm_xchunk_bytes(nsp);
}

uint32_t gemm_stage_one_launch_cols() { return kStatsThreads * kStatsPer; }

cudaError_t launch_gemm_stage_x(GemmX a, cudaStream_t s, bool pdl) {
    if (!a.nseq || a.nseq > 32 || a.cols % kChunk || !a.x || !a.bx || !a.xinv || !a.stats) return cudaErrorInvalidValue;
    a.nsp = (a.nseq + 15) / 16 * 16;  // the MMA's N (M = 128 needs a multiple of 16)
    cudaLaunchAttribute at[1];
    // rows of up to kStatsThreads * kStatsPer values: one launch, a CTA per sequence
    // (padding ones included) computes the statistics and stages its row
    const bool one = a.cols <= kStatsThreads * kStatsPer;
    // a row split over a cluster of kStageSplit CTAs when it divides into whole 256-value
    // chunks (EVELYN_STAGE_SPLIT=0: one CTA per sequence)
    static const bool split_off = [] {
        const char* e = std::getenv("EVELYN_STAGE_SPLIT");
        return e && e[0] == '0';
    }();
    if (one && a.cols % (kStageSplit * kChunk) == 0 && !split_off) {
        cudaLaunchAttribute at2[2];
        auto cfg = cfg_of(dim3(a.nsp * kStageSplit), dim3(kStatsThreads), 0, s, pdl, at2);
        at2[cfg.numAttrs].id = cudaLaunchAttributeClusterDimension;
        at2[cfg.numAttrs].val.clusterDim.x = kStageSplit;
        at2[cfg.numAttrs].val.clusterDim.y = 1;
        at2[cfg.numAttrs].val.clusterDim.z = 1;
        cfg.numAttrs += 1;
        return cudaLaunchKernelEx(&cfg, gemm_stage_cluster_kernel, a);
    }
    auto cfg = cfg_of(dim3(one ? a.nsp : a.nseq), dim3(kStatsThreads), 0, s, pdl, at);
    cudaError_t e = cudaLaunchKernelEx(&cfg, gemm_stage_stats_kernel, a);
    if (e != cudaSuccess || one) return e;
    auto cfg2 = cfg_of(dim3(a.nsp, a.cols / kChunk), dim3(kChunk), 0, s, pdl, at);
    return cudaLaunchKernelEx(&cfg2, gemm_stage_x_kernel, a);
}

uint32_t gemm_ksplit(const QGemmDev& w, int sms) {
    const uint32_t want = (uint32_t)std::max(1, (2 * sms + (int)w.mtiles / 2) / (int)w.mtiles);
    return std::max<uint32_t>(1, std::min<uint32_t>(want, w.nchunks));
}

cudaError_t launch_qgemm(const GemmArgs& a, cudaStream_t s, bool pdl) {
    if (!a.w.q || !a.bx || !a.part || !a.xinv || !a.nseq || a.nseq > 32 || !a.ksplit) return cudaErrorInvalidValue;
    if (a.w.type != GGML_Q4_K && a.w.type != GGML_Q6_K && a.w.type != GGML_Q8_0) return cudaErrorInvalidValue;
    auto kernel = a.w.type == GGML_Q4_K ? qgemm_kernel<GGML_Q4_K>
                  : a.w.type == GGML_Q6_K ? qgemm_kernel<GGML_Q6_K> : qgemm_kernel<GGML_Q8_0>;
    GemmPlan P{};
    P.a = a;
    P.nsp = (a.nseq + 15) / 16 * 16;
    P.N = 2 * P.nsp;
    P.ksplit = a.ksplit;
    P.items = a.w.mtiles * a.ksplit;
    P.xchunk = gemm_xchunk_bytes(P.nsp);
    P.sub_per_chunk = a.w.type == GGML_Q4_K ? 4 : 8;
    P.eu_per_chunk = a.w.type == GGML_Q8_0 ? 8 : 1;
    int dev = 0, sms = 148;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    // at least 116 KB so that no two CTAs share an SM: each allocates all 512 TMEM columns
    const uint32_t stage_bytes = a.w.block_bytes + P.xchunk;
    P.stages = std::min<uint32_t>(kMaxStages, (225u * 1024) / stage_bytes);
    if (P.stages < 2) return cudaErrorInvalidValue;
    // at least 116 KB so that no two CTAs share an SM: each allocates all 512 TMEM columns
    const size_t smem = std::max<size_t>((size_t)P.stages * stage_bytes, 116 * 1024);
    if (dev >= 0 && dev < 64 && !g_gemm_attr[dev]) {
        for (auto k : {qgemm_kernel<GGML_Q4_K>, qgemm_kernel<GGML_Q6_K>, qgemm_kernel<GGML_Q8_0>}) {
            e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 225 * 1024);
            if (e != cudaSuccess) return e;
        }
        g_gemm_attr[dev] = 1;
    }
    cudaLaunchAttribute at[1];
    auto cfg = cfg_of(dim3(std::min<uint32_t>(P.items, (uint32_t)sms)), dim3(kGemmThreads), smem, s, pdl, at);
    return cudaLaunchKernelEx(&cfg, kernel, P);
}

cudaError_t launch_gemm_reduce(const GemmReduce& a, cudaStream_t s, bool pdl) {
    if (!a.part || !a.y || !a.nseq || !a.rows || !a.ksplit) return cudaErrorInvalidValue;
    const uint64_t n = (uint64_t)a.nseq * a.rows;
    cudaLaunchAttribute at[1];
    auto cfg = cfg_of(dim3((unsigned)((n + 255) / 256)), dim3(256), 0, s, pdl, at);
    return cudaLaunchKernelEx(&cfg, gemm_reduce_kernel, a);
}

cudaError_t launch_gemm_reduce_n(const GemmReduce* a, uint32_t n, cudaStream_t s, bool pdl) {
    if (!a || n < 1 || n > 3) return cudaErrorInvalidValue;
    GemmReduceN r{};
    r.n = n;
    uint64_t tot = 0;
    for (uint32_t k = 0; k < n; ++k) {
        if (!a[k].part || !a[k].y || !a[k].nseq || !a[k].rows || !a[k].ksplit) return cudaErrorInvalidValue;
        r.r[k] = a[k];
        tot += (uint64_t)a[k].nseq * a[k].rows;
        r.end[k] = tot;
    }
    cudaLaunchAttribute at[1];
    auto cfg = cfg_of(dim3((unsigned)((tot + 255) / 256)), dim3(256), 0, s, pdl, at);
    return cudaLaunchKernelEx(&cfg, gemm_reduce_n_kernel, r);
}

}  // namespace evl
