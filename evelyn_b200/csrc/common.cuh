// common.cuh -- device-side types shared by the decode kernels.
//
// Quantised weights live in HBM in a repack of the GGUF blocks (the reference keeps
// the raw GGUF bytes, src/runtime.rs:23-51) ordered for the matvec's warp-level
// integer MMA (mma.sync m16n8k32, one 16-row x 32-value A tile per instruction). A
// unit is 64 values of one row. Rows are padded to a multiple of 16 and stored as
// 16-row slabs; a slab is cut into panels of up to 32 units (2048 values), panel g
// holding units [32g, 32g + U) of the slab's 16 rows, so one TMA bulk copy moves one
// panel. Inside a panel the bytes of the 16 rows are interleaved so that lane
// L = 4*g8 + t of a warp (g8 = L/4, t = L%4; MMA rows g8 and g8 + 8) finds its A
// fragments in one 16-byte word per load:
//
//   Q4_K  per super-block (4 units, 2304 B): 4 qs groups j x 512 B, lane L at
//         j*512 + 16L holding the qs words (bytes 4w..4w+3 of group j) w = t and
//         w = 4 + t of rows g8 and g8 + 8 as [w=t row g8, w=t row g8+8, w=4+t row g8,
//         w=4+t row g8+8]; then the 16-byte header (d, dmin, scales[12]) of each row.
//   Q6_K  per super-block (3360 B): halves H = 0, 1 of 1536 B, lane L at H*1536 + 48L
//         holding ql words at 64H + 16a + 4t (a = 0..3) and qh words at 32H + 16a + 4t
//         (a = 0, 1) of rows g8 and g8 + 8 as
//         [ql a0 g8, ql a1 g8, ql a0 g8+8, ql a1 g8+8 | ql a2 .., ql a3 .. | qh a0 g8,
//          qh a1 g8, qh a0 g8+8, qh a1 g8+8]; then the 16 int8 scales of each row, then
//         the f16 d of each row.
//   Q8_0  per unit (two 32-value blocks A, B; 1088 B): halves h = 0, 1 of 512 B, lane L
//         at h*512 + 16L holding the q words at bytes 16h + 4t of A row g8, A row g8+8,
//         B row g8, B row g8+8; then the f16 scales (A, B) of each row.
//   F16, BF16, F32: plain values, each row of the panel contiguous.
//   Q5_K  per super-block (2816 B): the qs groups as Q4_K (2048 B), then the qh words
//         of each lane (bytes 4t..4t+3 and 16+4t.. of rows g8 and g8 + 8, the fifth bits
//         of the values its qs words hold) at 2048 + 16L in the same order, then the
//         16-byte header (d, dmin, scales[12]) of each row.
// No byte is added or dropped: a slab of Q4_K / Q5_K / Q6_K / Q8_0 is exactly 16 rows
// of GGUF blocks, and block_byte_address maps every GGUF byte to its place (4-byte
// payload words stay contiguous).
#pragma once
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace evl {

constexpr uint32_t GGML_F32 = 0, GGML_F16 = 1, GGML_Q8_0 = 8, GGML_Q4_K = 12, GGML_Q5_K = 13, GGML_Q6_K = 14,
                   GGML_BF16 = 30;

// Device view of one repacked matrix.
struct QMatDev {
    uint32_t type = 0;
    uint32_t rows = 0, cols = 0;
    uint32_t nunits = 0;         // 64-value units per row
    uint32_t row_bytes = 0;      // bytes per row; a 16-row slab is 16 * row_bytes
    const uint8_t* q = nullptr;  // ceil(rows / 16) slabs
};

constexpr uint32_t kSlabRows = 16;
constexpr uint32_t kPanelUnits = 32;

// Bytes of one unit over the 16 rows of a slab.
__host__ __device__ inline uint32_t unit16_bytes(uint32_t type) {
    switch (type) {
        case GGML_Q4_K: return 576;   // 16 x 144 / 4
        case GGML_Q5_K: return 704;   // 16 x 176 / 4
        case GGML_Q6_K: return 840;   // 16 x 210 / 4
        case GGML_Q8_0: return 1088;  // 16 x 2 x 34
        case GGML_F16:
        case GGML_BF16: return 2048;
        case GGML_F32: return 4096;
        default: return 0;
    }
}
// Units in panel g of a row of `nunits` units.
__host__ __device__ inline uint32_t group_units(uint32_t nunits, uint32_t g) {
    const uint32_t rest = nunits - g * kPanelUnits;
    return rest < kPanelUnits ? rest : kPanelUnits;
}
__host__ __device__ inline uint32_t slab_row_bytes(uint32_t type, uint32_t nunits) {
    return nunits * unit16_bytes(type) / kSlabRows;
}
// Byte offset, inside a slab, of panel g; and the panel's size.
__host__ __device__ inline uint32_t panel_offset(uint32_t type, uint32_t g) {
    return g * kPanelUnits * unit16_bytes(type);
}
__host__ __device__ inline uint32_t panel_bytes(uint32_t type, uint32_t U) { return U * unit16_bytes(type); }

// Byte offset from the start of the matrix of byte `o` of GGUF block `b` of row r
// (Q4_K / Q6_K: 256-value super-block, o < 144 / 210; Q8_0: 32-value block, o < 34).
// Bytes o..o+3 of a payload word (o % 4 == 0 for Q4_K qs, Q6_K ql/qh; o % 4 == 2 for
// Q8_0 q) are contiguous, as are the 16 header bytes of a Q4_K block and the 16
// scales of a Q6_K block.
__host__ __device__ inline uint64_t block_byte_address(const QMatDev& m, uint32_t r, uint32_t b, uint32_t o) {
    const uint32_t T = m.type, r16 = r % kSlabRows, g8 = r16 & 7, hi = r16 >> 3;
    const uint64_t slab = (uint64_t)(r / kSlabRows) * kSlabRows * m.row_bytes;
    if (T == GGML_Q8_0) {
        const uint32_t u = b >> 1, blk = b & 1;
        const uint64_t base = slab + panel_offset(T, u / kPanelUnits) + (u % kPanelUnits) * 1088u;
        if (o < 2) return base + 1024u + r16 * 4u + blk * 2u + o;
        const uint32_t q = o - 2, h = q >> 4, t = (q >> 2) & 3;
        return base + h * 512u + (g8 * 4u + t) * 16u + (blk * 2u + hi) * 4u + (q & 3u);
    }
    const uint32_t u = 4 * b;
    const uint64_t base = slab + panel_offset(T, u / kPanelUnits) + ((u % kPanelUnits) / 4u) * 4u * unit16_bytes(T);
    if (T == GGML_Q4_K) {
        if (o < 16) return base + 2048u + r16 * 16u + o;
        const uint32_t q = o - 16, j = q >> 5, w = (q >> 2) & 7, t = w & 3;
        return base + j * 512u + (g8 * 4u + t) * 16u + ((w >> 2) * 2u + hi) * 4u + (q & 3u);
    }
    if (T == GGML_Q5_K) {
        if (o < 16) return base + 2560u + r16 * 16u + o;
        if (o < 48) {  // qh: byte l holds the fifth bits of value l of the eight sub-blocks
            const uint32_t q = o - 16, w = q >> 2, t = w & 3;
            return base + 2048u + (g8 * 4u + t) * 16u + ((w >> 2) * 2u + hi) * 4u + (q & 3u);
        }
        const uint32_t q = o - 48, j = q >> 5, w = (q >> 2) & 7, t = w & 3;
        return base + j * 512u + (g8 * 4u + t) * 16u + ((w >> 2) * 2u + hi) * 4u + (q & 3u);
    }
    // Q6_K
    if (o < 128) {
        const uint32_t H = o >> 6, oo = o & 63, a = oo >> 4, t = (oo >> 2) & 3;
        return base + H * 1536u + (g8 * 4u + t) * 48u + (a >> 1) * 16u + (hi * 2u + (a & 1)) * 4u + (oo & 3u);
    }
    if (o < 192) {
        const uint32_t q = o - 128, H = q >> 5, oo = q & 31, a = oo >> 4, t = (oo >> 2) & 3;
        return base + H * 1536u + (g8 * 4u + t) * 48u + 32u + (hi * 2u + a) * 4u + (oo & 3u);
    }
    if (o < 208) return base + 3072u + r16 * 16u + (o - 192);
    return base + 3328u + r16 * 2u + (o - 208);
}

// Plain types: byte offset of value c of row r (element size eb).
__host__ __device__ inline uint64_t plain_value_address(const QMatDev& m, uint32_t r, uint32_t c, uint32_t eb) {
    const uint32_t u = c / 64, g = u / kPanelUnits, U = group_units(m.nunits, g);
    return (uint64_t)(r / kSlabRows) * kSlabRows * m.row_bytes + panel_offset(m.type, g) +
           (uint64_t)(r % kSlabRows) * U * 64u * eb + (uint64_t)(c - g * kPanelUnits * 64u) * eb;
}

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// The reference's sigmoid (src/runtime.rs:476-483): 1 / (1 + e^-x) for x >= 0, else
// e^x / (1 + e^x).
__device__ __forceinline__ float sigmoid_ref(float x) {
    if (x >= 0.0f) return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x)));
    const float e = expf(x);
    return __fdiv_rn(e, __fadd_rn(1.0f, e));
}

__device__ __forceinline__ uint4 ldg_nc(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ uint4 ldg_nc_keep(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}

// Programmatic dependent launch: wait for the producing grid's memory, and let the
// next grid in the stream start launching.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

// ------------------------------------------------------------------ mbarrier + TMA bulk copies
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}
// One non-tensor TMA copy global -> this CTA's shared memory, completing on `bar`.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void tma_load_1d(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}
// An L2 policy under which the lines a copy brings in are the first to be evicted: the
// weight stream (each byte read once per step, gigabytes against a 126 MB L2) then does
// not push out the code, kernel parameters, norm weights, activations and KV pages
// that the following kernels read again.
__device__ __forceinline__ uint64_t l2_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ void tma_load_1d_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                                 uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}
__device__ __forceinline__ void prefetch_l2_bulk(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, 100000;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(phase)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Bounded wait: after kWaitNs of wall time the wait gives up and reports false;
// callers record the error and return instead of spinning forever.
constexpr uint64_t kWaitNs = 2000000000ull;
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t phase) {
    if (mbar_try_wait(bar, phase)) return true;
    const uint64_t t0 = global_ns();
    while (!mbar_try_wait(bar, phase))
        if (global_ns() - t0 > kWaitNs) return false;
    return true;
}

// Device error flags, read by the host after a step (0 = ok).
enum DeviceError : int { DEV_OK = 0, DEV_ERR_TOKEN = 1, DEV_ERR_WAIT_TIMEOUT = 2, DEV_ERR_POSITION = 3 };

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// byte of a 32-bit word selected by `sel` (0x7650 | k) as an exact float via the
// 2^23 magic: the bits 0x4B0000bb are the float 8388608 + bb.
__device__ __forceinline__ float byte_magic(uint32_t w, uint32_t sel) {
    return __uint_as_float(__byte_perm(w, 0x4B000000u, sel));
}

}  // namespace evl
