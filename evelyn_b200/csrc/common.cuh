// common.cuh -- device-side types shared by the decode kernels.
//
// Quantised weights live in HBM in a tiled repack of the GGUF blocks (the
// reference keeps the raw GGUF bytes, src/runtime.rs:23-51). A unit is 64 values of
// one row; a row is cut into tiles, each covering a group of up to 32 units (the last
// group of a row may be shorter, U units). Rows are padded to a multiple of 16 and
// stored as 16-row slabs: slab b holds, for each group g in turn, the 16 tiles
// (b*16 + i, g), i = 0..15, back to back -- so one TMA bulk copy moves 16 rows of one
// column group. A tile is self-contained and 16-byte aligned:
//
//   [payload: chunk-major, chunk c of unit u at c*U*16 + u*16 (16 B per chunk)]
//   [aux: block scales, padded to 16 B] [d: Q6_K super-block scales, padded to 16 B]
//
//   Q4_K  unit = 32-byte qs group j of super-block i (values 256i+64j+[0,64)),
//         2 chunks; aux = the 16-byte header (d, dmin, scales[12]) of each of the
//         U/4 super-blocks.
//   Q6_K  unit = (super-block i, half h, l0 in {0,16}) (values 256i+128h+32k+l0+[0,16),
//         k=0..3): 3 chunks (ql[64h+l0..+16], ql[64h+32+l0..+16], qh[32h+l0..+16]);
//         aux = u32 per unit with the 4 int8 scales sc[8h+l0/16+2k]; d = f16 per
//         super-block.
//   Q8_0  unit = two 32-value blocks: 4 chunks; aux = u32 per unit with the two
//         f16 block scales.
//   F16, BF16, F32: plain values, 8 (16) chunks per unit, no aux.
// Q5_K has no device-matrix layout (it is read only through the raw dequantiser).
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
    uint32_t row_bytes = 0;      // bytes of one row's tiles; a 16-row slab is 16 * row_bytes
    const uint8_t* q = nullptr;  // ceil(rows / 16) slabs
};

constexpr uint32_t kSlabRows = 16;

__host__ __device__ inline uint32_t chunks_per_unit(uint32_t type) {
    switch (type) {
        case GGML_Q4_K: return 2;
        case GGML_Q6_K: return 3;
        case GGML_Q8_0: return 4;
        case GGML_F16:
        case GGML_BF16: return 8;
        case GGML_F32: return 16;
        default: return 0;
    }
}

__host__ __device__ inline uint32_t pad16(uint32_t v) { return (v + 15u) & ~15u; }

// Sections of one tile of U units.
__host__ __device__ inline uint32_t tile_payload_bytes(uint32_t type, uint32_t U) {
    return U * chunks_per_unit(type) * 16u;
}
__host__ __device__ inline uint32_t tile_aux_bytes(uint32_t type, uint32_t U) {
    switch (type) {
        case GGML_Q4_K: return (U / 4u) * 16u;
        case GGML_Q6_K:
        case GGML_Q8_0: return pad16(U * 4u);
        default: return 0;
    }
}
__host__ __device__ inline uint32_t tile_d_bytes(uint32_t type, uint32_t U) {
    return type == GGML_Q6_K ? pad16((U / 4u) * 2u) : 0u;
}
__host__ __device__ inline uint32_t tile_bytes(uint32_t type, uint32_t U) {
    return tile_payload_bytes(type, U) + tile_aux_bytes(type, U) + tile_d_bytes(type, U);
}
// Units in group g of a row of `nunits` units.
__host__ __device__ inline uint32_t group_units(uint32_t nunits, uint32_t g) {
    const uint32_t rest = nunits - g * 32u;
    return rest < 32u ? rest : 32u;
}
__host__ __device__ inline uint32_t row_tile_bytes(uint32_t type, uint32_t nunits) {
    return (nunits / 32u) * tile_bytes(type, 32u) + ((nunits % 32u) ? tile_bytes(type, nunits % 32u) : 0u);
}
// Byte offset, inside a 16-row slab, of the 16 tiles of group g.
__host__ __device__ inline uint32_t slab_group_offset(uint32_t type, uint32_t g) {
    return g * kSlabRows * tile_bytes(type, 32u);
}
// Byte offset of tile (r, g) from the start of the matrix.
__host__ __device__ inline uint64_t tile_address(uint32_t type, uint32_t nunits, uint32_t row_bytes, uint32_t r,
                                                 uint32_t g) {
    return (uint64_t)(r / kSlabRows) * kSlabRows * row_bytes + slab_group_offset(type, g) +
           (r % kSlabRows) * tile_bytes(type, group_units(nunits, g));
}
// Offsets inside one tile of unit u (u's group is u >> 5; lane = u & 31).
__host__ __device__ inline uint32_t chunk_in_tile(uint32_t nunits, uint32_t u, uint32_t c) {
    return c * group_units(nunits, u >> 5) * 16u + (u & 31u) * 16u;
}
// aux entry of unit u (Q6_K, Q8_0: u32 per unit; Q4_K: 16-byte header of u's super-block)
__host__ __device__ inline uint32_t aux_in_tile(uint32_t type, uint32_t nunits, uint32_t u) {
    const uint32_t base = tile_payload_bytes(type, group_units(nunits, u >> 5));
    return type == GGML_Q4_K ? base + ((u & 31u) / 4u) * 16u : base + (u & 31u) * 4u;
}
// Q6_K f16 super-block scale of unit u
__host__ __device__ inline uint32_t d_in_tile(uint32_t type, uint32_t nunits, uint32_t u) {
    const uint32_t U = group_units(nunits, u >> 5);
    return tile_payload_bytes(type, U) + tile_aux_bytes(type, U) + ((u & 31u) / 4u) * 2u;
}

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

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
