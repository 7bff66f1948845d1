// common.cuh -- device-side types shared by the decode kernels.
//
// Quantised weights live in HBM in a "unit-interleaved" repack of the GGUF
// blocks (the reference keeps the raw GGUF bytes, src/runtime.rs:23-51). A unit is
// 64 consecutive values of one row; units are grouped 32 at a time, and inside a
// group the k-th 16-byte chunk of every unit is stored contiguously, so the 32
// lanes of a warp that each own one unit read 512 contiguous bytes per 128-bit load.
//
//   Q4_K  unit = 32-byte qs group j of super-block i (values 256i+64j+[0,64)),
//         2 chunks/unit;  aux = the 16-byte block header (d, dmin, scales[12]) per
//         super-block, [rows][nb][16].
//   Q6_K  unit = (super-block i, half h, l0 in {0,16}): 3 chunks/unit
//         (ql[64h+l0..+16], ql[64h+32+l0..+16], qh[32h+l0..+16]);
//         aux = u32 per unit holding the 4 int8 scales sc[8h+l0/16+2k], k=0..3;
//         d = f16 bits per super-block.
//   Q8_0  unit = two 32-value blocks: 4 chunks/unit; aux = u32 per unit with
//         the two f16 block scales.
//   F16, BF16, F32: plain values, 8 (16) chunks per unit.
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
    uint32_t nunits = 0;          // 64-value units per row
    const uint8_t* q = nullptr;   // chunk payload, row stride = nunits * chunks * 16
    const uint8_t* aux = nullptr; // see above
    const uint16_t* d = nullptr;  // Q6_K super-block scales
};

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

// Byte offset of chunk c of unit u inside one row's payload.
__host__ __device__ inline uint64_t chunk_offset(uint32_t nunits, uint32_t chunks, uint32_t u, uint32_t c) {
    uint32_t g = u >> 5, lane = u & 31;
    uint32_t rest = nunits - (g << 5);
    uint32_t gsize = rest < 32u ? rest : 32u;
    return (uint64_t)g * 32u * chunks * 16u + (uint64_t)c * gsize * 16u + (uint64_t)lane * 16u;
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
