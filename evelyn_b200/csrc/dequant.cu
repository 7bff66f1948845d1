// dequant.cu -- exact GGUF dequantisation on the device.
//
// Bit-exact restatement of src/gguf.rs:338-430 (see dequant.cuh for the value
// functions). Two entry points: one reads raw GGUF blocks, the other reads the
// repacked device layout of common.cuh (and so also proves that the repack is
// lossless).
#include "dequant.cuh"
#include "kernels.h"

namespace evl {

__global__ void dequant_raw_kernel(uint32_t type, const uint8_t* __restrict__ raw, uint64_t n,
                                   float* __restrict__ out) {
    uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float v;
    switch (type) {
        case GGML_F32: v = __uint_as_float(*(const uint32_t*)(raw + 4 * i)); break;
        case GGML_F16: v = f16_exact(ld_u16(raw + 2 * i)); break;
        case GGML_BF16: v = __uint_as_float(ld_u16(raw + 2 * i) << 16); break;
        case GGML_Q8_0: v = dq_raw_value(type, raw + (i / 32) * 34, (uint32_t)(i % 32)); break;
        case GGML_Q4_K: v = dq_raw_value(type, raw + (i / 256) * 144, (uint32_t)(i % 256)); break;
        case GGML_Q5_K: v = dq_raw_value(type, raw + (i / 256) * 176, (uint32_t)(i % 256)); break;
        case GGML_Q6_K: v = dq_raw_value(type, raw + (i / 256) * 210, (uint32_t)(i % 256)); break;
        default: v = 0.f;
    }
    out[i] = v;
}

__global__ void dequant_repacked_kernel(QMatDev m, uint32_t row0, uint32_t nrows, float* __restrict__ out) {
    uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    uint64_t n = (uint64_t)nrows * m.cols;
    if (i >= n) return;
    uint32_t r = (uint32_t)(i / m.cols), c = (uint32_t)(i % m.cols);
    out[i] = dq_repacked_value(m, row0 + r, c);
}

// Repack on the device: one thread per (row, GGUF block) -- per 64-value unit for the
// plain types -- copies the block's bytes out of the raw tensor rows into the matvec
// layout, each run of bytes to block_byte_address (the addresses the exact dequantiser
// reads back). Raw blocks of 34 / 210 bytes sit at any alignment, so they are read
// bytewise; every destination run is contiguous.
__device__ __forceinline__ void put_bytes(const QMatDev& d, uint8_t* dst, uint32_t r, uint32_t b, uint32_t o,
                                          const uint8_t* from, uint32_t n) {
    uint8_t* to = dst + block_byte_address(d, r, b, o);
    for (uint32_t i = 0; i < n; ++i) to[i] = from[i];
}

__global__ void repack_kernel(const QMatDev d, uint8_t* __restrict__ dst, const uint8_t* __restrict__ raw,
                              uint64_t stride, uint32_t rows, uint32_t per_row) {
    const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= (uint64_t)rows * per_row) return;
    const uint32_t r = (uint32_t)(idx / per_row), b = (uint32_t)(idx % per_row), T = d.type;
    const uint8_t* src = raw + r * stride;
    switch (T) {  // the byte runs of repack.cpp's layout, block by block (common.cuh)
        case GGML_Q4_K: {
            const uint8_t* blk = src + (uint64_t)b * 144;
            put_bytes(d, dst, r, b, 0, blk, 16);
            for (uint32_t o = 16; o < 144; o += 4) put_bytes(d, dst, r, b, o, blk + o, 4);
            break;
        }
        case GGML_Q5_K: {
            const uint8_t* blk = src + (uint64_t)b * 176;
            put_bytes(d, dst, r, b, 0, blk, 16);
            for (uint32_t o = 16; o < 176; o += 4) put_bytes(d, dst, r, b, o, blk + o, 4);
            break;
        }
        case GGML_Q6_K: {
            const uint8_t* blk = src + (uint64_t)b * 210;
            for (uint32_t o = 0; o < 192; o += 4) put_bytes(d, dst, r, b, o, blk + o, 4);
            put_bytes(d, dst, r, b, 192, blk + 192, 16);
            put_bytes(d, dst, r, b, 208, blk + 208, 2);
            break;
        }
        case GGML_Q8_0: {
            const uint8_t* blk = src + (uint64_t)b * 34;
            put_bytes(d, dst, r, b, 0, blk, 2);
            for (uint32_t o = 2; o < 34; o += 4) put_bytes(d, dst, r, b, o, blk + o, 4);
            break;
        }
        default: {  // F16 / BF16 / F32: unit b (64 values) of the row, contiguous in its panel row
            const uint32_t eb = T == GGML_F32 ? 4 : 2;
            const uint8_t* from = src + (uint64_t)b * 64 * eb;
            uint8_t* to = dst + plain_value_address(d, r, b * 64, eb);
            for (uint32_t i = 0; i < 64 * eb; ++i) to[i] = from[i];
        }
    }
}

cudaError_t launch_repack(const QMatDev& d, uint8_t* dst, uint64_t dst_bytes, const void* raw, uint64_t stride,
                          cudaStream_t s) {
    if (!d.rows || !d.cols || !dst || !raw) return cudaErrorInvalidValue;
    const uint32_t T = d.type;
    uint32_t per_row;
    if (T == GGML_Q4_K || T == GGML_Q5_K || T == GGML_Q6_K) per_row = d.cols / 256;
    else if (T == GGML_Q8_0) per_row = d.cols / 32;
    else if (T == GGML_F16 || T == GGML_BF16 || T == GGML_F32) per_row = d.cols / 64;
    else return cudaErrorInvalidValue;
    cudaError_t e = cudaMemsetAsync(dst, 0, dst_bytes, s);  // padding rows of the last slab
    if (e != cudaSuccess) return e;
    const uint64_t n = (uint64_t)d.rows * per_row;
    repack_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(d, dst, (const uint8_t*)raw, stride, d.rows, per_row);
    return cudaGetLastError();
}

cudaError_t launch_dequant_raw(uint32_t type, const void* raw, uint64_t n, float* out, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    uint64_t blocks = (n + 255) / 256;
    dequant_raw_kernel<<<(unsigned)blocks, 256, 0, s>>>(type, (const uint8_t*)raw, n, out);
    return cudaGetLastError();
}

cudaError_t launch_dequant_repacked(const QMatDev& m, uint32_t row0, uint32_t nrows, float* out, cudaStream_t s) {
    uint64_t n = (uint64_t)nrows * m.cols;
    if (n == 0) return cudaSuccess;
    uint64_t blocks = (n + 255) / 256;
    dequant_repacked_kernel<<<(unsigned)blocks, 256, 0, s>>>(m, row0, nrows, out);
    return cudaGetLastError();
}

}  // namespace evl
