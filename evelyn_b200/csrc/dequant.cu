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
