// plain_matvec.cu -- y = W x for matrices stored unquantised, as F16, BF16 or F32
// (QMatrix::matvec, src/runtime.rs:72-88, over the tensor types gguf.rs:338-352 reads).
//
// One warp per output row: the row's values are read straight from the plain panel
// layout (each row of a 16-row slab contiguous inside a 32-unit panel, common.cuh
// plain_value_address) with 16-byte loads, multiplied by x (times the RMSNorm weight,
// staged once per CTA in f32 in shared memory) and summed per lane, then across the
// warp; 1/rms and the epilogue (store, residual add, SiLU(gate) * up) are the quantised
// matvec's. A quantised segment of a launch that also holds an unquantised one is read
// through the exact dequantiser, and so are gate and up matrices of two different
// quantised types (the quantised kernel streams both through one ring of one layout).
// Unquantised projection matrices are rare in the GGUFs
// this engine serves, so the kernel is built for coverage: it reads every weight byte
// once, but does not pipeline its loads like the quantised matvec.
#include <algorithm>
#include <atomic>

#include "dequant.cuh"
#include "kernels.h"

namespace evl {

namespace {

constexpr int kPW = 16;  // warps per CTA

__device__ __forceinline__ bool plain_type(uint32_t t) { return t == GGML_F16 || t == GGML_BF16 || t == GGML_F32; }

__device__ __forceinline__ float half_bits(uint32_t T, uint32_t h) {
    return T == GGML_F16 ? f16_exact(h) : __uint_as_float(h << 16);
}

// sum over the row's cols values of W[r][c] * xs[c], lane partial sums added across the warp
__device__ float row_dot(const QMatDev& m, uint32_t r, const float* xs, uint32_t cols, int lane) {
    float acc = 0.f;
    const uint32_t T = m.type;
    if (plain_type(T)) {
        const uint32_t eb = T == GGML_F32 ? 4 : 2;
        for (uint32_t g = 0; g * kPanelUnits < m.nunits; ++g) {
            const uint32_t c0 = g * kPanelUnits * 64, n = group_units(m.nunits, g) * 64;
            const uint8_t* base = m.q + plain_value_address(m, r, c0, eb);
            for (uint32_t c = 8 * (uint32_t)lane; c < n; c += 256) {  // 8 values per lane and step
                float w[8];
                if (eb == 2) {
                    const uint4 v = *reinterpret_cast<const uint4*>(base + (size_t)c * 2);
                    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        w[2 * k] = half_bits(T, u[k] & 0xffffu);
                        w[2 * k + 1] = half_bits(T, u[k] >> 16);
                    }
                } else {
                    const float4 v0 = *reinterpret_cast<const float4*>(base + (size_t)c * 4);
                    const float4 v1 = *reinterpret_cast<const float4*>(base + (size_t)c * 4 + 16);
                    w[0] = v0.x; w[1] = v0.y; w[2] = v0.z; w[3] = v0.w;
                    w[4] = v1.x; w[5] = v1.y; w[6] = v1.z; w[7] = v1.w;
                }
                const float4 x0 = *reinterpret_cast<const float4*>(xs + c0 + c);
                const float4 x1 = *reinterpret_cast<const float4*>(xs + c0 + c + 4);
                const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
                for (int e = 0; e < 8; ++e) acc = fmaf(w[e], xv[e], acc);
            }
        }
    } else {
        for (uint32_t c = (uint32_t)lane; c < cols; c += 32) acc = fmaf(dq_repacked_value(m, r, c), xs[c], acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    return acc;
}

__device__ __forceinline__ float silu(float z) { return __fdiv_rn(z, __fadd_rn(1.0f, expf(-z))); }

__global__ void __launch_bounds__(kPW * 32) plain_matvec_kernel(const __grid_constant__ MatvecArgs a, uint32_t r1,
                                                                uint32_t r2, uint32_t total) {
    extern __shared__ __align__(16) float xs[];  // a.cols floats
    __shared__ float red[kPW];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t K = a.cols;
    pdl_wait();
    float ss = 0.f;
    for (uint32_t i = tid; i < K; i += blockDim.x) {
        const float v = __ldcg(a.x + i);
        ss += v * v;
        xs[i] = a.norm_w ? __fmul_rn(v, a.norm_w[i]) : v;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float inv = 1.f;
    if (a.norm_w) {
        float t = 0.f;
        for (int w = 0; w < kPW; ++w) t += red[w];
        inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)K), a.eps)));
    }
    pdl_launch_dependents();
    for (uint32_t row = blockIdx.x * kPW + warp; row < total; row += gridDim.x * kPW) {
        const int si = row >= r2 ? 2 : row >= r1 ? 1 : 0;
        const MatvecSeg& sg = a.seg[si];
        const uint32_t local = row - (si == 2 ? r2 : si == 1 ? r1 : 0);
        const float v = __fmul_rn(row_dot(sg.m, local, xs, K, lane), inv);
        // the up row: every lane takes part, the sum ends with a full-warp shuffle
        const float u = sg.epi == EPI_SWIGLU ? __fmul_rn(row_dot(sg.m2, local, xs, K, lane), inv) : 0.f;
        if (lane) continue;
        if (sg.epi == EPI_SWIGLU) {
            sg.y[local] = __fmul_rn(silu(v), u);
        } else if (sg.epi == EPI_ADD) {
            sg.y[local] = __ldcg(sg.y + local) + v;
        } else {
            sg.y[local] = v;
        }
    }
}

// dynamic shared memory opted in: the 227 KB a block may hold, less room for the
// static reduction array (the attribute counts only the dynamic part)
constexpr int kSmemOptIn = 226 * 1024;
constexpr int kMaxDevices = 64;
std::atomic<bool> g_opt_in[kMaxDevices];  // per device: the shared-memory opt-in is set

}  // namespace

bool matvec_has_plain(const MatvecArgs& a) {
    auto plain = [](uint32_t t) { return t == GGML_F16 || t == GGML_BF16 || t == GGML_F32; };
    for (int i = 0; i < a.nseg && i < kMaxSegs; ++i) {
        const MatvecSeg& sg = a.seg[i];
        if (plain(sg.m.type)) return true;
        // gate and up of different types: the quantised kernel streams both through one ring
        if (sg.epi == EPI_SWIGLU && (plain(sg.m2.type) || sg.m2.type != sg.m.type)) return true;
    }
    return false;
}

cudaError_t launch_plain_matvec(const MatvecArgs& a, cudaStream_t s, bool pdl) {
    if (a.nseg < 1 || a.nseg > kMaxSegs || a.cols == 0 || a.cols % 64 || !a.x || !a.err) return cudaErrorInvalidValue;
    uint32_t begin[kMaxSegs + 1] = {0, 0, 0, 0};
    for (int i = 0; i < kMaxSegs; ++i) {
        uint32_t rows = 0;
        if (i < a.nseg) {
            const MatvecSeg& sg = a.seg[i];
            if (sg.m.cols != a.cols || !sg.m.rows || !sg.y) return cudaErrorInvalidValue;
            if (sg.epi == EPI_SWIGLU && (sg.m2.rows != sg.m.rows || sg.m2.cols != a.cols)) return cudaErrorInvalidValue;
            if (sg.epi != EPI_STORE && sg.epi != EPI_ADD && sg.epi != EPI_SWIGLU) return cudaErrorInvalidValue;
            rows = sg.m.rows;
        }
        begin[i + 1] = begin[i] + rows;
    }
    const size_t smem = (size_t)a.cols * 4;
    if (smem > kSmemOptIn) return cudaErrorInvalidValue;
    {  // the shared-memory opt-in (x alone takes 48 KB at 12288 values), once per device
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return e;
        if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
        if (!g_opt_in[dev].load()) {
            e = cudaFuncSetAttribute(plain_matvec_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemOptIn);
            if (e != cudaSuccess) return e;
            g_opt_in[dev] = true;
        }
    }
    const uint32_t total = begin[a.nseg];
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(std::min<uint32_t>((total + kPW - 1) / kPW, 4 * 148));
    cfg.blockDim = dim3(kPW * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, plain_matvec_kernel, a, begin[1], begin[2], total);
}

}  // namespace evl
