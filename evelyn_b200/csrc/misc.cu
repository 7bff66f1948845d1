// misc.cu -- embedding lookup, RMSNorm, residual add and greedy argmax.
//
//   embed   QMatrix::row (src/runtime.rs:54-69): one exactly dequantised row per
//           token, with the out-of-vocabulary check of validate_token_ids
//           (src/runtime.rs:125-135) mirrored as a device error flag.
//   rmsnorm rms_norm (src/runtime.rs:193-196) in the reference's v*inv*g order.
//   argmax  src/runtime.rs:897-905: strict '>' from f32::MIN, so the first maximum
//           wins and NaN is never picked; also feeds the next token on the device.
#include <cfloat>

#include "dequant.cuh"
#include "kernels.h"

namespace evl {

namespace {

cudaLaunchConfig_t cfg_of(dim3 grid, dim3 block, cudaStream_t s, bool pdl, cudaLaunchAttribute* attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = s;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cfg;
}

// grid (ceil(cols/256), batch)
__global__ void embed_kernel(QMatDev m, const int32_t* __restrict__ tokens, float* __restrict__ x, int32_t* err) {
    pdl_wait();
    const uint32_t b = blockIdx.y, c = blockIdx.x * blockDim.x + threadIdx.x;
    const int32_t tok = tokens[b];
    if (tok < 0 || (uint32_t)tok >= m.rows) {
        if (c == 0) atomicExch(err, DEV_ERR_TOKEN);
        return;
    }
    if (c < m.cols) x[(uint64_t)b * m.cols + c] = dq_repacked_value(m, (uint32_t)tok, c);
    pdl_launch_dependents();
}

// grid (batch), block 256
__global__ void rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w, float* __restrict__ y,
                               uint32_t n, float eps) {
    __shared__ float red[8];
    pdl_wait();
    const float* xb = x + (uint64_t)blockIdx.x * n;
    float* yb = y + (uint64_t)blockIdx.x * n;
    float ss = 0.f;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) ss += xb[i] * xb[i];
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    ss = 0.f;
    for (uint32_t i = 0; i < blockDim.x / 32; ++i) ss += red[i];
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) yb[i] = __fmul_rn(__fmul_rn(xb[i], inv), w[i]);
    pdl_launch_dependents();
}

__global__ void add_kernel(float* __restrict__ x, const float* __restrict__ y, uint64_t n) {
    pdl_wait();
    const uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) x[i] += y[i];
    pdl_launch_dependents();
}

// candidate order: larger value, then smaller index
__device__ __forceinline__ void better(float& bv, int32_t& bi, float v, int32_t i) {
    if (v > bv || (v == bv && i < bi)) {
        bv = v;
        bi = i;
    }
}

// grid (parts, batch), block 256: each part scans a contiguous slice
__global__ void argmax_part_kernel(const float* __restrict__ logits, uint32_t n, float* part_v, int32_t* part_i) {
    pdl_wait();
    const uint32_t b = blockIdx.y, parts = gridDim.x;
    const uint32_t per = (n + parts - 1) / parts;
    const uint32_t lo = blockIdx.x * per, hi = min(n, lo + per);
    const float* lb = logits + (uint64_t)b * n;
    float bv = -FLT_MAX;  // f32::MIN: only values strictly above it are taken
    int32_t bi = INT32_MAX;
    for (uint32_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        const float v = lb[i];
        if (v > bv) {  // strict: ties keep the earlier index of this thread; NaN never wins
            bv = v;
            bi = (int32_t)i;
        }
    }
    __shared__ float sv[256];
    __shared__ int32_t si[256];
    sv[threadIdx.x] = bv;
    si[threadIdx.x] = bi;
    __syncthreads();
    for (uint32_t s = blockDim.x / 2; s > 0; s >>= 1) {
        if (threadIdx.x < s) {
            float v = sv[threadIdx.x];
            int32_t i = si[threadIdx.x];
            better(v, i, sv[threadIdx.x + s], si[threadIdx.x + s]);
            sv[threadIdx.x] = v;
            si[threadIdx.x] = i;
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        part_v[b * parts + blockIdx.x] = sv[0];
        part_i[b * parts + blockIdx.x] = si[0];
    }
    pdl_launch_dependents();
}

// grid (batch), block 32. Also ends the step: the chosen token becomes the next
// input (greedy loop on the device), is logged at hist[b][pos], and pos advances
// (Session::step's `self.pos += 1`, src/runtime.rs:806).
__global__ void argmax_final_kernel(const float* part_v, const int32_t* part_i, uint32_t parts, int32_t* out,
                                    int32_t* next_tokens, int32_t* pos, int32_t* hist, uint32_t hist_stride,
                                    uint32_t* epoch) {
    pdl_wait();
    const uint32_t b = blockIdx.x;
    float bv = -FLT_MAX;
    int32_t bi = INT32_MAX;
    for (uint32_t p = threadIdx.x; p < parts; p += 32) better(bv, bi, part_v[b * parts + p], part_i[b * parts + p]);
    for (int o = 16; o > 0; o >>= 1) {
        const float v = __shfl_xor_sync(0xffffffffu, bv, o);
        const int32_t i = __shfl_xor_sync(0xffffffffu, bi, o);
        better(bv, bi, v, i);
    }
    if (threadIdx.x == 0) {
        const int32_t r = bi == INT32_MAX ? 0 : bi;  // nothing above f32::MIN: index 0
        out[b] = r;
        if (next_tokens) next_tokens[b] = r;
        if (pos) {
            const int32_t p = pos[b];
            if (hist && (uint32_t)p < hist_stride) hist[(uint64_t)b * hist_stride + p] = r;
            pos[b] = p + 1;
        }
        if (epoch && b == 0) *epoch += 1;  // the step is complete: the next one's tags
    }
    pdl_launch_dependents();
}

// ---- sampling (src/server.rs:326-352, sample_token): max, f32 weights exp((v - max) / T)
// summed in f64, one xorshift64* draw, the first index whose running sum reaches
// draw * total. The sum runs in parts (a fixed order, so a result never changes from
// run to run); its rounding can differ from the reference's left-to-right f64 sum only
// in the last bits, which moves the pick only when the draw lands within that of a
// boundary between two tokens.

// grid (parts, batch), block 256: per part the maximum (f32::max: NaN ignored)
__global__ void sample_max_kernel(const float* __restrict__ logits, uint32_t n, float* part_m) {
    const uint32_t b = blockIdx.y, parts = gridDim.x, per = (n + parts - 1) / parts;
    const uint32_t lo = blockIdx.x * per, hi = min(n, lo + per);
    const float* lb = logits + (uint64_t)b * n;
    float m = -INFINITY;
    for (uint32_t i = lo + threadIdx.x; i < hi; i += blockDim.x) m = fmaxf(m, lb[i]);
    m = warp_max(m);
    __shared__ float sm[8];
    if ((threadIdx.x & 31) == 0) sm[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        float r = sm[0];
        for (uint32_t w = 1; w < blockDim.x / 32; ++w) r = fmaxf(r, sm[w]);
        part_m[b * parts + blockIdx.x] = r;
    }
}

__device__ __forceinline__ float seq_max(const float* part_m, uint32_t b, uint32_t parts) {
    float m = -INFINITY;
    for (uint32_t p = 0; p < parts; ++p) m = fmaxf(m, part_m[b * parts + p]);
    return m;
}
__device__ __forceinline__ double sample_weight(float v, float maximum, float temperature) {
    return (double)expf(__fdiv_rn(__fsub_rn(v, maximum), temperature));
}

// grid (parts, batch), block 256: per part the f64 sum of the weights (fixed tree order)
__global__ void sample_sum_kernel(const float* __restrict__ logits, uint32_t n, const float* part_m, float temperature,
                                  double* part_s) {
    const uint32_t b = blockIdx.y, parts = gridDim.x, per = (n + parts - 1) / parts;
    const uint32_t lo = blockIdx.x * per, hi = min(n, lo + per);
    const float* lb = logits + (uint64_t)b * n;
    const float maximum = seq_max(part_m, b, parts);
    double s = 0.0;
    for (uint32_t i = lo + threadIdx.x; i < hi; i += blockDim.x) s += sample_weight(lb[i], maximum, temperature);
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    __shared__ double sd[8];
    if ((threadIdx.x & 31) == 0) sd[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double r = 0.0;
        for (uint32_t w = 0; w < blockDim.x / 32; ++w) r += sd[w];
        part_s[b * parts + blockIdx.x] = r;
    }
}

// grid (batch), block 32: the draw, the part holding the threshold, then the index
// inside it (32 weights at a time, an f64 scan across the lanes); the greedy pick
// `argmax[b]` when the total is not finite and positive or nothing reaches the draw.
__global__ void sample_pick_kernel(const float* __restrict__ logits, uint32_t n, const float* part_m,
                                   const double* part_s, uint32_t parts, float temperature, uint64_t* rng,
                                   const int32_t* argmax, int32_t* out) {
    const uint32_t b = blockIdx.x, lane = threadIdx.x;
    const float* lb = logits + (uint64_t)b * n;
    const float maximum = seq_max(part_m, b, parts);
    double total = 0.0;
    for (uint32_t p = 0; p < parts; ++p) total += part_s[b * parts + p];
    int32_t pick = argmax[b];
    if (isfinite(total) && total > 0.0) {
        uint64_t x = rng[b];
        x ^= x >> 12;
        x ^= x << 25;
        x ^= x >> 27;
        __syncwarp();
        if (lane == 0) rng[b] = x;
        const double unit = (double)((x * 0x2545F4914F6CDD1Dull) >> 11) / 9007199254740992.0;  // / 2^53
        const double threshold = unit * total;
        double cum = 0.0;
        uint32_t p = 0;
        for (; p < parts; ++p) {
            if (cum + part_s[b * parts + p] >= threshold) break;
            cum += part_s[b * parts + p];
        }
        if (p < parts) {
            const uint32_t per = (n + parts - 1) / parts, lo = p * per, hi = min(n, lo + per);
            for (uint32_t i0 = lo; i0 < hi; i0 += 32) {
                const uint32_t i = i0 + lane;
                double w = i < hi ? sample_weight(lb[i], maximum, temperature) : 0.0;
                for (int o = 1; o < 32; o <<= 1) {  // inclusive scan
                    const double t = __shfl_up_sync(0xffffffffu, w, o);
                    if (lane >= (uint32_t)o) w += t;
                }
                const unsigned hit = __ballot_sync(0xffffffffu, i < hi && cum + w >= threshold);
                if (hit) {
                    pick = (int32_t)(i0 + __ffs(hit) - 1);
                    break;
                }
                cum += __shfl_sync(0xffffffffu, w, 31);
            }
        }
    }
    if (lane == 0) out[b] = pick;
}

}  // namespace

cudaError_t launch_sample(const float* logits, uint32_t n, uint32_t batch, float temperature, uint64_t* rng,
                          const int32_t* argmax, float* part_m, double* part_s, uint32_t parts, int32_t* out,
                          cudaStream_t s) {
    if (!parts || !batch) return cudaErrorInvalidValue;
    sample_max_kernel<<<dim3(parts, batch), 256, 0, s>>>(logits, n, part_m);
    sample_sum_kernel<<<dim3(parts, batch), 256, 0, s>>>(logits, n, part_m, temperature, part_s);
    sample_pick_kernel<<<batch, 32, 0, s>>>(logits, n, part_m, part_s, parts, temperature, rng, argmax, out);
    return cudaGetLastError();
}

cudaError_t launch_embed(const QMatDev& embed, const int32_t* tokens, uint32_t batch, float* x, int32_t* err,
                         cudaStream_t s, bool pdl) {
    cudaLaunchAttribute at[1];
    auto cfg = cfg_of(dim3((embed.cols + 255) / 256, batch), dim3(256), s, pdl, at);
    return cudaLaunchKernelEx(&cfg, embed_kernel, embed, tokens, x, err);
}

cudaError_t launch_rmsnorm(const float* x, const float* w, float* y, uint32_t n, uint32_t batch, float eps,
                           cudaStream_t s, bool pdl) {
    cudaLaunchAttribute at[1];
    auto cfg = cfg_of(dim3(batch), dim3(256), s, pdl, at);
    return cudaLaunchKernelEx(&cfg, rmsnorm_kernel, x, w, y, n, eps);
}

__global__ void l2_prefetch_kernel(const __grid_constant__ L2Ranges r) {
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x, first = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
    for (int i = 0; i < 4; ++i) {
        if (!r.base[i]) continue;
        const uint64_t chunks = (r.bytes[i] + 16383) / 16384;
        for (uint64_t c = first; c < chunks; c += stride) {
            const uint64_t off = c * 16384, n = (r.bytes[i] - off < 16384 ? r.bytes[i] - off : 16384) & ~15ull;
            if (n) prefetch_l2_bulk(r.base[i] + off, (uint32_t)n);
        }
    }
}

cudaError_t launch_l2_prefetch(const L2Ranges& r, cudaStream_t s) {
    for (int i = 0; i < 4; ++i)
        if (r.base[i] && (reinterpret_cast<uintptr_t>(r.base[i]) & 15)) return cudaErrorMisalignedAddress;
    cudaLaunchAttribute at[1];
    auto cfg = cfg_of(dim3(148), dim3(32), s, false, at);
    return cudaLaunchKernelEx(&cfg, l2_prefetch_kernel, r);
}

cudaError_t launch_add(float* x, const float* y, uint64_t n, cudaStream_t s, bool pdl) {
    cudaLaunchAttribute at[1];
    auto cfg = cfg_of(dim3((unsigned)((n + 255) / 256)), dim3(256), s, pdl, at);
    return cudaLaunchKernelEx(&cfg, add_kernel, x, y, n);
}

cudaError_t launch_argmax(const float* logits, uint32_t n, uint32_t batch, float* part_v, int32_t* part_i,
                          uint32_t parts, int32_t* out, int32_t* next_tokens, int32_t* pos, int32_t* hist,
                          uint32_t hist_stride, cudaStream_t s, bool pdl, uint32_t* epoch) {
    cudaLaunchAttribute at[1];
    auto cfg = cfg_of(dim3(parts, batch), dim3(256), s, pdl, at);
    cudaError_t e = cudaLaunchKernelEx(&cfg, argmax_part_kernel, logits, n, part_v, part_i);
    if (e != cudaSuccess) return e;
    auto cfg2 = cfg_of(dim3(batch), dim3(32), s, pdl, at);
    return cudaLaunchKernelEx(&cfg2, argmax_final_kernel, (const float*)part_v, (const int32_t*)part_i, parts, out,
                              next_tokens, pos, hist, hist_stride, epoch);
}

}  // namespace evl
