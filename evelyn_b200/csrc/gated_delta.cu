// gated_delta.cu -- the recurrent half of a Qwen3.5 gated-delta layer
// (gated_delta_attention, src/runtime.rs:551-630, and gated_delta_step, :493-528). (The
// sigmoid query gate of its full-attention layers, :753-761, is applied by the
// attention kernels as they write their output.)
//
// The projections around it are ordinary matvec launches: attn_qkv, attn_gate (z) and
// ssm_alpha | ssm_beta (stacked at load into one matrix) in one, ssm_out with the
// residual add after it.
// One CTA per (value head, sequence) then does everything between:
//   * the depthwise causal convolution of the channels it reads (its key head's q and
//     k channels, its own v channels) over the kernel - 1 previous projections and this
//     token's, then x * sigmoid(x);
//   * the L2 normalisation of q and k (sqrt(sum + eps));
//   * decay = exp(softplus(alpha + dt) * a), beta = sigmoid(beta);
//   * the delta rule on its [key_dim][value_dim] state, one thread per value column:
//     the decayed column's prediction k.S, the correction (v - k.S) * beta added as
//     k (x) delta, the read-out q.S / sqrt(key_dim); the state is read twice (the second
//     read from L2) and written once;
//   * the per-head RMSNorm with ssm_norm and the SiLU(z) gate.
// Products and sums keep the reference's f32 operation order where it is sequential
// (one rounding per multiply and per add, no fused multiply-add), except the q, k and
// output sums of squares, which are block reductions.
//
// Convolution history. A key head's q and k channels are read by every value head that
// maps to it (head % key_heads) but written by one; so that no CTA reads history that
// another has already moved on, each sequence keeps two copies of its kernel - 1 rows
// and the token at position p reads copy p % 2 and writes copy (p + 1) % 2. The CTA of
// value head h writes its v channels and, when h < key_heads, key head h's q and k
// channels (a key head that no value head maps to is never read).
//
// The state update is the kernel's cost: 2 x 4 x key_dim x value_dim bytes per head
// read and written. One CTA per head reading its columns with one thread each (the
// first version) leaves the loads waiting on memory latency. The cluster variant
// splits a head's value columns over a cluster of up to 4 CTAs, each of which stages
// its [key_dim][cols] slice of the state in shared memory with 16-byte loads, works on
// it with several threads per column (the keys dealt round-robin, the partial sums
// added in key-group order), and writes it back. The per-head RMSNorm's sum of squares
// meets through distributed shared memory: every CTA stores its partial into slot
// `rank` of every CTA of the cluster, which add the slots in rank order.
#include <algorithm>
#include <atomic>
#include <cooperative_groups.h>
#include <cstdlib>

#include "common.cuh"
#include "kernels.h"

namespace evl {

namespace cg = cooperative_groups;

namespace {

constexpr int kThreads = 128;

// runtime.rs:485-487
__device__ __forceinline__ float softplus_ref(float x) { return x > 20.0f ? x : log1pf(expf(x)); }

// 16-byte asynchronous copy global -> shared (completes at cp_async_wait)
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(smem)),
                 "l"(gmem)
                 : "memory");
}
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

// sum over the block (kThreads threads); every thread gets the total
__device__ float block_sum(float v, float* red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();  // red may still be read by a previous call
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) t += red[w];
    return t;
}

__global__ void __launch_bounds__(kThreads) gated_delta_kernel(const __grid_constant__ GatedDeltaArgs a) {
    extern __shared__ __align__(16) float sm[];
    __shared__ float red[kThreads / 32];
    const uint32_t KD = a.key_dim, VD = a.value_dim, CH = a.channels, KW = a.key_dim * a.key_heads;
    float* qs = sm;         // [KD] q, then q / |q|
    float* ks = qs + KD;    // [KD]
    float* vs = ks + KD;    // [VD]
    float* os = vs + VD;    // [VD] the read-out
    const uint32_t head = blockIdx.x, seq = blockIdx.y, kh = head % a.key_heads;
    const int tid = threadIdx.x;
    pdl_wait();
    const int32_t p = a.pos[seq];
    const uint32_t K1 = a.kernel - 1;
    const float* proj = a.proj + (uint64_t)seq * CH;
    const float* hr = a.hist + (uint64_t)seq * a.hist_stride + (uint64_t)(p & 1) * K1 * CH;
    float* hw = a.hist + (uint64_t)seq * a.hist_stride + (uint64_t)((p + 1) & 1) * K1 * CH;
    // ---- convolution (runtime.rs:562-579) of this CTA's 2 KD + VD channels
    for (uint32_t i = tid; i < 2 * KD + VD; i += kThreads) {
        const uint32_t ch = i < KD ? kh * KD + i : i < 2 * KD ? KW + kh * KD + (i - KD) : 2 * KW + head * VD + (i - 2 * KD);
        float sum = 0.0f;
        for (uint32_t tap = 0; tap < a.kernel; ++tap) {
            const float in = tap < K1 ? hr[(uint64_t)tap * CH + ch] : proj[ch];
            sum = __fadd_rn(sum, __fmul_rn(in, a.conv[(uint64_t)ch * a.kernel + tap]));
        }
        const float c = __fmul_rn(sum, sigmoid_ref(sum));
        if (i < KD) qs[i] = c; else if (i < 2 * KD) ks[i - KD] = c; else vs[i - 2 * KD] = c;
        if (i >= 2 * KD || head == kh)  // this CTA owns the channel's history
            for (uint32_t tap = 0; tap < K1; ++tap)
                hw[(uint64_t)tap * CH + ch] = tap + 1 < K1 ? hr[(uint64_t)(tap + 1) * CH + ch] : proj[ch];
    }
    __syncthreads();
    // ---- q and k over their L2 norms (runtime.rs:596-600)
    float sq = 0.f, sk = 0.f;
    for (uint32_t i = tid; i < KD; i += kThreads) {
        sq += qs[i] * qs[i];
        sk += ks[i] * ks[i];
    }
    const float qn = __fsqrt_rn(__fadd_rn(block_sum(sq, red), a.eps));
    const float kn = __fsqrt_rn(__fadd_rn(block_sum(sk, red), a.eps));
    for (uint32_t i = tid; i < KD; i += kThreads) {
        qs[i] = __fdiv_rn(qs[i], qn);
        ks[i] = __fdiv_rn(ks[i], kn);
    }
    const float* ab = a.ab + (uint64_t)seq * 2 * a.value_heads;
    const float decay = expf(__fmul_rn(softplus_ref(__fadd_rn(ab[head], a.dt[head])), a.a[head]));
    const float beta = sigmoid_ref(ab[a.value_heads + head]);
    __syncthreads();
    // ---- the delta rule (runtime.rs:493-528), one thread per value column
    float* S = a.state + (uint64_t)seq * a.state_stride + (uint64_t)head * KD * VD;
    const float root = __fsqrt_rn((float)KD);
    for (uint32_t v = tid; v < VD; v += kThreads) {
        float pred = 0.0f;
        for (uint32_t key = 0; key < KD; ++key)
            pred = __fadd_rn(pred, __fmul_rn(__fmul_rn(S[(uint64_t)key * VD + v], decay), ks[key]));
        const float delta = __fmul_rn(__fsub_rn(vs[v], pred), beta);
        float acc = 0.0f;
        for (uint32_t key = 0; key < KD; ++key) {
            const uint64_t o = (uint64_t)key * VD + v;
            const float s = __fadd_rn(__fmul_rn(S[o], decay), __fmul_rn(ks[key], delta));
            S[o] = s;
            acc = __fadd_rn(acc, __fmul_rn(s, qs[key]));
        }
        os[v] = __fdiv_rn(acc, root);
    }
    __syncthreads();
    // ---- per-head RMSNorm and the SiLU(z) gate (runtime.rs:617-628, 193-196)
    float ss = 0.f;
    for (uint32_t v = tid; v < VD; v += kThreads) ss += os[v] * os[v];
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(block_sum(ss, red), (float)VD), a.eps)));
    const uint64_t o0 = (uint64_t)seq * a.value_heads * VD + (uint64_t)head * VD;
    for (uint32_t v = tid; v < VD; v += kThreads) {
        const float zz = a.z[o0 + v];
        a.out[o0 + v] = __fmul_rn(__fmul_rn(__fmul_rn(os[v], inv), a.norm[v]), __fmul_rn(zz, sigmoid_ref(zz)));
    }
}

// CTAs per head (cluster size), value columns per CTA, threads per column
struct SliceShape {
    uint32_t S = 0, C = 0, G = 0;
};
constexpr uint32_t kMaxCluster = 4;
constexpr size_t kSliceSmemCap = 160 * 1024;

SliceShape slice_shape(uint32_t value_dim) {
    for (uint32_t S = kMaxCluster; S >= 1; S /= 2) {
        if (value_dim % (4 * S)) continue;  // whole float4 rows per CTA
        SliceShape sh;
        sh.S = S;
        sh.C = value_dim / S;
        sh.G = (sh.C <= (uint32_t)kThreads && kThreads % sh.C == 0) ? kThreads / sh.C : 1;
        return sh;
    }
    return SliceShape{};
}
size_t slice_smem(uint32_t key_dim, const SliceShape& sh) {
    return 4ull * ((uint64_t)key_dim * sh.C + 2 * key_dim + 3 * sh.C + (uint64_t)sh.G * sh.C + kMaxCluster);
}

__global__ void __launch_bounds__(kThreads) gated_delta_slice_kernel(const __grid_constant__ GatedDeltaArgs a,
                                                                      uint32_t S, uint32_t C, uint32_t G) {
    extern __shared__ __align__(16) float sm[];
    __shared__ float red[kThreads / 32];
    cg::cluster_group cl = cg::this_cluster();
    const uint32_t KD = a.key_dim, VD = a.value_dim, CH = a.channels, KW = a.key_dim * a.key_heads;
    float* Ss = sm;               // [KD][C] this CTA's slice of the state
    float* qs = Ss + KD * C;      // [KD]
    float* ks = qs + KD;          // [KD]
    float* vs = ks + KD;          // [C]
    float* os = vs + C;           // [C] the read-out
    float* dl = os + C;           // [C] the delta rule's correction
    float* part = dl + C;         // [G][C] per key group partial sums
    float* ssq = part + G * C;    // [kMaxCluster] the cluster's sums of squares, by rank
    const uint32_t head = blockIdx.x / S, rank = blockIdx.x % S, seq = blockIdx.y, kh = head % a.key_heads;
    const uint32_t c0 = rank * C;
    const int tid = threadIdx.x;
    pdl_wait();
    const int32_t p = a.pos[seq];
    const uint32_t K1 = a.kernel - 1;
    const float* proj = a.proj + (uint64_t)seq * CH;
    const float* hr = a.hist + (uint64_t)seq * a.hist_stride + (uint64_t)(p & 1) * K1 * CH;
    float* hw = a.hist + (uint64_t)seq * a.hist_stride + (uint64_t)((p + 1) & 1) * K1 * CH;
    float* St = a.state + (uint64_t)seq * a.state_stride + (uint64_t)head * KD * VD;
    // ---- the state slice into shared memory (rows of C floats at column c0), in flight
    // during the convolution and the q / k norms
    const uint32_t q4 = C / 4;
    for (uint32_t i = tid; i < KD * q4; i += kThreads)
        cp_async16(Ss + 4 * i, St + (uint64_t)(i / q4) * VD + c0 + 4 * (i % q4));
    // ---- convolution of the key head's q and k channels and this slice's v channels
    // (up to 8 taps with their loads issued together, longer kernels tap by tap)
    for (uint32_t i = tid; i < 2 * KD + C; i += kThreads) {
        const uint32_t ch =
            i < KD ? kh * KD + i : i < 2 * KD ? KW + kh * KD + (i - KD) : 2 * KW + head * VD + c0 + (i - 2 * KD);
        float sum = 0.0f;
        if (a.kernel <= 8) {
            float in[8], w[8];
#pragma unroll
            for (uint32_t tap = 0; tap < 8; ++tap)
                if (tap < a.kernel) {
                    in[tap] = tap < K1 ? hr[(uint64_t)tap * CH + ch] : proj[ch];
                    w[tap] = a.conv[(uint64_t)ch * a.kernel + tap];
                }
#pragma unroll
            for (uint32_t tap = 0; tap < 8; ++tap)
                if (tap < a.kernel) sum = __fadd_rn(sum, __fmul_rn(in[tap], w[tap]));
        } else {
            for (uint32_t tap = 0; tap < a.kernel; ++tap) {
                const float in = tap < K1 ? hr[(uint64_t)tap * CH + ch] : proj[ch];
                sum = __fadd_rn(sum, __fmul_rn(in, a.conv[(uint64_t)ch * a.kernel + tap]));
            }
        }
        const float c = __fmul_rn(sum, sigmoid_ref(sum));
        if (i < KD) qs[i] = c; else if (i < 2 * KD) ks[i - KD] = c; else vs[i - 2 * KD] = c;
        if (i >= 2 * KD || (head == kh && rank == 0))  // this CTA owns the channel's history
            for (uint32_t tap = 0; tap < K1; ++tap)
                hw[(uint64_t)tap * CH + ch] = tap + 1 < K1 ? hr[(uint64_t)(tap + 1) * CH + ch] : proj[ch];
    }
    __syncthreads();
    float sq = 0.f, sk = 0.f;
    for (uint32_t i = tid; i < KD; i += kThreads) {
        sq += qs[i] * qs[i];
        sk += ks[i] * ks[i];
    }
    const float qn = __fsqrt_rn(__fadd_rn(block_sum(sq, red), a.eps));
    const float kn = __fsqrt_rn(__fadd_rn(block_sum(sk, red), a.eps));
    for (uint32_t i = tid; i < KD; i += kThreads) {
        qs[i] = __fdiv_rn(qs[i], qn);
        ks[i] = __fdiv_rn(ks[i], kn);
    }
    const float* ab = a.ab + (uint64_t)seq * 2 * a.value_heads;
    const float decay = expf(__fmul_rn(softplus_ref(__fadd_rn(ab[head], a.dt[head])), a.a[head]));
    const float beta = sigmoid_ref(ab[a.value_heads + head]);
    cp_async_wait();  // this thread's slice copies
    __syncthreads();  // everyone's, and the normalised q / k
    // ---- the delta rule: thread (key group kg, column c) takes keys kg, kg + G, ...
    const uint32_t kg = G > 1 ? tid / C : 0;
    const uint32_t cfirst = G > 1 ? tid % C : (uint32_t)tid, cstride = G > 1 ? C : (uint32_t)kThreads;
    for (uint32_t c = cfirst; c < C; c += cstride) {
        float pr = 0.0f;
        for (uint32_t key = kg; key < KD; key += G)
            pr = __fadd_rn(pr, __fmul_rn(__fmul_rn(Ss[key * C + c], decay), ks[key]));
        part[kg * C + c] = pr;
    }
    __syncthreads();
    for (uint32_t c = tid; c < C; c += kThreads) {
        float pred = 0.0f;
        for (uint32_t g = 0; g < G; ++g) pred = __fadd_rn(pred, part[g * C + c]);
        dl[c] = __fmul_rn(__fsub_rn(vs[c], pred), beta);
    }
    __syncthreads();
    for (uint32_t c = cfirst; c < C; c += cstride) {
        const float d = dl[c];
        float acc = 0.0f;
        for (uint32_t key = kg; key < KD; key += G) {
            const float v = __fadd_rn(__fmul_rn(Ss[key * C + c], decay), __fmul_rn(ks[key], d));
            Ss[key * C + c] = v;
            acc = __fadd_rn(acc, __fmul_rn(v, qs[key]));
        }
        part[kg * C + c] = acc;
    }
    __syncthreads();
    for (uint32_t i = tid; i < KD * q4; i += kThreads)
        *reinterpret_cast<float4*>(St + (uint64_t)(i / q4) * VD + c0 + 4 * (i % q4)) =
            reinterpret_cast<const float4*>(Ss)[i];
    const float root = __fsqrt_rn((float)KD);
    float ss = 0.f;
    for (uint32_t c = tid; c < C; c += kThreads) {
        float acc = 0.0f;
        for (uint32_t g = 0; g < G; ++g) acc = __fadd_rn(acc, part[g * C + c]);
        const float o = __fdiv_rn(acc, root);
        os[c] = o;
        ss += o * o;
    }
    // ---- the per-head RMSNorm over the cluster's columns, then the SiLU(z) gate
    const float ssc = block_sum(ss, red);
    if ((uint32_t)tid < S) *cl.map_shared_rank(ssq + rank, (unsigned)tid) = ssc;
    cl.sync();
    float tot = 0.f;
    for (uint32_t r = 0; r < S; ++r) tot += ssq[r];
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)VD), a.eps)));
    const uint64_t o0 = (uint64_t)seq * a.value_heads * VD + (uint64_t)head * VD + c0;
    for (uint32_t c = tid; c < C; c += kThreads) {
        const float zz = a.z[o0 + c];
        a.out[o0 + c] = __fmul_rn(__fmul_rn(__fmul_rn(os[c], inv), a.norm[c0 + c]), __fmul_rn(zz, sigmoid_ref(zz)));
    }
}

cudaLaunchConfig_t cfg_of(dim3 grid, dim3 block, size_t smem, cudaStream_t s, bool pdl, cudaLaunchAttribute* attr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cfg;
}

}  // namespace

size_t gated_delta_smem(uint32_t key_dim, uint32_t value_dim) { return 4ull * (2 * key_dim + 2 * value_dim); }

cudaError_t launch_gated_delta(const GatedDeltaArgs& a, cudaStream_t s, bool pdl) {
    if (!a.proj || !a.z || !a.ab || !a.conv || !a.a || !a.dt || !a.norm || !a.hist || !a.state || !a.out || !a.pos)
        return cudaErrorInvalidValue;
    if (!a.batch || !a.kernel || !a.key_dim || !a.key_heads || !a.value_dim || !a.value_heads ||
        a.channels != 2 * a.key_dim * a.key_heads + a.value_dim * a.value_heads)
        return cudaErrorInvalidValue;
    if (a.hist_stride < 2ull * (a.kernel - 1) * a.channels ||
        a.state_stride < (uint64_t)a.value_heads * a.key_dim * a.value_dim)
        return cudaErrorInvalidValue;
    const SliceShape sh = slice_shape(a.value_dim);
    const size_t ssm = sh.S ? slice_smem(a.key_dim, sh) : 0;
    const char* ve = std::getenv("EVELYN_DELTA_SLICES");  // 0: the one-CTA-per-head kernel (tests)
    if (sh.S && ssm <= kSliceSmemCap && !(ve && ve[0] == '0')) {
        if (ssm > 48 * 1024) {  // the opt-in, once per device
            static std::atomic<bool> done[64];
            int dev = 0;
            cudaError_t e = cudaGetDevice(&dev);
            if (e != cudaSuccess) return e;
            if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
            if (!done[dev].load()) {
                e = cudaFuncSetAttribute(gated_delta_slice_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)kSliceSmemCap);
                if (e != cudaSuccess) return e;
                done[dev] = true;
            }
        }
        cudaLaunchAttribute at[2];
        auto cfg = cfg_of(dim3(a.value_heads * sh.S, a.batch), dim3(kThreads), ssm, s, pdl, at);
        at[cfg.numAttrs].id = cudaLaunchAttributeClusterDimension;
        at[cfg.numAttrs].val.clusterDim.x = sh.S;
        at[cfg.numAttrs].val.clusterDim.y = 1;
        at[cfg.numAttrs].val.clusterDim.z = 1;
        cfg.numAttrs += 1;
        return cudaLaunchKernelEx(&cfg, gated_delta_slice_kernel, a, sh.S, sh.C, sh.G);
    }
    const size_t smem = gated_delta_smem(a.key_dim, a.value_dim);
    if (smem > 48 * 1024) return cudaErrorInvalidValue;  // key_dim + value_dim up to 6144
    cudaLaunchAttribute at[1];
    auto cfg = cfg_of(dim3(a.value_heads, a.batch), dim3(kThreads), smem, s, pdl, at);
    return cudaLaunchKernelEx(&cfg, gated_delta_kernel, a);
}

}  // namespace evl
