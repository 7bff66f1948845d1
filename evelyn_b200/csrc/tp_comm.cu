// tp_comm.cu -- the tensor-parallel exchanges of a decode step over NVLink peer memory.
//
// Megatron tensor parallelism needs two sums per layer (the partial outputs of the
// row-split attn_output and ffn_down, each bs x d_model floats, 16 KB at bs1 for the
// 8B shape) and, at the end of the step, the greedy pick over the vocabulary shards of
// the LM head. Those are tiny, latency-bound exchanges: here each one is a single small
// kernel that stores this rank's values straight into every rank's inbox (peer memory
// mapped into this process) and then waits for the other ranks' values in its own.
// Every value travels as a tagged word -- (tag << 32) | f32 bits, one 8-byte store --
// so a reader knows a word is this step's without any flag or fence; the tag is
// `epoch * period + 1 + slot` (slot: which exchange of the step), and the step's pick
// advances the epoch. No collective library call remains inside the step, so the
// whole step stays one CUDA graph with programmatic dependent launches.
//
// The sums are added in rank order on every rank, so all ranks hold the same x.
// An inbox slot is written again only one step later for the same exchange, and a
// rank can only get there after every other rank has passed the reads of the previous
// use (each exchange of the next step needs this rank's contribution to the exchanges
// in between). Every wait is bounded (2 s) and reports DEV_ERR_WAIT_TIMEOUT.
#include <cfloat>

#include "kernels.h"

namespace evl {

namespace {

__device__ __forceinline__ void st_word(uint64_t* p, float v, uint32_t tag) {
    const uint64_t w = ((uint64_t)tag << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ uint64_t ld_word(const uint64_t* p) {
    uint64_t w;
    asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
__device__ __forceinline__ uint32_t tag_of(uint64_t w) { return (uint32_t)(w >> 32); }
__device__ __forceinline__ float val_of(uint64_t w) { return __uint_as_float((uint32_t)w); }

__device__ __forceinline__ uint64_t* slot_of(const TpPeers& P, uint32_t owner, uint32_t purpose, uint32_t sender) {
    return P.inbox[owner] + ((uint64_t)purpose * P.size + sender) * P.cap;
}

// Waits until the words w[0 .. n) (re-read from p[r * stride]) all carry `tag`.
__device__ __forceinline__ bool wait_words(const uint64_t* p, uint64_t stride, uint32_t n, uint32_t tag,
                                           uint64_t (&w)[kMaxPeers]) {
#pragma unroll
    for (int r = 0; r < kMaxPeers; ++r)
        if ((uint32_t)r < n) w[r] = ld_word(p + r * stride);
    uint64_t t0 = 0;
    for (;;) {
        bool all = true;
#pragma unroll
        for (int r = 0; r < kMaxPeers; ++r)
            if ((uint32_t)r < n) all &= tag_of(w[r]) == tag;
        if (all) return true;
        const uint64_t t = global_ns();
        if (!t0) t0 = t;
        else if (t - t0 > kWaitNs) return false;
#pragma unroll
        for (int r = 0; r < kMaxPeers; ++r)
            if ((uint32_t)r < n && tag_of(w[r]) != tag) w[r] = ld_word(p + r * stride);
    }
}

// x[i] += part_0[i] + part_1[i] + ... (rank order): the sum of the row-split matvec's
// partial outputs (o-proj / down-proj) fused with the residual add (src/runtime.rs:
// 798-800, 802-804).
__global__ void tp_allreduce_add_kernel(const TpPeers P, uint32_t purpose, uint32_t slot, float* __restrict__ x,
                                        const float* __restrict__ part, uint32_t n, int* err) {
    pdl_wait();
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    const uint32_t tag = *P.epoch * P.period + 1u + slot;
    if (i < n) {
        const float v = part[i];
        for (uint32_t r = 0; r < P.size; ++r) st_word(slot_of(P, r, purpose, P.rank) + i, v, tag);
        uint64_t w[kMaxPeers];
        if (wait_words(slot_of(P, P.rank, purpose, 0) + i, P.cap, P.size, tag, w)) {
            float sum = val_of(w[0]);
            for (uint32_t r = 1; r < P.size; ++r) sum += val_of(w[r]);
            x[i] = x[i] + sum;
        } else {
            atomicExch(err, DEV_ERR_WAIT_TIMEOUT);
        }
    }
    pdl_launch_dependents();
}

// candidate order: larger value, then smaller index (first maximum wins)
__device__ __forceinline__ void better(float& bv, int32_t& bi, float v, int32_t i) {
    if (v > bv || (v == bv && i < bi)) {
        bv = v;
        bi = i;
    }
}

// grid (parts, batch), block 256: this rank's vocabulary shard [v0, v0 + n) of each
// sequence's logits row (row stride `stride`), global indices
__global__ void tp_argmax_part_kernel(const float* __restrict__ logits, uint32_t stride, uint32_t v0, uint32_t n,
                                      float* part_v, int32_t* part_i) {
    pdl_wait();
    const uint32_t b = blockIdx.y, parts = gridDim.x;
    const uint32_t per = (n + parts - 1) / parts;
    const uint32_t lo = blockIdx.x * per, hi = min(n, lo + per);
    const float* lb = logits + (uint64_t)b * stride + v0;
    float bv = -FLT_MAX;  // f32::MIN (src/runtime.rs:897-905): only values strictly above it count
    int32_t bi = INT32_MAX;
    for (uint32_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        const float v = lb[i];
        if (v > bv) {
            bv = v;
            bi = (int32_t)(v0 + i);
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

// one block, warp b = sequence b: this rank's best (value, index) goes to every rank,
// the ranks' bests are compared in the same order everywhere, and the step ends as
// argmax_final_kernel ends it (next token, history, position) and advances the epoch.
__global__ void tp_argmax_pick_kernel(const TpPeers P, uint32_t slot, const float* part_v, const int32_t* part_i,
                                      uint32_t parts, int32_t* out, int32_t* next_tokens, int32_t* pos, int32_t* hist,
                                      uint32_t hist_stride, uint32_t* epoch, int* err) {
    pdl_wait();
    const uint32_t b = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t tag = *P.epoch * P.period + 1u + slot;
    float bv = -FLT_MAX;
    int32_t bi = INT32_MAX;
    for (uint32_t p = lane; p < parts; p += 32) better(bv, bi, part_v[b * parts + p], part_i[b * parts + p]);
    for (int o = 16; o > 0; o >>= 1) {
        const float v = __shfl_xor_sync(0xffffffffu, bv, o);
        const int32_t i = __shfl_xor_sync(0xffffffffu, bi, o);
        better(bv, bi, v, i);
    }
    if (lane < P.size) {  // lane r sends this rank's best to rank r
        __threadfence_system();  // the logits shard (earlier kernels) before the word that announces it
        uint64_t* dst = slot_of(P, lane, TP_PICK, P.rank) + 2 * b;
        st_word(dst, bv, tag);
        st_word(dst + 1, __int_as_float(bi), tag);
    }
    // lane r reads rank r's best
    float rv = -FLT_MAX;
    int32_t ri = INT32_MAX;
    bool ok = true;
    if (lane < P.size) {
        const uint64_t* src = slot_of(P, P.rank, TP_PICK, lane) + 2 * b;
        uint64_t w0 = ld_word(src), w1 = ld_word(src + 1), t0 = 0;
        while (tag_of(w0) != tag || tag_of(w1) != tag) {
            const uint64_t t = global_ns();
            if (!t0) t0 = t;
            else if (t - t0 > kWaitNs) {
                ok = false;
                break;
            }
            w0 = ld_word(src);
            w1 = ld_word(src + 1);
        }
        if (ok) {
            rv = val_of(w0);
            ri = __float_as_int(val_of(w1));
        }
    }
    if (!ok) atomicExch(err, DEV_ERR_WAIT_TIMEOUT);
    for (int o = 16; o > 0; o >>= 1) {
        const float v = __shfl_xor_sync(0xffffffffu, rv, o);
        const int32_t i = __shfl_xor_sync(0xffffffffu, ri, o);
        better(rv, ri, v, i);
    }
    if (lane == 0) {
        const int32_t r = ri == INT32_MAX ? 0 : ri;  // nothing above f32::MIN: index 0
        out[b] = r;
        if (next_tokens) next_tokens[b] = r;
        if (pos) {
            const int32_t p = pos[b];
            if (hist && (uint32_t)p < hist_stride) hist[(uint64_t)b * hist_stride + p] = r;
            pos[b] = p + 1;
        }
    }
    __syncthreads();  // every warp has read the epoch
    if (threadIdx.x == 0 && epoch) *epoch += 1;
    pdl_launch_dependents();
}

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

}  // namespace

cudaError_t launch_tp_allreduce_add(const TpPeers& P, uint32_t purpose, uint32_t slot, float* x, const float* part,
                                    uint32_t n, int* err, cudaStream_t s, bool pdl) {
    if (!P.size || P.size > (uint32_t)kMaxPeers || n > P.cap || purpose >= TP_PURPOSES) return cudaErrorInvalidValue;
    cudaLaunchAttribute at[1];
    auto cfg = cfg_of(dim3((n + 255) / 256), dim3(256), s, pdl, at);
    return cudaLaunchKernelEx(&cfg, tp_allreduce_add_kernel, P, purpose, slot, x, part, n, err);
}

cudaError_t launch_tp_argmax(const TpPeers& P, uint32_t slot, const float* logits, uint32_t stride, uint32_t v0,
                             uint32_t n, uint32_t batch, float* part_v, int32_t* part_i, uint32_t parts, int32_t* out,
                             int32_t* next_tokens, int32_t* pos, int32_t* hist, uint32_t hist_stride, uint32_t* epoch,
                             int* err, cudaStream_t s, bool pdl) {
    if (!P.size || P.size > (uint32_t)kMaxPeers || !batch || batch > 32 || 2 * batch > P.cap || !parts)
        return cudaErrorInvalidValue;
    cudaLaunchAttribute at[1];
    auto cfg = cfg_of(dim3(parts, batch), dim3(256), s, pdl, at);
    cudaError_t e = cudaLaunchKernelEx(&cfg, tp_argmax_part_kernel, logits, stride, v0, n, part_v, part_i);
    if (e != cudaSuccess) return e;
    auto cfg2 = cfg_of(dim3(1), dim3(32 * batch), s, pdl, at);
    return cudaLaunchKernelEx(&cfg2, tp_argmax_pick_kernel, P, slot, (const float*)part_v, (const int32_t*)part_i,
                              parts, out, next_tokens, pos, hist, hist_stride, epoch, err);
}

}  // namespace evl
