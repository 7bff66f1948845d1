// qmatvec.cu -- the standalone dequant-fused matvec launch (QMatrix::matvec,
// src/runtime.rs:72-88): one persistent CTA per SM running the producer/consumer
// machinery of matvec_core.cuh over its contiguous range of row blocks.
#include <algorithm>
#include <atomic>

#include "matvec_core.cuh"

namespace evl {

namespace {

using namespace mv;

__global__ void __launch_bounds__(kThreads, 1) qmatvec_kernel(const __grid_constant__ Plan p, uint32_t stages) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t full[kMaxStages], empty[kMaxStages];
    __shared__ float red[kCW];
    __shared__ volatile int abort_flag;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    uint32_t rb0, rb1;
    cta_rows(p, blockIdx.x, gridDim.x, rb0, rb1);
    const Ring r{smem, full, empty, stages, p.item_bytes};
    uint8_t* xs = smem + stages * p.item_bytes;

    if (tid == 0) {
        abort_flag = 0;
        for (uint32_t s = 0; s < stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kCW);
        }
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == kCW) {  // producer: needs nothing from the previous kernel
        if (lane != 0) return;
        RingPos rp;
        if (produce_items(p, r, rb0, rb1, rp, &abort_flag)) prefetch_next(p, blockIdx.x, gridDim.x);
        if (abort_flag) drain_ring(r, rp.n);
        return;
    }

    NormRegs nr;
    load_norm_regs(p, warp, lane, nr);
    pdl_wait();
    prefetch_rows(p, xs, rb0, rb1, (uint32_t)tid);
    const float inv = stage_input(p, xs, warp, lane, red, nr);
    pdl_launch_dependents();
    RingPos rp;
    if (!consume_items(p, r, xs, rb0, rb1, rp, warp, lane, &abort_flag, inv) && lane == 0)
        atomicExch(p.err, DEV_ERR_WAIT_TIMEOUT);
}

constexpr int kMaxDevices = 64;
std::atomic<int> g_sms[kMaxDevices];  // SM count per device, 0 until set up (zero-initialised static)

}  // namespace

cudaError_t launch_qmatvec(const MatvecArgs& a, cudaStream_t s, bool pdl) {
    if (matvec_has_plain(a)) return launch_plain_matvec(a, s, pdl);
    Plan p;
    cudaError_t e = plan_matvec(a, p);
    if (e != cudaSuccess) return e;
    const uint32_t stages = std::min<uint32_t>(kMaxStages, (kSmemBudget - p.xbytes) / p.item_bytes);
    // per-device set-up once: SM count and the kernel's shared-memory opt-in
    int dev = 0;
    e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    if (!g_sms[dev]) {
        int sms = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(qmatvec_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBudget);
        if (e != cudaSuccess) return e;
        g_sms[dev] = sms;
    }
    cudaLaunchConfig_t cfg = {};
    uint32_t grid = std::min<uint32_t>(p.rb_begin[kMaxSegs], (uint32_t)g_sms[dev]);
    if (a.max_ctas) grid = std::min(grid, a.max_ctas);
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = stages * p.item_bytes + p.xbytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, qmatvec_kernel, p, stages);
}

}  // namespace evl
