// attention_noalloc.cu -- evl_attention_decode_noalloc: the decode attention of
// evl_attention_decode with its split scratch in a fixed device array instead of a
// per-call allocation.
//
// Who needs it: callers that may not allocate device memory inside a decode call --
// a serving process whose HBM is wholly owned by its own pool (reserved at start-up,
// so a cudaMalloc here fails or forces the pool to give memory back), and callers
// that must not let a library cudaFree synchronise the whole device in the middle of
// their step. This entry point calls no cudaMalloc, cudaFree or any other allocating
// routine; its only device memory is the array below, sized at compile time.
//
// Limits and rules:
//   * The scratch is kNoAllocScratchBytes (1.5 MiB) per device: a 256-byte header
//     holding the device error flag, then the split partials,
//     heads * nsplit * (head_dim + 2) floats. nsplit is the same split count
//     evl_attention_decode uses (min(ceil(t / 16), 2 * SMs / kv_heads)), so on a
//     148-SM B200 every shape the kernels accept fits; a request that would need
//     more is rejected with EVL_ERR_INVALID_INPUT before anything is launched.
//   * The error flag must read zero when the kernels start; each call clears it with
//     cudaMemsetAsync on `stream` first. The partials need no initial value: every
//     split the combine step reads is written by its split kernel in the same call.
//   * One scratch per device per process: calls on the same device that overlap in
//     time (from two host threads) race on it and can corrupt each other's output.
//     Callers serialise them.
//   * The first call on a device does the set-up (it resolves the array's device
//     address with cudaGetSymbolAddress, which may load this library's device code).
//   * Every call reads the error flag back into host memory and synchronises
//     `stream`, so the entry point cannot be used inside a CUDA stream capture;
//     evl_attention_decode_ws is the asynchronous variant on caller memory.
#include <cstdio>
#include <mutex>

#include "engine.hpp"

using namespace evl;

namespace {

constexpr size_t kNoAllocScratchBytes = 1536u * 1024u;
constexpr size_t kNoAllocHeader = 256;  // int32 error flag, padded so the partials stay aligned
constexpr int kMaxDevices = 64;

static __device__ __align__(256) uint8_t g_attn_scratch[kNoAllocScratchBytes];

std::mutex g_setup_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of g_attn_scratch on the current device, resolved once per device.
uint8_t* scratch_for_current_device() {
    int dev = 0;
    cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
    if (dev < 0 || dev >= kMaxDevices) raise(EVL_ERR_UNSUPPORTED, "device index beyond the no-alloc scratch table");
    std::lock_guard<std::mutex> lk(g_setup_mu);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_attn_scratch);
        if (e != cudaSuccess || !p) {
            cudaGetLastError();
            raise(EVL_ERR_CUDA, std::string("cudaGetSymbolAddress(no-alloc attention scratch): ") +
                                    cudaGetErrorString(e));
        }
        g_scratch_ptr[dev] = p;
    }
    return static_cast<uint8_t*>(g_scratch_ptr[dev]);
}

void run(const float* d_q, const void* d_k_pages, const void* d_v_pages, const int32_t* d_page_table, uint32_t t,
         uint32_t heads, uint32_t kv_heads, uint32_t head_dim, uint32_t page_size, float* d_out, cudaStream_t s) {
    // the same checks, split count and launch as evl_attention_decode (abi.cpp); only
    // where the partials and the error flag live differs
    check_attention_args(d_q, d_k_pages, d_v_pages, d_page_table, t, heads, kv_heads, head_dim, page_size, d_out);
    const uint32_t nsplit = attention_splits(t, kv_heads, page_size);
    const size_t need = kNoAllocHeader + attention_part_bytes(heads, nsplit, head_dim);
    if (need > kNoAllocScratchBytes) {
        char msg[192];
        std::snprintf(msg, sizeof msg,
                      "no-alloc attention needs %zu bytes of scratch for this shape; its fixed scratch holds %zu",
                      need, kNoAllocScratchBytes);
        raise(EVL_ERR_INVALID_INPUT, msg);
    }

    uint8_t* scratch = scratch_for_current_device();
    int32_t* d_err = reinterpret_cast<int32_t*>(scratch);
    cuda_check(cudaMemsetAsync(d_err, 0, sizeof(int32_t), s), "memset");
    attention_standalone(d_q, d_k_pages, d_v_pages, d_page_table, t, heads, kv_heads, head_dim, page_size, d_out,
                         reinterpret_cast<float*>(scratch + kNoAllocHeader), nsplit, d_err, s);

    int32_t err = 0;
    cuda_check(cudaMemcpyAsync(&err, d_err, sizeof(int32_t), cudaMemcpyDeviceToHost, s), "D2H");
    cuda_check(cudaStreamSynchronize(s), "attention");
    if (err == DEV_ERR_WAIT_TIMEOUT) raise(EVL_ERR_TIMEOUT, "a device wait for KV pages timed out");
}

}  // namespace

extern "C" evl_status evl_attention_decode_noalloc(const float* d_q, const void* d_k_pages, const void* d_v_pages,
                                                   const int32_t* d_page_table, uint32_t t, uint32_t heads,
                                                   uint32_t kv_heads, uint32_t head_dim, uint32_t page_size,
                                                   float* d_out, void* stream) {
    try {
        run(d_q, d_k_pages, d_v_pages, d_page_table, t, heads, kv_heads, head_dim, page_size, d_out,
            static_cast<cudaStream_t>(stream));
        return EVL_OK;
    } catch (const Error& e) {
        set_last_error(e.msg);
        return e.code;
    } catch (const std::exception& e) {
        set_last_error(e.what());
        return EVL_ERR_IO;
    }
}
