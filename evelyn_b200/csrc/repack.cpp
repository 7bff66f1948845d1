// repack.cpp -- GGUF blocks -> the MMA-fragment device layout of common.cuh.
//
// The reference keeps each QMatrix as the raw GGUF bytes (src/runtime.rs:23-51) and
// re-reads whole 144/210/34-byte blocks per row. On the GPU the 16 rows of a slab are
// interleaved word by word so that each lane of the matvec's MMA warps loads its
// fragments with 16-byte shared-memory reads, and a panel of 32 units is one bulk
// copy. Every byte of the original survives at block_byte_address: the exact
// dequantiser reads this layout back bit-for-bit (dequant.cuh).
#include <algorithm>
#include <cstring>
#include <thread>

#include "engine.hpp"

namespace evl {

void repack_sizes(QMatrix& m) {
    const uint64_t cols = m.cols;
    switch (m.type) {
        case GGML_Q4_K:
        case GGML_Q5_K:
        case GGML_Q6_K:
            if (cols % 256) raise(EVL_ERR_INVALID_DATA, m.name + ": row length is not a multiple of 256");
            break;
        case GGML_Q8_0:
        case GGML_F16:
        case GGML_BF16:
        case GGML_F32:
            if (cols % 64) raise(EVL_ERR_UNSUPPORTED, m.name + ": row length is not a multiple of 64");
            break;
        default:
            raise(EVL_ERR_UNSUPPORTED, m.name + ": ggml type " + std::to_string(m.type) + " (" + type_name(m.type) +
                                           ") is not supported for device matrices");
    }
    const uint32_t nunits = (uint32_t)(cols / 64);
    m.dev.type = m.type;
    m.dev.rows = m.rows;
    m.dev.cols = m.cols;
    m.dev.nunits = nunits;
    m.dev.row_bytes = slab_row_bytes(m.type, nunits);
    const uint64_t slabs = (m.rows + kSlabRows - 1) / kSlabRows;
    m.total_bytes = (slabs * kSlabRows * m.dev.row_bytes + 255) / 256 * 256;
}

void place(QMatrix& m, uint8_t* base) { m.dev.q = base + m.offset; }

namespace {

void repack_rows(const QMatrix& m, const uint8_t* raw, size_t stride, uint8_t* dst, uint32_t r0, uint32_t r1) {
    const uint32_t T = m.type;
    const QMatDev& d = m.dev;
    for (uint32_t r = r0; r < r1; ++r) {
        const uint8_t* src = raw + (size_t)r * stride;
        auto put = [&](uint32_t b, uint32_t o, const uint8_t* from, uint32_t n) {
            std::memcpy(dst + block_byte_address(d, r, b, o), from, n);
        };
        switch (T) {
            case GGML_Q4_K:
                for (uint32_t b = 0; b < m.cols / 256; ++b) {
                    const uint8_t* blk = src + (size_t)b * 144;
                    put(b, 0, blk, 16);
                    for (uint32_t o = 16; o < 144; o += 4) put(b, o, blk + o, 4);
                }
                break;
            case GGML_Q5_K:
                for (uint32_t b = 0; b < m.cols / 256; ++b) {
                    const uint8_t* blk = src + (size_t)b * 176;
                    put(b, 0, blk, 16);
                    for (uint32_t o = 16; o < 176; o += 4) put(b, o, blk + o, 4);
                }
                break;
            case GGML_Q6_K:
                for (uint32_t b = 0; b < m.cols / 256; ++b) {
                    const uint8_t* blk = src + (size_t)b * 210;
                    for (uint32_t o = 0; o < 192; o += 4) put(b, o, blk + o, 4);
                    put(b, 192, blk + 192, 16);
                    put(b, 208, blk + 208, 2);
                }
                break;
            case GGML_Q8_0:
                for (uint32_t b = 0; b < m.cols / 32; ++b) {
                    const uint8_t* blk = src + (size_t)b * 34;
                    put(b, 0, blk, 2);
                    for (uint32_t o = 2; o < 34; o += 4) put(b, o, blk + o, 4);
                }
                break;
            default: {  // F16 / BF16 / F32: each panel row contiguous
                const uint32_t eb = T == GGML_F32 ? 4 : 2;
                for (uint32_t g = 0; g * kPanelUnits < d.nunits; ++g) {
                    const uint32_t c0 = g * kPanelUnits * 64, n = group_units(d.nunits, g) * 64;
                    std::memcpy(dst + plain_value_address(d, r, c0, eb), src + (size_t)c0 * eb, (size_t)n * eb);
                }
            }
        }
    }
}

}  // namespace

void repack_host(const QMatrix& m, const uint8_t* raw, size_t stride, uint8_t* dst, int threads) {
    std::memset(dst, 0, m.bytes());
    threads = std::max(1, std::min<int>(threads, (int)(m.rows / 64) + 1));
    if (threads == 1) {
        repack_rows(m, raw, stride, dst, 0, m.rows);
        return;
    }
    std::vector<std::thread> ts;
    const uint32_t per = (m.rows + threads - 1) / threads;
    for (int t = 0; t < threads; ++t) {
        const uint32_t a = t * per, b = std::min<uint32_t>(m.rows, a + per);
        if (a >= b) break;
        ts.emplace_back([&, a, b] { repack_rows(m, raw, stride, dst, a, b); });
    }
    for (auto& t : ts) t.join();
}

}  // namespace evl
