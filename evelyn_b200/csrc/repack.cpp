// repack.cpp -- GGUF blocks -> the tiled device layout of common.cuh.
//
// The reference keeps each QMatrix as the raw GGUF bytes (src/runtime.rs:23-51) and
// re-reads whole 144/210/34-byte blocks per row. On the GPU a row is cut into tiles of
// up to 32 units (64 values each); inside a tile the 16-byte chunks are stored
// chunk-major so the 32 lanes of a warp read consecutive 16-byte pieces, and the
// block scales of the tile follow its payload, so one bulk copy moves a whole tile.
// Every byte of the original survives: the exact dequantiser reads this layout back
// bit-for-bit (dequant.cuh).
#include <algorithm>
#include <cstring>
#include <thread>

#include "engine.hpp"

namespace evl {

void repack_sizes(QMatrix& m) {
    const uint64_t cols = m.cols;
    switch (m.type) {
        case GGML_Q4_K:
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
    m.dev.row_bytes = row_tile_bytes(m.type, nunits);
    const uint64_t slabs = (m.rows + kSlabRows - 1) / kSlabRows;
    m.total_bytes = (slabs * kSlabRows * m.dev.row_bytes + 255) / 256 * 256;
}

void place(QMatrix& m, uint8_t* base) { m.dev.q = base + m.offset; }

namespace {

void repack_rows(const QMatrix& m, const uint8_t* raw, size_t stride, uint8_t* dst, uint32_t r0, uint32_t r1) {
    const uint32_t T = m.type, N = m.dev.nunits, nb = m.cols / 256, ch = chunks_per_unit(T), RB = m.dev.row_bytes;
    for (uint32_t r = r0; r < r1; ++r) {
        const uint8_t* src = raw + (size_t)r * stride;
        // tile of unit u in this row
        auto tile = [&](uint32_t u) { return dst + tile_address(T, N, RB, r, u >> 5); };
        switch (T) {
            case GGML_Q4_K:
                for (uint32_t sb = 0; sb < nb; ++sb) {
                    const uint8_t* blk = src + (size_t)sb * 144;
                    std::memcpy(tile(sb * 4) + aux_in_tile(T, N, sb * 4), blk, 16);
                    for (uint32_t j = 0; j < 4; ++j) {
                        const uint32_t u = sb * 4 + j;
                        for (uint32_t c = 0; c < 2; ++c)
                            std::memcpy(tile(u) + chunk_in_tile(N, u, c), blk + 16 + 32 * j + 16 * c, 16);
                    }
                }
                break;
            case GGML_Q6_K:
                for (uint32_t sb = 0; sb < nb; ++sb) {
                    const uint8_t* blk = src + (size_t)sb * 210;
                    const uint8_t* ql = blk;
                    const uint8_t* qh = blk + 128;
                    const uint8_t* sc = blk + 192;
                    std::memcpy(tile(sb * 4) + d_in_tile(T, N, sb * 4), blk + 208, 2);
                    for (uint32_t h = 0; h < 2; ++h)
                        for (uint32_t b = 0; b < 2; ++b) {
                            const uint32_t u = sb * 4 + h * 2 + b, l0 = 16 * b;
                            uint8_t* t = tile(u);
                            std::memcpy(t + chunk_in_tile(N, u, 0), ql + 64 * h + l0, 16);
                            std::memcpy(t + chunk_in_tile(N, u, 1), ql + 64 * h + 32 + l0, 16);
                            std::memcpy(t + chunk_in_tile(N, u, 2), qh + 32 * h + l0, 16);
                            uint8_t w[4];
                            for (uint32_t k = 0; k < 4; ++k) w[k] = sc[8 * h + b + 2 * k];
                            std::memcpy(t + aux_in_tile(T, N, u), w, 4);
                        }
                }
                break;
            case GGML_Q8_0:
                for (uint32_t u = 0; u < N; ++u) {
                    const uint8_t* b0 = src + (size_t)(2 * u) * 34;
                    const uint8_t* b1 = b0 + 34;
                    uint8_t* t = tile(u);
                    std::memcpy(t + chunk_in_tile(N, u, 0), b0 + 2, 16);
                    std::memcpy(t + chunk_in_tile(N, u, 1), b0 + 18, 16);
                    std::memcpy(t + chunk_in_tile(N, u, 2), b1 + 2, 16);
                    std::memcpy(t + chunk_in_tile(N, u, 3), b1 + 18, 16);
                    const uint8_t w[4] = {b0[0], b0[1], b1[0], b1[1]};
                    std::memcpy(t + aux_in_tile(T, N, u), w, 4);
                }
                break;
            default: {  // F16 / BF16 / F32: plain values, chunked
                const uint32_t eb = T == GGML_F32 ? 4 : 2;
                for (uint32_t u = 0; u < N; ++u)
                    for (uint32_t c = 0; c < ch; ++c)
                        std::memcpy(tile(u) + chunk_in_tile(N, u, c), src + (size_t)u * 64 * eb + 16 * c, 16);
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
