// repack.cpp -- GGUF blocks -> the MMA-fragment device layout of common.cuh.
//
// The reference keeps each QMatrix as the raw GGUF bytes (src/runtime.rs:23-51) and
// re-reads whole 144/210/34-byte blocks per row. On the GPU the 16 rows of a slab are
// interleaved word by word so that each lane of the matvec's MMA warps loads its
// fragments with 16-byte shared-memory reads, and a panel of 32 units is one bulk
// copy. Every byte of the original survives at block_byte_address: the exact
// dequantiser reads this layout back bit-for-bit (dequant.cuh). The bytes are moved
// into place on the device (dequant.cu, launch_repack); this file sizes and places
// the matrices.
#include <algorithm>

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

}  // namespace evl
