// dequant.cuh -- exact GGUF dequantisation of single values (device functions).
//
// Bit-exact restatement of src/gguf.rs:300-320 (f16_to_f32, including subnormals,
// inf and NaN payloads), :327-336 (get_scale_min_k4) and :338-430 (F32, F16, BF16,
// Q8_0, Q4_K, Q5_K, Q6_K). Every product and difference uses the _rn intrinsics so
// nvcc cannot contract `d*s*q - dmin*m` into an FMA: the reference evaluates it as
// ((d*s)*q) - (dmin*m) with three roundings.
#pragma once
#include "common.cuh"

namespace evl {

// gguf.rs:300-320, as integer operations so NaN payloads survive bit-for-bit.
__device__ __forceinline__ float f16_exact(uint32_t h) {
    uint32_t sign = (h >> 15) << 31, exp = (h >> 10) & 0x1f, frac = h & 0x3ff, bits;
    if (exp == 0 && frac == 0) {
        bits = sign;
    } else if (exp == 0) {
        // shift until bit 10 is set; each shift lowers the exponent by one
        uint32_t sh = __clz(frac) - 21;  // frac < 0x400: clz >= 22
        uint32_t e = 127 - 15 + 1 - sh;
        bits = sign | (e << 23) | (((frac << sh) & 0x3ff) << 13);
    } else if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (frac << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (frac << 13);
    }
    return __uint_as_float(bits);
}

__device__ __forceinline__ uint32_t ld_u16(const uint8_t* p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8); }

__device__ __forceinline__ void scale_min_bytes(int j, const uint8_t* q, float* s, float* m) {
    if (j < 4) {
        *s = (float)(q[j] & 63);
        *m = (float)(q[j + 4] & 63);
    } else {
        *s = (float)((q[j + 4] & 0xf) | ((q[j - 4] >> 6) << 4));
        *m = (float)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

// Value `e` of one Q8_0 (e < 32) or K-quant (e < 256) block in raw GGUF bytes.
__device__ __forceinline__ float dq_raw_value(uint32_t type, const uint8_t* b, uint32_t e) {
    switch (type) {
        case GGML_Q8_0: {  // gguf.rs:353-358
            float d = f16_exact(ld_u16(b));
            return __fmul_rn(d, (float)(int8_t)b[2 + e]);
        }
        case GGML_Q4_K: {  // gguf.rs:359-372
            float d = f16_exact(ld_u16(b)), dmin = f16_exact(ld_u16(b + 2));
            uint32_t blk = e >> 6, hi = (e >> 5) & 1, l = e & 31;
            float s, m;
            scale_min_bytes(2 * blk + hi, b + 4, &s, &m);
            uint8_t v = b[16 + blk * 32 + l];
            float q = (float)(hi ? (v >> 4) : (v & 0xf));
            return __fsub_rn(__fmul_rn(__fmul_rn(d, s), q), __fmul_rn(dmin, m));
        }
        case GGML_Q5_K: {  // gguf.rs:373-396
            float d = f16_exact(ld_u16(b)), dmin = f16_exact(ld_u16(b + 2));
            uint32_t blk = e >> 6, hi = (e >> 5) & 1, l = e & 31;
            float s, m;
            scale_min_bytes(2 * blk + hi, b + 4, &s, &m);
            uint8_t v = b[48 + blk * 32 + l];
            uint8_t qh = b[16 + l];
            uint32_t bit = 2 * blk + hi;
            int q = (hi ? (v >> 4) : (v & 0xf)) + (((qh >> bit) & 1) ? 16 : 0);
            return __fsub_rn(__fmul_rn(__fmul_rn(d, s), (float)q), __fmul_rn(dmin, m));
        }
        case GGML_Q6_K: {  // gguf.rs:397-420
            float d = f16_exact(ld_u16(b + 208));
            uint32_t half = e >> 7, r = e & 127, k = r >> 5, l = r & 31;
            const uint8_t* ql = b + half * 64;
            const uint8_t* qh = b + 128 + half * 32;
            const int8_t* sc = (const int8_t*)(b + 192 + half * 8);
            uint32_t lo = (k & 1) ? ql[l + 32] : ql[l];
            uint32_t nib = (k >> 1) ? (lo >> 4) : (lo & 0xf);
            int q = (int)(nib | (((qh[l] >> (2 * k)) & 3) << 4)) - 32;
            uint32_t is = l / 16;
            return __fmul_rn(__fmul_rn(d, (float)sc[is + 2 * k]), (float)q);
        }
        default: return 0.f;
    }
}

// Value `c` of row `r` from the repacked layout (common.cuh).
__device__ __forceinline__ float dq_repacked_value(const QMatDev& m, uint32_t r, uint32_t c) {
    const uint32_t T = m.type, N = m.nunits;
    const uint32_t u_of_c = (T == GGML_Q6_K) ? (c >> 8) * 4 + ((c & 255) >> 7) * 2 + ((c >> 4) & 1) : c >> 6;
    const uint8_t* tile = m.q + tile_address(T, N, m.row_bytes, r, u_of_c >> 5);
    switch (T) {
        case GGML_Q4_K: {
            uint32_t sb = c >> 8, e = c & 255, j = e >> 6, hi = (e >> 5) & 1, l = e & 31;
            uint32_t u = sb * 4 + j;
            uint8_t v = tile[chunk_in_tile(N, u, l >> 4) + (l & 15)];
            const uint8_t* h = tile + aux_in_tile(T, N, u);
            float d = f16_exact(ld_u16(h)), dmin = f16_exact(ld_u16(h + 2));
            float s, mm;
            scale_min_bytes(2 * j + hi, h + 4, &s, &mm);
            float q = (float)(hi ? (v >> 4) : (v & 0xf));
            return __fsub_rn(__fmul_rn(__fmul_rn(d, s), q), __fmul_rn(dmin, mm));
        }
        case GGML_Q6_K: {
            uint32_t sb = c >> 8, e = c & 255, half = e >> 7, rr = e & 127, k = rr >> 5, l = rr & 31;
            uint32_t u = sb * 4 + half * 2 + (l >> 4);
            uint32_t li = l & 15;
            uint8_t lo = tile[chunk_in_tile(N, u, k & 1) + li];
            uint8_t qh = tile[chunk_in_tile(N, u, 2) + li];
            uint32_t nib = (k >> 1) ? (lo >> 4) : (lo & 0xf);
            int q = (int)(nib | (((qh >> (2 * k)) & 3) << 4)) - 32;
            uint32_t scw = *reinterpret_cast<const uint32_t*>(tile + aux_in_tile(T, N, u));
            float sc = (float)(int8_t)((scw >> (8 * k)) & 0xff);
            float d = f16_exact(ld_u16(tile + d_in_tile(T, N, u)));
            return __fmul_rn(__fmul_rn(d, sc), (float)q);
        }
        case GGML_Q8_0: {
            uint32_t u = c >> 6, e = c & 63;
            int8_t q = (int8_t)tile[chunk_in_tile(N, u, e >> 4) + (e & 15)];
            uint32_t dw = *reinterpret_cast<const uint32_t*>(tile + aux_in_tile(T, N, u));
            float d = f16_exact((e < 32) ? (dw & 0xffff) : (dw >> 16));
            return __fmul_rn(d, (float)q);
        }
        case GGML_F16:
        case GGML_BF16: {
            uint32_t u = c >> 6, e = c & 63;
            uint32_t h = ld_u16(tile + chunk_in_tile(N, u, e >> 3) + (e & 7) * 2);
            return T == GGML_F16 ? f16_exact(h) : __uint_as_float(h << 16);
        }
        case GGML_F32: {
            uint32_t u = c >> 6, e = c & 63;
            return __uint_as_float(*(const uint32_t*)(tile + chunk_in_tile(N, u, e >> 2) + (e & 3) * 4));
        }
        default: return 0.f;
    }
}

}  // namespace evl
