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

// Value `c` of row `r` from the repacked layout (common.cuh): the bytes of the
// value's GGUF block are fetched through block_byte_address and fed to the same
// arithmetic as the raw path.
__device__ __forceinline__ float dq_repacked_value(const QMatDev& m, uint32_t r, uint32_t c) {
    const uint32_t T = m.type;
    auto byte = [&](uint32_t b, uint32_t o) { return m.q[block_byte_address(m, r, b, o)]; };
    switch (T) {
        case GGML_Q4_K: {
            const uint32_t b = c >> 8, e = c & 255;
            uint8_t blk[16];
            for (uint32_t i = 0; i < 16; ++i) blk[i] = byte(b, i);
            float d = f16_exact(ld_u16(blk)), dmin = f16_exact(ld_u16(blk + 2));
            const uint32_t j = e >> 6, hi = (e >> 5) & 1, l = e & 31;
            float s, mm;
            scale_min_bytes(2 * j + hi, blk + 4, &s, &mm);
            const uint8_t v = byte(b, 16 + j * 32 + l);
            float q = (float)(hi ? (v >> 4) : (v & 0xf));
            return __fsub_rn(__fmul_rn(__fmul_rn(d, s), q), __fmul_rn(dmin, mm));
        }
        case GGML_Q5_K: {
            const uint32_t b = c >> 8, e = c & 255;
            uint8_t blk[16];
            for (uint32_t i = 0; i < 16; ++i) blk[i] = byte(b, i);
            float d = f16_exact(ld_u16(blk)), dmin = f16_exact(ld_u16(blk + 2));
            const uint32_t j = e >> 6, hi = (e >> 5) & 1, l = e & 31;
            float s, mm;
            scale_min_bytes(2 * j + hi, blk + 4, &s, &mm);
            const uint8_t v = byte(b, 48 + j * 32 + l);
            const uint8_t qh = byte(b, 16 + l);
            const int q = (hi ? (v >> 4) : (v & 0xf)) + (((qh >> (2 * j + hi)) & 1) ? 16 : 0);
            return __fsub_rn(__fmul_rn(__fmul_rn(d, s), (float)q), __fmul_rn(dmin, mm));
        }
        case GGML_Q6_K: {
            const uint32_t b = c >> 8, e = c & 255, half = e >> 7, rr = e & 127, k = rr >> 5, l = rr & 31;
            const uint8_t lo = byte(b, 64 * half + ((k & 1) ? 32 : 0) + l);
            const uint8_t qh = byte(b, 128 + 32 * half + l);
            const uint32_t nib = (k >> 1) ? (lo >> 4) : (lo & 0xf);
            const int q = (int)(nib | (((qh >> (2 * k)) & 3) << 4)) - 32;
            const float sc = (float)(int8_t)byte(b, 192 + 8 * half + l / 16 + 2 * k);
            const float d = f16_exact((uint32_t)byte(b, 208) | ((uint32_t)byte(b, 209) << 8));
            return __fmul_rn(__fmul_rn(d, sc), (float)q);
        }
        case GGML_Q8_0: {
            const uint32_t b = c >> 5, e = c & 31;
            const float d = f16_exact((uint32_t)byte(b, 0) | ((uint32_t)byte(b, 1) << 8));
            return __fmul_rn(d, (float)(int8_t)byte(b, 2 + e));
        }
        case GGML_F16:
        case GGML_BF16: {
            const uint32_t h = ld_u16(m.q + plain_value_address(m, r, c, 2));
            return T == GGML_F16 ? f16_exact(h) : __uint_as_float(h << 16);
        }
        case GGML_F32: return __uint_as_float(*(const uint32_t*)(m.q + plain_value_address(m, r, c, 4)));
        default: return 0.f;
    }
}

}  // namespace evl
