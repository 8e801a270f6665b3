// trc_quant.cuh -- device decode of GGUF legacy quantized blocks (shared by the dequant kernel and
// the fused dequant-prologue GEMM).
//
// Semantics follow train.cpp's host dequantizers (src/io/trc_gguf.cpp:320-417) bit for bit:
//   Q4_0 [d:f16][qs:16]        w[j] = (nib(j) - 8) * d
//   Q4_1 [d][m][qs:16]         w[j] = nib(j) * d + m
//   Q5_0 [d][qh:u32][qs:16]    w[j] = ((nib(j) | bit_j(qh) << 4) - 16) * d
//   Q5_1 [d][m][qh][qs:16]     w[j] = (nib(j) | bit_j(qh) << 4) * d + m
//   Q8_0 [d][qs:i8 x 32]       w[j] = qs[j] * d
// with nib(j) = low nibble of qs[j] for j < 16 and high nibble of qs[j-16] for j >= 16.
// q*d is exact in fp32 (|q| < 2^8, d carries 11 significant bits), so the reference's separately
// rounded q*d + m equals one fused multiply-add: both round q*d + m once.
#pragma once

#include <cstdint>

#include <cuda_fp16.h>

namespace trc {

template <int TYPE>
struct QuantTraits;

template <> struct QuantTraits<0> { static constexpr int kBytes = 0;  static constexpr int kQs = 0; };  // F32: no blocks
template <> struct QuantTraits<2> { static constexpr int kBytes = 18; static constexpr int kQs = 2; };  // Q4_0
template <> struct QuantTraits<3> { static constexpr int kBytes = 20; static constexpr int kQs = 4; };  // Q4_1
template <> struct QuantTraits<6> { static constexpr int kBytes = 22; static constexpr int kQs = 6; };  // Q5_0
template <> struct QuantTraits<7> { static constexpr int kBytes = 24; static constexpr int kQs = 8; };  // Q5_1
template <> struct QuantTraits<8> { static constexpr int kBytes = 34; static constexpr int kQs = 2; };  // Q8_0

// Little-endian reads from a block in shared or global memory that is only 2-byte aligned.
__device__ __forceinline__ uint32_t ld_u16(const uint8_t* p) { return *reinterpret_cast<const uint16_t*>(p); }
__device__ __forceinline__ uint32_t ld_u32_a2(const uint8_t* p) { return ld_u16(p) | (ld_u16(p + 2) << 16); }

// Raw 16-bit words a quad (weights j0..j0+3, j0 a multiple of 4) needs: the scale d, the minimum m
// (_1 formats), the 16-bit word of qh holding bits j0..j0+3 (Q5 formats) and the two words holding
// the four quant bytes. Loading them into registers first lets a later stage's loads overlap the
// decode of the current one.
struct QuadWords {
    uint32_t d, m, qh, q0, q1;
};

template <int TYPE>
__device__ __forceinline__ void load_quad_words(const uint8_t* blk, int j0, QuadWords& r) {
    const uint16_t* p16 = reinterpret_cast<const uint16_t*>(blk);
    r.d = p16[0];
    if constexpr (TYPE == 8) {
        r.q0 = p16[1 + (j0 >> 1)];
        r.q1 = p16[2 + (j0 >> 1)];
    } else {
        constexpr int qs16 = QuantTraits<TYPE>::kQs / 2;
        r.q0 = p16[qs16 + ((j0 & 15) >> 1)];
        r.q1 = p16[qs16 + ((j0 & 15) >> 1) + 1];
        if constexpr (TYPE == 3 || TYPE == 7) r.m = p16[1];
        if constexpr (TYPE == 6) r.qh = p16[1 + (j0 >> 4)];
        if constexpr (TYPE == 7) r.qh = p16[2 + (j0 >> 4)];
    }
}

// load_quad_words for a block in shared memory, addressed by its shared-window address (explicit
// ld.shared: a generic pointer into shared memory loses its address space through the kernel's
// aligned-pointer arithmetic and would be loaded with generic loads).
__device__ __forceinline__ uint32_t lds_u16(uint32_t saddr) {
    uint16_t v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(saddr));
    return v;
}

template <int TYPE>
__device__ __forceinline__ void load_quad_words_smem(uint32_t blk, int j0, QuadWords& r) {
    r.d = lds_u16(blk);
    if constexpr (TYPE == 8) {
        r.q0 = lds_u16(blk + 2 + 2 * (j0 >> 1));
        r.q1 = lds_u16(blk + 4 + 2 * (j0 >> 1));
    } else {
        constexpr int qs = QuantTraits<TYPE>::kQs;
        r.q0 = lds_u16(blk + qs + 2 * ((j0 & 15) >> 1));
        r.q1 = lds_u16(blk + qs + 2 + 2 * ((j0 & 15) >> 1));
        if constexpr (TYPE == 3 || TYPE == 7) r.m = lds_u16(blk + 2);
        if constexpr (TYPE == 6) r.qh = lds_u16(blk + 2 + 2 * (j0 >> 4));
        if constexpr (TYPE == 7) r.qh = lds_u16(blk + 4 + 2 * (j0 >> 4));
    }
}

// Decode weights j0 .. j0+3 from their raw words, exactly as the reference's dequantizers do:
// - the four codes are gathered into the four bytes of one word (Q5: the high bit of weight e is
//   moved to bit 4 of byte e by one multiply, whose partial products fall in disjoint bits; Q8_0:
//   the sign bit is flipped, so the byte is the int8 value + 128);
// - one byte permute per weight builds the float 2^23 + code, and subtracting 2^23 + the format's
//   offset gives the quant value q exactly;
// - the scale d and minimum m go through the hardware half -> float conversion, exact for every
//   finite or infinite half (a NaN stays a NaN);
// - y = q * d, or fma(q, d, m) for the _1 formats: the reference's q * d + m rounds twice, but
//   q * d is exact in fp32 (|q| < 2^8, d has 11 significant bits), so one fma is the same value.
template <int TYPE>
__device__ __forceinline__ void decode_quad_words(const QuadWords& r, int j0, float (&w)[4]) {
    const float    d = __half2float(__ushort_as_half(static_cast<unsigned short>(r.d)));
    const uint32_t q = r.q0 | (r.q1 << 16);
    uint32_t codes;
    if constexpr (TYPE == 8) {
        codes = q ^ 0x80808080u;
    } else {
        codes = (j0 >= 16 ? (q >> 4) : q) & 0x0F0F0F0Fu;
        if constexpr (TYPE == 6 || TYPE == 7) {
            const uint32_t hb = (r.qh >> (j0 & 15)) & 0xFu;       // high bits of weights j0 .. j0+3
            codes |= ((hb * 0x00204081u) & 0x01010101u) << 4;     // bit e -> bit 4 of byte e
        }
    }
    constexpr float kBias = 8388608.0f + (TYPE == 2 ? 8.0f : TYPE == 6 ? 16.0f : TYPE == 8 ? 128.0f : 0.0f);
    float m = 0.0f;
    if constexpr (TYPE == 3 || TYPE == 7) m = __half2float(__ushort_as_half(static_cast<unsigned short>(r.m)));
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        // 0x4B0000cc: byte 0 = code e, bytes 1-2 = 0, byte 3 = 0x4B (the exponent of 2^23)
        const float qf = __fsub_rn(__uint_as_float(__byte_perm(codes, 0x4B000000u, 0x7440u + e)), kBias);
        if constexpr (TYPE == 3 || TYPE == 7) w[e] = __fmaf_rn(qf, d, m);
        else w[e] = __fmul_rn(qf, d);
    }
}

}  // namespace trc
