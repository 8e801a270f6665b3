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

namespace trc {

// IEEE-754 binary16 -> binary32 from the format's definition: exact for finite values; a NaN keeps
// its payload and comes out quiet (what the reference's arithmetic decode gives on x86).
__host__ __device__ __forceinline__ float half_bits_to_float(uint32_t h) {
    const uint32_t sign = (h & 0x8000u) << 16;
    const uint32_t e    = (h >> 10) & 0x1Fu;
    const uint32_t m    = h & 0x3FFu;
    uint32_t       out;
    if (e == 0x1Fu) {
        out = sign | 0x7F800000u | (m << 13) | (m != 0 ? 0x00400000u : 0u);
    } else if (e != 0) {
        out = sign | ((e + 112u) << 23) | (m << 13);
    } else if (m == 0) {
        out = sign;
    } else {
#ifdef __CUDA_ARCH__
        const uint32_t s = static_cast<uint32_t>(__clz(m)) - 21u;  // shift that brings bit 10 up
#else
        uint32_t s = 0;
        while (((m << s) & 0x400u) == 0) ++s;
#endif
        out = sign | ((113u - s) << 23) | (((m << s) & 0x3FFu) << 13);
    }
#ifdef __CUDA_ARCH__
    return __uint_as_float(out);
#else
    float f;
    __builtin_memcpy(&f, &out, 4);
    return f;
#endif
}

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

// Decode weights 4c .. 4c+3 (c in 0..7) of the block at `blk` (2-byte aligned).
template <int TYPE>
__device__ __forceinline__ void decode_quad(const uint8_t* blk, int c, float (&w)[4]) {
    const float d = half_bits_to_float(ld_u16(blk));
    const int   j0 = 4 * c;
    if constexpr (TYPE == 8) {
        const uint32_t q4 = ld_u32_a2(blk + 2 + j0);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int q = static_cast<int>(static_cast<int8_t>((q4 >> (8 * e)) & 0xFFu));
            w[e] = static_cast<float>(q) * d;
        }
    } else {
        constexpr int kQs   = QuantTraits<TYPE>::kQs;
        const uint32_t q4    = ld_u32_a2(blk + kQs + 4 * (c & 3));  // qs[4(c&3)] .. +3
        const int      shift = (c >> 2) * 4;                          // low nibbles for j < 16
        uint32_t       qh    = 0;
        if constexpr (TYPE == 6) qh = ld_u32_a2(blk + 2);
        if constexpr (TYPE == 7) qh = ld_u32_a2(blk + 4);
        float m = 0.0f;
        if constexpr (TYPE == 3 || TYPE == 7) m = half_bits_to_float(ld_u16(blk + 2));
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            int q = static_cast<int>((q4 >> (8 * e + shift)) & 0xFu);
            if constexpr (TYPE == 6 || TYPE == 7) q |= static_cast<int>(((qh >> (j0 + e)) & 1u) << 4);
            if constexpr (TYPE == 2) w[e] = static_cast<float>(q - 8) * d;
            if constexpr (TYPE == 6) w[e] = static_cast<float>(q - 16) * d;
            if constexpr (TYPE == 3 || TYPE == 7) w[e] = __fmaf_rn(static_cast<float>(q), d, m);
        }
    }
}

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

template <int TYPE>
__device__ __forceinline__ void decode_quad_words(const QuadWords& r, int j0, float (&w)[4]) {
    const float    d = half_bits_to_float(r.d);
    const uint32_t q = r.q0 | (r.q1 << 16);
    if constexpr (TYPE == 8) {
#pragma unroll
        for (int e = 0; e < 4; ++e) w[e] = static_cast<float>(static_cast<int>(static_cast<int8_t>((q >> (8 * e)) & 0xFFu))) * d;
    } else {
        const int shift = j0 >= 16 ? 4 : 0;
        float m = 0.0f;
        if constexpr (TYPE == 3 || TYPE == 7) m = half_bits_to_float(r.m);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            int v = static_cast<int>((q >> (8 * e + shift)) & 0xFu);
            if constexpr (TYPE == 6 || TYPE == 7) v |= static_cast<int>(((r.qh >> ((j0 & 15) + e)) & 1u) << 4);
            if constexpr (TYPE == 2) w[e] = static_cast<float>(v - 8) * d;
            if constexpr (TYPE == 6) w[e] = static_cast<float>(v - 16) * d;
            if constexpr (TYPE == 3 || TYPE == 7) w[e] = __fmaf_rn(static_cast<float>(v), d, m);
        }
    }
}

}  // namespace trc
