// The block formats served on the CUDA cores only (the warp-per-row matvec of the operator seam
// and the expert kernels): Q4_K, Q5_K, Q6_K, IQ2_S and MXFP4. Their blocks keep the ggml byte
// order on the device, except for two shifts that align every field a kernel loads as a word
// (vlb_upload_matrix writes them):
//
//   type   slot  layout (byte offsets)
//   Q4_K   144   d 0, dmin 2, 12 packed 6-bit scale/min bytes 4, 128 nibble bytes 16
//   Q5_K   176   d 0, dmin 2, scale bytes 4, 32 fifth-bit bytes 16, 128 nibble bytes 48
//   Q6_K   212   128 low-nibble bytes 0, 64 high-bit bytes 128, 16 int8 scales 192, d 208
//   IQ2_S   84   d 0, (2 pad), 32 grid-index bytes 4, 32 sign bytes 36, 8 high-bit bytes 68,
//                8 scale bytes 76
//   MXFP4   20   16 nibble bytes 0, the E8M0 scale byte 16, (3 pad)
//
// Slots are tiled like the other formats (blk_index). Every decoder reproduces the reference's
// f32 weight exactly: the same operations in the same order, each rounded to f32 (__fmul_rn /
// __fsub_rn keep the compiler from contracting a product into a subtraction).
#pragma once

#include "vlb_internal.cuh"

namespace vlb {

__host__ __device__ constexpr bool raw_type(uint32_t t) {
    return t == kTypeQ4K || t == kTypeQ5K || t == kTypeQ6K || t == kTypeIq2S || t == kTypeMxfp4;
}
__host__ __device__ constexpr uint32_t raw_slot_bytes(uint32_t t) {
    return t == kTypeQ4K ? 144u : t == kTypeQ5K ? 176u : t == kTypeQ6K ? 212u : t == kTypeIq2S ? 84u : 20u;
}
// 32-weight groups per block
__host__ __device__ constexpr uint32_t raw_groups(uint32_t t) { return t == kTypeMxfp4 ? 1u : 8u; }

// The doubled E2M1 values of MXFP4 (decode_mxfp4_block, ggml_quantization.cpp:44-47,381-398) and
// half the power of two of an E8M0 byte (e8m0_to_float_half, :112-120): bytes 0 and 1 give the two
// smallest half-scaled powers (subnormal floats), byte e >= 2 the normal 2^(e - 128).
__device__ __forceinline__ float mxfp4_value(uint32_t nibble) {
    const int v = (int)(0xC8643210u >> (4u * (nibble & 7u)) & 15u);  // 0 1 2 3 4 6 8 12
    return (float)((nibble & 8u) ? -v : v);
}
__device__ __forceinline__ float e8m0_half(uint32_t e) {
    return __uint_as_float(e < 2u ? 0x00200000u << e : (e - 1u) << 23);
}

// qk_scale_min (ggml_quantization.cpp:437-455): 6-bit scale and minimum of sub-block j of a
// Q4_K / Q5_K block from its 12 packed bytes s[0..11].
__device__ __forceinline__ void qk_scale_min(uint32_t j, const uint8_t* s, uint32_t& sc, uint32_t& mn) {
    if (j < 4u) {
        sc = s[j] & 63u;
        mn = s[j + 4u] & 63u;
    } else {
        sc = (s[j + 4u] & 15u) | ((uint32_t)(s[j - 4u] >> 6) << 4);
        mn = (s[j + 4u] >> 4) | ((uint32_t)(s[j] >> 6) << 4);
    }
}

// What one 32-weight group needs besides its quant bytes.
struct RawGroup {
    float s0, s1;  // scales: Q4_K/Q5_K d*sc and dmin*m; Q6_K the two 16-weight scales; IQ2_S the
                   // scales of sub-blocks 0-1 and 2-3; MXFP4 the block scale
    uint32_t off;  // quant byte offset in the slot (Q4_K/Q5_K/Q6_K)
    uint32_t a, b, c;
};

__device__ __forceinline__ uint32_t ldu32(const uint8_t* p) { return __ldg(reinterpret_cast<const uint32_t*>(p)); }

// Group gg (of the block at slot p): its scales and word offsets.
template <uint32_t FMT>
__device__ __forceinline__ RawGroup raw_group(const uint8_t* p, uint32_t gg) {
    RawGroup r{};
    if constexpr (FMT == kTypeQ4K || FMT == kTypeQ5K) {
        // decode_q4_k_block :457-493, decode_q5_k_block :495-539
        uint8_t s[12];
        const uint32_t w0 = ldu32(p + 4), w1 = ldu32(p + 8), w2 = ldu32(p + 12);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            s[i] = (uint8_t)(w0 >> (8 * i));
            s[4 + i] = (uint8_t)(w1 >> (8 * i));
            s[8 + i] = (uint8_t)(w2 >> (8 * i));
        }
        uint32_t sc, mn;
        qk_scale_min(gg, s, sc, mn);
        const uint32_t dd = ldu32(p);
        r.s0 = __fmul_rn(h2f((uint16_t)dd), (float)sc);
        r.s1 = __fmul_rn(h2f((uint16_t)(dd >> 16)), (float)mn);
        r.off = (FMT == kTypeQ4K ? 16u : 48u) + 32u * (gg >> 1);
        r.a = 4u * (gg & 1u);  // nibble shift
        r.b = gg;              // Q5_K: the fifth bit of weight l is bit gg of byte 16 + l
    } else if constexpr (FMT == kTypeQ6K) {
        // decode_q6_k_block :541-590: group gg = half h, quarter i; weights 16 l' .. use scale
        // 8 h + 2 i (first 16) and 8 h + 2 i + 1 (last 16)
        const uint32_t h = gg >> 2, i = gg & 3u;
        const float d = h2f((uint16_t)ldu32(p + 208));
        const uint32_t sw = ldu32(p + 192 + 8u * h + 4u * (i >> 1));
        const int8_t s0 = (int8_t)(sw >> (16u * (i & 1u))), s1 = (int8_t)(sw >> (16u * (i & 1u) + 8u));
        r.s0 = __fmul_rn(d, (float)s0);
        r.s1 = __fmul_rn(d, (float)s1);
        r.off = 64u * h + 32u * (i & 1u);  // low-nibble bytes
        r.a = (i >> 1) * 4u;               // nibble shift
        r.b = 128u + 32u * h;              // high-bit bytes
        r.c = 2u * i;                      // high-bit shift
    } else if constexpr (FMT == kTypeIq2S) {
        // decode_iq2_s_block :285-334
        const float d = h2f((uint16_t)ldu32(p));
        const uint32_t sc = (ldu32(p + 76 + (gg & 4u)) >> (8u * (gg & 3u))) & 0xffu;
        r.s0 = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)(sc & 15u))), 0.25f);
        r.s1 = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)(sc >> 4))), 0.25f);
        r.a = ldu32(p + 4 + 4u * gg);   // grid-index bytes of sub-blocks 0-3
        r.b = ldu32(p + 36 + 4u * gg);  // their sign bytes
        r.c = (ldu32(p + 68 + (gg & 4u)) >> (8u * (gg & 3u))) & 0xffu;  // high index bits
    } else {  // MXFP4
        r.s0 = e8m0_half(ldu32(p + 16) & 0xffu);
    }
    return r;
}

// Weights 8 j .. 8 j + 7 of a group into w (grid: the IQ2_S codebook).
template <uint32_t FMT>
__device__ __forceinline__ void raw_sub(const uint8_t* p, const RawGroup& r, int j, const uint64_t* grid,
                                        float* w) {
    if constexpr (FMT == kTypeQ4K || FMT == kTypeQ5K) {
        const uint32_t q0 = ldu32(p + r.off + 8u * j), q1 = ldu32(p + r.off + 8u * j + 4u);
        uint32_t h0 = 0, h1 = 0;
        if constexpr (FMT == kTypeQ5K) {
            h0 = ldu32(p + 16 + 8u * j);
            h1 = ldu32(p + 20 + 8u * j);
        }
#pragma unroll
        for (int l = 0; l < 8; ++l) {
            const uint32_t byte = (l < 4 ? q0 : q1) >> (8 * (l & 3));
            uint32_t v = (byte >> r.a) & 15u;
            if constexpr (FMT == kTypeQ5K) v += (((l < 4 ? h0 : h1) >> (8 * (l & 3) + r.b)) & 1u) ? 16u : 0u;
            w[l] = __fsub_rn(__fmul_rn(r.s0, (float)v), r.s1);
        }
    } else if constexpr (FMT == kTypeQ6K) {
        const uint32_t q0 = ldu32(p + r.off + 8u * j), q1 = ldu32(p + r.off + 8u * j + 4u);
        const uint32_t h0 = ldu32(p + r.b + 8u * j), h1 = ldu32(p + r.b + 8u * j + 4u);
        const float s = j < 2 ? r.s0 : r.s1;
#pragma unroll
        for (int l = 0; l < 8; ++l) {
            const uint32_t lo = ((l < 4 ? q0 : q1) >> (8 * (l & 3) + r.a)) & 15u;
            const uint32_t hi = ((l < 4 ? h0 : h1) >> (8 * (l & 3) + r.c)) & 3u;
            w[l] = __fmul_rn(s, (float)((int)(lo | (hi << 4)) - 32));
        }
    } else if constexpr (FMT == kTypeIq2S) {
        const uint32_t idx = ((r.a >> (8 * j)) & 0xffu) | ((r.c << (8 - 2 * j)) & 0x300u);
        const uint64_t gv = grid[idx];
        const uint32_t sg = (r.b >> (8 * j)) & 0xffu;
        const float s = j < 2 ? r.s0 : r.s1;
#pragma unroll
        for (int l = 0; l < 8; ++l) {
            const float m = __fmul_rn(s, (float)((uint32_t)(gv >> (8 * l)) & 0xffu));
            w[l] = (sg >> l) & 1u ? -m : m;
        }
    } else {  // MXFP4: weight i < 16 the low nibble of byte i, i >= 16 the high nibble of byte i - 16
        const uint32_t q0 = ldu32(p + 8u * (j & 1)), q1 = ldu32(p + 8u * (j & 1) + 4u);
        const uint32_t shift = j >= 2 ? 4u : 0u;
#pragma unroll
        for (int l = 0; l < 8; ++l)
            w[l] = __fmul_rn(mxfp4_value(((l < 4 ? q0 : q1) >> (8 * (l & 3) + shift)) & 15u), r.s0);
    }
}

// The 32 weights of group gg of the block at slot p (dequantize).
template <uint32_t FMT>
__device__ __forceinline__ void raw_decode_group(const uint8_t* p, uint32_t gg, const uint64_t* grid, float* w) {
    const RawGroup r = raw_group<FMT>(p, gg);
#pragma unroll
    for (int j = 0; j < 4; ++j) raw_sub<FMT>(p, r, j, grid, w + 8 * j);
}

}  // namespace vlb
