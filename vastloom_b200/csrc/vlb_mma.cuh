// Operand decoders shared by the tensor-core expert kernels: the decode kernels on the warp-level
// MMA (mma.sync m16n8k16, fp16 operands, f32 accumulation; vlb_decode.cu) and the prefill
// producers that write fp16 operands into tensor memory (vlb_prefill.cu), for IQ2_XXS and Q8_0.
//
// Why this shape. A decode step reads every selected expert's weights once, with only 1-4 tokens
// per expert, so the work per weight is: decode it, multiply it by a few activations. On B200 the
// integer pipe runs at half the FP32 rate (64 lanes/clk/SM), so a CUDA-core dot product spends
// more issue slots decoding and multiplying than HBM delivers weights. Here the multiply-add goes
// to the MMA unit; the SM only decodes each weight once into an A-fragment register.
//
// Exactness of the operands (so the products are exact and only the f32 sums round):
//   * IQ2_XXS weight = d * (0.5 + s)/4 * m * sign, m in {8, 25, 43}: the factor (1 + 2s) * m / 8
//     has at most 11 significant bits, so A = sign * (0.5 + s)/4 * m is an exact fp16; the fp16
//     block scale d is applied in f32 when a 256-column block's partial sums are read out. The
//     signs come from the pair-layout sign word (vlb_internal.cuh): one shift per fp16 pair.
//   * Q8_0 weight = d * q: A = q (int8) is an exact fp16; d is applied per 32-column block.
//   * Activations: x * 2^e (a per-token power of two bringing max|x| into [2^14, 2^15)) is split
//     into hi = fp16(x') and lo = fp16(x' - hi), 22 significant bits; both pieces are B columns
//     (n = 2 * token + piece) and the two partial sums are added at the end, then scaled by 2^-e.
//   Against the reference's f64 row sums this leaves ~2^-22 relative error per product plus f32
//   accumulation error: well inside the 1e-5 layer tolerance.
//
// Fragment mapping. In m16n8k16 a lane (g = lane/4, q = lane%4) holds A rows g and g+8 at k slots
// {2q, 2q+1, 2q+8, 2q+9}. The k order inside an MMA is free, so each lane's slots are mapped to
// the 8 consecutive weights of ONE sub-block (two MMAs of the same k-step pair): lane q takes
// sub-block s%4 of group 2q + s/4 in k-step pair s = 0..7 of a 256-column IQ2_XXS block (one
// whole 32-column Q8_0 block per pair). With that mapping a single 16-byte load per row gives a
// lane the two groups it owns, a 16-byte shared load gives its 8 activation values, and no data
// moves between lanes. B columns use the same permutation.
#pragma once

#include <cuda_fp16.h>

#include "vlb_internal.cuh"

namespace vlb {
namespace mma {

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

__device__ __forceinline__ uint32_t hsub2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(sel));
    return d;
}

// a ^ (b & 0x80008000): flips the two fp16 sign bits selected by b
__device__ __forceinline__ uint32_t flip_signs(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, 0x80008000, 0x78;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}

__device__ __forceinline__ uint4 lds128(const void* p) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"((uint32_t)__cvta_generic_to_shared(p)));
    return v;
}

// The power-of-two prescale of a row whose largest magnitude is `amax`: max|x * s| in
// [2^14, 2^15), far from fp16 overflow, and the lo piece stays a normal fp16 for all but values
// 2^-27 below the maximum.
__device__ __forceinline__ float prescale_for(float amax) {
    if (!(amax > 0.f) || !isfinite(amax)) return 1.f;
    int e;
    frexpf(amax, &e);  // amax = m * 2^e, m in [0.5, 1)
    return ldexpf(1.f, 15 - e);
}

// fp16 IQ2_XXS magnitude table: entry e = 8 fp16 magnitudes, replicated 8 times so that replica r
// sits in bank quad r (entry stride 128 bytes). Lane l reads replica l % 8: conflict-free.
__device__ __forceinline__ void build_iq2_table(uint4* tab, const uint64_t* grid) {
    if (!grid) return;
    for (uint32_t i = threadIdx.x; i < 256u * 8u; i += blockDim.x) {
        const uint64_t gv = grid[i >> 3];
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const __half a = __uint2half_rn((uint32_t)(gv >> (16 * j)) & 0xffu);
            const __half b = __uint2half_rn((uint32_t)(gv >> (16 * j + 8)) & 0xffu);
            w[j] = (uint32_t)__half_as_ushort(a) | ((uint32_t)__half_as_ushort(b) << 16);
        }
        tab[i] = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Decodes one IQ2_XXS sub-block of one row into 4 fp16x2 registers (pairs 0..3): magnitudes from
// the table, times the group factor kk, signs flipped from the pair-layout sign word `sw` (the
// signs of pair j of sub-block `sub` sit at bits 4 sub + j and 4 sub + j + 16, so shifting left by
// 15 - 4 sub - j lands them on the fp16 sign bits 15 and 31).
__device__ __forceinline__ void decode_iq2_sub(const uint4* tab, uint32_t lane7, uint32_t idx4,
                                               uint32_t sw, uint32_t sub, uint32_t kk,
                                               uint32_t (&v)[4]) {
    const uint32_t idx = prmt(idx4, 0u, 0x4440u | sub);  // grid index byte `sub`
    const uint4 g = tab[idx * 8u + lane7];
    v[0] = flip_signs(hmul2(g.x, kk), sw << (15u - 4u * sub));
    v[1] = flip_signs(hmul2(g.y, kk), sw << (14u - 4u * sub));
    v[2] = flip_signs(hmul2(g.z, kk), sw << (13u - 4u * sub));
    v[3] = flip_signs(hmul2(g.w, kk), sw << (12u - 4u * sub));
}

// The same decode with the table address built in two instructions (byte permute, multiply-add
// onto the lane's replica base `tab_lane`, a shared-memory address) and an explicit 32-bit
// shared-memory load (measured ~4% faster in the decode kernel than the generic-pointer form).
__device__ __forceinline__ void decode_iq2_sub_lane(uint32_t tab_lane, uint32_t idx4, uint32_t sw, uint32_t sub,
                                                    uint32_t kk, uint32_t (&v)[4]) {
    const uint32_t idx = prmt(idx4, 0u, 0x4440u | sub);
    uint32_t addr;
    asm("mad.lo.u32 %0, %1, 128, %2;" : "=r"(addr) : "r"(idx), "r"(tab_lane));
    uint4 g;
    asm("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(g.x), "=r"(g.y), "=r"(g.z), "=r"(g.w) : "r"(addr));
    v[0] = flip_signs(hmul2(g.x, kk), sw << (15u - 4u * sub));
    v[1] = flip_signs(hmul2(g.y, kk), sw << (14u - 4u * sub));
    v[2] = flip_signs(hmul2(g.z, kk), sw << (13u - 4u * sub));
    v[3] = flip_signs(hmul2(g.w, kk), sw << (12u - 4u * sub));
}

// IQ1_S grid as fp16: entry e = its 8 values q in {-1, 0, 1} (16 bytes), one copy (2048 entries
// fill 32 KB).
__device__ __forceinline__ void build_iq1s_table(uint4* tab, const uint64_t* grid) {
    if (!grid) return;
    for (uint32_t i = threadIdx.x; i < 2048u; i += blockDim.x) {
        const uint64_t gv = grid[i];
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const __half a = __int2half_rn((int)(int8_t)(uint8_t)(gv >> (16 * j)));
            const __half b = __int2half_rn((int)(int8_t)(uint8_t)(gv >> (16 * j + 8)));
            w[j] = (uint32_t)__half_as_ushort(a) | ((uint32_t)__half_as_ushort(b) << 16);
        }
        tab[i] = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

// IQ3_XXS grid as fp16: entry e = its 4 magnitudes (8 bytes), replicated 16 times so that replica
// r sits at byte 8 r of the entry's 128-byte row: the 16 lanes of an 8-byte load phase read
// replicas lane % 16, free of bank conflicts.
__device__ __forceinline__ void build_iq3_table(uint2* tab, const uint32_t* grid) {
    if (!grid) return;
    for (uint32_t i = threadIdx.x; i < 256u * 16u; i += blockDim.x) {
        const uint32_t gv = grid[i >> 4];
        uint32_t w[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const __half a = __uint2half_rn((gv >> (16 * j)) & 0xffu);
            const __half b = __uint2half_rn((gv >> (16 * j + 8)) & 0xffu);
            w[j] = (uint32_t)__half_as_ushort(a) | ((uint32_t)__half_as_ushort(b) << 16);
        }
        tab[i] = make_uint2(w[0], w[1]);
    }
}

// IQ1_S sub-block `sub` of one row: 11-bit grid index = qs byte `sub` | 3 bits of the group's qh
// word, the 8 grid values q from the table, A = q * (2s + 1) + delta * (2s + 1) (kk, dk: those
// factors as fp16 pairs) - an exact fp16 (at most 8 significant bits), the reference's weight
// ls * (q + delta) without the fp16 block scale d.
__device__ __forceinline__ void decode_iq1_sub(uint32_t tab, uint32_t qs4, uint32_t h, uint32_t sub, uint32_t kk,
                                               uint32_t dk, uint32_t (&v)[4]) {
    const uint32_t idx = prmt(qs4, 0u, 0x4440u | sub) | (((h >> (3u * sub)) & 7u) << 8);
    uint32_t addr;
    asm("mad.lo.u32 %0, %1, 16, %2;" : "=r"(addr) : "r"(idx), "r"(tab));
    uint4 g;
    asm("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(g.x), "=r"(g.y), "=r"(g.z), "=r"(g.w) : "r"(addr));
    v[0] = hfma2(g.x, kk, dk);
    v[1] = hfma2(g.y, kk, dk);
    v[2] = hfma2(g.z, kk, dk);
    v[3] = hfma2(g.w, kk, dk);
}

// (2s + 1, 2s + 1) and (delta (2s + 1), delta (2s + 1)) as fp16 pairs from an IQ1_S group word h
// (s = bits 12-14, delta = -1/8 when bit 15 is set, else +1/8): exact.
__device__ __forceinline__ void iq1_group_factors(uint32_t h, uint32_t& kk, uint32_t& dk) {
    const uint32_t n = 2u * ((h >> 12) & 7u) + 1u;
    kk = hsub2((n * 0x10001u) | 0x64006400u, 0x64006400u);
    dk = hmul2(kk, (h & 0x8000u) ? 0xB000B000u : 0x30003000u);
}

// IQ3_XXS sub-block `sub` of one row: two grid indices (bytes 2 (sub & 1), 2 (sub & 1) + 1 of
// `word`, the group's index word holding this sub-block), 4 magnitudes each from the replicated
// table, times the group factor kk = (0.5 + s) / 2, signs from the pair-layout sign word `sw` as
// for IQ2_XXS. A = sign * (0.5 + s) / 2 * m is an exact fp16 (at most 10 significant bits).
__device__ __forceinline__ void decode_iq3_sub(uint32_t tab_lane, uint32_t word, uint32_t sw, uint32_t sub,
                                               uint32_t kk, uint32_t (&v)[4]) {
    const uint32_t i0 = prmt(word, 0u, 0x4440u | (2u * (sub & 1u)));
    const uint32_t i1 = prmt(word, 0u, 0x4440u | (2u * (sub & 1u) + 1u));
    uint32_t a0, a1;
    asm("mad.lo.u32 %0, %1, 128, %2;" : "=r"(a0) : "r"(i0), "r"(tab_lane));
    asm("mad.lo.u32 %0, %1, 128, %2;" : "=r"(a1) : "r"(i1), "r"(tab_lane));
    uint2 A, B;
    asm("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(A.x), "=r"(A.y) : "r"(a0));
    asm("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(B.x), "=r"(B.y) : "r"(a1));
    v[0] = flip_signs(hmul2(A.x, kk), sw << (15u - 4u * sub));
    v[1] = flip_signs(hmul2(A.y, kk), sw << (14u - 4u * sub));
    v[2] = flip_signs(hmul2(B.x, kk), sw << (13u - 4u * sub));
    v[3] = flip_signs(hmul2(B.y, kk), sw << (12u - 4u * sub));
}

// (0.5 + s)/2 for the IQ3_XXS group scale s, as a pair of equal fp16 values (exact):
// fp16(1024 + s) * 0.5 - 511.75.
__device__ __forceinline__ uint32_t iq3_group_scale_h2(uint32_t s4) {
    return hfma2((s4 * 0x10001u) | 0x64006400u, 0x38003800u, 0xDFFFDFFFu);
}

// (0.5 + s)/4 for the 4-bit group scale s, as a pair of equal fp16 values (exact):
// fp16(1024 + s) is built from its bits, then (1024 + s) / 4 - 255.875 rounds exactly.
__device__ __forceinline__ uint32_t group_scale_h2(uint32_t s4) {
    return hfma2((s4 * 0x10001u) | 0x64006400u, 0x34003400u, 0xdbffdbffu);
}

// Q8_0: 8 int8 quants (two words) -> 4 fp16x2 registers with the exact integer values.
__device__ __forceinline__ void decode_q8_sub(uint32_t lo, uint32_t hi, uint32_t (&v)[4]) {
    const uint32_t ul = lo ^ 0x80808080u, uh = hi ^ 0x80808080u;  // biased to unsigned
    const uint32_t bias = 0x64806480u;                            // fp16(1152) x 2
    v[0] = hsub2(prmt(ul, 0x64646464u, 0x4140u), bias);
    v[1] = hsub2(prmt(ul, 0x64646464u, 0x4342u), bias);
    v[2] = hsub2(prmt(uh, 0x64646464u, 0x4140u), bias);
    v[3] = hsub2(prmt(uh, 0x64646464u, 0x4342u), bias);
}

}  // namespace mma
}  // namespace vlb
