// Decode expert kernels on the tensor cores' warp-level MMA (mma.sync m16n8k16, fp16 operands,
// f32 accumulation), for the IQ2_XXS and Q8_0 formats.
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
// whole 32-column Q8_0 block per pair). With that mapping a single coalesced 16-byte load per row
// gives a lane the two groups it owns, a 16-byte shared load gives its 8 activation values, and no
// data moves between lanes. B columns use the same permutation.
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

__device__ __forceinline__ uint4 ldg128(const void* p) {
    return __ldg(reinterpret_cast<const uint4*>(p));
}

// ---- activation staging -------------------------------------------------------------------
// xs holds 8 B columns (n = 2 * token + piece) of K fp16 values, as 16-byte chunks with an XOR
// swizzle inside each 128-byte segment so that the 8 lanes of a shared-load phase (two n values x
// four lanes q) always hit 8 different bank quads.
__device__ __forceinline__ uint32_t xs_chunk(uint32_t n, uint32_t ch, uint32_t k_chunks) {
    return n * k_chunks + (ch ^ (((ch >> 3) & 3u) | ((n & 1u) << 2)));
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

// Stages rows[t] (f32, K floats; null = zero) scaled by scale[t] into xs as fp16 hi/lo pieces.
// Only the first n_tokens token slots are written (null rows become zeros); slots above stay as
// they are, which the caller guarantees to be zero.
__device__ __forceinline__ void stage_pieces(uint4* xs, const float* const* rows,
                                             const float* scale, uint32_t K, uint32_t n_tokens) {
    const uint32_t k_chunks = K / 8u;
    const uint32_t total = n_tokens * k_chunks;
    constexpr int kBatch = 4;  // loads issued together, for memory-level parallelism
    for (uint32_t i0 = threadIdx.x; i0 < total; i0 += kBatch * blockDim.x) {
        float4 a[kBatch], b[kBatch];
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            const uint32_t i = i0 + j * blockDim.x;
            a[j] = b[j] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (i < total) {
                const uint32_t t = i / k_chunks, ch = i % k_chunks;
                if (rows[t]) {
                    a[j] = *reinterpret_cast<const float4*>(rows[t] + ch * 8u);
                    b[j] = *reinterpret_cast<const float4*>(rows[t] + ch * 8u + 4u);
                }
            }
        }
#pragma unroll
        for (int j = 0; j < kBatch; ++j) {
            const uint32_t i = i0 + j * blockDim.x;
            if (i >= total) break;
            const uint32_t t = i / k_chunks, ch = i % k_chunks;
            const float v[8] = {a[j].x, a[j].y, a[j].z, a[j].w, b[j].x, b[j].y, b[j].z, b[j].w};
            const float s = scale[t];
            uint32_t hi[4], lo[4];
#pragma unroll
            for (int w = 0; w < 4; ++w) {
                const float x0 = v[2 * w] * s, x1 = v[2 * w + 1] * s;  // exact: s is 2^k
                const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
                const __half l0 = __float2half_rn(x0 - __half2float(h0));
                const __half l1 = __float2half_rn(x1 - __half2float(h1));
                hi[w] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
                lo[w] = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
            }
            xs[xs_chunk(2u * t, ch, k_chunks)] = make_uint4(hi[0], hi[1], hi[2], hi[3]);
            xs[xs_chunk(2u * t + 1u, ch, k_chunks)] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        }
    }
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

constexpr int kTiles = 2;  // 16-row tiles per warp

// Per-tile row pointers of this lane's two fragment rows (g and g+8).
struct TileRows {
    const uint8_t* body_lo[kTiles];
    const uint8_t* body_hi[kTiles];
    const uint16_t* d_lo[kTiles];
    const uint16_t* d_hi[kTiles];
    const uint32_t* s_lo[kTiles];  // IQ2_XXS group scale words
    const uint32_t* s_hi[kTiles];
};

__device__ __forceinline__ void tile_rows(const DevMat* const (&mats)[kTiles],
                                          const uint32_t (&rows_lo)[kTiles],
                                          const uint32_t (&rows_hi)[kTiles], uint32_t body_bytes,
                                          TileRows& tr) {
#pragma unroll
    for (int i = 0; i < kTiles; ++i) {
        const DevMat m = *mats[i];
        tr.body_lo[i] = m.body + blk_index(m.bpr, rows_lo[i], 0) * body_bytes;
        tr.body_hi[i] = m.body + blk_index(m.bpr, rows_hi[i], 0) * body_bytes;
        tr.d_lo[i] = m.d + blk_index(m.bpr, rows_lo[i], 0);
        tr.d_hi[i] = m.d + blk_index(m.bpr, rows_hi[i], 0);
        tr.s_lo[i] = m.scales ? m.scales + blk_index(m.bpr, rows_lo[i], 0) : nullptr;
        tr.s_hi[i] = m.scales ? m.scales + blk_index(m.bpr, rows_hi[i], 0) : nullptr;
    }
}

// One 256-column IQ2_XXS block of this lane's rows: two 16-byte pieces (groups 2q, 2q+1) and
// the fp16 block scale, per tile and fragment row.
struct Iq2Block {
    uint4 a[kTiles], b[kTiles];
    float da[kTiles], db[kTiles];
    uint32_t sa[kTiles], sb[kTiles];  // group scale words
};

__device__ __forceinline__ void load_iq2_block(const TileRows& tr, uint32_t blk, uint32_t q,
                                               Iq2Block& r) {
#pragma unroll
    for (int i = 0; i < kTiles; ++i) {
        r.a[i] = ldg128(tr.body_lo[i] + (size_t)blk * (kTileRows * 64u) + 16u * q);
        r.b[i] = ldg128(tr.body_hi[i] + (size_t)blk * (kTileRows * 64u) + 16u * q);
        r.da[i] = h2f(__ldg(tr.d_lo[i] + (size_t)blk * kTileRows));
        r.db[i] = h2f(__ldg(tr.d_hi[i] + (size_t)blk * kTileRows));
        r.sa[i] = __ldg(tr.s_lo[i] + (size_t)blk * kTileRows);
        r.sb[i] = __ldg(tr.s_hi[i] + (size_t)blk * kTileRows);
    }
}

// Accumulates acc[i][0..3] over columns [k0, k1) for the warp's tiles of an IQ2_XXS matrix. The
// next block's packed weights are loaded while the current one is decoded and multiplied.
__device__ __forceinline__ void iq2_rows(const TileRows& tr, uint32_t k0, uint32_t k1,
                                         const uint4* xs, uint32_t k_chunks, const uint4* tab,
                                         float (&acc)[kTiles][4]) {
    const uint32_t lane = threadIdx.x & 31u, q = lane & 3u, n = lane >> 2, lane7 = lane & 7u;
    const uint32_t b0 = k0 / 256u, b1 = k1 / 256u;
    if (b0 >= b1) return;
    Iq2Block cur;
    load_iq2_block(tr, b0, q, cur);
    for (uint32_t b = b0; b < b1; ++b) {
        Iq2Block nxt;
        if (b + 1 < b1) load_iq2_block(tr, b + 1, q, nxt);
        float D[kTiles][4];
#pragma unroll
        for (int i = 0; i < kTiles; ++i) D[i][0] = D[i][1] = D[i][2] = D[i][3] = 0.f;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            uint32_t kka[kTiles], kkb[kTiles];
#pragma unroll
            for (int i = 0; i < kTiles; ++i) {
                kka[i] = group_scale_h2((cur.sa[i] >> (4u * (2u * q + half))) & 15u);
                kkb[i] = group_scale_h2((cur.sb[i] >> (4u * (2u * q + half))) & 15u);
            }
#pragma unroll
            for (int sub = 0; sub < 4; ++sub) {
                const uint32_t ch = b * 32u + (2u * q + half) * 4u + sub;
                const uint4 xb = lds128(xs + xs_chunk(n, ch, k_chunks));
#pragma unroll
                for (int i = 0; i < kTiles; ++i) {
                    uint32_t va[4], vb[4];
                    decode_iq2_sub(tab, lane7, half ? cur.a[i].z : cur.a[i].x,
                                   half ? cur.a[i].w : cur.a[i].y, sub, kka[i], va);
                    decode_iq2_sub(tab, lane7, half ? cur.b[i].z : cur.b[i].x,
                                   half ? cur.b[i].w : cur.b[i].y, sub, kkb[i], vb);
                    mma16816(D[i], va[0], vb[0], va[1], vb[1], xb.x, xb.y);
                    mma16816(D[i], va[2], vb[2], va[3], vb[3], xb.z, xb.w);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < kTiles; ++i) {
            acc[i][0] = fmaf(cur.da[i], D[i][0], acc[i][0]);
            acc[i][1] = fmaf(cur.da[i], D[i][1], acc[i][1]);
            acc[i][2] = fmaf(cur.db[i], D[i][2], acc[i][2]);
            acc[i][3] = fmaf(cur.db[i], D[i][3], acc[i][3]);
        }
        if (b + 1 < b1) cur = nxt;
    }
}

// The same for a Q8_0 matrix (one 32-column block per k-step pair), two blocks per step so the
// next pair's quants are in flight while the current ones are multiplied.
__device__ __forceinline__ void q8_rows(const TileRows& tr, uint32_t k0, uint32_t k1,
                                        const uint4* xs, uint32_t k_chunks,
                                        float (&acc)[kTiles][4]) {
    const uint32_t lane = threadIdx.x & 31u, q = lane & 3u, n = lane >> 2;
    const uint32_t b0 = k0 / 32u, b1 = k1 / 32u;
    uint2 qa[kTiles], qb[kTiles];
    float da[kTiles], db[kTiles];
    auto load = [&](uint32_t b, uint2 (&xa)[kTiles], uint2 (&xb)[kTiles], float (&ya)[kTiles],
                    float (&yb)[kTiles]) {
#pragma unroll
        for (int i = 0; i < kTiles; ++i) {
            xa[i] = __ldg(reinterpret_cast<const uint2*>(tr.body_lo[i] + (size_t)b * (kTileRows * 32u) + 8u * q));
            xb[i] = __ldg(reinterpret_cast<const uint2*>(tr.body_hi[i] + (size_t)b * (kTileRows * 32u) + 8u * q));
            ya[i] = h2f(__ldg(tr.d_lo[i] + (size_t)b * kTileRows));
            yb[i] = h2f(__ldg(tr.d_hi[i] + (size_t)b * kTileRows));
        }
    };
    if (b0 >= b1) return;
    load(b0, qa, qb, da, db);
    for (uint32_t b = b0; b < b1; ++b) {
        uint2 na[kTiles], nb[kTiles];
        float nda[kTiles], ndb[kTiles];
        if (b + 1 < b1) load(b + 1, na, nb, nda, ndb);
        const uint4 xv = lds128(xs + xs_chunk(n, b * 4u + q, k_chunks));
#pragma unroll
        for (int i = 0; i < kTiles; ++i) {
            uint32_t va[4], vb[4];
            decode_q8_sub(qa[i].x, qa[i].y, va);
            decode_q8_sub(qb[i].x, qb[i].y, vb);
            float D[4] = {0.f, 0.f, 0.f, 0.f};
            mma16816(D, va[0], vb[0], va[1], vb[1], xv.x, xv.y);
            mma16816(D, va[2], vb[2], va[3], vb[3], xv.z, xv.w);
            acc[i][0] = fmaf(da[i], D[0], acc[i][0]);
            acc[i][1] = fmaf(da[i], D[1], acc[i][1]);
            acc[i][2] = fmaf(db[i], D[2], acc[i][2]);
            acc[i][3] = fmaf(db[i], D[3], acc[i][3]);
        }
        if (b + 1 < b1) {
#pragma unroll
            for (int i = 0; i < kTiles; ++i) {
                qa[i] = na[i];
                qb[i] = nb[i];
                da[i] = nda[i];
                db[i] = ndb[i];
            }
        }
    }
}

}  // namespace mma
}  // namespace vlb
