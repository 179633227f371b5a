// Warp-level dequant-dot engine of the decode path (few tokens per expert).
//
// A warp owns R rows of one or two resident matrices and up to TOKC tokens; its 32 lanes split
// the columns by 32-weight groups (lane l takes groups l, l+32, ...), so the raw block data a
// warp reads for one row is one contiguous, coalesced span. Each lane decodes a group sub-block
// (8 weights) at a time into registers and multiplies it against TOKC activation rows held in
// shared memory. The activation for a sub-block is loaded once and reused by all R rows, which
// is what keeps shared-memory traffic well below the FMA rate. Partial sums are reduced across
// the warp at the end.
//
// Shared-memory activation layout (conflict-free 16-byte loads for consecutive groups):
//   xs[((t*4 + j)*2 + h)*ngroups + g][e] = x[t][g*32 + j*8 + h*4 + e]
#pragma once

#include "vlb_formats.cuh"
#include "vlb_internal.cuh"

namespace vlb {

struct GridSmem {
    const uint64_t* iq1s;
    const uint64_t* iq2xxs;
    const uint32_t* iq3xxs;
    const uint64_t* iq2s;
};

__device__ __forceinline__ uint32_t xs_index(uint32_t t, uint32_t j, uint32_t h, uint32_t g,
                                             uint32_t ngroups) {
    return (((t * 4u + j) * 2u + h) * ngroups + g) * 4u;
}

// Per-(row, group) raw data held in registers while the four sub-blocks are processed.
struct GroupRaw {
    uint32_t a, b, c, e;  // format-specific words
    float ls;             // group scale
    float delta;          // IQ1_S delta
};

template <uint32_t FMT>
__device__ __forceinline__ void load_group(const DevMat& m, uint32_t row, uint32_t g,
                                           GroupRaw& r) {
    if constexpr (FMT == kTypeQ8_0) {
        // one 32-weight block per group; the 32 quants are loaded per sub-block pair below
        r.ls = h2f(__ldg(m.d + blk_index(m.bpr, row, g)));
    } else if constexpr (FMT == kTypeIq2Xxs) {
        const uint32_t blk = g >> 3, gg = g & 7u;
        const float d = h2f(__ldg(m.d + blk_index(m.bpr, row, blk)));
        const uint2 v = __ldg(reinterpret_cast<const uint2*>(
            m.body + blk_index(m.bpr, row, blk) * 64u + gg * 8u));
        const uint32_t ls4 = (__ldg(m.scales + blk_index(m.bpr, row, blk)) >> (4u * gg)) & 15u;
        r.a = v.x;
        r.b = v.y;  // pair-layout sign word
        r.ls = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)ls4)), 0.25f);
    } else if constexpr (FMT == kTypeIq3Xxs) {
        const uint32_t blk = g >> 3, gg = g & 7u;
        const float d = h2f(__ldg(m.d + blk_index(m.bpr, row, blk)));
        const uint8_t* body = m.body + blk_index(m.bpr, row, blk) * 96u;
        const uint2 v = __ldg(reinterpret_cast<const uint2*>(body + gg * 8u));
        const uint32_t ls4 = (__ldg(m.scales + blk_index(m.bpr, row, blk)) >> (4u * gg)) & 15u;
        r.a = v.x;
        r.b = v.y;
        r.c = __ldg(reinterpret_cast<const uint32_t*>(body + 64u + gg * 4u));  // pair-layout sign word
        r.ls = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)ls4)), 0.5f);
    } else {  // IQ1_S
        const uint32_t blk = g >> 3, gg = g & 7u;
        const float d = h2f(__ldg(m.d + blk_index(m.bpr, row, blk)));
        const uint8_t* body = m.body + blk_index(m.bpr, row, blk) * 48u;
        const uint32_t qs4 = __ldg(reinterpret_cast<const uint32_t*>(body + gg * 4u));
        const uint32_t h = __ldg(reinterpret_cast<const uint16_t*>(body + 32u + gg * 2u));
        r.a = qs4;
        r.b = h;
        r.ls = __fmul_rn(d, (float)(2u * ((h >> 12) & 7u) + 1u));
        r.delta = (h & 0x8000u) ? -0.125f : 0.125f;
    }
}

// Decodes sub-block j (8 weights) of a group into w[8], bit-exact with the reference decoders.
template <uint32_t FMT>
__device__ __forceinline__ void decode_sub(const DevMat& m, uint32_t row, uint32_t g,
                                           const GroupRaw& r, int j, const GridSmem& gs,
                                           float* w) {
    if constexpr (FMT == kTypeQ8_0) {
        const uint2 q = __ldg(reinterpret_cast<const uint2*>(
            m.body + blk_index(m.bpr, row, g) * 32u + j * 8u));
#pragma unroll
        for (int l = 0; l < 8; ++l) {
            const uint32_t word = l < 4 ? q.x : q.y;
            w[l] = __fmul_rn(r.ls, (float)(int8_t)((word >> (8 * (l & 3))) & 0xffu));
        }
    } else if constexpr (FMT == kTypeIq2Xxs) {
        const uint64_t gv = gs.iq2xxs[(r.a >> (8 * j)) & 0xffu];
        const uint32_t signs = iq2_sub_signs(r.b, j);
#pragma unroll
        for (int l = 0; l < 8; ++l) {
            const float p = __fmul_rn(r.ls, (float)((uint32_t)(gv >> (8 * l)) & 0xffu));
            w[l] = (signs >> l) & 1u ? -p : p;
        }
    } else if constexpr (FMT == kTypeIq3Xxs) {
        const uint32_t word = j < 2 ? r.a : r.b;
        const uint32_t g1 = gs.iq3xxs[(word >> (16 * (j & 1))) & 0xffu];
        const uint32_t g2 = gs.iq3xxs[(word >> (16 * (j & 1) + 8)) & 0xffu];
        const uint32_t signs = iq2_sub_signs(r.c, j);
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const float p1 = __fmul_rn(r.ls, (float)((g1 >> (8 * l)) & 0xffu));
            const float p2 = __fmul_rn(r.ls, (float)((g2 >> (8 * l)) & 0xffu));
            w[l] = (signs >> l) & 1u ? -p1 : p1;
            w[l + 4] = (signs >> (l + 4)) & 1u ? -p2 : p2;
        }
    } else {
        const uint32_t idx = ((r.a >> (8 * j)) & 0xffu) | (((r.b >> (3 * j)) & 7u) << 8);
        const uint64_t gv = gs.iq1s[idx];
#pragma unroll
        for (int l = 0; l < 8; ++l) {
            const float q = (float)(int8_t)(uint8_t)((gv >> (8 * l)) & 0xffu);
            w[l] = __fmul_rn(r.ls, __fadd_rn(q, r.delta));
        }
    }
}

// warp_dot for the whole-block formats (vlb_formats.cuh): the same column split and activation
// layout, each group's scales read once per row, its weights decoded 8 at a time.
template <uint32_t FMT, int RA, int RB, int TOKC>
__device__ __forceinline__ void warp_dot_raw(const DevMat& ma, const DevMat& mb, uint32_t row_a,
                                             uint32_t row_b, const float* __restrict__ xs,
                                             uint32_t ngroups, const GridSmem& gs,
                                             float (&acc)[RA + RB][TOKC]) {
    constexpr int R = RA + RB;
    constexpr uint32_t gpb = raw_groups(FMT), slot = raw_slot_bytes(FMT);
    const uint32_t lane = threadIdx.x & 31u;
    for (uint32_t g = lane; g < ngroups; g += 32u) {
        const uint32_t blk = g / gpb, gg = g % gpb;
        const uint8_t* pb[R];
        RawGroup raw[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const DevMat& m = r < RA ? ma : mb;
            const uint32_t row = r < RA ? row_a + r : row_b + (r - RA);
            pb[r] = m.body + blk_index(m.bpr, row, blk) * slot;
            raw[r] = raw_group<FMT>(pb[r], gg);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float xv[TOKC][8];
#pragma unroll
            for (int t = 0; t < TOKC; ++t) {
                const float4 lo = *reinterpret_cast<const float4*>(xs + xs_index(t, j, 0, g, ngroups));
                const float4 hi = *reinterpret_cast<const float4*>(xs + xs_index(t, j, 1, g, ngroups));
                xv[t][0] = lo.x; xv[t][1] = lo.y; xv[t][2] = lo.z; xv[t][3] = lo.w;
                xv[t][4] = hi.x; xv[t][5] = hi.y; xv[t][6] = hi.z; xv[t][7] = hi.w;
            }
#pragma unroll
            for (int r = 0; r < R; ++r) {
                float w[8];
                raw_sub<FMT>(pb[r], raw[r], j, gs.iq2s, w);
#pragma unroll
                for (int t = 0; t < TOKC; ++t)
#pragma unroll
                    for (int l = 0; l < 8; ++l) acc[r][t] = fmaf(w[l], xv[t][l], acc[r][t]);
            }
        }
    }
}

// acc[r][t] += sum over this lane's columns of W[row_r][c] * x[t][c], for the R rows
// rows[0..R) of matrix ma (first RA rows) and mb (the rest). Both matrices share the columns.
template <uint32_t FMT, int RA, int RB, int TOKC>
__device__ __forceinline__ void warp_dot_split(const DevMat& ma, const DevMat& mb, uint32_t row_a,
                                               uint32_t row_b, const float* __restrict__ xs,
                                               uint32_t ngroups, const GridSmem& gs,
                                               float (&acc)[RA + RB][TOKC]) {
    constexpr int R = RA + RB;
    const uint32_t lane = threadIdx.x & 31u;
    for (uint32_t g = lane; g < ngroups; g += 32u) {
        GroupRaw raw[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
            if (r < RA) load_group<FMT>(ma, row_a + r, g, raw[r]);
            else load_group<FMT>(mb, row_b + (r - RA), g, raw[r]);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float xv[TOKC][8];
#pragma unroll
            for (int t = 0; t < TOKC; ++t) {
                const float4 lo = *reinterpret_cast<const float4*>(xs + xs_index(t, j, 0, g, ngroups));
                const float4 hi = *reinterpret_cast<const float4*>(xs + xs_index(t, j, 1, g, ngroups));
                xv[t][0] = lo.x; xv[t][1] = lo.y; xv[t][2] = lo.z; xv[t][3] = lo.w;
                xv[t][4] = hi.x; xv[t][5] = hi.y; xv[t][6] = hi.z; xv[t][7] = hi.w;
            }
#pragma unroll
            for (int r = 0; r < R; ++r) {
                float w[8];
                if (r < RA) decode_sub<FMT>(ma, row_a + r, g, raw[r], j, gs, w);
                else decode_sub<FMT>(mb, row_b + (r - RA), g, raw[r], j, gs, w);
#pragma unroll
                for (int t = 0; t < TOKC; ++t)
#pragma unroll
                    for (int l = 0; l < 8; ++l) acc[r][t] = fmaf(w[l], xv[t][l], acc[r][t]);
            }
        }
    }
}

template <uint32_t FMT, int RA, int RB, int TOKC>
__device__ __forceinline__ void warp_dot(const DevMat& ma, const DevMat& mb, uint32_t row_a,
                                         uint32_t row_b, const float* __restrict__ xs,
                                         uint32_t ngroups, const GridSmem& gs,
                                         float (&acc)[RA + RB][TOKC]) {
    if constexpr (raw_type(FMT))
        warp_dot_raw<FMT, RA, RB, TOKC>(ma, mb, row_a, row_b, xs, ngroups, gs, acc);
    else
        warp_dot_split<FMT, RA, RB, TOKC>(ma, mb, row_a, row_b, xs, ngroups, gs, acc);
}

template <int R, int TOKC>
__device__ __forceinline__ void warp_reduce(float (&acc)[R][TOKC]) {
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int t = 0; t < TOKC; ++t) {
            float v = acc[r][t];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            acc[r][t] = v;
        }
}

// Copies TOKC activation rows (row pointers may be null -> zeros) of `cols` floats into the
// permuted shared layout. All threads of the CTA participate.
template <int TOKC>
__device__ __forceinline__ void stage_x(float* xs, const float* const* rows, uint32_t cols) {
    const uint32_t ngroups = cols / 32u;
    const uint32_t n4 = cols / 4u;  // float4 per row
    for (uint32_t i = threadIdx.x; i < TOKC * n4; i += blockDim.x) {
        const uint32_t t = i / n4, q = i % n4;
        const uint32_t c = q * 4u;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (rows[t]) v = *reinterpret_cast<const float4*>(rows[t] + c);
        const uint32_t g = c >> 5, j = (c >> 3) & 3u, h = (c >> 2) & 1u;
        *reinterpret_cast<float4*>(xs + xs_index(t, j, h, g, ngroups)) = v;
    }
}

}  // namespace vlb
