// Internal definitions shared by the vlb200 CUDA sources: the device matrix layout, the
// bit-exact block decoders and the launch-side workspace structures.
//
// Device layout of a resident ggml matrix (chosen at upload, vlb_upload_matrix):
//   d      : fp16 block scales (the 2-byte header of every ggml block)
//   scales : IQ2_XXS and IQ3_XXS: one u32 per block holding the 8 group scales (nibble g = group
//            g's 4-bit scale, the top nibble of the ggml group word)
//   body   : the rest of each block, padded to a 16-byte multiple
//            Q8_0    : 32 int8 quants                                   (32 B)
//            IQ2_XXS : 8 groups x (4 grid-index bytes, u32 sign word)    (64 B)
//            IQ3_XXS : 64 grid-index bytes, then 8 x u32 pair sign words  (96 B)
//            IQ1_S   : 32 low-index bytes, then 8 x u16 high bits/scale   (48 B)
// all three in 128-row tiles: entry (row, block) sits at ((row / 128) * blocks_per_row + block) *
// 128 + row % 128, so one block column of a tile (128 rows x one block) is contiguous. The ggml
// block is 34/66/98/50 bytes, so splitting the scale off makes every body 16-byte aligned; the
// tiling makes the GEMMs' per-stage weight tile one contiguous run (bulk copies) and a decode
// warp's 8 consecutive rows of a block 512 contiguous bytes. Rows are padded to a multiple of 128
// (zero blocks).
//
// IQ2_XXS / IQ3_XXS sign word. The ggml group word holds four 7-bit sign fields (the eighth sign
// of each 8-weight sub-block is the even parity of the seven) and the group scale. The upload
// rewrites it with all 32 signs laid out in pairs: the signs of weights 2j and 2j + 1 of sub-block
// s are bits 4 s + j and 4 s + j + 16. One shift then puts a pair's two signs on the sign bits
// (15, 31) of an fp16x2 register, which is what the tensor-core decoders flip. The scale moves to
// `scales` (4 more bytes per 256 weights: 70 instead of 66 for IQ2_XXS, 102 instead of 98 for
// IQ3_XXS).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/vlb200.h"

namespace vlb {

constexpr uint32_t kTypeQ8_0 = VLB_TYPE_Q8_0;
constexpr uint32_t kTypeIq2Xxs = VLB_TYPE_IQ2_XXS;
constexpr uint32_t kTypeIq3Xxs = VLB_TYPE_IQ3_XXS;
constexpr uint32_t kTypeIq1S = VLB_TYPE_IQ1_S;
constexpr uint32_t kTypeQ4K = VLB_TYPE_Q4_K;
constexpr uint32_t kTypeQ5K = VLB_TYPE_Q5_K;
constexpr uint32_t kTypeQ6K = VLB_TYPE_Q6_K;
constexpr uint32_t kTypeIq2S = VLB_TYPE_IQ2_S;
constexpr uint32_t kTypeMxfp4 = VLB_TYPE_MXFP4;

struct TypeLayout {
    uint32_t block_elems;  // weights per ggml block
    uint32_t block_bytes;  // ggml block size (file/payload layout)
    uint32_t body_bytes;   // device body size (block minus the fp16 scale, 16-byte multiple)
};

__host__ __device__ inline bool type_layout(uint32_t type, TypeLayout* l) {
    switch (type) {
        case kTypeQ8_0: *l = {32u, 34u, 32u}; return true;
        case kTypeIq2Xxs: *l = {256u, 66u, 64u}; return true;
        case kTypeIq3Xxs: *l = {256u, 98u, 96u}; return true;
        case kTypeIq1S: *l = {256u, 50u, 48u}; return true;
        // served on the CUDA cores from whole-block slots (vlb_formats.cuh)
        case kTypeQ4K: *l = {256u, 144u, 144u}; return true;
        case kTypeQ5K: *l = {256u, 176u, 176u}; return true;
        case kTypeQ6K: *l = {256u, 210u, 212u}; return true;
        case kTypeIq2S: *l = {256u, 82u, 84u}; return true;
        case kTypeMxfp4: *l = {32u, 17u, 20u}; return true;
        default: return false;
    }
}

constexpr uint32_t kTileRows = 128;

// Layer error flag (MoeParams::counters[3]) of a Hyper-Connection reduced row that is not finite
// (deepseek_v4_hc_pre rejects it, deepseek_v4_reference.cpp:544-545).
constexpr uint32_t kLayerErrHcNonFinite = 32u;
// ... and of a Hyper-Connection entry whose weight-streaming wait ran out of time.
constexpr uint32_t kLayerErrHcTimeout = 64u;

// Index of block `blk` of row `row` in the tiled d / body arrays of a matrix with `bpr` blocks per
// row; consecutive blocks of one row are kTileRows entries apart.
__host__ __device__ __forceinline__ size_t blk_index(uint32_t bpr, uint32_t row, uint32_t blk) {
    return ((size_t)(row / kTileRows) * bpr + blk) * kTileRows + (row % kTileRows);
}

// Kernel-side view of a resident matrix.
struct DevMat {
    uint32_t type;
    uint32_t rows;
    uint32_t cols;
    uint32_t bpr;  // blocks per row
    const uint16_t* d;
    const uint8_t* body;
    const uint32_t* scales;  // IQ2_XXS / IQ3_XXS group scales (one u32 per block, tiled like d); else null
    // Power of two applied to the weights when the prefill kernels decode them to fp16: chosen at
    // upload from the largest block scale so that every |weight| * pscale stays below 2^14 (no
    // overflow) while small weights stay clear of the fp16 subnormal range.
    float pscale;
};

struct Grids {
    const uint64_t* iq1s;    // 2048 entries, 8 x int8
    const uint64_t* iq2xxs;  // 256 entries, 8 x uint8 magnitudes
    const uint32_t* iq3xxs;  // 256 entries, 4 x uint8 magnitudes
    const uint64_t* iq2s;    // 1024 entries, 8 x uint8 magnitudes
};

// fp16 -> f32. The hardware conversion is exact (every half, subnormals included, is a float),
// so it equals the reference's bit-level fp16_to_float (ggml_quantization.cpp:101-124).
__device__ __forceinline__ float h2f(uint16_t bits) {
    return __half2float(__ushort_as_half(bits));
}

// One bit per device storage type, for sets of types.
__host__ __device__ constexpr uint32_t fmt_bit(uint32_t type) {
    return type == kTypeQ8_0    ? 1u
           : type == kTypeIq2Xxs ? 2u
           : type == kTypeIq3Xxs ? 4u
           : type == kTypeIq1S   ? 8u
           : type == kTypeQ4K    ? 16u
           : type == kTypeQ5K    ? 32u
           : type == kTypeQ6K    ? 64u
           : type == kTypeIq2S   ? 128u
           : type == kTypeMxfp4  ? 256u
                                 : 0u;
}

// ---- bit-exact block decoders (one 32-weight group at a time) ------------------------------
// Each writes the 32 weights of group g (0..7 for the 256-weight formats; 0 for Q8_0) exactly as
// the reference's decode_*_block computes them: the same operations in the same order, every one
// rounded to f32 (no contraction is possible: no product feeds an addition).

// decode_q8_0_block, ggml_quantization.cpp:419-435
__device__ __forceinline__ void decode_group_q8_0(float d, const uint8_t* body, float* w) {
#pragma unroll
    for (int i = 0; i < 32; ++i) w[i] = __fmul_rn(d, (float)(int8_t)body[i]);
}

// The IQ2_XXS sign word of one ggml group word `aux` (see the layout note at the top): the four
// sub-blocks' 8-bit sign masks (seven stored bits plus even parity, ksigns_iq2xs semantics of
// ggml_quantization.cpp:268-271) regrouped into weight pairs.
__host__ __device__ inline uint32_t iq2_pair_signs(uint32_t aux) {
    uint32_t s = 0;
    for (uint32_t sub = 0; sub < 4; ++sub) {
        uint32_t s7 = (aux >> (7 * sub)) & 127u, par = 0;
        for (uint32_t b = 0; b < 7; ++b) par ^= (s7 >> b) & 1u;
        const uint32_t s8 = s7 | (par << 7);
        for (uint32_t l = 0; l < 8; ++l)
            if ((s8 >> l) & 1u) s |= 1u << (4 * sub + (l >> 1) + 16 * (l & 1));
    }
    return s;
}

// The 8-bit sign mask (bit l = weight l negative) of sub-block `sub` from a pair-layout sign word.
__device__ __forceinline__ uint32_t iq2_sub_signs(uint32_t sw, int sub) {
    const uint32_t lo = (sw >> (4 * sub)) & 15u, hi = (sw >> (4 * sub + 16)) & 15u;
    uint32_t r = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) r |= (((lo >> j) & 1u) << (2 * j)) | (((hi >> j) & 1u) << (2 * j + 1));
    return r;
}

// decode_iq2_xxs_block, ggml_quantization.cpp:250-283 (device layout: grid indices and the pair
// sign word in the body, the 4-bit group scale `ls4` from the scales word)
__device__ __forceinline__ void decode_group_iq2_xxs(float d, const uint8_t* body, int g, uint32_t ls4,
                                                     const uint64_t* grid, float* w) {
    const uint32_t idx4 = *reinterpret_cast<const uint32_t*>(body + g * 8);
    const uint32_t sw = *reinterpret_cast<const uint32_t*>(body + g * 8 + 4);
    const float ls = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)ls4)), 0.25f);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint64_t gv = grid[(idx4 >> (8 * j)) & 0xffu];
        const uint32_t signs = iq2_sub_signs(sw, j);
#pragma unroll
        for (int l = 0; l < 8; ++l) {
            const float m = (float)((uint32_t)(gv >> (8 * l)) & 0xffu);
            const float p = __fmul_rn(ls, m);
            w[j * 8 + l] = (signs >> l) & 1u ? -p : p;
        }
    }
}

// decode_iq3_xxs_block, ggml_quantization.cpp:336-379 (device layout: grid indices and the pair
// sign word in the body, the 4-bit group scale `ls4` from the scales word)
__device__ __forceinline__ void decode_group_iq3_xxs(float d, const uint8_t* body, int g, uint32_t ls4,
                                                     const uint32_t* grid, float* w) {
    const uint32_t sw = *reinterpret_cast<const uint32_t*>(body + 64 + g * 4);
    const uint2 idx8 = *reinterpret_cast<const uint2*>(body + g * 8);
    const float ls = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)ls4)), 0.5f);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t word = j < 2 ? idx8.x : idx8.y;
        const uint32_t g1 = grid[(word >> (16 * (j & 1))) & 0xffu];
        const uint32_t g2 = grid[(word >> (16 * (j & 1) + 8)) & 0xffu];
        const uint32_t signs = iq2_sub_signs(sw, j);
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const float p1 = __fmul_rn(ls, (float)((g1 >> (8 * l)) & 0xffu));
            const float p2 = __fmul_rn(ls, (float)((g2 >> (8 * l)) & 0xffu));
            w[j * 8 + l] = (signs >> l) & 1u ? -p1 : p1;
            w[j * 8 + l + 4] = (signs >> (l + 4)) & 1u ? -p2 : p2;
        }
    }
}

// decode_iq1_s_block, ggml_quantization.cpp:217-248
__device__ __forceinline__ void decode_group_iq1_s(float d, const uint8_t* body, int g,
                                                   const uint64_t* grid, float* w) {
    const uint32_t qs4 = *reinterpret_cast<const uint32_t*>(body + g * 4);
    const uint32_t h = *reinterpret_cast<const uint16_t*>(body + 32 + g * 2);
    const float ls = __fmul_rn(d, (float)(2u * ((h >> 12) & 7u) + 1u));
    const float delta = (h & 0x8000u) ? -0.125f : 0.125f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t idx = ((qs4 >> (8 * j)) & 0xffu) | (((h >> (3 * j)) & 7u) << 8);
        const uint64_t gv = grid[idx];
#pragma unroll
        for (int l = 0; l < 8; ++l) {
            const float q = (float)(int8_t)(uint8_t)((gv >> (8 * l)) & 0xffu);
            w[j * 8 + l] = __fmul_rn(ls, __fadd_rn(q, delta));
        }
    }
}

// ---- workspace of one MoE layer forward ----------------------------------------------------
// A "unit" is one expert's slice of at most kUnitTokens (token, slot) pairs; every (unit, row
// tile) pair is one work item of the expert kernels. Units are ordered by expert id ascending
// (the shared expert last), so a CTA walking consecutive items keeps the same activations.
constexpr int kUnitTokens = 4;

struct Unit {
    uint32_t expert;      // routed expert id, or E for the shared expert
    uint32_t pair_begin;  // first pair (row of the act/out workspaces)
    uint32_t count;       // pairs in this unit (1..kUnitTokens)
    uint32_t pad;
};

struct MoeParams {
    uint32_t H, I, E, k, T;
    int score;
    int hash_routing;
    int weight_after_down;
    float route_scale;
    float routed_limit;
    float shared_limit;
    uint32_t vocab;
    int has_shared;
    int has_legacy;          // some expert uses a format the prefill GEMMs do not serve (IQ3_XXS, IQ1_S)
    int has_mma;             // some expert uses a format the prefill GEMMs serve (IQ2_XXS, Q8_0)
    uint32_t fmt_gu, fmt_dn; // storage types present among the W1/W3 and the W2 matrices (fmt_bit)
    // weights
    const double* router;    // [E x H], the f32 router weights widened to f64 at layer creation
    const float* bias;       // [E]
    const uint32_t* tid2eid; // [vocab x k]
    const DevMat* mats;      // [3 x (E+1)]: w1[0..E], w3[0..E], w2[0..E]; index E = shared
    Grids grids;
    // per-call inputs
    const float* x;          // [T x H]
    const uint32_t* token_ids;
    const float* logits_in;  // optional [T x E]
    const uint32_t* routes_idx;  // optional [T x k]: given routes (skip the router and top-k)
    const float* routes_w;       // [T x k] their weights
    // optional half-row input (one route per row): rows fp16(x * 2^e) with, per row, meta
    // [expert id, route weight bits, max|x| bits]; replaces x, routes_idx and routes_w
    const __half* x_half;        // [T x H]
    const uint32_t* routes_meta; // [T x 3]
    // workspace
    float* logits;           // [T x E]
    float* scores;           // [T x E]
    uint32_t* idx;           // [T x k]
    float* weights;          // [T x k]
    uint32_t* offsets;       // [E + 2]
    uint32_t* pair_token;    // [T*k + T]
    uint32_t* pair_slot;     // [T*k + T]
    float* pair_weight;      // [T*k + T]
    Unit* units;             // [max_units]
    uint32_t* counters;      // [8]: n_units, n_active, gate/up next item, error flags, down next item,
                             //      prefill gate/up next item, prefill down next item, n_ptiles
    uint32_t* combine_pairs; // [T x k]: each token's pairs in (expert, slot) order
    float* act;              // [(T*k + T) x I]
    float* y;                // [(T*k + T) x H]
    float* out;              // [T x H]
    uint32_t* xmax;          // [T]: bits of max|x| per token (zeroed with the counters)
    double* xd;              // [T x H]: the router's input rows widened to f64
    uint32_t* act_max;       // [T*k + T]: bits of max|act| per pair (non-negative floats order as ints)
    // residual block (input norm set): the layer runs on xn = RMSNorm(x) (rows of x_norm) and the
    // combine adds the original rows back: out = x + MoE(xn)
    const float* norm_w;     // [H] or null
    float norm_eps;
    float* x_norm;           // [T x H] workspace
    const float* x_residual; // set by launch_moe for a residual block: the original rows
    // Hyper-Connection block (hc_m > 0; the input norm is set too): x and out hold m copies of
    // each token's hidden state, [T x m x H]. The entry computes the token's split (pre, post,
    // combination) and its reduced row, then the input norm; the combine writes
    // out[t, d] = post[d] * MoE[t] + sum_s comb[s][d] * x[t, s]
    uint32_t hc_m;           // 0: no Hyper-Connection
    uint32_t hc_iters;       // Sinkhorn iterations
    float hc_eps;            // the split's epsilon (the mixing RMS uses norm_eps)
    const double* hc_fn;     // [(2+m)m x mH] mixing weight, widened to f64 at set time
    const float* hc_scale;   // [3]
    const float* hc_base;    // [(2+m)m]
    float* hc_pre;           // [T x m] workspace: the split of the last forward
    float* hc_post;          // [T x m]
    float* hc_comb;          // [T x m x m], [source][destination]
    const float* hc_state;   // set by launch_moe: the original [T x m x H] rows
    uint32_t max_units;
    uint32_t* disp_counts;   // [ceil(T*k / 1024) x E]: per-chunk expert counts of the multi-CTA dispatch
    // K-split scratch of the decode kernels (small batches): 16 warps x 32 lanes x 8 floats of
    // partial sums per split item, and one arrival counter per (row group, warp), zeroed with the
    // counters before each forward; null: no splitting
    float* split_part;
    uint32_t* split_cnt;
    uint32_t split_items;    // split items the scratch holds
    // 1: a one-route-per-row forward (k = 1, given routes) without a shared expert whose route
    // weight is applied before the down product: each row's output is its single expert's down
    // product, so the down kernels write it straight to out[token] and no combine pass runs
    int direct_out;
    // prefill (tensor-core grouped GEMM) path
    int prefill;             // 1: this forward runs the expert products on tcgen05 (fp16 operands)
    __half* xperm;           // [(T*k + T) x H]: pair p's token row, fp16(x * 2^e_t) (the token's xmax power of two)
    __half* act_h;           // [(T*k + T) x I]: fp16(act * 2^e_p), the per-pair power of two of act_max
    Unit* ptiles;            // [max_ptiles]: (expert, first pair, pairs <= 256) GEMM column tiles
    uint32_t max_ptiles;
    // TMA descriptors of xperm and act_h (rows = max_tokens * (k + 1), 64 x 16 boxes, 128-byte
    // swizzle): the prefill GEMMs' B operands
    CUtensorMap bmap_x;
    CUtensorMap bmap_act;
};

}  // namespace vlb
