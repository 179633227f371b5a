// Decode expert products (one to four tokens per expert unit) for the IQ2_XXS and Q8_0 formats:
// warp-level tensor-core MMAs (mma.sync m16n8k16, exact fp16 operands, f32 accumulation; see
// vlb_mma.cuh for the exactness argument) fed by a bulk-copy ring in shared memory.
//
// Reference semantics: the expert loop of moe_forward (deepseek_v4_graph.cpp:2134-2227,
// execute_expert :1826-1895) and of the OLMoE layer (olmoe_runtime.cpp:1226-1285): gate = W1 x,
// up = W3 x, act = SwiGLU(gate, up) (route weight before the down product for DeepSeek V4, after
// it for OLMoE), y = W2 act, each row a sum of double(w) * double(x) in the reference. Here every
// product is exact and only the f32 sums round: ~1e-7 relative per row, inside the 1e-5 layer
// tolerance.
//
// Why this shape. A decode step reads every selected expert's weights once, with a handful of
// tokens each, so the kernel is a stream of weights through the SMs: each weight is decoded once
// into an A-fragment register and multiplied against 4 tokens x (hi, lo) activation pieces. The
// SM-side cost per weight (table lookup, scale, sign flip) is what bounds it, so nothing else may
// stall the decoding warps: one loader warp per CTA moves the packed weights and the unit's
// activations for the same columns with bulk copies into a 4-stage ring (~160 KB in flight per
// SM), and 16 consumer warps only decode and multiply. The activations come from an image that
// dc_image_kernel writes once per token (gate/up) or pair (down) before the launch.
//
// Work decomposition. A unit (<= 4 pairs of one expert, ordered by expert) and a row group form
// an item: gate/up items cover 256 rows of W1 and the same 256 rows of W3, down items 512 rows of
// W2. A stage is one K-chunk of the item: four 128-row tile block columns ("slices", 8 KB of
// packed weights each: 256 IQ2_XXS or 64 Q8_0 columns) with their block scales, and the unit's
// activation columns. Consumer warp w owns 16 rows of two slices (gate: W1 and W3 of tile w / 8;
// down: tiles w / 8 and 2 + w / 8), so every warp reads every stage and finishes its rows' sums
// itself: no cross-warp reduction. The loader takes items from a global counter in chunks of
// neighbouring items, fetching each item's scalars one item ahead, and tells the consumers what a
// stage holds through its stage header (item, K range, unit, storage type, the tokens' prescale
// words): the consumers make no global loads at item boundaries.
//
// Every wait is bounded by a 2 s limit; one that runs out sets error bit 8 of the layer flags and
// an abort word that ends every other wait of the CTA, so a broken pipeline ends the kernel with
// an error instead of hanging the GPU.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <mutex>
#include <vector>

#include "vlb_launch.h"
#include "vlb_mma.cuh"
#include "vlb_tcgen05.cuh"

namespace vlb {
namespace {

constexpr uint32_t kDcConsumerWarps = 16;
constexpr uint32_t kDcConsumers = kDcConsumerWarps * 32;
constexpr uint32_t kDcThreads = kDcConsumers + 32;             // + the loader warp
constexpr uint32_t kDcSlices = 4;
constexpr uint32_t kDcD = 512;                                 // fp16 block scales (<= 2 blocks)
constexpr uint32_t kDcSc = kTileRows * 4u;                     // IQ2_XXS / IQ3_XXS group scale words
constexpr uint32_t kDcTabBytes = 32768u;  // the IQ codebook in fp16 (layout per format: dc_build_table)
// Stage carve for slices of BODY bytes of packed weights: 8 KB holds a 128-row tile block column
// of IQ2_XXS (64 B a row), IQ1_S (48 B) or two Q8_0 blocks (2 x 32 B); IQ3_XXS (96 B a row) needs
// 12 KB and is launched with the larger carve.
constexpr uint32_t kDcBodySmall = kTileRows * 64u;
constexpr uint32_t kDcBodyLarge = kTileRows * 96u;
// A stage also holds the unit's activations for the stage's columns, streamed from the activation
// image (below) with the weights: 8 columns n = 2 token + piece (piece 0 = hi, 1 = lo) of one
// 512-byte block record each, 576 bytes apart (the 64-byte shift puts columns 2m and 2m + 1 in
// different bank halves).
constexpr uint32_t kDcXsCol = 576;
constexpr uint32_t kDcXsStage = 8u * kDcXsCol;
template <uint32_t BODY>
struct DcL {
    static constexpr uint32_t Body = BODY;
    static constexpr uint32_t Ring = BODY <= kDcBodySmall ? 4u : 3u;  // stages in flight
    static constexpr uint32_t Slice = BODY + kDcD + kDcSc;
    static constexpr uint32_t XsOff = kDcSlices * Slice;  // the activations, within a stage
    static constexpr uint32_t Stage = XsOff + kDcXsStage;
    static constexpr uint32_t RingOff = kDcTabBytes;
    static constexpr uint32_t HdrOff = RingOff + Ring * Stage;
    static constexpr uint32_t BarOff = HdrOff + Ring * 48u;  // three uint4 per stage header
    static constexpr uint32_t MiscOff = BarOff + 64u;        // abort word
    static constexpr uint32_t End = MiscOff + 16u;
    static_assert(Stage % 128 == 0 && HdrOff % 16 == 0, "shared-memory carve alignment");
    static_assert(2u * Ring * 8u <= 64u, "barriers fit their slot");
};
constexpr uint64_t kDcWaitNs = 2000000000ull;
constexpr uint32_t kDcSleepNs = 1000;  // suspend hint of one barrier test
constexpr uint32_t kDcErrTimeout = 8u;
constexpr uint32_t kDcEnd = 0xffffffffu;
#ifndef VLB_DC_MAX_CHUNK
#define VLB_DC_MAX_CHUNK 4
#endif
constexpr uint32_t kDcMaxChunk = VLB_DC_MAX_CHUNK;
constexpr uint32_t kDcMaxSplits = 8;

// Activation image: the decode kernels' B operand, converted once per row (a token's x for
// gate/up, a pair's act for down) instead of once per unit in every CTA. Row r is K / 256 records
// of 1 KB, one per 256-column block: the fp16 hi pieces of the block's values x * s (s the row's
// power-of-two prescale: max|x * s| in [2^14, 2^15)), then the lo pieces x * s - hi, each 32
// 16-byte chunks with chunk c (columns 8 c .. 8 c + 7) at position 4 (c % 8) + c / 8. In that
// order the consumer lanes' 16-byte loads are free of bank conflicts: in a 256-column stage lane
// q reads chunk 8 q + j (j = 4 half + sub-block), at position 4 j + q. A row takes 4 K bytes, the
// size of its f32 row, so the down phase converts act in place.
__global__ void __launch_bounds__(256) dc_image_kernel(const float* src, uint32_t K, const uint32_t* __restrict__ maxbits,
                                                       unsigned char* dst) {
    extern __shared__ __align__(16) float row_s[];
    const uint32_t r = blockIdx.x;
    const float* row = src + (size_t)r * K;
    // the whole row first: the down phase writes over its own input
    for (uint32_t i = threadIdx.x; i < K / 4u; i += blockDim.x)
        reinterpret_cast<float4*>(row_s)[i] = reinterpret_cast<const float4*>(row)[i];
    const float s = mma::prescale_for(__uint_as_float(maxbits[r]));
    __syncthreads();
    unsigned char* out = dst + (size_t)r * K * 4u;
    for (uint32_t c = threadIdx.x; c < K / 8u; c += blockDim.x) {
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            const float x0 = row_s[8u * c + 2u * w] * s, x1 = row_s[8u * c + 2u * w + 1u] * s;  // exact: s is a power of two
            const __half h0 = __float2half_rn(x0), h1 = __float2half_rn(x1);
            const __half l0 = __float2half_rn(x0 - __half2float(h0));
            const __half l1 = __float2half_rn(x1 - __half2float(h1));
            hi[w] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
            lo[w] = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
        }
        const uint32_t cb = c & 31u, pos = 4u * (cb & 7u) + (cb >> 3);
        unsigned char* rec = out + (size_t)(c >> 5) * 1024u + pos * 16u;
        *reinterpret_cast<uint4*>(rec) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4*>(rec + 512u) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
}

// One bounded wait on an mbarrier phase; false on abort or after the time limit. After a first
// test the thread suspends in the barrier (woken when the phase completes) instead of spinning.
__device__ __forceinline__ bool dc_wait(uint64_t* bar, uint32_t parity, volatile uint32_t* abort) {
    if (tc::mbar_try(bar, parity)) return true;
    const uint64_t t0 = tc::global_ns();
    for (uint32_t i = 1; i < (1u << 30); ++i) {
        if (tc::mbar_try_sleep(bar, parity, kDcSleepNs)) return true;
        if (*abort) return false;
        if (tc::global_ns() - t0 > kDcWaitNs) return false;
    }
    return false;
}

__device__ __forceinline__ void dc_fail(uint32_t* flags, volatile uint32_t* abort) {
    *abort = 1u;
    atomicOr(flags, kDcErrTimeout);
}

// Item geometry shared by the loader and the consumers.
struct DcItem {
    uint32_t unit, group;       // unit index, row group
    const DevMat* m[kDcSlices];  // matrix of each slice
    uint32_t tile[kDcSlices];    // 128-row tile of each slice
    bool valid[kDcSlices];
    uint32_t fmt;                // storage type of the item's matrices
    uint32_t st0, st1;           // this item's K-chunks: [st0, st1) of the row group's K
};

// Packed bytes per (row, block) of the device body, per type.
__device__ __forceinline__ uint32_t dc_body_bytes(uint32_t fmt) {
    return fmt == kTypeQ8_0 ? 32u : fmt == kTypeIq2Xxs ? 64u : fmt == kTypeIq1S ? 48u : 96u;
}

// Items are (unit, row group, K split): item = (unit * groups + group) * splits + split, so the
// splits of one row group are neighbours (they share the staged activations).
template <bool GATEUP>
__device__ __forceinline__ DcItem dc_item(const MoeParams& p, uint32_t item, const Unit& u, uint32_t fmt,
                                          uint32_t groups, uint32_t splits) {
    DcItem it;
    const uint32_t split = item % splits, rg = item / splits;
    it.unit = rg / groups;
    it.group = rg % groups;
    const uint32_t rows = GATEUP ? p.I : p.H;
    const uint32_t tiles = (rows + kTileRows - 1u) / kTileRows;
#pragma unroll
    for (uint32_t s = 0; s < kDcSlices; ++s) {
        if (GATEUP) {
            it.m[s] = p.mats + (s < 2u ? 0u : (p.E + 1u)) + u.expert;  // W1 for slices 0-1, W3 for 2-3
            it.tile[s] = 2u * it.group + (s & 1u);
        } else {
            it.m[s] = p.mats + 2u * (p.E + 1u) + u.expert;
            it.tile[s] = 4u * it.group + s;
        }
        it.valid[s] = it.tile[s] < tiles;
    }
    const uint32_t K = GATEUP ? p.H : p.I;
    it.fmt = fmt;
    const uint32_t stages = it.fmt != kTypeQ8_0 ? K / 256u : (K / 32u + 1u) / 2u;
    it.st0 = (uint32_t)((uint64_t)stages * split / splits);
    it.st1 = (uint32_t)((uint64_t)stages * (split + 1u) / splits);
    return it;
}

// The consumer warp's view of an item: its two slices' tiles (scalars, no indexed arrays).
struct DcWarpItem {
    uint32_t unit;
    uint32_t tile0, tile1;  // tiles of slices s0 and s1
    bool valid0, valid1;
    uint32_t fmt;
    uint32_t bpr;
};

// Built from the stage header's second word (unit count | storage type << 8, first pair, expert,
// blocks per row), which the loader writes: no global loads at an item boundary.
template <bool GATEUP>
__device__ __forceinline__ DcWarpItem dc_warp_item(const MoeParams& p, uint32_t item, const uint4& h2,
                                                   uint32_t groups, uint32_t splits, uint32_t s0, uint32_t s1) {
    DcWarpItem w;
    const uint32_t rg = item / splits;
    w.unit = rg / groups;
    const uint32_t group = rg % groups;
    const uint32_t rows = GATEUP ? p.I : p.H;
    const uint32_t tiles = (rows + kTileRows - 1u) / kTileRows;
    w.tile0 = GATEUP ? 2u * group + (s0 & 1u) : 4u * group + s0;
    w.tile1 = GATEUP ? 2u * group + (s1 & 1u) : 4u * group + s1;
    w.valid0 = w.tile0 < tiles;
    w.valid1 = w.tile1 < tiles;
    w.fmt = (h2.x >> 8) & 0xffu;
    w.bpr = h2.w;
    return w;
}

// ---- loader warp --------------------------------------------------------------------------------
// Lane 0 takes the items and does the ring bookkeeping; the copies of a stage are issued by
// different lanes at once (one copy per lane): a bulk copy costs its issuing thread a few hundred
// cycles, so a single issuing lane would cap the stage rate well below HBM bandwidth.
template <bool GATEUP, uint32_t BODY>
__device__ void dc_loader(const MoeParams& p, unsigned char* smem, uint32_t groups, uint32_t splits,
                          uint64_t n_items, uint32_t chunk, uint32_t tfmt, volatile uint32_t* abort) {
    using Lay = DcL<BODY>;
    constexpr uint32_t R = Lay::Ring;
    const uint32_t lane = threadIdx.x & 31u;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + Lay::BarOff);
    uint64_t* empty = full + R;
    uint4* hdr = reinterpret_cast<uint4*>(smem + Lay::HdrOff);
    uint32_t* next_item = p.counters + (GATEUP ? 2 : 4);
    const uint32_t mat_off = GATEUP ? 0u : 2u * (p.E + 1u);
    const uint32_t K = GATEUP ? p.H : p.I;
    // the activation image: gate/up in the prefill operand buffer (idle in a decode forward), down
    // in act (converted in place)
    const unsigned char* image = GATEUP ? reinterpret_cast<const unsigned char*>(p.xperm)
                                        : reinterpret_cast<const unsigned char*>(p.act);
    uint32_t g = 0;
    bool ok = true;
    // every lane runs this (warp-uniform result)
    auto acquire = [&](uint32_t slot) -> bool {
        bool got = true;
        if (lane == 0 && g >= R && !dc_wait(empty + slot, ((g / R) - 1u) & 1u, abort)) {
            dc_fail(p.counters + 3, abort);
            got = false;
        }
        return __shfl_sync(0xffffffffu, got ? 1u : 0u, 0) != 0;
    };
    // chunks of neighbouring items (one unit's row groups share the activation rows) while much work
    // is left, single items towards the end so that the CTAs finish together; [c0, c1) is the chunk
    auto claim = [&](uint64_t& c0, uint64_t& c1) {
        uint64_t a = 0;
        uint32_t take = 1;
        if (lane == 0) {
            const uint64_t seen = *reinterpret_cast<volatile uint32_t*>(next_item);
            take = seen < n_items ? (uint32_t)((n_items - seen) / (2ull * gridDim.x)) : 1u;
            take = take < 1u ? 1u : (take > chunk ? chunk : take);
            a = atomicAdd(next_item, take);
        }
        c0 = __shfl_sync(0xffffffffu, (unsigned long long)a, 0);
        take = __shfl_sync(0xffffffffu, take, 0);
        c1 = c0 < n_items ? (c0 + take < n_items ? c0 + take : n_items) : c0;
    };
    // an item's scalars, loaded one item ahead so that their latency hides behind the stages issued
    // meanwhile: its unit, storage type and, on lane 12 + 2 t + piece, token t's image row and
    // (piece 0) the row's max-bits word
    struct Pre {
        Unit u;
        uint32_t type;
        uint32_t row, maxbits;
    };
    const uint32_t xt = (lane - 12u) >> 1, xpiece = (lane - 12u) & 1u;
    auto fetch = [&](uint64_t item) -> Pre {
        Pre f;
        f.u = p.units[(uint32_t)(item / ((uint64_t)groups * splits))];
        f.type = p.mats[mat_off + f.u.expert].type;
        f.row = 0;
        f.maxbits = 0;
        if (lane >= 12u && lane < 12u + 2u * kUnitTokens && xt < f.u.count) {
            const uint32_t pair = f.u.pair_begin + xt;
            f.row = GATEUP ? p.pair_token[pair] : pair;
            if (!xpiece) f.maxbits = GATEUP ? p.xmax[f.row] : p.act_max[pair];
        }
        return f;
    };
    uint64_t c0 = 0, c1 = 0;
    claim(c0, c1);
    uint64_t n0 = 0, n1 = 0;  // the next chunk, claimed while the current one's last item is issued
    bool have_next = false;
    uint64_t item = c0;
    Pre cur{};
    if (item < c1) cur = fetch(item);
    while (ok && item < c1) {
        // the next item: in this chunk, else the first of the next chunk (claimed now)
        uint64_t nitem = item + 1;
        if (nitem >= c1) {
            claim(n0, n1);
            have_next = n0 < n1;
            nitem = n0;
        }
        Pre nxt{};
        if (nitem < n_items && (nitem < c1 || have_next)) nxt = fetch(nitem);
        const Unit u = cur.u;
        const uint32_t t = cur.type;
        if (t == tfmt || t == kTypeQ8_0) {  // else served by the CUDA-core kernels
            const DcItem it = dc_item<GATEUP>(p, (uint32_t)item, u, t, groups, splits);
            const bool xlane = lane >= 12u && lane < 12u + 2u * kUnitTokens && xt < u.count;
            const unsigned char* xrow = xlane ? image + (size_t)cur.row * K * 4u + xpiece * 512u : nullptr;
            const uint4 hmax = make_uint4(__shfl_sync(0xffffffffu, cur.maxbits, 12), __shfl_sync(0xffffffffu, cur.maxbits, 14),
                                          __shfl_sync(0xffffffffu, cur.maxbits, 16), __shfl_sync(0xffffffffu, cur.maxbits, 18));
            const uint32_t bpr = it.m[0]->bpr;
            for (uint32_t st = it.st0; st < it.st1; ++st, ++g) {
                const uint32_t slot = g % R;
                if (!(ok = acquire(slot))) break;
                // Q8_0: blocks 2 st and 2 st + 1 (the second may be past the row end)
                const bool q8 = it.fmt == kTypeQ8_0;
                const bool scaled = it.fmt == kTypeIq2Xxs || it.fmt == kTypeIq3Xxs;
                const uint32_t nblk = q8 ? (2u * st + 1u < bpr ? 2u : 1u) : 1u;
                const uint32_t bb = dc_body_bytes(it.fmt);
                const uint32_t body = nblk * kTileRows * bb;
                const uint32_t dbytes = nblk * kTileRows * 2u;
                const uint32_t sbase = tc::smem_u32(smem + Lay::RingOff + slot * Lay::Stage);
                if (lane == 0) {
                    uint32_t bytes = u.count * 1024u;
#pragma unroll
                    for (uint32_t s = 0; s < kDcSlices; ++s)
                        if (it.valid[s]) bytes += body + dbytes + (scaled ? kDcSc : 0u);
                    hdr[3u * slot] = make_uint4((uint32_t)item, st, it.st1, it.st0);
                    hdr[3u * slot + 1u] = make_uint4(u.count | (it.fmt << 8), u.pair_begin, u.expert, bpr);
                    hdr[3u * slot + 2u] = hmax;
                    tc::mbar_arrive_expect_tx(full + slot, bytes);
                }
                __syncwarp();
                if (lane < 12u) {
                    // lane 3 s + c: slice s, copy c (0 packed weights, 1 block scales, 2 group scales)
                    const uint32_t s = lane / 3u, c = lane % 3u;
                    const DevMat* ms = it.m[0];
                    uint32_t tile = 0;
                    bool valid = false;
#pragma unroll
                    for (uint32_t k = 0; k < kDcSlices; ++k)  // constant indices keep the item in registers
                        if (k == s) {
                            ms = it.m[k];
                            tile = it.tile[k];
                            valid = it.valid[k];
                        }
                    if (valid && (c < 2u || scaled)) {
                        const DevMat& m = *ms;
                        const uint32_t blk = q8 ? 2u * st : st;
                        const size_t at = blk_index(m.bpr, tile * kTileRows, blk);
                        const uint32_t sd = sbase + s * Lay::Slice;
                        if (c == 0) tc::bulk_load(sd, m.body + at * bb, body, full + slot);
                        else if (c == 1) tc::bulk_load(sd + BODY, m.d + at, dbytes, full + slot);
                        else tc::bulk_load(sd + BODY + kDcD, m.scales + at, kDcSc, full + slot);
                    }
                } else if (xlane) {
                    // the 256-column block holding the stage's columns (a Q8_0 stage: a quarter of it)
                    const uint32_t blk = q8 ? st >> 2 : st;
                    tc::bulk_load(sbase + Lay::XsOff + (2u * xt + xpiece) * kDcXsCol, xrow + (size_t)blk * 1024u, 512u,
                                  full + slot);
                }
                __syncwarp();
            }
        }
        if (item + 1 >= c1) {  // move to the chunk claimed above
            if (!have_next) break;
            c0 = n0;
            c1 = n1;
            have_next = false;
        }
        item = nitem;
        cur = nxt;
    }
    if (ok) {  // end marker: a stage with no copies
        const uint32_t slot = g % R;
        if (acquire(slot)) {
            if (lane == 0) {
                hdr[3u * slot] = make_uint4(kDcEnd, 0u, 0u, 0u);
                tc::mbar_arrive(full + slot);
            }
            ++g;
        }
    }
    // no bulk copy may still be landing in shared memory when the CTA exits
    if (lane == 0)
        for (uint32_t j = g > R ? g - R : 0u; j < g; ++j)
            if (!dc_wait(full + j % R, (j / R) & 1u, abort)) break;
}

// ---- consumer warps -------------------------------------------------------------------------------
// One output of the gate/up epilogue: act = SwiGLU(gate, up), for DeepSeek V4 with the optional
// clamp and the route weight before the down product (execute_expert, deepseek_v4_graph.cpp:
// 1865-1890, double arithmetic), for OLMoE the float SwiGLU with expf (olmoe_runtime.cpp:1279).
// pw: the pair's route weight (read when the item starts).
__device__ __forceinline__ float dc_act_value(const MoeParams& p, float gv, float uv, bool shared, float pw) {
    if (p.weight_after_down) return __fmul_rn(__fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv))), uv);
    const float limit = shared ? p.shared_limit : p.routed_limit;
    double gd = (double)gv, ud = (double)uv;
    if (limit > 0.f) {
        gd = fmin(gd, (double)limit);
        ud = fmin(fmax(ud, -(double)limit), (double)limit);
    }
    double v = gd / (1.0 + exp(-gd)) * ud;
    if (!shared) v *= (double)pw;
    return (float)v;
}

// IQ2_XXS stage: one 256-column block of this warp's two slices (rows rt + gq and rt + gq + 8).
template <uint32_t BODY>
__device__ __forceinline__ void dc_iq2_stage(uint32_t st_addr, uint32_t s0, uint32_t s1, uint32_t rt,
                                             uint32_t gq, uint32_t q, uint32_t xrow, uint32_t tab_lane,
                                             float (&acc)[2][4]) {
    uint4 ra[2], rb[2];
    float da[2], db[2];
    uint32_t sa[2], sb[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const uint32_t sl = st_addr + (i ? s1 : s0) * DcL<BODY>::Slice;
        const uint32_t ba = sl + (rt + gq) * 64u + 16u * q, bb = ba + 8u * 64u;
        asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(ra[i].x), "=r"(ra[i].y), "=r"(ra[i].z), "=r"(ra[i].w) : "r"(ba));
        asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(rb[i].x), "=r"(rb[i].y), "=r"(rb[i].z), "=r"(rb[i].w) : "r"(bb));
        unsigned short ha, hb;
        asm volatile("ld.shared.u16 %0, [%1];" : "=h"(ha) : "r"(sl + BODY + (rt + gq) * 2u));
        asm volatile("ld.shared.u16 %0, [%1];" : "=h"(hb) : "r"(sl + BODY + (rt + gq + 8u) * 2u));
        da[i] = h2f(ha);
        db[i] = h2f(hb);
        uint32_t wa, wb;
        asm volatile("ld.shared.u32 %0, [%1];" : "=r"(wa) : "r"(sl + BODY + kDcD + (rt + gq) * 4u));
        asm volatile("ld.shared.u32 %0, [%1];" : "=r"(wb) : "r"(sl + BODY + kDcD + (rt + gq + 8u) * 4u));
        sa[i] = wa >> (8u * q);  // this lane's groups 2q, 2q + 1 in the low byte
        sb[i] = wb >> (8u * q);
    }
    float D[2][4] = {}, E[2][4] = {};
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        uint32_t kka[2], kkb[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            kka[i] = mma::group_scale_h2((sa[i] >> (4 * half)) & 15u);
            kkb[i] = mma::group_scale_h2((sb[i] >> (4 * half)) & 15u);
        }
#pragma unroll
        for (int sub = 0; sub < 4; ++sub) {
            uint4 xb;
            asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                         : "=r"(xb.x), "=r"(xb.y), "=r"(xb.z), "=r"(xb.w)
                         : "r"(xrow + (uint32_t)(4 * half + sub) * 64u));
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                uint32_t va[4], vb[4];
                mma::decode_iq2_sub_lane(tab_lane, half ? ra[i].z : ra[i].x, half ? ra[i].w : ra[i].y,
                                         (uint32_t)sub, kka[i], va);
                mma::decode_iq2_sub_lane(tab_lane, half ? rb[i].z : rb[i].x, half ? rb[i].w : rb[i].y,
                                         (uint32_t)sub, kkb[i], vb);
                float (&A)[4] = (sub & 1) ? E[i] : D[i];
                mma::mma16816(A, va[0], vb[0], va[1], vb[1], xb.x, xb.y);
                mma::mma16816(A, va[2], vb[2], va[3], vb[3], xb.z, xb.w);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        acc[i][0] = fmaf(da[i], D[i][0] + E[i][0], acc[i][0]);
        acc[i][1] = fmaf(da[i], D[i][1] + E[i][1], acc[i][1]);
        acc[i][2] = fmaf(db[i], D[i][2] + E[i][2], acc[i][2]);
        acc[i][3] = fmaf(db[i], D[i][3] + E[i][3], acc[i][3]);
    }
}

// Q8_0 stage: 32-column blocks 2 st and 2 st + 1 (nblk of them) of the warp's two slices.
template <uint32_t BODY>
// xq: this lane's activations in the stage: column n's record holds chunk 4 j + q of the stage's
// 64 columns at position 4 (4 j + q) + (stage % 4), i.e. xq + 256 j.
__device__ __forceinline__ void dc_q8_stage(uint32_t st_addr, uint32_t s0, uint32_t s1, uint32_t rt, uint32_t gq,
                                            uint32_t q, uint32_t xq, uint32_t nblk, float (&acc)[2][4]) {
    uint2 qa[2][2], qb[2][2];
    float da[2][2], db[2][2];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const uint32_t sl = st_addr + (i ? s1 : s0) * DcL<BODY>::Slice;
            const uint32_t ba = sl + j * (kTileRows * 32u) + (rt + gq) * 32u + 8u * q, bb = ba + 8u * 32u;
            asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(qa[i][j].x), "=r"(qa[i][j].y) : "r"(ba));
            asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(qb[i][j].x), "=r"(qb[i][j].y) : "r"(bb));
            unsigned short ha, hb;
            asm volatile("ld.shared.u16 %0, [%1];" : "=h"(ha) : "r"(sl + BODY + j * (kTileRows * 2u) + (rt + gq) * 2u));
            asm volatile("ld.shared.u16 %0, [%1];"
                         : "=h"(hb)
                         : "r"(sl + BODY + j * (kTileRows * 2u) + (rt + gq + 8u) * 2u));
            da[i][j] = h2f(ha);
            db[i][j] = h2f(hb);
        }
#pragma unroll
    for (uint32_t j = 0; j < 2; ++j) {
        if (j >= nblk) break;
        uint4 xv;
        asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(xv.x), "=r"(xv.y), "=r"(xv.z), "=r"(xv.w)
                     : "r"(xq + j * 256u));
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            uint32_t va[4], vb[4];
            mma::decode_q8_sub(qa[i][j].x, qa[i][j].y, va);
            mma::decode_q8_sub(qb[i][j].x, qb[i][j].y, vb);
            float D[4] = {0.f, 0.f, 0.f, 0.f};
            mma::mma16816(D, va[0], vb[0], va[1], vb[1], xv.x, xv.y);
            mma::mma16816(D, va[2], vb[2], va[3], vb[3], xv.z, xv.w);
            acc[i][0] = fmaf(da[i][j], D[0], acc[i][0]);
            acc[i][1] = fmaf(da[i][j], D[1], acc[i][1]);
            acc[i][2] = fmaf(db[i][j], D[2], acc[i][2]);
            acc[i][3] = fmaf(db[i][j], D[3], acc[i][3]);
        }
    }
}

// IQ1_S stage: one 256-column block (48 bytes a row: 32 qs bytes, 8 qh words) of this warp's two
// slices. Lane q owns groups 2q and 2q + 1 as for IQ2_XXS; the fp16 block scale d is applied per
// block on the accumulators.
template <uint32_t BODY>
__device__ __forceinline__ void dc_iq1_stage(uint32_t st_addr, uint32_t s0, uint32_t s1, uint32_t rt,
                                             uint32_t gq, uint32_t q, uint32_t xrow, uint32_t tab,
                                             float (&acc)[2][4]) {
    uint2 qa[2], qb[2];
    uint32_t ha[2], hb[2];
    float da[2], db[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const uint32_t sl = st_addr + (i ? s1 : s0) * DcL<BODY>::Slice;
        const uint32_t ba = sl + (rt + gq) * 48u, bb = ba + 8u * 48u;
        asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(qa[i].x), "=r"(qa[i].y) : "r"(ba + 8u * q));
        asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(qb[i].x), "=r"(qb[i].y) : "r"(bb + 8u * q));
        asm volatile("ld.shared.u32 %0, [%1];" : "=r"(ha[i]) : "r"(ba + 32u + 4u * q));
        asm volatile("ld.shared.u32 %0, [%1];" : "=r"(hb[i]) : "r"(bb + 32u + 4u * q));
        unsigned short xa, xb;
        asm volatile("ld.shared.u16 %0, [%1];" : "=h"(xa) : "r"(sl + BODY + (rt + gq) * 2u));
        asm volatile("ld.shared.u16 %0, [%1];" : "=h"(xb) : "r"(sl + BODY + (rt + gq + 8u) * 2u));
        da[i] = h2f(xa);
        db[i] = h2f(xb);
    }
    float D[2][4] = {}, E[2][4] = {};
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        uint32_t kka[2], dka[2], kkb[2], dkb[2], hga[2], hgb[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            hga[i] = (ha[i] >> (16 * half)) & 0xffffu;
            hgb[i] = (hb[i] >> (16 * half)) & 0xffffu;
            mma::iq1_group_factors(hga[i], kka[i], dka[i]);
            mma::iq1_group_factors(hgb[i], kkb[i], dkb[i]);
        }
#pragma unroll
        for (int sub = 0; sub < 4; ++sub) {
            uint4 xv;
            asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                         : "=r"(xv.x), "=r"(xv.y), "=r"(xv.z), "=r"(xv.w)
                         : "r"(xrow + (uint32_t)(4 * half + sub) * 64u));
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                uint32_t va[4], vb[4];
                mma::decode_iq1_sub(tab, half ? qa[i].y : qa[i].x, hga[i], (uint32_t)sub, kka[i], dka[i], va);
                mma::decode_iq1_sub(tab, half ? qb[i].y : qb[i].x, hgb[i], (uint32_t)sub, kkb[i], dkb[i], vb);
                float (&A)[4] = (sub & 1) ? E[i] : D[i];
                mma::mma16816(A, va[0], vb[0], va[1], vb[1], xv.x, xv.y);
                mma::mma16816(A, va[2], vb[2], va[3], vb[3], xv.z, xv.w);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        acc[i][0] = fmaf(da[i], D[i][0] + E[i][0], acc[i][0]);
        acc[i][1] = fmaf(da[i], D[i][1] + E[i][1], acc[i][1]);
        acc[i][2] = fmaf(db[i], D[i][2] + E[i][2], acc[i][2]);
        acc[i][3] = fmaf(db[i], D[i][3] + E[i][3], acc[i][3]);
    }
}

// IQ3_XXS stage: one 256-column block (96 bytes a row: 64 grid-index bytes, 8 pair-layout sign
// words; group scales in the stage's scale words) of this warp's two slices.
template <uint32_t BODY>
__device__ __forceinline__ void dc_iq3_stage(uint32_t st_addr, uint32_t s0, uint32_t s1, uint32_t rt,
                                             uint32_t gq, uint32_t q, uint32_t xrow, uint32_t tab_lane,
                                             float (&acc)[2][4]) {
    uint4 ia[2], ib[2];
    uint2 wa[2], wb[2];
    uint32_t sca[2], scb[2];
    float da[2], db[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const uint32_t sl = st_addr + (i ? s1 : s0) * DcL<BODY>::Slice;
        const uint32_t ba = sl + (rt + gq) * 96u, bb = ba + 8u * 96u;
        asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(ia[i].x), "=r"(ia[i].y), "=r"(ia[i].z), "=r"(ia[i].w) : "r"(ba + 16u * q));
        asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(ib[i].x), "=r"(ib[i].y), "=r"(ib[i].z), "=r"(ib[i].w) : "r"(bb + 16u * q));
        asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(wa[i].x), "=r"(wa[i].y) : "r"(ba + 64u + 8u * q));
        asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(wb[i].x), "=r"(wb[i].y) : "r"(bb + 64u + 8u * q));
        unsigned short xa, xb;
        asm volatile("ld.shared.u16 %0, [%1];" : "=h"(xa) : "r"(sl + BODY + (rt + gq) * 2u));
        asm volatile("ld.shared.u16 %0, [%1];" : "=h"(xb) : "r"(sl + BODY + (rt + gq + 8u) * 2u));
        da[i] = h2f(xa);
        db[i] = h2f(xb);
        uint32_t ta, tb;
        asm volatile("ld.shared.u32 %0, [%1];" : "=r"(ta) : "r"(sl + BODY + kDcD + (rt + gq) * 4u));
        asm volatile("ld.shared.u32 %0, [%1];" : "=r"(tb) : "r"(sl + BODY + kDcD + (rt + gq + 8u) * 4u));
        sca[i] = ta >> (8u * q);  // this lane's groups 2q, 2q + 1 in the low byte
        scb[i] = tb >> (8u * q);
    }
    float D[2][4] = {}, E[2][4] = {};
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        uint32_t kka[2], kkb[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            kka[i] = mma::iq3_group_scale_h2((sca[i] >> (4 * half)) & 15u);
            kkb[i] = mma::iq3_group_scale_h2((scb[i] >> (4 * half)) & 15u);
        }
#pragma unroll
        for (int sub = 0; sub < 4; ++sub) {
            uint4 xv;
            asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                         : "=r"(xv.x), "=r"(xv.y), "=r"(xv.z), "=r"(xv.w)
                         : "r"(xrow + (uint32_t)(4 * half + sub) * 64u));
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                // the group's index words: (x, y) for group 2q, (z, w) for 2q + 1; sub-blocks 0-1
                // in the first word, 2-3 in the second
                const uint32_t wla = half ? (sub < 2 ? ia[i].z : ia[i].w) : (sub < 2 ? ia[i].x : ia[i].y);
                const uint32_t wlb = half ? (sub < 2 ? ib[i].z : ib[i].w) : (sub < 2 ? ib[i].x : ib[i].y);
                uint32_t va[4], vb[4];
                mma::decode_iq3_sub(tab_lane, wla, half ? wa[i].y : wa[i].x, (uint32_t)sub, kka[i], va);
                mma::decode_iq3_sub(tab_lane, wlb, half ? wb[i].y : wb[i].x, (uint32_t)sub, kkb[i], vb);
                float (&A)[4] = (sub & 1) ? E[i] : D[i];
                mma::mma16816(A, va[0], vb[0], va[1], vb[1], xv.x, xv.y);
                mma::mma16816(A, va[2], vb[2], va[3], vb[3], xv.z, xv.w);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        acc[i][0] = fmaf(da[i], D[i][0] + E[i][0], acc[i][0]);
        acc[i][1] = fmaf(da[i], D[i][1] + E[i][1], acc[i][1]);
        acc[i][2] = fmaf(db[i], D[i][2] + E[i][2], acc[i][2]);
        acc[i][3] = fmaf(db[i], D[i][3] + E[i][3], acc[i][3]);
    }
}

// K-split join. Every split of a row group writes its warp's partial sums (8 floats a lane) to the
// layer's split scratch and counts itself in on the (row group, warp) counter; the warp that
// arrives last adds the splits' partials in split order (the same sum whatever CTA ran which
// split) and runs the epilogue, and resets the counter. Returns true for that last warp, with acc
// holding the full sums.
__device__ __noinline__ bool dc_join_splits(const MoeParams& p, uint32_t item, uint32_t splits, uint32_t warp,
                                               uint32_t lane, float (&acc)[2][4]) {
    const uint32_t rg = item / splits;
    float4* part = reinterpret_cast<float4*>(p.split_part);
    const size_t mine = (((size_t)item * kDcConsumerWarps + warp) * 32u + lane) * 2u;
    __stcg(part + mine, make_float4(acc[0][0], acc[0][1], acc[0][2], acc[0][3]));
    __stcg(part + mine + 1, make_float4(acc[1][0], acc[1][1], acc[1][2], acc[1][3]));
    __threadfence();
    __syncwarp();
    uint32_t old = 0;
    if (lane == 0) old = atomicAdd(p.split_cnt + (size_t)rg * kDcConsumerWarps + warp, 1u);
    old = __shfl_sync(0xffffffffu, old, 0);
    if (old + 1u != splits) return false;
    // every split has arrived: the counter goes back to zero for the next kernel (gate/up and down
    // use the same counters, one after the other)
    if (lane == 0) p.split_cnt[(size_t)rg * kDcConsumerWarps + warp] = 0u;
    __threadfence();
#pragma unroll
    for (int i = 0; i < 2; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
    for (uint32_t sp = 0; sp < splits; ++sp) {
        const size_t at = ((((size_t)rg * splits + sp) * kDcConsumerWarps + warp) * 32u + lane) * 2u;
        const float4 a = __ldcg(part + at), b = __ldcg(part + at + 1);
        acc[0][0] += a.x; acc[0][1] += a.y; acc[0][2] += a.z; acc[0][3] += a.w;
        acc[1][0] += b.x; acc[1][1] += b.y; acc[1][2] += b.z; acc[1][3] += b.w;
    }
    return true;
}

// TFMT: the IQ storage type whose codebook the CTA holds (IQ2_XXS, IQ1_S or IQ3_XXS); items of
// that type and of Q8_0 run here, any other type on the CUDA-core kernels. One instance per type
// keeps each instance's register allocation to its own decoder.
template <bool GATEUP, uint32_t BODY, uint32_t TFMT>
__global__ void __launch_bounds__(kDcThreads, 1) decode_experts_kernel(const __grid_constant__ MoeParams p,
                                                                       uint32_t chunk, uint32_t splits) {
    constexpr uint32_t tfmt = TFMT;
    using Lay = DcL<BODY>;
    constexpr uint32_t R = Lay::Ring;
    extern __shared__ __align__(1024) unsigned char smem[];
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    volatile uint32_t* abort = reinterpret_cast<volatile uint32_t*>(smem + Lay::MiscOff);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + Lay::BarOff);
    uint64_t* empty = full + R;
    if constexpr (TFMT == kTypeIq2Xxs) mma::build_iq2_table(reinterpret_cast<uint4*>(smem), p.grids.iq2xxs);
    if constexpr (TFMT == kTypeIq1S) mma::build_iq1s_table(reinterpret_cast<uint4*>(smem), p.grids.iq1s);
    if constexpr (TFMT == kTypeIq3Xxs) mma::build_iq3_table(reinterpret_cast<uint2*>(smem), p.grids.iq3xxs);
    if (threadIdx.x == 0) {
        for (uint32_t s = 0; s < R; ++s) {
            tc::mbar_init(full + s, 1);
            tc::mbar_init(empty + s, kDcConsumerWarps);
        }
        *abort = 0u;
        tc::mbar_fence_init();
    }
    __syncthreads();
    const uint32_t rows = GATEUP ? p.I : p.H;
    const uint32_t groups = (rows + (GATEUP ? 255u : 511u)) / (GATEUP ? 256u : 512u);
    const uint64_t n_items = (uint64_t)p.counters[0] * groups * splits;
    if (warp == kDcConsumerWarps) {
        dc_loader<GATEUP, BODY>(p, smem, groups, splits, n_items, chunk, tfmt, abort);
        return;
    }
    // consumer warp: 16 rows of slices (w / 8) and (2 + w / 8)
    const uint32_t s0 = warp >> 3, s1 = 2u + (warp >> 3), rt = (warp & 7u) * 16u;
    const uint32_t gq = lane >> 2, q = lane & 3u, n = lane >> 2, lane7 = lane & 7u;
    const uint4* hdr = reinterpret_cast<const uint4*>(smem + Lay::HdrOff);
    // this lane's activation column n in a stage: its chunk q (256-column formats), or 64 q bytes
    // further on for Q8_0
    const uint32_t xs_lane = Lay::XsOff + n * kDcXsCol + q * 16u;
    const uint32_t xs_lane_q8 = Lay::XsOff + n * kDcXsCol + q * 64u;
    const uint32_t tab = tc::smem_u32(smem);
    const uint32_t tab_lane = tab + (tfmt == kTypeIq3Xxs ? (lane & 15u) * 8u : lane7 * 16u);  // this lane's replica
    float acc[2][4] = {};
    DcWarpItem it{};
    Unit u{};
    float pw = 1.f;        // the pair's route weight (gate/up epilogue)
    float inv = 1.f;       // 1 / the power-of-two prescale of the pair's activations
    uint32_t out_row = 0;  // the pair's token (down epilogue writing out directly)
    for (uint32_t g = 0;; ++g) {
        const uint32_t slot = g % R;
        const bool ok = dc_wait(full + slot, (g / R) & 1u, abort);
        if (!__all_sync(0xffffffffu, ok)) {
            if (lane == 0) dc_fail(p.counters + 3, abort);
            break;
        }
        const uint4 h = hdr[3u * slot];
        if (h.x == kDcEnd) break;
        if (h.y == h.w) {  // first stage of an item
            const uint4 h2 = hdr[3u * slot + 1u];
            const uint4 hmax = hdr[3u * slot + 2u];
            it = dc_warp_item<GATEUP>(p, h.x, h2, groups, splits, s0, s1);
            u.count = h2.x & 0xffu;
            u.pair_begin = h2.y;
            u.expert = h2.z;
            // the epilogue's per-pair scalars, loaded now so that their latency hides behind the item
            if (q < u.count) {
                const uint32_t pair = u.pair_begin + q;
                inv = 1.f / mma::prescale_for(__uint_as_float(q == 0u ? hmax.x : q == 1u ? hmax.y : q == 2u ? hmax.z
                                                                                                      : hmax.w));  // exact
                if (GATEUP) pw = (u.expert != p.E && !p.weight_after_down) ? p.pair_weight[pair] : 1.f;
                else if (p.direct_out) out_row = p.pair_token[pair];
            }
#pragma unroll
            for (int i = 0; i < 2; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
        }
        const uint32_t st_addr = tc::smem_u32(smem + Lay::RingOff + slot * Lay::Stage);
        if (it.fmt != kTypeQ8_0) {  // the CTA's IQ type (the loader sends no other)
            if constexpr (TFMT == kTypeIq2Xxs)
                dc_iq2_stage<BODY>(st_addr, s0, s1, rt, gq, q, st_addr + xs_lane, tab_lane, acc);
            if constexpr (TFMT == kTypeIq1S)
                dc_iq1_stage<BODY>(st_addr, s0, s1, rt, gq, q, st_addr + xs_lane, tab, acc);
            if constexpr (TFMT == kTypeIq3Xxs)
                dc_iq3_stage<BODY>(st_addr, s0, s1, rt, gq, q, st_addr + xs_lane, tab_lane, acc);
        } else {
            const uint32_t nblk = 2u * h.y + 1u < it.bpr ? 2u : 1u;
            dc_q8_stage<BODY>(st_addr, s0, s1, rt, gq, q, st_addr + xs_lane_q8 + (h.y & 3u) * 16u, nblk, acc);
        }
        // the slot goes back to the loader once this warp's loads of it (weights and activations)
        // have completed: the MMAs that consume them have issued
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(empty + slot);
        if (h.y + 1u == h.z) {  // last stage of the item
            if (splits > 1u && !dc_join_splits(p, h.x, splits, warp, lane, acc)) continue;
            // this warp's rows are complete
            if (q < u.count) {
                const uint32_t pair = u.pair_begin + q;
                if (GATEUP) {
                    const bool shared = u.expert == p.E;
                    const uint32_t row_base = it.tile0 * kTileRows + rt + gq;
#pragma unroll
                    for (int hi = 0; hi < 2; ++hi) {  // fragment row gq / gq + 8
                        const uint32_t row = row_base + 8u * hi;
                        if (!it.valid0 || row >= p.I) continue;
                        const float gv = (acc[0][2 * hi] + acc[0][2 * hi + 1]) * inv;
                        const float uv = (acc[1][2 * hi] + acc[1][2 * hi + 1]) * inv;
                        const float a = dc_act_value(p, gv, uv, shared, pw);
                        p.act[(size_t)pair * p.I + row] = a;
                        atomicMax(p.act_max + pair, __float_as_uint(fabsf(a)));
                    }
                } else {
                    float* yrow = p.direct_out ? p.out + (size_t)out_row * p.H : p.y + (size_t)pair * p.H;
#pragma unroll
                    for (int i = 0; i < 2; ++i) {
                        if (!(i ? it.valid1 : it.valid0)) continue;
#pragma unroll
                        for (int hi = 0; hi < 2; ++hi) {
                            const uint32_t row = (i ? it.tile1 : it.tile0) * kTileRows + rt + gq + 8u * hi;
                            if (row < p.H) yrow[row] = (acc[i][2 * hi] + acc[i][2 * hi + 1]) * inv;
                        }
                    }
                }
            }
        }
    }
}

// The phase's IQ type and its stage carve: IQ2_XXS, else IQ1_S, else IQ3_XXS (0: Q8_0 only); a
// carve that does not fit the device's shared memory for this K leaves the IQ type to the
// CUDA-core kernels.
struct DcChoice {
    uint32_t tfmt;
    bool large;
    size_t smem;
};

static int g_optin_smem = 0;

static DcChoice dc_choice(const MoeParams& p, bool gateup) {
    const uint32_t mask = gateup ? p.fmt_gu : p.fmt_dn;
    const uint32_t K = gateup ? p.H : p.I;
    DcChoice c{0u, false, 0};
    if (mask & fmt_bit(kTypeIq2Xxs)) c.tfmt = kTypeIq2Xxs;
    else if (mask & fmt_bit(kTypeIq1S)) c.tfmt = kTypeIq1S;
    else if (mask & fmt_bit(kTypeIq3Xxs)) c.tfmt = kTypeIq3Xxs;
    c.large = c.tfmt == kTypeIq3Xxs;
    c.smem = c.large ? DcL<kDcBodyLarge>::End : DcL<kDcBodySmall>::End;
    if (g_optin_smem == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_optin_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    }
    if (c.large && c.smem > (size_t)g_optin_smem) {  // IQ3_XXS does not fit: CUDA cores take it
        c.tfmt = 0;
        c.large = false;
        c.smem = DcL<kDcBodySmall>::End;
    }
    return c;
}

template <bool GATEUP, uint32_t BODY, uint32_t TFMT>
cudaError_t launch_decode_carve(const MoeParams& p, unsigned n_sms, size_t smem, cudaStream_t s) {
    static std::mutex mu;
    static std::vector<size_t> configured;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (configured.size() <= (size_t)dev) configured.resize((size_t)dev + 1, 0);
        if (configured[(size_t)dev] < smem) {
            int optin = 0;
            if ((e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess)
                return e;
            if (smem > (size_t)optin) return cudaErrorInvalidValue;  // hidden size beyond this kernel's staging
            if ((e = cudaFuncSetAttribute(decode_experts_kernel<GATEUP, BODY, TFMT>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)) != cudaSuccess)
                return e;
            configured[(size_t)dev] = smem;
        }
    }
    const uint32_t K = GATEUP ? p.H : p.I;
    // items ~ units x row groups; the host does not know the unit count (it is on the device), so
    // the chunk follows the worst case of one unit per routed pair plus the shared expert's units
    const uint32_t rows = GATEUP ? p.I : p.H;
    const uint32_t groups = (rows + (GATEUP ? 255u : 511u)) / (GATEUP ? 256u : 512u);
    const uint64_t est = (uint64_t)(p.T * p.k < p.E ? p.T * p.k : p.E) * groups;
    // Small batches have fewer (unit, row group) items than SMs: split K so that about two items
    // reach every SM. The unit count is bounded by one per routed pair plus the shared expert's.
    const uint64_t max_items = ((uint64_t)p.T * p.k + (p.has_shared ? (p.T + kUnitTokens - 1u) / kUnitTokens : 0u)) *
                               groups;
    const uint32_t min_stages = K / 256u;  // a 256-column format's K-chunks (Q8_0 has more)
    uint32_t splits = 1;
    if (p.split_part && max_items < 2ull * n_sms) {
        splits = (uint32_t)((2ull * n_sms + max_items - 1) / max_items);
        if (splits > kDcMaxSplits) splits = kDcMaxSplits;
        if (splits > min_stages) splits = min_stages;
        while (splits > 1u && max_items * splits > p.split_items) --splits;
        if (splits < 1u) splits = 1;
    }
    uint32_t chunk = (uint32_t)((est * splits + 4ull * n_sms - 1) / (4ull * n_sms));
    chunk = chunk < 1u ? 1u : (chunk > kDcMaxChunk ? kDcMaxChunk : chunk);
    decode_experts_kernel<GATEUP, BODY, TFMT><<<n_sms, kDcThreads, smem, s>>>(p, chunk, splits);
    return cudaGetLastError();
}

// The phase's activation image (dc_image_kernel): gate/up converts the T token rows into the
// prefill operand buffer, down converts the pairs' act rows in place (after every reader of act
// as f32: the CUDA-core kernels of the phase run before).
// One record of the image kernel's shared-memory limit per device (both phases launch it): it
// only ever grows.
static std::mutex g_image_mu;
static std::vector<size_t> g_image_smem;

template <bool GATEUP>
cudaError_t launch_decode_image(const MoeParams& p, cudaStream_t s) {
    const uint32_t K = GATEUP ? p.H : p.I;
    const uint32_t rows = GATEUP ? p.T : p.T * p.k + (p.has_shared ? p.T : 0u);
    if (rows == 0) return cudaSuccess;
    const size_t smem = (size_t)K * sizeof(float);
    std::mutex& mu = g_image_mu;
    std::vector<size_t>& configured = g_image_smem;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (configured.size() <= (size_t)dev) configured.resize((size_t)dev + 1, 0);
        if (configured[(size_t)dev] < smem) {
            if ((e = cudaFuncSetAttribute(dc_image_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem)) !=
                cudaSuccess)
                return e;
            configured[(size_t)dev] = smem;
        }
    }
    dc_image_kernel<<<rows, 256, smem, s>>>(GATEUP ? p.x : p.act, K, GATEUP ? p.xmax : p.act_max,
                                            GATEUP ? reinterpret_cast<unsigned char*>(p.xperm)
                                                   : reinterpret_cast<unsigned char*>(p.act));
    return cudaGetLastError();
}

template <bool GATEUP>
cudaError_t launch_decode(const MoeParams& p, unsigned n_sms, cudaStream_t s) {
    cudaError_t e = launch_decode_image<GATEUP>(p, s);
    if (e != cudaSuccess) return e;
    const DcChoice c = dc_choice(p, GATEUP);
    if (c.tfmt == kTypeIq3Xxs) return launch_decode_carve<GATEUP, kDcBodyLarge, kTypeIq3Xxs>(p, n_sms, c.smem, s);
    if (c.tfmt == kTypeIq1S) return launch_decode_carve<GATEUP, kDcBodySmall, kTypeIq1S>(p, n_sms, c.smem, s);
    // IQ2_XXS, or Q8_0 alone (the IQ2_XXS instance builds no table without its codebook in use)
    return launch_decode_carve<GATEUP, kDcBodySmall, kTypeIq2Xxs>(p, n_sms, c.smem, s);
}

}  // namespace

cudaError_t launch_decode_gateup(const MoeParams& p, unsigned n_sms, cudaStream_t s) {
    return launch_decode<true>(p, n_sms, s);
}

cudaError_t launch_decode_down(const MoeParams& p, unsigned n_sms, cudaStream_t s) {
    return launch_decode<false>(p, n_sms, s);
}

uint32_t decode_ring_types(const MoeParams& p, bool gateup) {
    const DcChoice c = dc_choice(p, gateup);
    return fmt_bit(kTypeQ8_0) | (c.tfmt ? fmt_bit(c.tfmt) : 0u);
}

}  // namespace vlb
