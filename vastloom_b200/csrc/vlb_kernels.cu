// sm_100a kernels of the MoE routed-expert decode path, and their launchers.
//
//   dequant_kernel    bit-exact block decode (reference decode_*_block)
//   gemv_kernel       multi-token dequant-matvec over one resident matrix (the operator seam)
//   router_kernel     router projection (sequential f64 sums, bit-exact) + score function
//   route_kernel      warp-per-token top-k (ties to the lower id) and route weights
//   dispatch_kernel   stable counting sort of (token, slot) pairs by expert, work units
//                     (dispatch_count / scatter / finish for large batches)
//   expert_kernel     CUDA-core expert products for the IQ3_XXS / IQ1_S experts (bit-exact decode)
//   combine_kernel    per-token deterministic combine in the reference's order + shared expert
//   launch_moe        the whole layer: routing, dispatch, expert products (decode kernels in
//                     vlb_decode.cu or the tcgen05 prefill GEMMs in vlb_prefill.cu), combine
#include <cuda_runtime.h>

#include <cstdlib>
#include <mutex>
#include <utility>
#include <vector>

#include "vlb_gemv.cuh"
#include "vlb_launch.h"
#include "vlb_mma.cuh"
#include "vlb_tcgen05.cuh"

namespace vlb {

constexpr uint32_t kGridSmemBytes = 2048u * 8u + 256u * 8u + 256u * 4u + 1024u * 8u;  // 27,648

// Copies the codebooks of the storage types in `need` (fmt_bit set) into shared memory.
__device__ __forceinline__ GridSmem stage_grids(const Grids& g, unsigned char* smem, uint32_t need = ~0u) {
    uint64_t* s1 = reinterpret_cast<uint64_t*>(smem);
    uint64_t* s2 = s1 + 2048;
    uint32_t* s3 = reinterpret_cast<uint32_t*>(s2 + 256);
    uint64_t* s4 = reinterpret_cast<uint64_t*>(s3 + 256);
    if (g.iq2s && (need & fmt_bit(kTypeIq2S)))
        for (uint32_t i = threadIdx.x; i < 1024u; i += blockDim.x) s4[i] = g.iq2s[i];
    if (g.iq1s && (need & fmt_bit(kTypeIq1S)))
        for (uint32_t i = threadIdx.x; i < 2048u; i += blockDim.x) s1[i] = g.iq1s[i];
    if (g.iq2xxs && (need & fmt_bit(kTypeIq2Xxs)))
        for (uint32_t i = threadIdx.x; i < 256u; i += blockDim.x) s2[i] = g.iq2xxs[i];
    if (g.iq3xxs && (need & fmt_bit(kTypeIq3Xxs)))
        for (uint32_t i = threadIdx.x; i < 256u; i += blockDim.x) s3[i] = g.iq3xxs[i];
    return GridSmem{s1, s2, s3, s4};
}

// ---------------------------------------------------------------------------------------------
// dequantize: one thread per 32-weight group
__global__ void dequant_kernel(DevMat m, Grids g, float* __restrict__ out) {
    const uint32_t ngroups = m.cols / 32u;
    const size_t gid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (gid >= (size_t)m.rows * ngroups) return;
    const uint32_t row = (uint32_t)(gid / ngroups), grp = (uint32_t)(gid % ngroups);
    float w[32];
    if (raw_type(m.type)) {
        const uint32_t gpb = raw_groups(m.type), blk = grp / gpb, gg = grp % gpb;
        const uint8_t* pb = m.body + blk_index(m.bpr, row, blk) * raw_slot_bytes(m.type);
        switch (m.type) {
            case kTypeQ4K: raw_decode_group<kTypeQ4K>(pb, gg, g.iq2s, w); break;
            case kTypeQ5K: raw_decode_group<kTypeQ5K>(pb, gg, g.iq2s, w); break;
            case kTypeQ6K: raw_decode_group<kTypeQ6K>(pb, gg, g.iq2s, w); break;
            case kTypeIq2S: raw_decode_group<kTypeIq2S>(pb, gg, g.iq2s, w); break;
            default: raw_decode_group<kTypeMxfp4>(pb, gg, g.iq2s, w); break;
        }
    } else if (m.type == kTypeQ8_0) {
        decode_group_q8_0(h2f(m.d[blk_index(m.bpr, row, grp)]),
                          m.body + blk_index(m.bpr, row, grp) * 32u, w);
    } else {
        const uint32_t blk = grp >> 3, gg = grp & 7u;
        const float d = h2f(m.d[blk_index(m.bpr, row, blk)]);
        if (m.type == kTypeIq2Xxs)
            decode_group_iq2_xxs(d, m.body + blk_index(m.bpr, row, blk) * 64u, gg,
                                 (m.scales[blk_index(m.bpr, row, blk)] >> (4u * gg)) & 15u, g.iq2xxs, w);
        else if (m.type == kTypeIq3Xxs)
            decode_group_iq3_xxs(d, m.body + blk_index(m.bpr, row, blk) * 96u, gg,
                                 (m.scales[blk_index(m.bpr, row, blk)] >> (4u * gg)) & 15u, g.iq3xxs, w);
        else
            decode_group_iq1_s(d, m.body + blk_index(m.bpr, row, blk) * 48u, gg, g.iq1s, w);
    }
    float* o = out + (size_t)row * m.cols + (size_t)grp * 32u;
#pragma unroll
    for (int i = 0; i < 32; i += 4) *reinterpret_cast<float4*>(o + i) = make_float4(w[i], w[i + 1], w[i + 2], w[i + 3]);
}

// ---------------------------------------------------------------------------------------------
// Standalone multi-token GEMV: CTA = 8 warps x gemv_rows(TOKC) rows; tokens in chunks of TOKC. A
// warp's rows share each activation load; few rows per warp keep a single matrix spread over
// every SM (a 4096-row matrix is 256 CTAs at one token).
constexpr int kGemvWarps = 8;
__host__ __device__ constexpr int gemv_rows(int tokc) { return tokc == 1 ? 2 : 4; }

template <uint32_t FMT, int TOKC>
__global__ void __launch_bounds__(256) gemv_kernel(DevMat m, Grids grids, const float* __restrict__ x,
                                                   uint32_t ntok, uint32_t xstride,
                                                   float* __restrict__ y, uint32_t ystride) {
    constexpr int kGemvRows = gemv_rows(TOKC);
    extern __shared__ __align__(16) unsigned char smem[];
    const GridSmem gs = stage_grids(grids, smem, fmt_bit(FMT));
    float* xs = reinterpret_cast<float*>(smem + kGridSmemBytes);
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t row0 = blockIdx.x * (kGemvRows * kGemvWarps) + warp * kGemvRows;
    const uint32_t ngroups = m.cols / 32u;
    const uint32_t rbase = row0 < m.rows ? row0 : 0u;
    for (uint32_t t0 = 0; t0 < ntok; t0 += TOKC) {
        const float* rows[TOKC];
#pragma unroll
        for (int t = 0; t < TOKC; ++t) rows[t] = t0 + t < ntok ? x + (size_t)(t0 + t) * xstride : nullptr;
        __syncthreads();
        stage_x<TOKC>(xs, rows, m.cols);
        __syncthreads();
        if (row0 >= m.rows) continue;
        float acc[kGemvRows][TOKC];
#pragma unroll
        for (int r = 0; r < kGemvRows; ++r)
#pragma unroll
            for (int t = 0; t < TOKC; ++t) acc[r][t] = 0.f;
        if (rbase + kGemvRows <= m.rows) {
            warp_dot<FMT, kGemvRows, 0, TOKC>(m, m, rbase, 0u, xs, ngroups, gs, acc);
        } else {
            // tail: one row at a time
            for (int r = 0; r < kGemvRows; ++r) {
                if (rbase + r >= m.rows) break;
                float a1[1][TOKC];
#pragma unroll
                for (int t = 0; t < TOKC; ++t) a1[0][t] = 0.f;
                warp_dot<FMT, 1, 0, TOKC>(m, m, rbase + r, 0u, xs, ngroups, gs, a1);
#pragma unroll
                for (int t = 0; t < TOKC; ++t) acc[r][t] = a1[0][t];
            }
        }
        warp_reduce<kGemvRows, TOKC>(acc);
#pragma unroll
        for (int r = 0; r < kGemvRows; ++r)
#pragma unroll
            for (int t = 0; t < TOKC; ++t)
                if (lane == (uint32_t)(r * TOKC + t) % 32u && rbase + r < m.rows && t0 + t < ntok)
                    y[(size_t)(t0 + t) * ystride + rbase + r] = acc[r][t];
    }
}

// ---------------------------------------------------------------------------------------------
// Router projection (deepseek_v4_graph.cpp:735-767 `linear`; qwen3_8_flash_next_reference.cpp:311
// `linear_f`): logits[t][e] = f32(sum over columns c = 0, 1, ... of double(x[t][c]) *
// double(w[e][c])), one f64 rounding per added term, in column order. Every product of two f32
// values is exact in f64, so fma(x, w, s) rounds exactly like s + x * w, and a thread that walks
// the columns in order reproduces the reference's logit bit for bit. That order is the whole cost:
// each logit is a chain of H dependent f64 additions, so the kernel is latency-bound (H times the
// 8-cycle DFMA latency) and, with many tokens, by the FP64 pipe (measured on B200: about 8 DFMA
// per clock per SM). It is built to keep every chain fed:
//   * the operands arrive already widened to f64 (the layer keeps its router weights as f64; the
//     activations are widened by the entry step): an f32 -> f64 conversion per use would cost
//     more issue time than the DFMA chain itself;
//   * a CTA computes a tile of 32 experts (the lanes) x 4 warps x kRtChains tokens; 128-column
//     slices of the tile's weights and activations stream into a 4-stage shared-memory ring with
//     cp.async: three slices (about 1.9 us of chain steps) in flight, more than the memory latency,
//     so the chains do not wait for their operands;
//   * warps whose tokens are all past T skip the chain (they only help stage), which leaves the
//     SM's FP64 pipe to the chains that count.
#ifndef VLB_RT_CHAINS
#define VLB_RT_CHAINS 1
#endif
constexpr uint32_t kRtExperts = 32;
constexpr uint32_t kRtWarps = 4;
constexpr uint32_t kRtChains = VLB_RT_CHAINS;          // tokens per warp: independent chains per thread
constexpr uint32_t kRtTokens = kRtWarps * kRtChains;  // tokens per CTA
constexpr uint32_t kRtCols = 128;
constexpr uint32_t kRtStages = 4;
constexpr uint32_t kRtWStride = kRtCols + 2;  // doubles per staged weight row: a 16-byte phase shift per row
constexpr uint32_t kRtThreads = kRtExperts * kRtWarps;
constexpr uint32_t kRtStageDoubles = kRtExperts * kRtWStride + kRtTokens * kRtCols;
constexpr size_t kRtSmemBytes = (size_t)kRtStages * kRtStageDoubles * 8u;

__device__ __forceinline__ float sqrt_softplus_dev(float v) {
    const double p = (double)v;
    const double sp = fmax(p, 0.0) + log1p(exp(-fabs(p)));
    return (float)sqrt(sp);
}
__device__ __forceinline__ float sigmoid_dev(float v) {
    const double p = (double)v;
    if (p >= 0.0) return (float)(1.0 / (1.0 + exp(-p)));
    const double e = exp(p);
    return (float)(e / (1.0 + e));
}
__device__ __forceinline__ float score_dev(int score, float logit) {
    if (score == VLB_SCORE_SIGMOID) return sigmoid_dev(logit);
    if (score == VLB_SCORE_SQRT_SOFTPLUS) return sqrt_softplus_dev(logit);
    return logit;  // the softmax routers work on the logits themselves
}

__device__ __forceinline__ double2 lds_f64x2(uint32_t addr) {
    double2 v;
    asm("ld.shared.v2.f64 {%0, %1}, [%2];" : "=d"(v.x), "=d"(v.y) : "r"(addr));
    return v;
}

// wd: f64 router weights [E x H]; xd: f64 activations [T x H]; H % 2 == 0.
__global__ void __launch_bounds__(kRtThreads) router_kernel(const double* __restrict__ wd,
                                                            const double* __restrict__ xd, uint32_t T,
                                                            uint32_t H, uint32_t E, int score,
                                                            float* __restrict__ logits,
                                                            float* __restrict__ scores) {
    extern __shared__ __align__(16) double ring[];
    const uint32_t lane = threadIdx.x & 31u, warp = threadIdx.x >> 5;
    const uint32_t e0 = blockIdx.x * kRtExperts, t0 = blockIdx.y * kRtTokens;
    const uint32_t slices = (H + kRtCols - 1u) / kRtCols;
    // slice `sl` into stage sl % kRtStages: the weight tile's double2s and the token rows' double2s,
    // spread over the threads; rows past E / T and columns past H are zero-filled
    auto issue = [&](uint32_t sl) {
        double* st = ring + (sl % kRtStages) * kRtStageDoubles;
        const uint32_t c0 = sl * kRtCols;
#pragma unroll
        for (uint32_t i = 0; i < kRtExperts * kRtCols / 2u / kRtThreads; ++i) {
            const uint32_t f = threadIdx.x + i * kRtThreads;
            const uint32_t r = f / (kRtCols / 2u), c = (f % (kRtCols / 2u)) * 2u;
            const bool ok = e0 + r < E && c0 + c < H;
            tc::cp_async16(st + r * kRtWStride + c, ok ? wd + (size_t)(e0 + r) * H + c0 + c : wd, ok ? 16u : 0u);
        }
#pragma unroll
        for (uint32_t i = 0; i < (kRtTokens * kRtCols / 2u + kRtThreads - 1u) / kRtThreads; ++i) {
            const uint32_t f = threadIdx.x + i * kRtThreads;
            if (f >= kRtTokens * kRtCols / 2u) break;
            const uint32_t r = f / (kRtCols / 2u), c = (f % (kRtCols / 2u)) * 2u;
            const bool ok = t0 + r < T && c0 + c < H;
            tc::cp_async16(st + kRtExperts * kRtWStride + r * kRtCols + c, ok ? xd + (size_t)(t0 + r) * H + c0 + c : xd,
                           ok ? 16u : 0u);
        }
    };
    for (uint32_t sl = 0; sl < kRtStages - 1u; ++sl) {
        if (sl < slices) issue(sl);
        tc::cp_async_commit();  // (an empty group past the last slice keeps the count uniform)
    }
    double acc[kRtChains];
#pragma unroll
    for (uint32_t h = 0; h < kRtChains; ++h) acc[h] = 0.0;
    const uint32_t ring_a = tc::smem_u32(ring);
    for (uint32_t sl = 0; sl < slices; ++sl) {
        asm volatile("cp.async.wait_group %0;" ::"n"(kRtStages - 2u) : "memory");  // slice sl has landed
        __syncthreads();  // ... for every thread; and every thread is done with slice sl - 1's stage
        if (sl + kRtStages - 1u < slices) issue(sl + kRtStages - 1u);
        tc::cp_async_commit();
        const uint32_t st = ring_a + (sl % kRtStages) * kRtStageDoubles * 8u;
        const uint32_t wa = st + lane * kRtWStride * 8u;
        const uint32_t xa = st + (kRtExperts * kRtWStride + warp * kRtChains * kRtCols) * 8u;
        const uint32_t n = H - sl * kRtCols;  // even (H % 2 == 0)
        if (t0 + warp * kRtChains >= T) continue;  // no valid token in this warp: keep the FP64 pipe free
        if (n >= kRtCols) {
#pragma unroll
            for (uint32_t c = 0; c < kRtCols; c += 2u) {
                const double2 wv = lds_f64x2(wa + 8u * c);
#pragma unroll
                for (uint32_t h = 0; h < kRtChains; ++h) {
                    const double2 xv = lds_f64x2(xa + 8u * (h * kRtCols + c));
                    acc[h] = __fma_rn(xv.x, wv.x, acc[h]);
                    acc[h] = __fma_rn(xv.y, wv.y, acc[h]);
                }
            }
        } else {
            for (uint32_t c = 0; c < n; c += 2u) {
                const double2 wv = lds_f64x2(wa + 8u * c);
#pragma unroll
                for (uint32_t h = 0; h < kRtChains; ++h) {
                    const double2 xv = lds_f64x2(xa + 8u * (h * kRtCols + c));
                    acc[h] = __fma_rn(xv.x, wv.x, acc[h]);
                    acc[h] = __fma_rn(xv.y, wv.y, acc[h]);
                }
            }
        }
    }
    tc::cp_async_wait_all();
    const uint32_t e = e0 + lane;
#pragma unroll
    for (uint32_t h = 0; h < kRtChains; ++h) {
        const uint32_t t = t0 + warp * kRtChains + h;
        if (e < E && t < T) {
            const float lg = (float)acc[h];
            logits[(size_t)t * E + e] = lg;
            scores[(size_t)t * E + e] = score_dev(score, lg);
        }
    }
}

__global__ void widen_kernel(const float* __restrict__ src, size_t n, double* __restrict__ dst) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        dst[i] = (double)src[i];
}

__global__ void score_kernel(const float* __restrict__ logits, size_t n, int score,
                             float* __restrict__ scores) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) scores[i] = score_dev(score, logits[i]);
}

// ---------------------------------------------------------------------------------------------
// Top-k routing, one warp per token (deepseek_v4_route_learned_logits / _hash_logits,
// deepseek_v4_reference.cpp:223-307; OLMoE softmax router, olmoe_runtime.cpp:1120-1137; Qwen
// router, qwen3_8_flash_next_reference.cpp:1186-1239). Selection key: learned = score + bias (f32
// add), OLMoE softmax = f32 probability, Qwen softmax = f64 probability; larger first, ties to the
// lower expert id (std::partial_sort / std::sort with that strict order). KT is the key type: f32
// for the f32-keyed routers, f64 for the Qwen router (a one-warp selection in f64 costs several
// times the f32 one on this GPU's FP64 pipe). E <= 32 * kMaxPerLane.
constexpr int kMaxPerLane = 16;  // E <= 512

__device__ __forceinline__ bool f64_softmax(int score) {
    return score == VLB_SCORE_SOFTMAX_F64 || score == VLB_SCORE_SOFTMAX_F64_NORM;
}

template <typename KT>
__global__ void __launch_bounds__(256) route_kernel(const float* __restrict__ scores,
                                                    const float* __restrict__ bias,
                                                    const uint32_t* __restrict__ token_ids,
                                                    const uint32_t* __restrict__ tid2eid,
                                                    uint32_t vocab, uint32_t T, uint32_t E,
                                                    uint32_t k, int score, int hash_routing,
                                                    float route_scale, uint32_t* __restrict__ idx,
                                                    float* __restrict__ weights,
                                                    uint32_t* __restrict__ error_flag) {
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    const uint32_t t = blockIdx.x * 8u + warp;
    if (t >= T) return;
    const float* s = scores + (size_t)t * E;
    KT key[kMaxPerLane];
    KT val[kMaxPerLane];
    if (score == VLB_SCORE_SOFTMAX) {
        // p_e = float exp of (logit - max); double denominator; float division (no renorm)
        float mx = -INFINITY;
        for (uint32_t e = lane; e < E; e += 32u) mx = fmaxf(mx, s[e]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        float p[kMaxPerLane];
        double den = 0.0;
#pragma unroll
        for (int i = 0; i < kMaxPerLane; ++i) {
            const uint32_t e = lane + 32u * i;
            p[i] = e < E ? (float)exp((double)__fsub_rn(s[e], mx)) : 0.f;
            den += (double)p[i];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) den += __shfl_xor_sync(0xffffffffu, den, o);
        const float fden = (float)den;
#pragma unroll
        for (int i = 0; i < kMaxPerLane; ++i) {
            val[i] = (KT)__fdiv_rn(p[i], fden);
            key[i] = lane + 32u * i < E ? val[i] : (KT)-INFINITY;
        }
    } else if (f64_softmax(score)) {
        // probs[e] = exp(double(l_e) - max) in double, summed in expert order (the reference's
        // sequential loop: each lane's values join the sum in turn), prob = probs[e] * (1 / sum)
        double mx = -INFINITY;
        for (uint32_t e = lane; e < E; e += 32u) mx = fmax(mx, (double)s[e]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mx = fmax(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        double pv[kMaxPerLane];
#pragma unroll
        for (int i = 0; i < kMaxPerLane; ++i) {
            const uint32_t e = lane + 32u * i;
            pv[i] = e < E ? exp(__dsub_rn((double)s[e], mx)) : 0.0;
        }
        double sum = 0.0;
#pragma unroll
        for (int i = 0; i < kMaxPerLane; ++i) {
            if (32u * (uint32_t)i >= E) break;
            for (uint32_t l = 0; l < 32u && 32u * i + l < E; ++l) sum = __dadd_rn(sum, __shfl_sync(0xffffffffu, pv[i], l));
        }
        const double inv = sum > 0.0 ? 1.0 / sum : 0.0;
#pragma unroll
        for (int i = 0; i < kMaxPerLane; ++i) {
            val[i] = (KT)__dmul_rn(pv[i], inv);
            key[i] = lane + 32u * i < E ? val[i] : (KT)-INFINITY;
        }
    } else {
#pragma unroll
        for (int i = 0; i < kMaxPerLane; ++i) {
            const uint32_t e = lane + 32u * i;
            if (e < E) {
                val[i] = (KT)s[e];
                key[i] = hash_routing ? (KT)0 : (KT)__fadd_rn(s[e], bias ? bias[e] : 0.f);
            } else {
                val[i] = (KT)0;
                key[i] = (KT)-INFINITY;
            }
        }
    }
    // slot j's expert and value end up in lane j (k <= 16 <= 32): no per-thread arrays
    uint32_t msel = 0;
    KT mval = (KT)0;
    if (hash_routing) {
        const uint32_t tok = token_ids[t];
        if (tok >= vocab) {
            if (lane == 0) atomicOr(error_flag, 1u);
            return;
        }
        for (uint32_t j = 0; j < k; ++j) {
            const uint32_t e = tid2eid[(size_t)tok * k + j];
            if (e >= E) {
                if (lane == 0) atomicOr(error_flag, 2u);
                return;
            }
            // fetch val of expert e from its owner lane
            const uint32_t owner = e & 31u, slot = e >> 5;
            KT mine = (KT)0;
#pragma unroll
            for (int i = 0; i < kMaxPerLane; ++i) if ((uint32_t)i == slot) mine = val[i];
            const KT v = __shfl_sync(0xffffffffu, mine, owner);
            if (lane == j) {
                msel = e;
                mval = v;
            }
        }
    } else {
        uint32_t removed = 0;  // bit i: this lane's entry i has been selected already
        for (uint32_t j = 0; j < k; ++j) {
            // lane-local best: larger key, ties to the lower id (= lower i within a lane)
            KT bk = (KT)0;
            uint32_t be = 0xffffffffu;
#pragma unroll
            for (int i = 0; i < kMaxPerLane; ++i) {
                const uint32_t e = lane + 32u * i;
                if (e < E && !((removed >> i) & 1u) && (be == 0xffffffffu || key[i] > bk)) {
                    bk = key[i];
                    be = e;
                }
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const KT ok = __shfl_xor_sync(0xffffffffu, bk, o);
                const uint32_t oe = __shfl_xor_sync(0xffffffffu, be, o);
                if (oe != 0xffffffffu && (be == 0xffffffffu || ok > bk || (ok == bk && oe < be))) {
                    bk = ok;
                    be = oe;
                }
            }
            const uint32_t owner = be & 31u, slot = be >> 5;
            KT mine = (KT)0;
#pragma unroll
            for (int i = 0; i < kMaxPerLane; ++i) if ((uint32_t)i == slot) mine = val[i];
            const KT v = __shfl_sync(0xffffffffu, mine, owner);
            if (lane == owner) removed |= 1u << slot;
            if (lane == j) {
                msel = be;
                mval = v;
            }
        }
    }
    // the selected values' sum in slot order (the reference's sequential loop), every lane alike
    double sum = 0.0;
    for (uint32_t j = 0; j < k; ++j) sum = __dadd_rn(sum, (double)__shfl_sync(0xffffffffu, mval, j));
    if (lane < k) {
        const size_t at = (size_t)t * k + lane;
        idx[at] = msel;
        if (score == VLB_SCORE_SOFTMAX) {
            weights[at] = (float)mval;
        } else if (f64_softmax(score)) {
            // weights = f32(prob); with norm_topk_prob each is rescaled by 1 / (the rank-order f64
            // sum of the selected probabilities)
            const bool norm = score == VLB_SCORE_SOFTMAX_F64_NORM && sum > 0.0;
            const float w = (float)mval;
            weights[at] = norm ? (float)__dmul_rn((double)w, 1.0 / sum) : w;
        } else {
            // route_from_indices, deepseek_v4_reference.cpp:80-121
            if (lane == 0 && (!(sum > 0.0) || isinf(sum))) atomicOr(error_flag, 4u);
            weights[at] = (float)((double)mval / sum * (double)route_scale);
        }
    }
}

// ---------------------------------------------------------------------------------------------
// Dispatch: one CTA. Stable counting sort of the T*k (token, slot) elements by expert; the
// shared expert's T pairs are appended at [T*k, T*k + T). Builds the work units (<= kUnitTokens
// pairs of one expert each, experts ascending, shared last) and each token's combine list.
constexpr int kDispatchThreads = 1024;
constexpr uint32_t kMaxExperts = 512;  // vlb_layer_create bound

// Exclusive scan of v[0..n) in shared memory by warp 0 (n <= a few thousand); returns the total.
__device__ __forceinline__ uint32_t warp0_exclusive_scan(uint32_t* v, uint32_t n, uint32_t* total) {
    if (threadIdx.x < 32u) {
        const uint32_t lane = threadIdx.x;
        uint32_t carry = 0;
        for (uint32_t b = 0; b < n; b += 32u) {
            const uint32_t i = b + lane;
            const uint32_t x = i < n ? v[i] : 0u;
            uint32_t incl = x;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= (uint32_t)o) incl += y;
            }
            if (i < n) v[i] = carry + incl - x;
            carry += __shfl_sync(0xffffffffu, incl, 31);
        }
        if (lane == 0) *total = carry;
    }
    __syncthreads();
    return *total;
}

// Stable placement of elements [c0, c0 + blockDim.x) (element i = token * k + slot): each goes to
// base[e] + (its rank among this chunk's elements of expert e, in element order), which is the
// reference's visit order (expert ascending, then token, then slot). base[] advances past the
// chunk. wcnt: [32 warps x E] shared scratch.
__device__ __forceinline__ void dispatch_place_chunk(const MoeParams& p, uint32_t c0, uint32_t* base,
                                                     uint32_t* wcnt) {
    const uint32_t E = p.E, k = p.k, n = p.T * p.k;
    const uint32_t tid = threadIdx.x, lane = tid & 31u, warp = tid >> 5;
    const uint32_t i = c0 + tid;
    const bool valid = i < n;
    const uint32_t e = valid ? p.idx[i] : 0xffffffffu;
    for (uint32_t q = tid; q < 32u * E; q += blockDim.x) wcnt[q] = 0;
    __syncthreads();
    const uint32_t peers = __match_any_sync(0xffffffffu, e);
    const uint32_t rank_in_warp = __popc(peers & ((1u << lane) - 1u));
    const uint32_t leader = __ffs(peers) - 1u;
    if (valid && lane == leader) wcnt[warp * E + e] = __popc(peers);
    __syncthreads();
    uint32_t before = 0;
    if (valid) for (uint32_t w = 0; w < warp; ++w) before += wcnt[w * E + e];
    __syncthreads();
    if (valid) {
        const uint32_t pos = base[e] + before + rank_in_warp;
        p.pair_token[pos] = i / k;
        p.pair_slot[pos] = i % k;
        p.pair_weight[pos] = p.weights[i];
        p.combine_pairs[i] = pos;  // element -> pair position (reordered by the tail)
    }
    __syncthreads();
    for (uint32_t ee = tid; ee < E; ee += blockDim.x) {
        uint32_t sum = 0;
        for (uint32_t w = 0; w < blockDim.x / 32u; ++w) sum += wcnt[w * E + ee];
        base[ee] += sum;
    }
    __syncthreads();
}

// After placement (off[0..E] = expert offsets in shared memory, nu: [E + 1] shared scratch):
// per-pair act_max reset, the shared expert's pairs, each token's combine order, the work units
// and the counters.
__device__ __forceinline__ void dispatch_tail(const MoeParams& p, const uint32_t* off, uint32_t* nu,
                                              uint32_t* total_s) {
    const uint32_t E = p.E, k = p.k, T = p.T, n = T * k, tid = threadIdx.x;
    for (uint32_t i = tid; i < n + (p.has_shared ? T : 0u); i += blockDim.x) p.act_max[i] = 0u;
    if (p.has_shared)
        for (uint32_t t = tid; t < T; t += blockDim.x) {
            p.pair_token[n + t] = t;
            p.pair_slot[n + t] = 0;
            p.pair_weight[n + t] = 1.f;
        }
    // combine order per token: V4 sums its pairs in pair order (expert ascending, then slot);
    // OLMoE keeps rank order.
    if (!p.weight_after_down)
        for (uint32_t t = tid; t < T; t += blockDim.x) {
            uint32_t* c = p.combine_pairs + (size_t)t * k;
            for (uint32_t a = 1; a < k; ++a) {
                const uint32_t v = c[a];
                uint32_t b = a;
                while (b > 0 && c[b - 1] > v) { c[b] = c[b - 1]; --b; }
                c[b] = v;
            }
        }
    // Work units: each expert's pairs split into <= kUnitTokens; the shared expert's units come
    // first (they are the heaviest: every token, usually the widest storage type), so dynamically
    // scheduled CTAs start on them and finish on light ones. Ordinal 0 = shared, e + 1 = expert e.
    for (uint32_t o = tid; o <= E; o += blockDim.x) {
        uint32_t c = 0;
        if (o == 0) c = p.has_shared ? T : 0u;
        else c = off[o] - off[o - 1];
        nu[o] = (c + kUnitTokens - 1) / kUnitTokens;
    }
    __syncthreads();
    const uint32_t n_units = warp0_exclusive_scan(nu, E + 1, total_s);
    for (uint32_t o = tid; o <= E; o += blockDim.x) {
        const uint32_t e = o == 0 ? E : o - 1u;
        const uint32_t b = o == 0 ? n : off[e];
        const uint32_t c = o == 0 ? (p.has_shared ? T : 0u) : off[e + 1] - off[e];
        uint32_t u = nu[o];
        for (uint32_t s = 0; s < c && u < p.max_units; s += kUnitTokens, ++u) {
            p.units[u].expert = e;
            p.units[u].pair_begin = b + s;
            p.units[u].count = min((uint32_t)kUnitTokens, c - s);
            p.units[u].pad = 0;
        }
    }
    if (tid == 0) {
        p.counters[0] = n_units < p.max_units ? n_units : p.max_units;
        uint32_t na = 0;
        for (uint32_t e = 0; e < E; ++e) na += off[e + 1] > off[e];
        p.counters[1] = na + (p.has_shared ? 1u : 0u);
    }
}

// Given routes (expert-parallel groups): copies them into the layer's route arrays; an expert id
// out of range is flagged (bit 2, "route selects an out-of-range expert") and replaced by 0 so
// that nothing downstream indexes past the expert table.
__global__ void routes_copy_kernel(const uint32_t* __restrict__ idx, const float* __restrict__ w, size_t n,
                                   uint32_t E, uint32_t* __restrict__ idx_out, float* __restrict__ w_out,
                                   uint32_t* flags) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    uint32_t e = idx[i];
    if (e >= E) {
        atomicOr(flags, 2u);
        e = 0;
    }
    idx_out[i] = e;
    w_out[i] = w[i];
}

// Half-row input: one route per row from its meta words (expert, weight bits, max|x| bits); the
// row's max|x| goes where the prescale kernel would have put it. Out-of-range ids as above.
__global__ void routes_meta_kernel(const uint32_t* __restrict__ meta, uint32_t n, uint32_t E,
                                   uint32_t* __restrict__ idx_out, float* __restrict__ w_out,
                                   uint32_t* __restrict__ xmax, uint32_t* flags) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    uint32_t e = meta[3u * i];
    if (e >= E) {
        atomicOr(flags, 2u);
        e = 0;
    }
    idx_out[i] = e;
    w_out[i] = __uint_as_float(meta[3u * i + 1u]);
    xmax[i] = meta[3u * i + 2u];
}

// Small batches: the whole dispatch in one CTA (chunks of blockDim.x elements in order).
__global__ void __launch_bounds__(kDispatchThreads) dispatch_kernel(MoeParams p) {
    extern __shared__ uint32_t dsm[];
    const uint32_t E = p.E, T = p.T, n = T * p.k;
    uint32_t* cnt = dsm;              // [E + 1]
    uint32_t* off = cnt + E + 1;      // [E + 1] expert offsets (kept)
    uint32_t* base = off + E + 1;     // [E + 1] running placement bases
    uint32_t* wcnt = base + E + 1;    // [32 warps x E] per-warp counts of the current chunk
    __shared__ uint32_t total_s;
    const uint32_t tid = threadIdx.x;
    for (uint32_t e = tid; e <= E; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (uint32_t i = tid; i < n; i += blockDim.x) atomicAdd(&cnt[p.idx[i]], 1u);
    __syncthreads();
    for (uint32_t e = tid; e <= E; e += blockDim.x) off[e] = cnt[e];
    __syncthreads();
    warp0_exclusive_scan(off, E + 1, &total_s);  // off[E] = n (cnt[E] = 0)
    for (uint32_t e = tid; e <= E; e += blockDim.x) {
        base[e] = off[e];
        p.offsets[e] = off[e];
    }
    if (tid == 0) p.offsets[E + 1] = n + (p.has_shared ? T : 0u);
    __syncthreads();
    for (uint32_t c0 = 0; c0 < n; c0 += blockDim.x) dispatch_place_chunk(p, c0, base, wcnt);
    dispatch_tail(p, off, base, &total_s);
}

// Large batches, three launches. (1) per-chunk expert counts, counts[chunk * E + e].
__global__ void __launch_bounds__(kDispatchThreads) dispatch_count_kernel(MoeParams p, uint32_t* counts) {
    __shared__ uint32_t cnt[kMaxExperts];
    const uint32_t E = p.E, n = p.T * p.k, tid = threadIdx.x;
    for (uint32_t e = tid; e < E; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    const uint32_t i = blockIdx.x * blockDim.x + tid;
    if (i < n) atomicAdd(&cnt[p.idx[i]], 1u);
    __syncthreads();
    for (uint32_t e = tid; e < E; e += blockDim.x) counts[(size_t)blockIdx.x * E + e] = cnt[e];
}

// (2) each chunk's base per expert = offset of the expert + the counts of earlier chunks, then the
// chunk's stable placement; block 0 publishes the offsets.
__global__ void __launch_bounds__(kDispatchThreads) dispatch_scatter_kernel(MoeParams p, const uint32_t* counts) {
    extern __shared__ uint32_t dsm[];
    const uint32_t E = p.E, T = p.T, n = T * p.k, tid = threadIdx.x, chunks = gridDim.x;
    uint32_t* off = dsm;              // [E + 1]
    uint32_t* base = off + E + 1;     // [E + 1]
    uint32_t* wcnt = base + E + 1;    // [32 warps x E]
    __shared__ uint32_t total_s;
    for (uint32_t e = tid; e <= E; e += blockDim.x) {
        uint32_t tot = 0, before = 0;
        if (e < E)
            for (uint32_t b = 0; b < chunks; ++b) {
                const uint32_t c = counts[(size_t)b * E + e];
                tot += c;
                before += b < blockIdx.x ? c : 0u;
            }
        off[e] = tot;
        base[e] = before;
    }
    __syncthreads();
    warp0_exclusive_scan(off, E + 1, &total_s);
    for (uint32_t e = tid; e <= E; e += blockDim.x) {
        base[e] += off[e];
        if (blockIdx.x == 0) p.offsets[e] = off[e];
    }
    if (blockIdx.x == 0 && tid == 0) p.offsets[E + 1] = n + (p.has_shared ? T : 0u);
    __syncthreads();
    dispatch_place_chunk(p, blockIdx.x * blockDim.x, base, wcnt);
}

// (3) the tail, one CTA, from the published offsets.
__global__ void __launch_bounds__(kDispatchThreads) dispatch_finish_kernel(MoeParams p) {
    __shared__ uint32_t off[kMaxExperts + 1];
    __shared__ uint32_t nu[kMaxExperts + 1];
    __shared__ uint32_t total_s;
    for (uint32_t e = threadIdx.x; e <= p.E; e += blockDim.x) off[e] = p.offsets[e];
    __syncthreads();
    dispatch_tail(p, off, nu, &total_s);
}

// ---------------------------------------------------------------------------------------------
// Expert kernels. Persistent CTAs walk a contiguous range of work items; an item is one unit
// (<= 4 pairs of one expert) x one row tile. Gate/up: a warp takes 4 gate rows and the same 4
// up rows, so the SwiGLU epilogue needs nothing from other warps.
constexpr int kGuRowsPerWarp = 4;
constexpr int kGuRowsPerCta = kGuRowsPerWarp * 8;  // 32 intermediate rows per item
constexpr int kDnRowsPerWarp = 8;
constexpr int kDnRowsPerCta = kDnRowsPerWarp * 8;  // 64 hidden rows per item

template <uint32_t FMT, int TOKC>
__device__ __forceinline__ void gateup_rows(const MoeParams& p, const DevMat& w1, const DevMat& w3,
                                            uint32_t row, const float* xs, const GridSmem& gs,
                                            const Unit& u, uint32_t e) {
    float acc[2 * kGuRowsPerWarp][TOKC];
#pragma unroll
    for (int r = 0; r < 2 * kGuRowsPerWarp; ++r)
#pragma unroll
        for (int t = 0; t < TOKC; ++t) acc[r][t] = 0.f;
    warp_dot<FMT, kGuRowsPerWarp, kGuRowsPerWarp, TOKC>(w1, w3, row, row, xs, p.H / 32u, gs, acc);
    warp_reduce<2 * kGuRowsPerWarp, TOKC>(acc);
    const uint32_t lane = threadIdx.x & 31u;
    const bool shared = e == p.E;
    const float limit = shared ? p.shared_limit : p.routed_limit;
#pragma unroll
    for (int r = 0; r < kGuRowsPerWarp; ++r)
#pragma unroll
        for (int t = 0; t < TOKC; ++t) {
            if (lane != (uint32_t)(r * TOKC + t) % 32u || (uint32_t)t >= u.count) continue;
            const uint32_t pair = u.pair_begin + t;
            const float g = acc[r][t], up = acc[kGuRowsPerWarp + r][t];
            float a;
            if (p.weight_after_down) {
                // OLMoE: float SwiGLU with expf (olmoe_runtime.cpp:1279)
                a = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), up);
            } else {
                // execute_expert: double SwiGLU, optional clamp, route weight before down
                // (deepseek_v4_graph.cpp:1865-1890)
                double gv = (double)g, uv = (double)up;
                if (limit > 0.f) {
                    gv = fmin(gv, (double)limit);
                    uv = fmin(fmax(uv, -(double)limit), (double)limit);
                }
                double v = gv / (1.0 + exp(-gv)) * uv;
                if (!shared) v *= (double)p.pair_weight[pair];
                a = (float)v;
            }
            p.act[(size_t)pair * p.I + row + r] = a;
            atomicMax(p.act_max + pair, __float_as_uint(fabsf(a)));
        }
}

template <uint32_t FMT, int TOKC>
__device__ __forceinline__ void down_rows(const MoeParams& p, const DevMat& w2, uint32_t row,
                                          const float* xs, const GridSmem& gs, const Unit& u) {
    float acc[kDnRowsPerWarp][TOKC];
#pragma unroll
    for (int r = 0; r < kDnRowsPerWarp; ++r)
#pragma unroll
        for (int t = 0; t < TOKC; ++t) acc[r][t] = 0.f;
    warp_dot<FMT, kDnRowsPerWarp, 0, TOKC>(w2, w2, row, 0u, xs, p.I / 32u, gs, acc);
    warp_reduce<kDnRowsPerWarp, TOKC>(acc);
    const uint32_t lane = threadIdx.x & 31u;
#pragma unroll
    for (int r = 0; r < kDnRowsPerWarp; ++r)
#pragma unroll
        for (int t = 0; t < TOKC; ++t)
            if (lane == (uint32_t)(r * TOKC + t) % 32u && (uint32_t)t < u.count)
                p.y[(size_t)(u.pair_begin + t) * p.H + row + r] = acc[r][t];
}

template <int TOKC>
__device__ __forceinline__ void gateup_dispatch(const MoeParams& p, const DevMat& w1,
                                                const DevMat& w3, uint32_t row, const float* xs,
                                                const GridSmem& gs, const Unit& u, uint32_t e) {
    switch (w1.type) {
        case kTypeIq2Xxs: gateup_rows<kTypeIq2Xxs, TOKC>(p, w1, w3, row, xs, gs, u, e); break;
        case kTypeQ8_0: gateup_rows<kTypeQ8_0, TOKC>(p, w1, w3, row, xs, gs, u, e); break;
        case kTypeIq3Xxs: gateup_rows<kTypeIq3Xxs, TOKC>(p, w1, w3, row, xs, gs, u, e); break;
        case kTypeQ4K: gateup_rows<kTypeQ4K, TOKC>(p, w1, w3, row, xs, gs, u, e); break;
        case kTypeQ5K: gateup_rows<kTypeQ5K, TOKC>(p, w1, w3, row, xs, gs, u, e); break;
        case kTypeQ6K: gateup_rows<kTypeQ6K, TOKC>(p, w1, w3, row, xs, gs, u, e); break;
        case kTypeIq2S: gateup_rows<kTypeIq2S, TOKC>(p, w1, w3, row, xs, gs, u, e); break;
        case kTypeMxfp4: gateup_rows<kTypeMxfp4, TOKC>(p, w1, w3, row, xs, gs, u, e); break;
        default: gateup_rows<kTypeIq1S, TOKC>(p, w1, w3, row, xs, gs, u, e); break;
    }
}

template <int TOKC>
__device__ __forceinline__ void down_dispatch(const MoeParams& p, const DevMat& w2, uint32_t row,
                                              const float* xs, const GridSmem& gs, const Unit& u) {
    switch (w2.type) {
        case kTypeIq2Xxs: down_rows<kTypeIq2Xxs, TOKC>(p, w2, row, xs, gs, u); break;
        case kTypeQ8_0: down_rows<kTypeQ8_0, TOKC>(p, w2, row, xs, gs, u); break;
        case kTypeIq3Xxs: down_rows<kTypeIq3Xxs, TOKC>(p, w2, row, xs, gs, u); break;
        case kTypeQ4K: down_rows<kTypeQ4K, TOKC>(p, w2, row, xs, gs, u); break;
        case kTypeQ5K: down_rows<kTypeQ5K, TOKC>(p, w2, row, xs, gs, u); break;
        case kTypeQ6K: down_rows<kTypeQ6K, TOKC>(p, w2, row, xs, gs, u); break;
        case kTypeIq2S: down_rows<kTypeIq2S, TOKC>(p, w2, row, xs, gs, u); break;
        case kTypeMxfp4: down_rows<kTypeMxfp4, TOKC>(p, w2, row, xs, gs, u); break;
        default: down_rows<kTypeIq1S, TOKC>(p, w2, row, xs, gs, u); break;
    }
}

// skip: fmt_bit set of the storage types another kernel of the phase serves.
template <bool GATEUP>
__global__ void __launch_bounds__(256) expert_kernel(MoeParams p, uint32_t skip) {
    extern __shared__ __align__(16) unsigned char smem[];
    const GridSmem gs = stage_grids(p.grids, smem);
    float* xs = reinterpret_cast<float*>(smem + kGridSmemBytes);
    const uint32_t n_units = p.counters[0];
    const uint32_t rows_per_item = GATEUP ? kGuRowsPerCta : kDnRowsPerCta;
    const uint32_t tiles = (GATEUP ? p.I : p.H) / rows_per_item;
    const uint32_t cols = GATEUP ? p.H : p.I;
    const uint64_t n_items = (uint64_t)n_units * tiles;
    const uint64_t begin = n_items * blockIdx.x / gridDim.x;
    const uint64_t end = n_items * (blockIdx.x + 1) / gridDim.x;
    const uint32_t warp = threadIdx.x >> 5;
    uint32_t staged = 0xffffffffu;
    for (uint64_t item = begin; item < end; ++item) {
        const uint32_t ui = (uint32_t)(item / tiles), tile = (uint32_t)(item % tiles);
        const Unit u = p.units[ui];
        if (skip & fmt_bit(p.mats[(GATEUP ? 0u : 2u * (p.E + 1)) + u.expert].type)) continue;
        if (ui != staged) {
            const float* rows[kUnitTokens];
#pragma unroll
            for (int t = 0; t < kUnitTokens; ++t) {
                const uint32_t pair = u.pair_begin + t;
                rows[t] = (uint32_t)t < u.count
                              ? (GATEUP ? p.x + (size_t)p.pair_token[pair] * p.H
                                        : p.act + (size_t)pair * p.I)
                              : nullptr;
            }
            __syncthreads();
            stage_x<kUnitTokens>(xs, rows, cols);
            __syncthreads();
            staged = ui;
        }
        const uint32_t row = tile * rows_per_item + warp * (GATEUP ? kGuRowsPerWarp : kDnRowsPerWarp);
        if (GATEUP) {
            const DevMat w1 = p.mats[u.expert];
            const DevMat w3 = p.mats[(p.E + 1) + u.expert];
            if (u.count == 1) gateup_dispatch<1>(p, w1, w3, row, xs, gs, u, u.expert);
            else if (u.count == 2) gateup_dispatch<2>(p, w1, w3, row, xs, gs, u, u.expert);
            else gateup_dispatch<4>(p, w1, w3, row, xs, gs, u, u.expert);
        } else {
            const DevMat w2 = p.mats[2 * (p.E + 1) + u.expert];
            if (u.count == 1) down_dispatch<1>(p, w2, row, xs, gs, u);
            else if (u.count == 2) down_dispatch<2>(p, w2, row, xs, gs, u);
            else down_dispatch<4>(p, w2, row, xs, gs, u);
        }
    }
}

__global__ void __launch_bounds__(256) token_prescale_kernel(const float* __restrict__ x, uint32_t T,
                                                             uint32_t H, uint32_t* __restrict__ xmax,
                                                             double* __restrict__ xd) {
    // grid (ceil(H / 1024), min(T, 65535)), rows strided over gridDim.y: each thread takes 4 columns
    // of one token; the token's max|x| (for the tensor-core activation prescale) is an atomic max
    // over float bits (non-negative floats order as integers); with xd the row is also widened to
    // f64 for the router projection
    const uint32_t c = (blockIdx.x * blockDim.x + threadIdx.x) * 4u;
    for (uint32_t t = blockIdx.y; t < T; t += gridDim.y) {
        float m = 0.f;
        if (c < H) {
            const float4 v = *reinterpret_cast<const float4*>(x + (size_t)t * H + c);
            m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
            if (xd) {
                double* o = xd + (size_t)t * H + c;
                *reinterpret_cast<double2*>(o) = make_double2(v.x, v.y);
                *reinterpret_cast<double2*>(o + 2) = make_double2(v.z, v.w);
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if ((threadIdx.x & 31u) == 0 && m > 0.f) atomicMax(xmax + t, __float_as_uint(m));
    }
}

// ---------------------------------------------------------------------------------------------
// Hyper-Connection around the MoE (the ffn half of block_prefill / block_incremental,
// deepseek_v4_graph.cpp:2391-2408: hc_pre, ffn_norm, moe_forward, hc_post).
constexpr size_t kHcSmemLimit = 224u * 1024u;  // dynamic shared memory of the entry kernel
constexpr uint32_t kHcMaxStages = 3;
constexpr uint32_t kHcSlots = 224;          // chain threads (warps 0-6); warp 7 streams the weight
constexpr uint32_t kHcProducerWarp = 7;
constexpr uint64_t kHcWaitNs = 2000000000ull;  // a stage wait that outlasts 2 s is a failure

// Entry, one CTA per token (deepseek_v4_hc_pre, deepseek_v4_reference.cpp:479-547, and the
// split, :387-477): the token's m x H state is staged in shared memory as f64; every mixing row
// r < (2+m)m and the sum of squares is one thread's sequential f64 chain in column order (each
// product of two f32 values is exact in f64, so fma(a, b, s) rounds like the reference's
// s + a * b), which makes the mixes bit-identical; the mixing weight (kept in f64) streams through
// a 3-stage shared-memory ring in column chunks (bulk copies by a producer warp, mbarrier
// hand-offs), so a chain never waits on memory: its floor is the dependent FMA (8.2 cycles on B200,
// measured); in this kernel a step costs about 19 cycles (a standalone loop of the same shape
// runs at 10.5-13). The split gives each combination element its own thread, which
// re-walks its row or column sum in the reference's order; the reduced row overwrites copy 0 of
// the staged state (each column is read by its own thread before it writes it), then the ffn norm
// runs as rms_norm_kernel does. Only CUDA's double exp can differ from the host's (at most 1 ulp of
// an f64, rarely visible after the f32 rounding).
__device__ __forceinline__ float hc_affine(float mix, float scale, float base) {
    return __fadd_rn(__fmul_rn(mix, scale), base);  // mixes * scale + base, no contraction
}

// Shared-memory plan of the entry: the token's state widened to f64 [m x H], then a ring of 3
// (else 2) stages of the f64 mixing weight, each `chunk` columns of all (2+m)m rows (row stride
// chunk + 2 doubles: 16-byte reads of different rows fall in different bank groups). chunk divides
// m x H (a multiple of 256). Operands are f64 in shared memory because a float-to-double conversion per
// chain step costs more issue slots than the chain's FMA latency (about 31 cycles a step against
// 8 on B200).
struct HcPlan {
    uint32_t chunk;   // columns per staged chunk (divides m x H)
    uint32_t stages;  // ring depth (3, else 2)
};
__host__ __device__ inline size_t hc_plan_bytes(uint32_t m, uint32_t H, HcPlan pl) {
    return (size_t)m * H * 8u + (size_t)pl.stages * (2u + m) * m * (pl.chunk + 2u) * 8u;
}
__host__ __device__ inline HcPlan hc_plan(uint32_t m, uint32_t H) {
    for (uint32_t st = 3; st >= 2u; --st)
        for (uint32_t c = 128; c >= 16u; c >>= 1)
            if (hc_plan_bytes(m, H, HcPlan{c, st}) <= kHcSmemLimit) return HcPlan{c, st};
    return HcPlan{16, 2};
}
__host__ __device__ inline size_t hc_entry_smem(uint32_t m, uint32_t H) { return hc_plan_bytes(m, H, hc_plan(m, H)); }

// Bounded wait on an mbarrier phase for the entry (false after the time limit or once another
// thread of the CTA gave up).
__device__ __forceinline__ bool hc_wait(uint64_t* bar, uint32_t parity, volatile uint32_t* abort) {
    if (tc::mbar_try(bar, parity)) return true;
    const uint64_t t0 = tc::global_ns();
    for (uint32_t i = 1; i < (1u << 30); ++i) {
        if (tc::mbar_try_sleep(bar, parity, 20000u)) return true;
        if (*abort) return false;
        if (tc::global_ns() - t0 > kHcWaitNs) return false;
    }
    return false;
}

// The chain warps' walk over the staged chunks (CH: the plan's chunk, a compile-time loop length
// so that the loads of the next columns are hoisted above the current FMAs).
template <uint32_t CH>
__device__ __forceinline__ void hc_consume(const double* stage, const double* hrow, uint64_t* full, uint64_t* empty,
                                           volatile uint32_t* abort, uint32_t* flags, uint32_t ns, uint32_t nk,
                                           uint32_t mw, uint32_t r0, uint32_t r1, bool a0, bool a1, uint32_t lane,
                                           double& s0, double& s1) {
    constexpr uint32_t cs = CH + 2u;
    for (uint32_t k = 0; k < nk; ++k) {
        bool ok = true;
        if (lane == 0) ok = hc_wait(full + k % ns, (k / ns) & 1u, abort);
        ok = __shfl_sync(0xffffffffu, ok ? 1u : 0u, 0) != 0u;
        if (!ok) {
            if (lane == 0) {
                *abort = 1u;
                atomicOr(flags, kLayerErrHcTimeout);
            }
            return;
        }
        const double* buf = stage + (size_t)(k % ns) * mw * cs;
        const double* xk = hrow + (size_t)k * CH;
        const double* w0 = r0 < mw ? buf + (size_t)r0 * cs : xk;
        if (a1) {
            const double* w1 = r1 < mw ? buf + (size_t)r1 * cs : xk;
#pragma unroll 16
            for (uint32_t c = 0; c < CH; c += 2u) {
                const double2 xv = *reinterpret_cast<const double2*>(xk + c);
                const double2 u = *reinterpret_cast<const double2*>(w0 + c);
                const double2 v = *reinterpret_cast<const double2*>(w1 + c);
                s0 = __fma_rn(xv.x, u.x, s0);
                s1 = __fma_rn(xv.x, v.x, s1);
                s0 = __fma_rn(xv.y, u.y, s0);
                s1 = __fma_rn(xv.y, v.y, s1);
            }
        } else if (a0) {
#pragma unroll 16
            for (uint32_t c = 0; c < CH; c += 2u) {
                const double2 xv = *reinterpret_cast<const double2*>(xk + c);
                const double2 u = *reinterpret_cast<const double2*>(w0 + c);
                s0 = __fma_rn(xv.x, u.x, s0);
                s0 = __fma_rn(xv.y, u.y, s0);
            }
        }
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(empty + k % ns);
    }
}

__global__ void __launch_bounds__(256) hc_entry_kernel(MoeParams p) {
    extern __shared__ __align__(16) double hsm[];
    __shared__ float mix[16 * 18];
    __shared__ float cmb[16 * 16];
    __shared__ float pre_s[16];
    __shared__ double inv_s, ninv_s;
    __shared__ float wmax[8];
    __shared__ __align__(8) uint64_t full[kHcMaxStages], empty[kHcMaxStages];
    __shared__ uint32_t abort_s;
    const uint32_t t = blockIdx.x, m = p.hc_m, H = p.H, fw = m * H, mw = (2u + m) * m;
    const HcPlan pl = hc_plan(m, H);
    const uint32_t chunk = pl.chunk, ns = pl.stages, cs = chunk + 2u, nk = fw / chunk;
    double* hrow = hsm;             // [m x H]
    double* stage = hsm + fw;       // [stages][mw][cs]
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u;
    // chain slots: consumer thread i < 224 walks mixing rows i and i + 224; slot mw walks the sum
    // of squares, whose "weights" are the state itself (the same instructions, so no divergence).
    // Warp 7 streams the mixing weight: chunk k of every row into stage k % stages with bulk
    // copies completing on full[k % stages]; the chain warps release a stage on empty[].
    const uint32_t r0 = threadIdx.x, r1 = threadIdx.x + kHcSlots;
    const uint32_t chain_warps = min(kHcSlots / 32u, (mw + 32u) / 32u);
    const bool consumer = warp < chain_warps, producer = warp == kHcProducerWarp;
    const bool a0 = consumer && r0 <= mw, a1 = consumer && r1 <= mw;
    if (threadIdx.x == 0) {
        for (uint32_t i = 0; i < ns; ++i) {
            tc::mbar_init(full + i, 1);
            tc::mbar_init(empty + i, chain_warps);
        }
        abort_s = 0;
        tc::mbar_fence_init();
    }
    __syncthreads();
    const uint32_t stage_bytes = mw * chunk * 8u;
    auto issue = [&](uint32_t k) {  // the whole producer warp
        double* dst = stage + (size_t)(k % ns) * mw * cs;
        if (lane == 0) tc::mbar_arrive_expect_tx(full + k % ns, stage_bytes);
        __syncwarp();
        for (uint32_t r = lane; r < mw; r += 32u)
            tc::bulk_load(tc::smem_u32(dst + (size_t)r * cs), p.hc_fn + (size_t)r * fw + (size_t)k * chunk,
                          chunk * 8u, full + k % ns);
    };
    if (producer)
        for (uint32_t k = 0; k < ns && k < nk; ++k) issue(k);
    const float* xr = p.x + (size_t)t * fw;
    for (uint32_t c = threadIdx.x * 4u; c < fw; c += blockDim.x * 4u) {
        const float4 v = *reinterpret_cast<const float4*>(xr + c);
        *reinterpret_cast<double2*>(hrow + c) = make_double2(v.x, v.y);
        *reinterpret_cast<double2*>(hrow + c + 2) = make_double2(v.z, v.w);
    }
    __syncthreads();
    double s0 = 0.0, s1 = 0.0;
    if (producer) {
        uint32_t issued = min(ns, nk);
        for (uint32_t k = ns; k < nk; ++k) {
            bool ok = true;
            if (lane == 0) ok = hc_wait(empty + k % ns, ((k / ns) - 1u) & 1u, &abort_s);
            ok = __shfl_sync(0xffffffffu, ok ? 1u : 0u, 0) != 0u;
            if (!ok) {
                if (lane == 0) {
                    abort_s = 1u;
                    atomicOr(p.counters + 3, kLayerErrHcTimeout);
                }
                break;
            }
            issue(k);
            issued = k + 1u;
        }
        // no copy may still be landing when the CTA leaves: wait (bounded) for every issued chunk
        if (lane == 0)
            for (uint32_t k = issued > ns ? issued - ns : 0u; k < issued; ++k)
                if (!hc_wait(full + k % ns, (k / ns) & 1u, &abort_s)) {
                    atomicOr(p.counters + 3, kLayerErrHcTimeout);
                    break;
                }
    } else if (consumer) {
        switch (chunk) {
            case 128: hc_consume<128>(stage, hrow, full, empty, &abort_s, p.counters + 3, ns, nk, mw, r0, r1, a0, a1, lane, s0, s1); break;
            case 64: hc_consume<64>(stage, hrow, full, empty, &abort_s, p.counters + 3, ns, nk, mw, r0, r1, a0, a1, lane, s0, s1); break;
            case 32: hc_consume<32>(stage, hrow, full, empty, &abort_s, p.counters + 3, ns, nk, mw, r0, r1, a0, a1, lane, s0, s1); break;
            default: hc_consume<16>(stage, hrow, full, empty, &abort_s, p.counters + 3, ns, nk, mw, r0, r1, a0, a1, lane, s0, s1); break;
        }
    }
    __syncthreads();
    if (a0 && r0 == mw) inv_s = 1.0 / sqrt(s0 / (double)fw + (double)p.norm_eps);
    if (a1 && r1 == mw) inv_s = 1.0 / sqrt(s1 / (double)fw + (double)p.norm_eps);
    double chain[2] = {s0, s1};
    uint32_t rows[2] = {a0 ? r0 : 0xffffffffu, a1 ? r1 : 0xffffffffu};
    __syncthreads();
    for (uint32_t i = 0; i < 2u; ++i)
        if (rows[i] < mw) mix[rows[i]] = (float)(chain[i] * inv_s);
    __syncthreads();
    // the split: thread i < m * m owns combination element (i / m, i % m); every row or column
    // sum is re-walked by each of its threads in the reference's order, so all of them see the
    // same value and the m * m divisions of a pass run at once. m * m <= 32 stays in warp 0.
    {
        const bool in_warp = m * m <= 32u;
        if (!in_warp || threadIdx.x < 32u) {
            const uint32_t i = threadIdx.x, r = i / m, j = i % m;
            const bool own = i < m * m;
            const float eps = p.hc_eps;
            const double deps = (double)eps;
            auto sync = [&] {
                if (in_warp) __syncwarp();
                else __syncthreads();
            };
            if (i < m) {
                const float pr = __fadd_rn(sigmoid_dev(hc_affine(mix[i], p.hc_scale[0], p.hc_base[i])), eps);
                const float po = __fmul_rn(2.0f, sigmoid_dev(hc_affine(mix[m + i], p.hc_scale[1], p.hc_base[m + i])));
                pre_s[i] = pr;
                p.hc_pre[(size_t)t * m + i] = pr;
                p.hc_post[(size_t)t * m + i] = po;
            }
            // row softmax plus eps (the row's maximum in column order, as std::max keeps it)
            float v = 0.f;
            if (own) {
                float mx = -INFINITY;
                for (uint32_t q = 0; q < m; ++q) {
                    const uint32_t at = 2u * m + r * m + q;
                    const float a = hc_affine(mix[at], p.hc_scale[2], p.hc_base[at]);
                    mx = mx < a ? a : mx;
                }
                const uint32_t at = 2u * m + r * m + j;
                v = (float)exp((double)__fsub_rn(hc_affine(mix[at], p.hc_scale[2], p.hc_base[at]), mx));
                cmb[i] = v;
            }
            sync();
            if (own) {
                double sum = 0.0;
                for (uint32_t q = 0; q < m; ++q) sum = __dadd_rn(sum, (double)cmb[r * m + q]);
                v = __fadd_rn((float)__ddiv_rn((double)v, sum), eps);
            }
            sync();
            if (own) cmb[i] = v;
            sync();
            for (uint32_t it = 0; it < p.hc_iters; ++it) {
                if (it > 0u) {  // rows
                    if (own) {
                        double sum = 0.0;
                        for (uint32_t q = 0; q < m; ++q) sum = __dadd_rn(sum, (double)cmb[r * m + q]);
                        v = (float)__ddiv_rn((double)v, __dadd_rn(sum, deps));
                    }
                    sync();
                    if (own) cmb[i] = v;
                    sync();
                }
                if (own) {  // columns
                    double sum = 0.0;
                    for (uint32_t q = 0; q < m; ++q) sum = __dadd_rn(sum, (double)cmb[q * m + j]);
                    v = (float)__ddiv_rn((double)v, __dadd_rn(sum, deps));
                }
                sync();
                if (own) cmb[i] = v;
                sync();
            }
            if (own) p.hc_comb[(size_t)t * m * m + i] = v;
        }
    }
    __syncthreads();
    // reduced[c] = sum over copies j of pre[j] * x[j][c] (f64, copy order), kept in copy 0's slot
    bool bad = false;
    for (uint32_t c = threadIdx.x; c < H; c += blockDim.x) {
        double s = 0.0;
        for (uint32_t j = 0; j < m; ++j) s = __fma_rn((double)pre_s[j], hrow[(size_t)j * H + c], s);
        const float rf = (float)s;
        bad |= !isfinite(rf);
        hrow[c] = (double)rf;
    }
    if (bad) atomicOr(p.counters + 3, kLayerErrHcNonFinite);
    __syncthreads();
    // the ffn norm of the reduced row (rms_norm_kernel's arithmetic)
    if (threadIdx.x == 0) {
        double sq = 0.0;
#pragma unroll 8
        for (uint32_t c = 0; c < H; c += 2u) {
            const double2 v = *reinterpret_cast<const double2*>(hrow + c);
            sq = __fma_rn(v.x, v.x, sq);
            sq = __fma_rn(v.y, v.y, sq);
        }
        ninv_s = 1.0 / sqrt(sq / (double)H + (double)p.norm_eps);
    }
    __syncthreads();
    const double inv = ninv_s;
    float mxv = 0.f;
    for (uint32_t c = threadIdx.x; c < H; c += blockDim.x) {
        const float o = (float)(__dmul_rn(__dmul_rn(hrow[c], inv), (double)p.norm_w[c]));
        p.x_norm[(size_t)t * H + c] = o;
        if (p.xd) p.xd[(size_t)t * H + c] = (double)o;
        mxv = fmaxf(mxv, fabsf(o));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mxv = fmaxf(mxv, __shfl_xor_sync(0xffffffffu, mxv, o));
    if ((threadIdx.x & 31u) == 0) wmax[threadIdx.x >> 5] = mxv;
    __syncthreads();
    if (threadIdx.x == 0) {
        float mm = 0.f;
        for (uint32_t i = 0; i < blockDim.x / 32u; ++i) mm = fmaxf(mm, wmax[i]);
        p.xmax[t] = __float_as_uint(mm);
    }
}

// Exit: out[t, d] = f32(post[d] * moe + sum over sources s of comb[s][d] * x[t, s]) in f64 (the
// reference's order; each product of two f32 values is exact in f64).
__device__ __forceinline__ void hc_post_store(const MoeParams& p, uint32_t t, uint32_t c4, float4 moe) {
    const uint32_t m = p.hc_m, H = p.H;
    const float* post = p.hc_post + (size_t)t * m;
    const float* comb = p.hc_comb + (size_t)t * m * m;
    const float* st = p.hc_state + (size_t)t * m * H + c4;
    for (uint32_t d = 0; d < m; ++d) {
        const double pd = (double)post[d];
        double v0 = __dmul_rn(pd, (double)moe.x), v1 = __dmul_rn(pd, (double)moe.y);
        double v2 = __dmul_rn(pd, (double)moe.z), v3 = __dmul_rn(pd, (double)moe.w);
        for (uint32_t s = 0; s < m; ++s) {
            const double cs = (double)comb[s * m + d];
            const float4 r = *reinterpret_cast<const float4*>(st + (size_t)s * H);
            v0 = __fma_rn(cs, (double)r.x, v0);
            v1 = __fma_rn(cs, (double)r.y, v1);
            v2 = __fma_rn(cs, (double)r.z, v2);
            v3 = __fma_rn(cs, (double)r.w, v3);
        }
        *reinterpret_cast<float4*>(p.out + ((size_t)t * m + d) * H + c4) =
            make_float4((float)v0, (float)v1, (float)v2, (float)v3);
    }
}

// ---------------------------------------------------------------------------------------------
// Combine (deepseek_v4_graph.cpp:2214-2227, :2263-2266; olmoe_runtime.cpp:1282-1285).
__global__ void __launch_bounds__(256) combine_kernel(MoeParams p) {
    const uint32_t c4 = (blockIdx.x * blockDim.x + threadIdx.x) * 4u;
    if (c4 >= p.H) return;
    for (uint32_t t = blockIdx.y; t < p.T; t += gridDim.y) {
        const uint32_t* cp = p.combine_pairs + (size_t)t * p.k;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (uint32_t j = 0; j < p.k; ++j) {
            const uint32_t pair = cp[j];
            const float4 v = *reinterpret_cast<const float4*>(p.y + (size_t)pair * p.H + c4);
            if (p.weight_after_down) {
                const float w = p.pair_weight[pair];
                acc.x = __fadd_rn(acc.x, __fmul_rn(w, v.x));
                acc.y = __fadd_rn(acc.y, __fmul_rn(w, v.y));
                acc.z = __fadd_rn(acc.z, __fmul_rn(w, v.z));
                acc.w = __fadd_rn(acc.w, __fmul_rn(w, v.w));
            } else {
                acc.x = __fadd_rn(acc.x, v.x);
                acc.y = __fadd_rn(acc.y, v.y);
                acc.z = __fadd_rn(acc.z, v.z);
                acc.w = __fadd_rn(acc.w, v.w);
            }
        }
        if (p.has_shared) {
            const float4 v = *reinterpret_cast<const float4*>(p.y + (size_t)(p.T * p.k + t) * p.H + c4);
            acc.x = __fadd_rn(acc.x, v.x);
            acc.y = __fadd_rn(acc.y, v.y);
            acc.z = __fadd_rn(acc.z, v.z);
            acc.w = __fadd_rn(acc.w, v.w);
        }
        if (p.hc_m) {  // Hyper-Connection exit (deepseek_v4_hc_post, deepseek_v4_reference.cpp:549-610)
            hc_post_store(p, t, c4, acc);
            continue;
        }
        if (p.x_residual) {  // residual block: x + MoE(RMSNorm(x)), one f32 addition
            const float4 v = *reinterpret_cast<const float4*>(p.x_residual + (size_t)t * p.H + c4);
            acc.x = __fadd_rn(v.x, acc.x);
            acc.y = __fadd_rn(v.y, acc.y);
            acc.z = __fadd_rn(v.z, acc.z);
            acc.w = __fadd_rn(v.w, acc.w);
        }
        *reinterpret_cast<float4*>(p.out + (size_t)t * p.H + c4) = acc;
    }
}

// ---------------------------------------------------------------------------------------------
// RMSNorm (deepseek_v4_reference.cpp:170-206), one CTA per row: out = f32(double(x) * inv *
// double(w)) with inv = 1 / sqrt(sum(double(x)^2) / width + eps). The sum of squares is the
// reference's sequential f64 sum (each square of an f32 is exact in f64, so fma(v, v, s) rounds
// like s + v * v): the CTA stages the row in shared memory as f64 (every thread converts a few
// values: a conversion per chain step would cost more than the chain) and one thread walks it in
// column order, so the result is bit-identical; division and square root are IEEE-rounded in CUDA
// as on the host. With xmax non-null the kernel is also the layer's entry step: it records
// max|out| of the row (bits of a non-negative float, for the tensor-core activation prescale), and
// with out_d the normalised row widened to f64 (the router projection's input).
__global__ void __launch_bounds__(256) rms_norm_kernel(const float* __restrict__ x,
                                                       const float* __restrict__ w,
                                                       uint32_t width, float eps,
                                                       float* __restrict__ out,
                                                       uint32_t* __restrict__ xmax,
                                                       double* __restrict__ out_d) {
    extern __shared__ __align__(16) double rowd[];
    __shared__ double inv_s;
    __shared__ float wmax[8];
    const float* xr = x + (size_t)blockIdx.x * width;
    for (uint32_t c = threadIdx.x * 4u; c < width; c += blockDim.x * 4u) {
        const float4 v = *reinterpret_cast<const float4*>(xr + c);
        *reinterpret_cast<double2*>(rowd + c) = make_double2(v.x, v.y);
        *reinterpret_cast<double2*>(rowd + c + 2) = make_double2(v.z, v.w);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        double sq = 0.0;
        uint32_t c = 0;
        for (; c + 8u <= width; c += 8u) {
            double v[8];
#pragma unroll
            for (int i = 0; i < 8; i += 2) {
                const double2 d2 = *reinterpret_cast<const double2*>(rowd + c + i);
                v[i] = d2.x;
                v[i + 1] = d2.y;
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) sq = __fma_rn(v[i], v[i], sq);
        }
        for (; c < width; ++c) sq = __fma_rn(rowd[c], rowd[c], sq);
        inv_s = 1.0 / sqrt(sq / (double)width + (double)eps);
    }
    __syncthreads();
    const double inv = inv_s;
    float m = 0.f;
    for (uint32_t c = threadIdx.x; c < width; c += blockDim.x) {
        const float o = (float)(__dmul_rn(__dmul_rn(rowd[c], inv), (double)w[c]));
        out[(size_t)blockIdx.x * width + c] = o;
        if (out_d) out_d[(size_t)blockIdx.x * width + c] = (double)o;
        m = fmaxf(m, fabsf(o));
    }
    if (!xmax) return;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31u) == 0) wmax[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        float mm = 0.f;
        for (uint32_t i = 0; i < blockDim.x / 32u; ++i) mm = fmaxf(mm, wmax[i]);
        xmax[blockIdx.x] = __float_as_uint(mm);
    }
}

// =============================================================================================
// launchers

// Raises a kernel's dynamic shared-memory limit once per process and size (a host call that must
// not sit on the per-forward path, and that graph capture would not record anyway).
template <typename K>
static cudaError_t set_smem_once(K kernel, size_t bytes) {
    static std::mutex mu;
    static std::vector<std::pair<const void*, size_t>> done;
    std::lock_guard<std::mutex> lock(mu);
    for (auto& d : done)
        if (d.first == (const void*)kernel && d.second >= bytes) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e == cudaSuccess) done.emplace_back((const void*)kernel, bytes);
    return e;
}
// grid.y for row-strided kernels (gridDim.y is limited to 65535)
static unsigned rows_grid(uint32_t rows) { return rows < 65535u ? (rows ? rows : 1u) : 65535u; }
static int g_num_sms = 0;
static int num_sms() {
    if (g_num_sms == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
        if (g_num_sms <= 0) g_num_sms = 148;
    }
    return g_num_sms;
}

cudaError_t launch_dequant(const DevMat& m, const Grids& g, float* out, cudaStream_t s) {
    const size_t groups = (size_t)m.rows * (m.cols / 32u);
    dequant_kernel<<<(unsigned)((groups + 255) / 256), 256, 0, s>>>(m, g, out);
    return cudaGetLastError();
}

template <uint32_t FMT, int TOKC>
static cudaError_t gemv_launch(const DevMat& m, const Grids& g, const float* x, uint32_t ntok,
                               uint32_t xs, float* y, uint32_t ys, cudaStream_t s) {
    const size_t smem = kGridSmemBytes + (size_t)TOKC * m.cols * sizeof(float);
    auto kern = gemv_kernel<FMT, TOKC>;
    cudaError_t e = set_smem_once(kern, smem);
    if (e != cudaSuccess) return e;
    const unsigned grid = (m.rows + gemv_rows(TOKC) * kGemvWarps - 1) / (gemv_rows(TOKC) * kGemvWarps);
    kern<<<grid, 256, smem, s>>>(m, g, x, ntok, xs, y, ys);
    return cudaGetLastError();
}

template <int TOKC>
static cudaError_t gemv_type(const DevMat& m, const Grids& g, const float* x, uint32_t ntok,
                             uint32_t xs, float* y, uint32_t ys, cudaStream_t s) {
    switch (m.type) {
        case kTypeQ8_0: return gemv_launch<kTypeQ8_0, TOKC>(m, g, x, ntok, xs, y, ys, s);
        case kTypeIq2Xxs: return gemv_launch<kTypeIq2Xxs, TOKC>(m, g, x, ntok, xs, y, ys, s);
        case kTypeIq3Xxs: return gemv_launch<kTypeIq3Xxs, TOKC>(m, g, x, ntok, xs, y, ys, s);
        case kTypeIq1S: return gemv_launch<kTypeIq1S, TOKC>(m, g, x, ntok, xs, y, ys, s);
        case kTypeQ4K: return gemv_launch<kTypeQ4K, TOKC>(m, g, x, ntok, xs, y, ys, s);
        case kTypeQ5K: return gemv_launch<kTypeQ5K, TOKC>(m, g, x, ntok, xs, y, ys, s);
        case kTypeQ6K: return gemv_launch<kTypeQ6K, TOKC>(m, g, x, ntok, xs, y, ys, s);
        case kTypeIq2S: return gemv_launch<kTypeIq2S, TOKC>(m, g, x, ntok, xs, y, ys, s);
        case kTypeMxfp4: return gemv_launch<kTypeMxfp4, TOKC>(m, g, x, ntok, xs, y, ys, s);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_gemv(const DevMat& m, const Grids& g, const float* x, uint32_t ntok,
                        uint32_t xstride, float* y, uint32_t ystride, cudaStream_t s) {
    if (ntok == 0) return cudaSuccess;
    if (ntok == 1) return gemv_type<1>(m, g, x, ntok, xstride, y, ystride, s);
    if (ntok == 2) return gemv_type<2>(m, g, x, ntok, xstride, y, ystride, s);
    return gemv_type<4>(m, g, x, ntok, xstride, y, ystride, s);
}

cudaError_t launch_router(const double* xd, const double* wd, uint32_t T, uint32_t H, uint32_t E, int score,
                          float* logits, float* scores, cudaStream_t s) {
    if (H % 2u) return cudaErrorInvalidValue;
    const dim3 grid((E + kRtExperts - 1u) / kRtExperts, (T + kRtTokens - 1u) / kRtTokens);
    if (grid.y > 65535u) return cudaErrorInvalidValue;
    cudaError_t e = set_smem_once(router_kernel, kRtSmemBytes);
    if (e != cudaSuccess) return e;
    router_kernel<<<grid, kRtThreads, kRtSmemBytes, s>>>(wd, xd, T, H, E, score, logits, scores);
    return cudaGetLastError();
}

cudaError_t launch_widen(const float* src, size_t n, double* dst, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    const size_t blocks = (n + 255) / 256;
    widen_kernel<<<(unsigned)(blocks < 4096 ? blocks : 4096), 256, 0, s>>>(src, n, dst);
    return cudaGetLastError();
}

cudaError_t launch_prescale(const float* x, uint32_t T, uint32_t H, uint32_t* xmax, double* xd, cudaStream_t s) {
    cudaError_t e = cudaMemsetAsync(xmax, 0, (size_t)T * 4u, s);
    if (e != cudaSuccess) return e;
    token_prescale_kernel<<<dim3((H + 1023) / 1024, rows_grid(T)), 256, 0, s>>>(x, T, H, xmax, xd);
    return cudaGetLastError();
}

cudaError_t launch_scores(const float* logits, size_t n, int score, float* scores,
                          cudaStream_t s) {
    score_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(logits, n, score, scores);
    return cudaGetLastError();
}

cudaError_t launch_route(const float* scores, const float* bias, const uint32_t* token_ids,
                         const uint32_t* tid2eid, uint32_t vocab, uint32_t T, uint32_t E,
                         uint32_t k, int score, int hash_routing, float route_scale,
                         uint32_t* idx, float* weights, uint32_t* error_flag, cudaStream_t s) {
    if (score == VLB_SCORE_SOFTMAX_F64 || score == VLB_SCORE_SOFTMAX_F64_NORM)
        route_kernel<double><<<(T + 7) / 8, 256, 0, s>>>(scores, bias, token_ids, tid2eid, vocab, T, E, k, score,
                                                         hash_routing, route_scale, idx, weights, error_flag);
    else
        route_kernel<float><<<(T + 7) / 8, 256, 0, s>>>(scores, bias, token_ids, tid2eid, vocab, T, E, k, score,
                                                        hash_routing, route_scale, idx, weights, error_flag);
    return cudaGetLastError();
}

cudaError_t launch_moe(const MoeParams& p_in, cudaStream_t s, cudaEvent_t* ev) {
    cudaError_t e;
    if (ev) cudaEventRecord(ev[0], s);
    MoeParams p = p_in;
    // routing: router projection (or supplied logits) -> scores -> top-k; or given routes; or
    // half rows that arrive with their max|x| and one route each
    const bool given = p.routes_idx != nullptr;
    if (p.x_half) {
        routes_meta_kernel<<<(p.T + 255) / 256, 256, 0, s>>>(p.routes_meta, p.T, p.E, p.idx, p.weights, p.xmax,
                                                             p.counters + 3);
        e = cudaGetLastError();
    } else {
        if (p.hc_m) {
            // Hyper-Connection entry: split + reduced row + ffn norm, one CTA per token; the
            // combine writes the m copies back
            const size_t smem = hc_entry_smem(p.hc_m, p.H);
            if ((e = set_smem_once(hc_entry_kernel, smem)) != cudaSuccess) return e;
            MoeParams q = p;
            q.xd = (p.logits_in || given) ? nullptr : p.xd;
            hc_entry_kernel<<<p.T, 256, smem, s>>>(q);
            if ((e = cudaGetLastError()) != cudaSuccess) return e;
            p.hc_state = p.x;
            p.x = p.x_norm;
        } else if (p.norm_w) {
            // residual block entry: xn = RMSNorm(x) with each row's max|xn| (the prescale); the
            // layer then runs on xn and the combine adds x back
            if ((e = launch_rms_norm(p.x, p.norm_w, p.T, p.H, p.norm_eps, p.x_norm, p.xmax,
                                     (p.logits_in || given) ? nullptr : p.xd, s)) != cudaSuccess)
                return e;
            p.x_residual = p.x;
            p.x = p.x_norm;
        } else {
            token_prescale_kernel<<<dim3((p.H + 1023) / 1024, rows_grid(p.T)), 256, 0, s>>>(
                p.x, p.T, p.H, p.xmax, (p.logits_in || given) ? nullptr : p.xd);
            if ((e = cudaGetLastError()) != cudaSuccess) return e;
        }
        if (given) {
            const size_t n = (size_t)p.T * p.k;
            routes_copy_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(p.routes_idx, p.routes_w, n, p.E,
                                                                           p.idx, p.weights, p.counters + 3);
            e = cudaGetLastError();
        } else {
            if (p.logits_in) {
                e = launch_scores(p.logits_in, (size_t)p.T * p.E, p.score, p.scores, s);
            } else {
                e = launch_router(p.xd, p.router, p.T, p.H, p.E, p.score, p.logits, p.scores, s);
            }
            if (e != cudaSuccess) return e;
            e = launch_route(p.scores, p.bias, p.token_ids, p.tid2eid, p.vocab, p.T, p.E, p.k, p.score,
                             p.hash_routing, p.route_scale, p.idx, p.weights, p.counters + 3, s);
        }
    }
    if (e != cudaSuccess) return e;
    if (ev) cudaEventRecord(ev[1], s);
    const uint32_t n_el = p.T * p.k;
    if (n_el <= 4u * kDispatchThreads || !p.disp_counts) {
        const size_t dsmem = ((size_t)(p.E + 1) * 3 + 32u * p.E) * sizeof(uint32_t);
        if ((e = set_smem_once(dispatch_kernel, dsmem)) != cudaSuccess) return e;
        dispatch_kernel<<<1, kDispatchThreads, dsmem, s>>>(p);
    } else {
        const unsigned chunks = (n_el + kDispatchThreads - 1) / kDispatchThreads;
        dispatch_count_kernel<<<chunks, kDispatchThreads, 0, s>>>(p, p.disp_counts);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
        const size_t ssmem = ((size_t)(p.E + 1) * 2 + 32u * p.E) * sizeof(uint32_t);
        if ((e = set_smem_once(dispatch_scatter_kernel, ssmem)) != cudaSuccess) return e;
        dispatch_scatter_kernel<<<chunks, kDispatchThreads, ssmem, s>>>(p, p.disp_counts);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
        dispatch_finish_kernel<<<1, kDispatchThreads, 0, s>>>(p);
    }
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    if (ev) cudaEventRecord(ev[2], s);
    // experts
    const int ctas_per_sm = 2;
    const unsigned grid = (unsigned)(num_sms() * ctas_per_sm);
    if (p.prefill && (e = launch_prefill_plan(p, s)) != cudaSuccess) return e;
    // which kernel serves which storage type: the prefill GEMMs take IQ2_XXS and Q8_0; the decode
    // kernels take Q8_0 and one IQ type per phase (decode_ring_types); the CUDA-core kernels the rest
    const uint32_t pf_types = fmt_bit(kTypeIq2Xxs) | fmt_bit(kTypeQ8_0);
    const uint32_t gu_fast = p.prefill ? pf_types : decode_ring_types(p, true);
    const uint32_t dn_fast = p.prefill ? pf_types : decode_ring_types(p, false);
    const size_t gu_smem = kGridSmemBytes + (size_t)kUnitTokens * p.H * sizeof(float);
    if ((p.fmt_gu & ~gu_fast) && (e = set_smem_once(expert_kernel<true>, gu_smem)) != cudaSuccess) return e;
    if (p.fmt_gu & ~gu_fast) expert_kernel<true><<<grid, 256, gu_smem, s>>>(p, gu_fast);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    if ((p.fmt_gu & gu_fast) && p.prefill) {
        if ((e = launch_prefill_gateup(p, (unsigned)num_sms(), s)) != cudaSuccess) return e;
    } else if (p.fmt_gu & gu_fast) {
        if ((e = launch_decode_gateup(p, (unsigned)num_sms(), s)) != cudaSuccess) return e;
    }
    if (ev) cudaEventRecord(ev[3], s);
    const size_t dn_smem = kGridSmemBytes + (size_t)kUnitTokens * p.I * sizeof(float);
    if ((p.fmt_dn & ~dn_fast) && (e = set_smem_once(expert_kernel<false>, dn_smem)) != cudaSuccess) return e;
    if (p.fmt_dn & ~dn_fast) expert_kernel<false><<<grid, 256, dn_smem, s>>>(p, dn_fast);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    if ((p.fmt_dn & dn_fast) && p.prefill) {
        if ((e = launch_prefill_down(p, (unsigned)num_sms(), s)) != cudaSuccess) return e;
    } else if (p.fmt_dn & dn_fast) {
        if ((e = launch_decode_down(p, (unsigned)num_sms(), s)) != cudaSuccess) return e;
    }
    if (ev) cudaEventRecord(ev[4], s);
    if (!p.direct_out) {
        dim3 cg((p.H / 4 + 255) / 256, rows_grid(p.T));
        combine_kernel<<<cg, 256, 0, s>>>(p);
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    if (ev) cudaEventRecord(ev[5], s);
    return cudaSuccess;
}

// Stable placement of p.idx's T*k elements by expert (offsets, pair_token / pair_slot /
// pair_weight, combine_pairs = element -> position) without the layer tail: count + scatter.
// p.idx must hold ids < p.E. p.disp_counts: [ceil(T*k / 1024) x E].
cudaError_t launch_stable_sort(const MoeParams& p, cudaStream_t s) {
    const uint32_t n_el = p.T * p.k;
    if (n_el == 0) return cudaSuccess;
    const unsigned chunks = (n_el + kDispatchThreads - 1) / kDispatchThreads;
    dispatch_count_kernel<<<chunks, kDispatchThreads, 0, s>>>(p, p.disp_counts);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    const size_t ssmem = ((size_t)(p.E + 1) * 2 + 32u * p.E) * sizeof(uint32_t);
    if ((e = set_smem_once(dispatch_scatter_kernel, ssmem)) != cudaSuccess) return e;
    dispatch_scatter_kernel<<<chunks, kDispatchThreads, ssmem, s>>>(p, p.disp_counts);
    return cudaGetLastError();
}

bool hc_entry_fits(uint32_t m, uint32_t H) {
    if (m == 0 || m > 16 || H == 0 || ((size_t)m * H) % 256u) return false;
    return hc_entry_smem(m, H) <= kHcSmemLimit;
}

cudaError_t launch_rms_norm(const float* x, const float* w, uint32_t rows, uint32_t width,
                            float eps, float* out, uint32_t* xmax, double* out_d, cudaStream_t s) {
    if (width % 4u || width > kRmsMaxWidth) return cudaErrorInvalidValue;
    const size_t smem = (size_t)width * 8u;
    cudaError_t e = set_smem_once(rms_norm_kernel, smem);
    if (e != cudaSuccess) return e;
    rms_norm_kernel<<<rows, 256, smem, s>>>(x, w, width, eps, out, xmax, out_d);
    return cudaGetLastError();
}

}  // namespace vlb
