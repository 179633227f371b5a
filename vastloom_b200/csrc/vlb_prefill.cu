// Prefill expert products: a grouped GEMM on the 5th-generation tensor cores (tcgen05.mma, f32
// accumulators in tensor memory) with the block dequantization fused into the operand path.
//
// Reference semantics: the same expert loop as the decode path (deepseek_v4_graph.cpp:2134-2227,
// olmoe_runtime.cpp:1226-1285): gate = W1 x, up = W3 x, act = SwiGLU(gate, up) (times the route
// weight before the down projection for DeepSeek V4, after it for OLMoE), y = W2 act, combined per
// token. The products here round their operands to fp16, so the layer output matches the
// reference's f32/f64 sums to about 1e-3 relative (the contract for this path is 2e-2).
//
// Work decomposition. Dispatch sorts the (token, slot) pairs by expert; prefill_plan_kernel cuts
// each expert's pairs into column tiles of at most 160 pairs (balanced, so 300 pairs -> 150 + 150).
// One work item is (column tile, 128-row block): gate/up computes 128 rows of W1 AND the same 128
// rows of W3 into two TMEM accumulators and applies SwiGLU in the epilogue; down computes two
// 128-row tiles of W2 the same way. A persistent CTA per SM takes items from an atomic counter;
// the shared expert's tiles come first (heaviest).
//
// Data path of one 64-column stage:
//   packed weights: the stage's 128-row tile block column is contiguous in the tiled device
//     layout (8 KB of Q8_0 per matrix; an IQ2_XXS 256-column block covers four stages), so the
//     loader warp brings it into a shared-memory ring with one bulk copy per matrix;
//   A (weights): the producer warps decode their rows from that ring to fp16 in registers and
//     write them straight into tensor memory (tcgen05.st): the MMA reads A from TMEM;
//   B (activations): N rows of the pair-ordered fp16 matrix (xperm for gate/up, act_h for down),
//     TMA-loaded as 80-row boxes into a shared-memory ring (K-major, 128-byte swizzle).
// CTA roles (608 threads, one CTA per SM):
//   warps 0-15  producers: thread t owns half (t / 128 % 2) of the 64 stage columns of row t % 128
//               of accumulator t / 256 (its TMEM lane is its row). Afterwards they are the
//               epilogue: tcgen05.ld of the accumulators, scaling, SwiGLU, stores.
//   warp 16     loader: lanes 0-5 issue the packed-weight bulk copies of a stage at once.
//   warp 17     TMA: lane 0 issues the B boxes.
//   warp 18     MMA: lane 0 issues the MMAs (M = 128, N = tile, K = 16; 8 per stage), commits
//               each stage's A and B slots back and the finished accumulators to the epilogue.
// TMEM (512 columns): accumulators at columns 0 and 160 (N <= 160 each), three A slots at
// 320 + slot * 64 (+ 32 for the second accumulator's rows).
// Every wait is bounded by a 2 s time limit; a wait that runs out sets error bit 8 of the layer's
// flags and an abort word that makes every other wait of the CTA give up, so a fault in the
// pipeline ends the kernel (and the host call reports it) instead of hanging the GPU.
//
// Operand scaling (exact powers of two, removed in the epilogue):
//   weights:      fp16(w * pscale), pscale per matrix (upload time) keeps |w * pscale| < 2^14;
//   activations:  fp16(x * s_t), s_t brings max|x| of token t into [2^14, 2^15) (xmax of the
//                 routing prescale); act likewise per pair from act_max.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <mutex>
#include <utility>
#include <vector>

#include "vlb_launch.h"
#include "vlb_mma.cuh"
#include "vlb_tcgen05.cuh"

namespace vlb {
namespace {

constexpr uint32_t kPfM = 128;                       // rows per accumulator (MMA M)
constexpr uint32_t kPfMaxN = 160;                    // pairs per column tile (MMA N)
constexpr uint32_t kPfKc = 64;                       // columns per stage: one 128-byte fp16 row
constexpr uint32_t kPfProducerWarps = 16;
constexpr uint32_t kPfProducers = kPfProducerWarps * 32;
constexpr uint32_t kPfLoadWarp = kPfProducerWarps;
constexpr uint32_t kPfTmaWarp = kPfProducerWarps + 1;
constexpr uint32_t kPfMmaWarp = kPfProducerWarps + 2;
constexpr uint32_t kPfThreads = kPfProducers + 96;
// B rows per TMA box. The TMA unit spends a fixed time per box besides the bytes (measured on
// B200: a 160-row stage as ten 16-row boxes takes ~1,260 cycles, as two 80-row boxes ~750, the
// time of the stage's MMAs), so a stage loads ceil(N / rows) large boxes and ignores the rows
// past N.
#ifndef VLB_PF_BOX_ROWS
#define VLB_PF_BOX_ROWS 80
#endif
constexpr uint32_t kPfBoxRows = VLB_PF_BOX_ROWS;
// The packed-weight copies of a stage are issued by separate lanes in one instruction (measured:
// ~2% faster than one lane issuing them in turn; lanes that each take a branch of their own were
// ~20% slower).
#ifndef VLB_PF_RAW_LANES
#define VLB_PF_RAW_LANES 1
#endif
constexpr bool kPfRawLanes = VLB_PF_RAW_LANES != 0;
constexpr uint32_t kPfASlots = 3;                    // A operand buffers in TMEM
// shared memory: B ring, packed-weight ring, IQ2 table, per-tile scalars, barriers
constexpr uint32_t kPfBStages = 5;                   // B (activation) ring slots
constexpr uint32_t kPfRing = 6;                      // stage barrier ring (>= A and B slots)
constexpr uint32_t kPfBStage = kPfMaxN * kPfKc * 2;  // 20 KB
constexpr uint32_t kPfRawStages = 5;                 // packed-weight ring: ~85 KB in flight
constexpr uint32_t kPfRawBody = kTileRows * 64u;     // 8 KB per matrix: one tile block column
constexpr uint32_t kPfRawD = 512;                    // its block scales (<= 2 blocks x 128 rows)
constexpr uint32_t kPfRawSc = kTileRows * 4u;        // IQ2_XXS group scale words (128 rows x u32)
constexpr uint32_t kPfRawStage = 2 * kPfRawBody + 2 * kPfRawD + 2 * kPfRawSc;
constexpr uint32_t kPfRawOff = kPfBStages * kPfBStage;
constexpr uint32_t kPfTabOff = kPfRawOff + kPfRawStages * kPfRawStage;
constexpr uint32_t kPfTabBytes = 256u * 8u * 16u;    // fp16 IQ2_XXS magnitudes, 8 replicas
constexpr uint32_t kPfInvOff = kPfTabOff + kPfTabBytes;
constexpr uint32_t kPfPwOff = kPfInvOff + kPfMaxN * 4;
constexpr uint32_t kPfBarOff = kPfPwOff + kPfMaxN * 4;
constexpr uint32_t kPfBars = 2 * kPfRawStages + 2 * kPfRing + 1;
constexpr uint32_t kPfSmemBytes = kPfBarOff + kPfBars * 8 + 32;
// tensor memory
constexpr uint32_t kPfTmemCols = 512;
constexpr uint32_t kPfAcc1Col = kPfMaxN;             // second accumulator's first column
constexpr uint32_t kPfACol = 2 * kPfMaxN;            // A slots
constexpr uint64_t kPfWaitNs = 2000000000ull;        // 2 s: no wait in a healthy kernel comes close
constexpr uint32_t kPfSleepNs = 20000;               // suspend hint of the mostly-waiting lanes
#ifndef VLB_PF_BACKOFF_NS
#define VLB_PF_BACKOFF_NS 128
#endif
// Producer warps park between polls: a spinning lane 0 in each of 16 warps would take the issue
// slots the decode and MMA lanes need.
constexpr uint32_t kPfBackoffNs = VLB_PF_BACKOFF_NS;
constexpr uint32_t kPfErrTimeout = 8u;
constexpr uint32_t kPfErrAlign = 16u;

static_assert(kPfSmemBytes <= 232448, "prefill rings exceed the shared memory of a CTA");
static_assert(kPfBStage % 1024 == 0 && kPfRawOff % 1024 == 0, "swizzle atoms must stay 1 KB aligned");
static_assert(kPfBoxRows * 128 % 1024 == 0, "TMA boxes must start on swizzle-atom boundaries");
static_assert(kPfMaxN % kPfBoxRows == 0 && kPfBoxRows <= 256, "a stage's boxes must fill its B slot exactly");
static_assert(kPfACol + kPfASlots * 64 <= kPfTmemCols, "TMEM budget");
static_assert(kPfRing >= kPfBStages + 1 && kPfRing >= kPfASlots + 1,
              "a slot's waiter must never fall two phases behind on the stage barrier ring");

__device__ __forceinline__ bool pf_mma_type(uint32_t t) { return t == kTypeIq2Xxs || t == kTypeQ8_0; }

// Waits for `parity` of `bar`; false when the CTA aborted or the time limit ran out. sleep_ns > 0
// lets the hardware suspend the thread inside each test; backoff_ns > 0 parks the warp between
// tests (a polling warp otherwise takes issue slots from the warps doing the work).
__device__ __forceinline__ bool pf_wait(uint64_t* bar, uint32_t parity, volatile uint32_t* abort,
                                        uint32_t sleep_ns, uint32_t backoff_ns = 0) {
    uint64_t t0 = 0;
    for (uint32_t i = 1;; ++i) {
        if (sleep_ns ? tc::mbar_try_sleep(bar, parity, sleep_ns) : tc::mbar_try(bar, parity)) return true;
        if (backoff_ns) __nanosleep(backoff_ns);
        if (sleep_ns || backoff_ns || (i & 63u) == 0) {
            if (*abort) return false;
            const uint64_t now = tc::global_ns();
            if (t0 == 0) t0 = now;
            else if (now - t0 > kPfWaitNs) return false;
            if (i >= (1u << 30)) return false;
        }
    }
}

__device__ __forceinline__ void pf_fail(uint32_t* flags, volatile uint32_t* abort) {
    *abort = 1u;
    atomicOr(flags, kPfErrTimeout);
}

// A producer warp's wait: lane 0 polls, the outcome is broadcast (and the warp reconverged).
__device__ __forceinline__ bool pf_wait_warp(uint64_t* bar, uint32_t parity, volatile uint32_t* abort) {
    bool ok = true;
    if ((threadIdx.x & 31u) == 0) ok = pf_wait(bar, parity, abort, 0, kPfBackoffNs);
    return __shfl_sync(0xffffffffu, ok ? 1u : 0u, 0) != 0;
}

// A producer warp's arrival: every lane's prior shared-memory reads and TMEM stores are ordered
// before lane 0's (release) arrival by the warp barrier; the mbarrier counts warps.
__device__ __forceinline__ void pf_arrive_warp(uint64_t* bar) {
    __syncwarp();
    if ((threadIdx.x & 31u) == 0) tc::mbar_arrive(bar);
}

// Position in a ring of n slots: slot and the parity of the slot's current use.
struct PfPos {
    uint32_t slot, ph;
    __device__ __forceinline__ void next(uint32_t n) {
        if (++slot == n) {
            slot = 0;
            ph ^= 1u;
        }
    }
};

__device__ __forceinline__ uint32_t h2_bits(float v) {
    const uint32_t u = __half_as_ushort(__float2half_rn(v));
    return u | (u << 16);
}

__device__ __forceinline__ uint32_t lds_u16(uint32_t addr) {
    unsigned short v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
    return v;
}

__device__ __forceinline__ uint32_t lds_u32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}

__device__ __forceinline__ uint4 lds_u4(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
    return v;
}

// Operand stages are numbered globally across the CTA's items (g = 0, 1, ...). Stage g uses A slot
// g % kPfASlots (TMEM), B slot g % kPfBStages (shared memory) and one pair of barriers, index
// g % kPfRing: full (16 producer-warp arrivals + the TMA lane's transaction bytes) and empty (one
// tcgen05.commit after the stage's MMAs, which frees both slots). One commit per stage matters:
// every commit costs the tensor pipe a short drain. The producers reuse an A slot after stage
// g - kPfASlots's commit, the TMA lane a B slot after stage g - kPfBStages's.
struct PfBars {
    uint64_t* raw_full;   // [kPfRawStages]  loader -> producers (bulk-copy bytes)
    uint64_t* raw_empty;  // [kPfRawStages]  producers -> loader
    uint64_t* full;       // [kPfRing]       producers + TMA bytes -> MMA
    uint64_t* empty;      // [kPfRing]       MMA commit -> producers, TMA
    uint64_t* acc_full;   //                 MMA commit -> epilogue
    volatile uint32_t* abort;
};

// Waits until stage g's commit (if g is a real stage: g >= 0) freed its slots.
__device__ __forceinline__ bool pf_wait_freed(const PfBars& br, int64_t g, uint32_t sleep_ns, uint32_t backoff_ns = 0) {
    if (g < 0) return true;
    return pf_wait(br.empty + (uint32_t)(g % kPfRing), (uint32_t)((g / kPfRing) & 1), br.abort, sleep_ns,
                   backoff_ns);
}

// ---- decode of one half-row stage to 16 fp16x2 words --------------------------------------------
// Q8_0 (decode_q8_0_block, ggml_quantization.cpp:419-435): w = d * q. q is an exact fp16, d * pscale
// too (a power-of-two scaling of an fp16); their product rounds once.
__device__ __forceinline__ void pf_decode_q8(uint4 q0, uint4 q1, uint32_t dbits, float ps, uint32_t (&v)[16]) {
    const uint32_t dh = h2_bits(h2f((uint16_t)dbits) * ps);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint4 q = j < 2 ? q0 : q1;
        uint32_t t[4];
        mma::decode_q8_sub((j & 1) ? q.z : q.x, (j & 1) ? q.w : q.y, t);
#pragma unroll
        for (int i = 0; i < 4; ++i) v[4 * j + i] = mma::hmul2(t[i], dh);
    }
}

// IQ2_XXS (decode_iq2_xxs_block, ggml_quantization.cpp:250-283): w = d * (0.5 + s) / 4 * m * sign.
// The group factor fp16(d * pscale * (0.5 + s) / 4) rounds once, its product with the exact grid
// magnitude m once more; the sign is a bit flip (pair-layout sign word `sw`, 4-bit scale `s4`).
__device__ __forceinline__ void pf_decode_iq2(uint32_t idx4, uint32_t sw, uint32_t s4, float d, const uint4* tab,
                                              uint32_t lane7, uint32_t (&v)[16]) {
    const uint32_t kk = h2_bits(d * (0.5f + (float)s4) * 0.25f);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        uint32_t t[4];
        mma::decode_iq2_sub(tab, lane7, idx4, sw, (uint32_t)j, kk, t);
#pragma unroll
        for (int i = 0; i < 4; ++i) v[4 * j + i] = t[i];
    }
}

// Issues the TMEM store of one decoded half-row stage (32 fp16 = 16 columns) into the A slot of
// global stage g once stage g - kPfASlots's MMAs released it. Completion is published later by
// pf_publish_a, so the warp decodes the next stage while the store is in flight.
__device__ __forceinline__ bool pf_store_a(const PfBars& br, uint32_t g, uint32_t taddr, const uint32_t (&v)[16]) {
    bool ok = true;
    if ((threadIdx.x & 31u) == 0) ok = pf_wait_freed(br, (int64_t)g - kPfASlots, 0, kPfBackoffNs);
    if (__shfl_sync(0xffffffffu, ok ? 1u : 0u, 0) == 0) return false;
    tc::fence_after_sync();
    tc::tmem_st16(taddr + (g % kPfASlots) * 64u, v);
    return true;
}

// Waits for the warp's outstanding TMEM store and arrives on stage g's full barrier.
__device__ __forceinline__ void pf_publish_a(const PfBars& br, uint32_t g) {
    tc::tmem_wait_st();
    tc::fence_before_sync();
    pf_arrive_warp(br.full + g % kPfRing);
}

// Q8_0 raw stage -> decoded half-row (block `half` of the stage's two, row r).
__device__ __forceinline__ bool pf_fetch_q8(const PfBars& br, uint32_t smem, uint32_t rs, uint32_t acc, uint32_t half,
                                            uint32_t r, float ps, uint32_t (&v)[16]) {
    const uint32_t rslot = rs % kPfRawStages;
    if (!pf_wait_warp(br.raw_full + rslot, (rs / kPfRawStages) & 1u, br.abort)) return false;
    const uint32_t st = smem + kPfRawOff + rslot * kPfRawStage;
    const uint32_t body = st + acc * kPfRawBody + (half * kTileRows + r) * 32u;
    const uint4 q0 = lds_u4(body), q1 = lds_u4(body + 16u);
    const uint32_t dbits = lds_u16(st + 2u * kPfRawBody + acc * kPfRawD + (half * kTileRows + r) * 2u);
    pf_arrive_warp(br.raw_empty + rslot);
    pf_decode_q8(q0, q1, dbits, ps, v);
    return true;
}

// One producer thread's main loop over an item: packed weights from the shared ring, decoded,
// into its TMEM lane, software-pipelined so that stage kc + 1's decode overlaps stage kc's TMEM
// store. g0 / rs0: global numbers of the item's first stage / raw stage.
template <uint32_t FMT>
__device__ __forceinline__ bool pf_produce(const PfBars& br, uint32_t smem, const uint4* tab, float ps,
                                           uint32_t acc, uint32_t half, uint32_t r, uint32_t t_a,
                                           uint32_t nk, uint32_t g0, uint32_t rs0) {
    const uint32_t lane7 = threadIdx.x & 7u;
    if constexpr (FMT == kTypeQ8_0) {
        // one raw stage per operand stage
        uint32_t v[16];
        if (!pf_fetch_q8(br, smem, rs0, acc, half, r, ps, v)) return false;
        for (uint32_t kc = 0; kc < nk; ++kc) {
            if (!pf_store_a(br, g0 + kc, t_a, v)) return false;
            if (kc + 1u < nk && !pf_fetch_q8(br, smem, rs0 + kc + 1u, acc, half, r, ps, v)) {
                tc::tmem_wait_st();
                return false;
            }
            pf_publish_a(br, g0 + kc);
        }
    } else {
        // one raw stage (a 256-column block) per four operand stages; this thread's groups are
        // half, 2 + half, 4 + half, 6 + half
        for (uint32_t kb = 0; kb < nk / 4u; ++kb) {
            const uint32_t rs = rs0 + kb, rslot = rs % kPfRawStages;
            if (!pf_wait_warp(br.raw_full + rslot, (rs / kPfRawStages) & 1u, br.abort)) return false;
            const uint32_t st = smem + kPfRawOff + rslot * kPfRawStage;
            const uint32_t body = st + acc * kPfRawBody + r * 64u;
            const uint4 c0 = lds_u4(body), c1 = lds_u4(body + 16u), c2 = lds_u4(body + 32u), c3 = lds_u4(body + 48u);
            const uint32_t dbits = lds_u16(st + 2u * kPfRawBody + acc * kPfRawD + r * 2u);
            const uint32_t scw = lds_u32(st + 2u * kPfRawBody + 2u * kPfRawD + acc * kPfRawSc + r * 4u);
            pf_arrive_warp(br.raw_empty + rslot);
            const float d = h2f((uint16_t)dbits) * ps;
            uint32_t v[16];
            pf_decode_iq2(half ? c0.z : c0.x, half ? c0.w : c0.y, (scw >> (4u * half)) & 15u, d, tab, lane7, v);
#pragma unroll
            for (uint32_t sub = 0; sub < 4u; ++sub) {  // groups 2 sub, 2 sub + 1
                const uint32_t g = g0 + 4u * kb + sub;
                if (!pf_store_a(br, g, t_a, v)) return false;
                if (sub < 3u) {
                    const uint4 c = sub == 0 ? c1 : sub == 1 ? c2 : c3;
                    pf_decode_iq2(half ? c.z : c.x, half ? c.w : c.y, (scw >> (4u * (2u * sub + 2u + half))) & 15u, d,
                                  tab, lane7, v);
                }
                pf_publish_a(br, g);
            }
        }
    }
    return true;
}

// Loader warp: the item's packed weights, one bulk copy per matrix body and per scale run. Lane 0
// waits for the ring slot and registers the stage's bytes; the copies are issued by lanes 2 c + i
// (matrix i, copy c: 0 packed weights, 1 block scales, 2 group scales) at once, since a bulk copy
// holds its issuing thread for a few hundred cycles. Every lane of the warp runs this.
__device__ __forceinline__ bool pf_load_raw(const PfBars& br, uint32_t smem, const DevMat& m0, const DevMat& m1,
                                            uint32_t rt0, uint32_t rt1, uint32_t nk, PfPos& raw) {
    const uint32_t lane = threadIdx.x & 31u;
    const bool q8 = m0.type == kTypeQ8_0;
    const uint32_t stages = q8 ? nk : nk / 4u;
    const uint32_t dbytes = q8 ? 2u * kTileRows * 2u : kTileRows * 2u;
    for (uint32_t rs = 0; rs < stages; ++rs) {
        bool ok = true;
        if (lane == 0) ok = pf_wait(br.raw_empty + raw.slot, raw.ph ^ 1u, br.abort, kPfSleepNs);
        if (__shfl_sync(0xffffffffu, ok ? 1u : 0u, 0) == 0) return false;
        const uint32_t dst = smem + kPfRawOff + raw.slot * kPfRawStage;
        if (lane == 0)
            tc::mbar_arrive_expect_tx(br.raw_full + raw.slot, 2u * (kPfRawBody + dbytes + (q8 ? 0u : kPfRawSc)));
        __syncwarp();
        const uint32_t blk = q8 ? 2u * rs : rs;
        if (kPfRawLanes) {
            // lane 2 c + i: copy c of matrix i, all issued by one instruction
            if (lane < (q8 ? 4u : 6u)) {
                const uint32_t i = lane & 1u, c = lane >> 1;
                const DevMat* m = i ? &m1 : &m0;
                const size_t at = blk_index(m->bpr, (i ? rt1 : rt0) * kTileRows, blk);
                const void* src = c == 0u ? (const void*)(m->body + at * (q8 ? 32u : 64u))
                                  : c == 1u ? (const void*)(m->d + at) : (const void*)(m->scales + at);
                const uint32_t to = c == 0u ? dst + i * kPfRawBody
                                    : c == 1u ? dst + 2u * kPfRawBody + i * kPfRawD
                                              : dst + 2u * kPfRawBody + 2u * kPfRawD + i * kPfRawSc;
                const uint32_t bytes = c == 0u ? kPfRawBody : c == 1u ? dbytes : kPfRawSc;
                tc::bulk_load(to, src, bytes, br.raw_full + raw.slot);
            }
        } else if (lane == 0) {
#pragma unroll
            for (uint32_t i = 0; i < 2u; ++i) {
                const DevMat& m = i ? m1 : m0;
                const size_t at = blk_index(m.bpr, (i ? rt1 : rt0) * kTileRows, blk);
                tc::bulk_load(dst + i * kPfRawBody, m.body + at * (q8 ? 32u : 64u), kPfRawBody, br.raw_full + raw.slot);
                tc::bulk_load(dst + 2u * kPfRawBody + i * kPfRawD, m.d + at, dbytes, br.raw_full + raw.slot);
                if (!q8)
                    tc::bulk_load(dst + 2u * kPfRawBody + 2u * kPfRawD + i * kPfRawSc, m.scales + at, kPfRawSc,
                                  br.raw_full + raw.slot);
            }
        }
        __syncwarp();
        raw.next(kPfRawStages);
    }
    return true;
}

// TMA lane: per stage, the B rows of the tile (pair order, starting at row0) as ceil(N / box)
// boxes; rows past N land in the slot unused (past the matrix end the TMA unit fills zeros).
__device__ __forceinline__ bool pf_load_b(const PfBars& br, uint32_t smem, const CUtensorMap* map,
                                          uint32_t row0, uint32_t nk, uint32_t N, uint32_t g0) {
    const uint32_t nbox = (N + kPfBoxRows - 1u) / kPfBoxRows;
    for (uint32_t kc = 0; kc < nk; ++kc) {
        const uint32_t g = g0 + kc, bar = g % kPfRing;
        if (!pf_wait_freed(br, (int64_t)g - kPfBStages, kPfSleepNs)) return false;
        tc::mbar_arrive_expect_tx(br.full + bar, nbox * kPfBoxRows * kPfKc * 2u);
        const uint32_t dst = smem + (g % kPfBStages) * kPfBStage;
        for (uint32_t j = 0; j < nbox; ++j)
            tc::tma_load_2d(dst + j * kPfBoxRows * 128u, map, (int32_t)(kc * kPfKc), (int32_t)(row0 + j * kPfBoxRows),
                            br.full + bar);
    }
    return true;
}

// MMA lane: per stage, 4 K-steps x 2 accumulators with A from TMEM and B from shared memory, then
// one commit that frees the stage's slots.
__device__ __forceinline__ bool pf_mma(const PfBars& br, uint32_t smem, uint32_t tmem, uint32_t nk, uint32_t N,
                                       uint32_t g0, bool& pending) {
    const uint32_t idesc = tc::idesc_f16(kPfM, N);
    for (uint32_t kc = 0; kc < nk; ++kc) {
        const uint32_t g = g0 + kc, bar = g % kPfRing;
        if (!pf_wait(br.full + bar, (g / kPfRing) & 1u, br.abort, kPfSleepNs)) return false;
        tc::fence_after_sync();
        const uint32_t bs = smem + (g % kPfBStages) * kPfBStage;
        const uint32_t ta = tmem + kPfACol + (g % kPfASlots) * 64u;
        pending = true;
#pragma unroll
        for (uint32_t ks = 0; ks < kPfKc / 16u; ++ks) {
            const uint64_t bd = tc::sw128_desc(bs + ks * 32u);
            const uint32_t accumulate = (kc | ks) ? 1u : 0u;
            tc::mma_f16_ts(tmem, ta + ks * 8u, bd, idesc, accumulate);
            tc::mma_f16_ts(tmem + kPfAcc1Col, ta + 32u + ks * 8u, bd, idesc, accumulate);
        }
        tc::mma_commit(br.empty + bar);
    }
    tc::mma_commit(br.acc_full);
    pending = false;
    return true;
}

// silu(g) * u from the definition g / (1 + e^-g), with the approximate exponential and reciprocal
// (relative error ~1e-6, far inside the prefill tolerance); e^-g = inf gives 0.
__device__ __forceinline__ float pf_silu_mul(float g, float u) {
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.f + __expf(-g)));
    return g * r * u;
}

// Max over the 32 lanes of each of 8 columns, as a reduce-scatter: on return lane l holds the
// maximum of column (l >> 2) & 7 (9 shuffles instead of 40).
__device__ __forceinline__ float pf_colmax8(const float (&v)[8]) {
    const uint32_t lane = threadIdx.x & 31u;
    float a4[4], a2[2];
    const bool b4 = lane & 16u, b3 = lane & 8u, b2 = lane & 4u;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float mine = b4 ? v[4 + i] : v[i], other = b4 ? v[i] : v[4 + i];
        a4[i] = fmaxf(mine, __shfl_xor_sync(0xffffffffu, other, 16));
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const float mine = b3 ? a4[2 + i] : a4[i], other = b3 ? a4[i] : a4[2 + i];
        a2[i] = fmaxf(mine, __shfl_xor_sync(0xffffffffu, other, 8));
    }
    float a1 = fmaxf(b2 ? a2[1] : a2[0], __shfl_xor_sync(0xffffffffu, b2 ? a2[0] : a2[1], 4));
    a1 = fmaxf(a1, __shfl_xor_sync(0xffffffffu, a1, 2));
    return fmaxf(a1, __shfl_xor_sync(0xffffffffu, a1, 1));
}

// Gate/up epilogue: warp w reads TMEM lanes 32 (w % 4) .. +31 (rows) and every fourth 8-column
// chunk starting at w / 4; writes act (f32) and the per-pair max |act|.
__device__ __forceinline__ void pf_epilogue_gateup(const MoeParams& p, uint32_t tmem, const Unit& tile,
                                                   uint32_t N, uint32_t row0, float inv_ps0,
                                                   float inv_ps1, const float* tok_inv,
                                                   const float* pw) {
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u, lq = warp & 3u;
    const uint32_t row = row0 + 32u * lq + lane;
    const uint32_t t_lane = tmem + ((32u * lq) << 16);
    const bool shared = tile.expert == p.E;
    const float limit = shared ? p.shared_limit : p.routed_limit;
    const bool clamp = !p.weight_after_down && limit > 0.f;
    const bool weigh = !p.weight_after_down && !shared;
    for (uint32_t j = warp >> 2; 8u * j < N; j += 4u) {
        float g[8], u[8];
        tc::tmem_ld8(t_lane + 8u * j, g);
        tc::tmem_ld8(t_lane + kPfAcc1Col + 8u * j, u);
        tc::tmem_wait_ld();
        const uint32_t n0 = 8u * j;
        float m[8];
#pragma unroll
        for (uint32_t i = 0; i < 8u; ++i) {
            m[i] = 0.f;
            const uint32_t n = n0 + i;
            if (n < tile.count) {
                const float inv = tok_inv[n];
                float gv = g[i] * inv * inv_ps0, uv = u[i] * inv * inv_ps1;
                if (clamp) {
                    gv = fminf(gv, limit);
                    uv = fminf(fmaxf(uv, -limit), limit);
                }
                float a = pf_silu_mul(gv, uv);
                if (weigh) a *= pw[n];
                p.act[(size_t)(tile.pair_begin + n) * p.I + row] = a;
                m[i] = fabsf(a);
            }
        }
        const float cm = pf_colmax8(m);
        const uint32_t col = (lane >> 2) & 7u;
        if ((lane & 3u) == 0 && n0 + col < tile.count)
            atomicMax(p.act_max + tile.pair_begin + n0 + col, __float_as_uint(cm));
    }
}

// Down epilogue: the two accumulators are rows row0.. and row0 + 128.. of W2; y in f32.
__device__ __forceinline__ void pf_epilogue_down(const MoeParams& p, uint32_t tmem, const Unit& tile,
                                                 uint32_t N, uint32_t row0, float inv_ps,
                                                 const float* tok_inv) {
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31u, lq = warp & 3u;
    const uint32_t r0 = row0 + 32u * lq + lane, r1 = r0 + kPfM;
    const uint32_t t_lane = tmem + ((32u * lq) << 16);
    for (uint32_t j = warp >> 2; 8u * j < N; j += 4u) {
        float a[8], b[8];
        tc::tmem_ld8(t_lane + 8u * j, a);
        tc::tmem_ld8(t_lane + kPfAcc1Col + 8u * j, b);
        tc::tmem_wait_ld();
#pragma unroll
        for (uint32_t i = 0; i < 8u; ++i) {
            const uint32_t n = 8u * j + i;
            if (n < tile.count) {
                const float inv = tok_inv[n] * inv_ps;
                const uint32_t pair = tile.pair_begin + n;
                float* yr = p.direct_out ? p.out + (size_t)p.pair_token[pair] * p.H : p.y + (size_t)pair * p.H;
                yr[r0] = a[i] * inv;
                yr[r1] = b[i] * inv;
            }
        }
    }
}

template <bool GATEUP>
__global__ void __launch_bounds__(kPfThreads, 1) prefill_gemm_kernel(const __grid_constant__ MoeParams p) {
    extern __shared__ __align__(1024) unsigned char pf_smem[];
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31u;
    const uint32_t smem = tc::smem_u32(pf_smem);
    if (smem & 1023u) {  // the swizzle atoms need 1 KB alignment; uniform across the CTA
        if (tid == 0) atomicOr(p.counters + 3, kPfErrAlign);
        return;
    }
    const uint4* tab = reinterpret_cast<const uint4*>(pf_smem + kPfTabOff);
    float* tok_inv = reinterpret_cast<float*>(pf_smem + kPfInvOff);
    float* pw = reinterpret_cast<float*>(pf_smem + kPfPwOff);
    uint64_t* bars = reinterpret_cast<uint64_t*>(pf_smem + kPfBarOff);
    uint32_t* misc = reinterpret_cast<uint32_t*>(bars + kPfBars);  // [0] TMEM base [1] item [2] abort
    PfBars br;
    br.raw_full = bars;
    br.raw_empty = br.raw_full + kPfRawStages;
    br.full = br.raw_empty + kPfRawStages;
    br.empty = br.full + kPfRing;
    br.acc_full = br.empty + kPfRing;
    br.abort = misc + 2;
    const CUtensorMap* bmap = GATEUP ? &p.bmap_x : &p.bmap_act;
    if (warp == kPfMmaWarp) tc::tmem_alloc(misc, kPfTmemCols);
    if (tid == 0) {
        for (uint32_t i = 0; i < kPfRawStages; ++i) {
            tc::mbar_init(br.raw_full + i, 1);
            tc::mbar_init(br.raw_empty + i, kPfProducerWarps);
        }
        for (uint32_t i = 0; i < kPfRing; ++i) {
            tc::mbar_init(br.full + i, kPfProducerWarps + 1);  // producer warps + the TMA lane
            tc::mbar_init(br.empty + i, 1);
        }
        tc::mbar_init(br.acc_full, 1);
        misc[2] = 0;
        tc::mbar_fence_init();
    }
    if (warp == kPfTmaWarp && lane == 0)
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(bmap)) : "memory");
    mma::build_iq2_table(reinterpret_cast<uint4*>(pf_smem + kPfTabOff), p.grids.iq2xxs);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = misc[0];

    const uint32_t K = GATEUP ? p.H : p.I;
    const uint32_t nk = K / kPfKc;
    const uint32_t per_tile = GATEUP ? p.I / kPfM : p.H / (2u * kPfM);
    const uint32_t n_items = p.counters[7] * per_tile;
    uint32_t* next = p.counters + (GATEUP ? 5 : 6);
    // producer geometry: row r of accumulator acc, column half `half` of each stage; its TMEM
    // lane is r (warp % 4 == r / 32), its A columns 16 * half of the accumulator's 32 per slot
    const uint32_t acc = tid >> 8, half = (tid >> 7) & 1u, r = tid & (kPfM - 1u);
    const uint32_t t_a = tmem + ((32u * (warp & 3u)) << 16) + kPfACol + acc * 32u + half * 16u;
    PfPos raw{0, 0};
    uint32_t gs0 = 0, rs0 = 0;  // global stage / raw-stage numbers of the item's first
    uint32_t item_it = 0, pending_parity = 0;
    bool pending = false, copies_dirty = false;
    for (;;) {
        __syncthreads();
        if (tid == 0) misc[1] = *br.abort ? 0xffffffffu : atomicAdd(next, 1u);
        __syncthreads();
        const uint32_t item = misc[1];
        if (item >= n_items) break;
        const Unit tile = p.ptiles[item / per_tile];
        const uint32_t mi = item % per_tile;
        const DevMat* m0 = p.mats + (GATEUP ? 0u : 2u * (p.E + 1)) + tile.expert;
        const DevMat* m1 = GATEUP ? p.mats + (p.E + 1) + tile.expert : m0;
        const uint32_t type = m0->type;
        if (!pf_mma_type(type)) continue;  // served by the CUDA-core expert kernels
        const uint32_t N = (tile.count + 15u) & ~15u;
        // row tiles (128 rows) of the two accumulators
        const uint32_t rt0 = GATEUP ? mi : 2u * mi, rt1 = GATEUP ? mi : 2u * mi + 1u;
        if (tid < tile.count) {
            const uint32_t pair = tile.pair_begin + tid;
            const uint32_t bits = GATEUP ? p.xmax[p.pair_token[pair]] : p.act_max[pair];
            tok_inv[tid] = 1.f / mma::prescale_for(__uint_as_float(bits));
            pw[tid] = p.pair_weight[pair];
        }
        __syncthreads();
        if (warp < kPfProducerWarps) {
            const float ps = (acc ? m1 : m0)->pscale;
            bool ok = type == kTypeQ8_0
                          ? pf_produce<kTypeQ8_0>(br, smem, tab, ps, acc, half, r, t_a, nk, gs0, rs0)
                          : pf_produce<kTypeIq2Xxs>(br, smem, tab, ps, acc, half, r, t_a, nk, gs0, rs0);
            ok = __all_sync(0xffffffffu, ok);
            if (ok) ok = pf_wait_warp(br.acc_full, item_it & 1u, br.abort);
            if (ok) {
                tc::fence_after_sync();
                if (GATEUP)
                    pf_epilogue_gateup(p, tmem, tile, N, rt0 * kPfM, 1.f / m0->pscale, 1.f / m1->pscale, tok_inv, pw);
                else
                    pf_epilogue_down(p, tmem, tile, N, rt0 * kPfM, 1.f / m0->pscale, tok_inv);
            } else {
                pf_fail(p.counters + 3, br.abort);
            }
            tc::fence_before_sync();
        } else if (warp == kPfLoadWarp) {
            copies_dirty = true;
            if (pf_load_raw(br, smem, *m0, *m1, rt0, rt1, nk, raw)) copies_dirty = false;
            else if (lane == 0) pf_fail(p.counters + 3, br.abort);
        } else if (warp == kPfTmaWarp) {
            if (lane == 0) {
                copies_dirty = true;
                if (pf_load_b(br, smem, bmap, tile.pair_begin, nk, N, gs0)) copies_dirty = false;
                else pf_fail(p.counters + 3, br.abort);
            }
        } else if (lane == 0) {
            pending_parity = item_it & 1u;
            if (!pf_mma(br, smem, tmem, nk, N, gs0, pending)) pf_fail(p.counters + 3, br.abort);
        }
        ++item_it;
        gs0 += nk;
        rs0 += type == kTypeQ8_0 ? nk : nk / 4u;
    }
    __syncthreads();
    if ((warp == kPfLoadWarp || warp == kPfTmaWarp) && lane == 0 && copies_dirty) {
        // after an abort, let copies already issued land before the CTA's shared memory goes away
        const uint64_t t0 = tc::global_ns();
        while (tc::global_ns() - t0 < 1000000ull) {
        }
    }
    if (warp == kPfMmaWarp) {
        // after an abort, MMAs already issued must finish before their TMEM is released
        if (lane == 0 && pending) {
            tc::mma_commit(br.acc_full);
            const uint64_t t0 = tc::global_ns();
            while (!tc::mbar_try(br.acc_full, pending_parity) && tc::global_ns() - t0 < kPfWaitNs) {
            }
        }
        __syncwarp();
        tc::fence_after_sync();
        tc::tmem_dealloc(tmem, kPfTmemCols);
    }
    __syncthreads();
}

// Column tiles of every expert's pairs (the shared expert first): an expert with c pairs gets
// ceil(c / 256) tiles of balanced size. One CTA.
__global__ void __launch_bounds__(512) prefill_plan_kernel(MoeParams p) {
    __shared__ uint32_t nt[513];
    __shared__ uint32_t warp_sum[16];
    const uint32_t E = p.E, n = p.T * p.k, tid = threadIdx.x;
    auto count_of = [&](uint32_t o, uint32_t* begin, uint32_t* expert) -> uint32_t {
        if (o == 0) {
            *begin = n;
            *expert = E;
            return p.has_shared ? p.T : 0u;
        }
        *begin = p.offsets[o - 1];
        *expert = o - 1;
        return p.offsets[o] - p.offsets[o - 1];
    };
    // exclusive scan of the tile counts over ordinals 0..E, blockDim.x ordinals per pass
    uint32_t running = 0;
    for (uint32_t base = 0; base <= E; base += blockDim.x) {
        const uint32_t o = base + tid;
        uint32_t b, e, c = 0;
        if (o <= E) c = count_of(o, &b, &e);
        const uint32_t v = (c + kPfMaxN - 1u) / kPfMaxN;
        uint32_t incl = v;
        const uint32_t lane = tid & 31u, w = tid >> 5;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const uint32_t y = __shfl_up_sync(0xffffffffu, incl, d);
            if (lane >= (uint32_t)d) incl += y;
        }
        if (lane == 31) warp_sum[w] = incl;
        __syncthreads();
        uint32_t before = running;
        for (uint32_t i = 0; i < w; ++i) before += warp_sum[i];
        if (o <= E) nt[o] = before + incl - v;  // exclusive
        uint32_t total = 0;
        for (uint32_t i = 0; i < blockDim.x / 32u; ++i) total += warp_sum[i];
        __syncthreads();
        running += total;
    }
    for (uint32_t o = tid; o <= E; o += blockDim.x) {
        uint32_t b, e;
        const uint32_t c = count_of(o, &b, &e);
        const uint32_t tiles = (c + kPfMaxN - 1u) / kPfMaxN;
        for (uint32_t j = 0; j < tiles; ++j) {
            const uint32_t at = nt[o] + j;
            if (at >= p.max_ptiles) break;
            const uint32_t lo = (uint32_t)((uint64_t)c * j / tiles), hi = (uint32_t)((uint64_t)c * (j + 1) / tiles);
            p.ptiles[at] = Unit{e, b + lo, hi - lo, 0u};
        }
    }
    if (tid == 0) p.counters[7] = running < p.max_ptiles ? running : p.max_ptiles;
}

// Pair-ordered fp16 activations: xperm[pair] = fp16(x[token(pair)] * s_token). 4 columns a thread;
// rows strided over gridDim.y (limited to 65535).
__global__ void __launch_bounds__(256) prefill_gather_kernel(const float* __restrict__ x,
                                                             const uint32_t* __restrict__ pair_token,
                                                             const uint32_t* __restrict__ xmax, uint32_t rows,
                                                             uint32_t width, __half* __restrict__ dst) {
    const uint32_t c = (blockIdx.x * blockDim.x + threadIdx.x) * 4u;
    if (c >= width) return;
    for (uint32_t pr = blockIdx.y; pr < rows; pr += gridDim.y) {
        const uint32_t t = pair_token[pr];
        const float s = mma::prescale_for(__uint_as_float(xmax[t]));
        const float4 v = *reinterpret_cast<const float4*>(x + (size_t)t * width + c);
        const __half2 a = __floats2half2_rn(v.x * s, v.y * s), b = __floats2half2_rn(v.z * s, v.w * s);
        uint2 o;
        o.x = *reinterpret_cast<const uint32_t*>(&a);
        o.y = *reinterpret_cast<const uint32_t*>(&b);
        *reinterpret_cast<uint2*>(dst + (size_t)pr * width + c) = o;
    }
}

// Pair-ordered fp16 activations from half-row input (already fp16(x * s_token)): a row copy.
__global__ void __launch_bounds__(256) prefill_copy_rows_kernel(const __half* __restrict__ src,
                                                                const uint32_t* __restrict__ pair_token, uint32_t rows,
                                                                uint32_t width, __half* __restrict__ dst) {
    const uint32_t c = (blockIdx.x * blockDim.x + threadIdx.x) * 8u;
    if (c >= width) return;
    for (uint32_t pr = blockIdx.y; pr < rows; pr += gridDim.y)
        *reinterpret_cast<uint4*>(dst + (size_t)pr * width + c) =
            *reinterpret_cast<const uint4*>(src + (size_t)pair_token[pr] * width + c);
}

// fp16(act * s) rows with s the power of two of each row's max (act_max); 4 columns a thread.
__global__ void __launch_bounds__(256) prefill_half_kernel(const float* __restrict__ src,
                                                           const uint32_t* __restrict__ rmax, uint32_t rows,
                                                           uint32_t width, __half* __restrict__ dst) {
    const uint32_t c = (blockIdx.x * blockDim.x + threadIdx.x) * 4u;
    if (c >= width) return;
    for (uint32_t r = blockIdx.y; r < rows; r += gridDim.y) {
        const float s = mma::prescale_for(__uint_as_float(rmax[r]));
        const float4 v = *reinterpret_cast<const float4*>(src + (size_t)r * width + c);
        const __half2 a = __floats2half2_rn(v.x * s, v.y * s), b = __floats2half2_rn(v.z * s, v.w * s);
        uint2 o;
        o.x = *reinterpret_cast<const uint32_t*>(&a);
        o.y = *reinterpret_cast<const uint32_t*>(&b);
        *reinterpret_cast<uint2*>(dst + (size_t)r * width + c) = o;
    }
}

template <typename Kern>
cudaError_t pf_smem_once(Kern kernel, size_t bytes) {
    static std::mutex mu;
    static std::vector<std::pair<const void*, size_t>> done;
    std::lock_guard<std::mutex> lock(mu);
    for (auto& d : done)
        if (d.first == (const void*)kernel && d.second >= bytes) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    if (e == cudaSuccess) done.emplace_back((const void*)kernel, bytes);
    return e;
}

uint32_t pairs_of(const MoeParams& p) { return p.T * p.k + (p.has_shared ? p.T : 0u); }

unsigned rows_grid(uint32_t rows) { return rows < 65535u ? (rows ? rows : 1u) : 65535u; }

}  // namespace

uint32_t prefill_max_tiles(uint32_t T, uint32_t k, uint32_t E) {
    return (T * k + T) / kPfMaxN + E + 2u;
}

uint32_t prefill_box_rows() { return kPfBoxRows; }

cudaError_t launch_prefill_plan(const MoeParams& p, cudaStream_t s) {
    prefill_plan_kernel<<<1, 512, 0, s>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_prefill_gateup(const MoeParams& p, unsigned grid, cudaStream_t s) {
    if (p.x_half)
        prefill_copy_rows_kernel<<<dim3((p.H / 8 + 255) / 256, rows_grid(pairs_of(p))), 256, 0, s>>>(
            p.x_half, p.pair_token, pairs_of(p), p.H, p.xperm);
    else
        prefill_gather_kernel<<<dim3((p.H / 4 + 255) / 256, rows_grid(pairs_of(p))), 256, 0, s>>>(
            p.x, p.pair_token, p.xmax, pairs_of(p), p.H, p.xperm);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    if ((e = pf_smem_once(prefill_gemm_kernel<true>, kPfSmemBytes)) != cudaSuccess) return e;
    prefill_gemm_kernel<true><<<grid, kPfThreads, kPfSmemBytes, s>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_prefill_down(const MoeParams& p, unsigned grid, cudaStream_t s) {
    prefill_half_kernel<<<dim3((p.I / 4 + 255) / 256, rows_grid(pairs_of(p))), 256, 0, s>>>(
        p.act, p.act_max, pairs_of(p), p.I, p.act_h);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    if ((e = pf_smem_once(prefill_gemm_kernel<false>, kPfSmemBytes)) != cudaSuccess) return e;
    prefill_gemm_kernel<false><<<grid, kPfThreads, kPfSmemBytes, s>>>(p);
    return cudaGetLastError();
}

}  // namespace vlb
