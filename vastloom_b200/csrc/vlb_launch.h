// Host-side launchers of the vlb200 kernels (implemented in vlb_kernels.cu).
#pragma once

#include <cuda_runtime.h>

#include "vlb_internal.cuh"

namespace vlb {

cudaError_t launch_dequant(const DevMat& m, const Grids& g, float* out, cudaStream_t s);
cudaError_t launch_gemv(const DevMat& m, const Grids& g, const float* x, uint32_t ntok,
                        uint32_t xstride, float* y, uint32_t ystride, cudaStream_t s);
// logits[t][e] = f32(sequential f64 sum of xd[t][c] * wd[e][c]), scores = score function of them;
// xd / wd are the f64 widenings of the f32 activations / router weights (H % 2 == 0)
cudaError_t launch_router(const double* xd, const double* wd, uint32_t T, uint32_t H, uint32_t E, int score,
                          float* logits, float* scores, cudaStream_t s);
cudaError_t launch_widen(const float* src, size_t n, double* dst, cudaStream_t s);
// per-token max|x| bits; with xd non-null also the rows widened to f64
cudaError_t launch_prescale(const float* x, uint32_t T, uint32_t H, uint32_t* xmax, double* xd, cudaStream_t s);
cudaError_t launch_scores(const float* logits, size_t n, int score, float* scores,
                          cudaStream_t s);
cudaError_t launch_route(const float* scores, const float* bias, const uint32_t* token_ids,
                         const uint32_t* tid2eid, uint32_t vocab, uint32_t T, uint32_t E,
                         uint32_t k, int score, int hash_routing, float route_scale,
                         uint32_t* idx, float* weights, uint32_t* error_flag, cudaStream_t s);
// The whole layer: routing, dispatch, gate/up + SwiGLU, down, combine (the expert products on the
// decode kernels, or on the prefill kernels when p.prefill is set).
// ev: optional 6 events recorded at the phase boundaries (start, routed, dispatched, gate/up done,
// down done, combined).
constexpr int kMoePhases = 5;
cudaError_t launch_moe(const MoeParams& p, cudaStream_t s, cudaEvent_t* ev = nullptr);
// Prefill path (vlb_prefill.cu): column-tile plan after dispatch, then the tcgen05 grouped GEMMs
// (each preceded by the fp16 conversion of its activations).
uint32_t prefill_max_tiles(uint32_t T, uint32_t k, uint32_t E);
uint32_t prefill_box_rows();  // rows of the B operand's TMA box
cudaError_t launch_prefill_plan(const MoeParams& p, cudaStream_t s);
cudaError_t launch_prefill_gateup(const MoeParams& p, unsigned grid, cudaStream_t s);
cudaError_t launch_prefill_down(const MoeParams& p, unsigned grid, cudaStream_t s);
cudaError_t launch_stable_sort(const MoeParams& p, cudaStream_t s);
// Decode path (vlb_decode.cu): IQ2_XXS / Q8_0 expert products on mma.sync fed by a bulk-copy ring,
// one CTA per SM.
cudaError_t launch_decode_gateup(const MoeParams& p, unsigned n_sms, cudaStream_t s);
// fmt_bit set of the storage types the decode kernel of a phase serves: Q8_0 and the phase's IQ
// type (IQ2_XXS before IQ1_S before IQ3_XXS when several are present) if its stage carve fits
uint32_t decode_ring_types(const MoeParams& p, bool gateup);
cudaError_t launch_decode_down(const MoeParams& p, unsigned n_sms, cudaStream_t s);
// Expert-parallel helpers (vlb_ep.cu)
cudaError_t launch_ep_validate(const uint32_t* idx, size_t n, uint32_t E, uint32_t* flag, cudaStream_t s);
// expert ids -> exchange slots (slot_of null: identity); out-of-range ids flagged and replaced by 0
cudaError_t launch_ep_slots(const uint32_t* idx, size_t n, uint32_t E, const uint32_t* slot_of, uint32_t* out,
                            uint32_t* flag, cudaStream_t s);
// f32 rows -> fp16 rows with a per-row power-of-two scale (scale[r] = the inverse factor)
cudaError_t launch_ep_pack_half(const float* y, uint32_t rows, uint32_t H, __half* out, float* scale, cudaStream_t s);
cudaError_t launch_ep_combine_half(const __half* rows, const float* scale, const uint32_t* elem_row, uint32_t T,
                                   uint32_t k, const float* shared_rows, uint32_t H, float* out, cudaStream_t s);
cudaError_t launch_ep_gather(const uint32_t* pair_token, const uint32_t* pair_slot, const uint32_t* idx,
                             uint32_t n, uint32_t k, uint32_t epr, const float* x, uint32_t H, float* send_x,
                             uint32_t* send_expert, cudaStream_t s);
// Half-row exchange: fp16 send rows + (expert, weight, max|x|) meta, and the own tokens' rows.
cudaError_t launch_ep_gather_half(const uint32_t* pair_token, const uint32_t* pair_slot, const uint32_t* idx,
                                  const float* sorted_w, uint32_t n, uint32_t k, uint32_t epr, const float* x,
                                  const uint32_t* xmax, uint32_t H, __half* rows, uint32_t* meta, cudaStream_t s);
cudaError_t launch_ep_own_rows(const float* x, const uint32_t* xmax, uint32_t T, uint32_t H, uint32_t epr,
                               __half* rows, uint32_t* meta, cudaStream_t s);
cudaError_t launch_ep_combine(const float* y, const uint32_t* elem_row, uint32_t T, uint32_t k,
                              const float* shared_rows, uint32_t H, float* out, cudaStream_t s);
// RMSNorm rows (bit-exact); xmax non-null: also each row's max|out| bits; out_d: the rows as f64.
// width % 4 == 0 and
// width <= kRmsMaxWidth (the row is staged in shared memory).
constexpr uint32_t kRmsMaxWidth = 24576;  // the row staged as f64 in shared memory
// Whether the Hyper-Connection entry kernel's shared-memory plan fits m copies of a hidden row.
bool hc_entry_fits(uint32_t m, uint32_t H);
cudaError_t launch_rms_norm(const float* x, const float* w, uint32_t rows, uint32_t width,
                            float eps, float* out, uint32_t* xmax, double* out_d, cudaStream_t s);

}  // namespace vlb
