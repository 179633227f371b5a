/*
 * TEST INFRASTRUCTURE ONLY - a CPU restatement of the vastloom reference arithmetic for the MoE
 * routed-expert path. It is the checker for the CUDA library: only tests/, __graft_entry__.smoke()
 * and bench.py's cpu_baseline leg may load it. Nothing in vastloom_b200/ links or calls it.
 *
 * Every function cites the reference file:line it restates (paths relative to the vastloom
 * source tree). Parity of this restatement is pinned two ways: against the reference's own
 * known-answer tests (tests/test_main.cpp hashes and outputs, tests/fixtures/*.json), and against
 * the reference library itself compiled from its sources into oracle/_ref.
 *
 * Codebooks (IQ grids) are not part of this file: callers pass them in, exactly as the reference's
 * device path receives them from iq*_grid_table().
 */
#ifndef VLB_ORACLE_H
#define VLB_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids (include/vastloom/inference/ggml_quantization.hpp:35-46) */
#define VLO_TYPE_F32 0u
#define VLO_TYPE_Q8_0 8u
#define VLO_TYPE_IQ2_XXS 16u
#define VLO_TYPE_IQ3_XXS 18u
#define VLO_TYPE_IQ1_S 19u
#define VLO_TYPE_Q4_K 12u
#define VLO_TYPE_Q5_K 13u
#define VLO_TYPE_Q6_K 14u
#define VLO_TYPE_IQ2_S 22u
#define VLO_TYPE_MXFP4 39u

/* Routing score functions. SQRT_SOFTPLUS and SOFTMAX are the reference's; SIGMOID has no
 * reference router (parity unpinned) and reuses route_from_indices semantics with a sigmoid
 * score (the sigmoid helper itself is deepseek_v4_reference.cpp:71-78). */
#define VLO_SCORE_SQRT_SOFTPLUS 0
#define VLO_SCORE_SIGMOID 1
#define VLO_SCORE_SOFTMAX 2
#define VLO_SCORE_SOFTMAX_F64 3      /* Qwen: qwen38_moe_route, norm_topk_prob = false */
#define VLO_SCORE_SOFTMAX_F64_NORM 4 /* Qwen: qwen38_moe_route, norm_topk_prob = true */

int vlo_block_layout(uint32_t type, size_t* block_elems, size_t* block_bytes);
float vlo_fp16_to_float(uint16_t v);
uint16_t vlo_float_to_fp16(float v);
uint64_t vlo_fnv1a_f32(const float* v, size_t n);
uint64_t vlo_fnv1a_bytes(const void* v, size_t n);

/* Decodes n_blocks consecutive blocks. Returns 0 on success, nonzero on a non-finite scale. */
int vlo_dequantize(uint32_t type, const uint8_t* enc, size_t n_blocks, const void* grid,
                   float* out);
/* y[r] = f32(sum over columns in order of double(w)*double(x)) */
int vlo_matvec(uint32_t type, const uint8_t* enc, size_t rows, size_t cols, const float* x,
               float* y, const void* grid);
int vlo_quantize_q8_0(const float* m, size_t rows, size_t logical_cols, size_t storage_cols,
                      uint8_t* out);

float vlo_sqrt_softplus(float v);
float vlo_sigmoid(float v);
/* logits[t*E+e] = f32(sum_c double(x)*double(w)) */
void vlo_router_logits(const float* x, const float* w, size_t T, size_t H, size_t E,
                       float* logits);
int vlo_route_learned(const float* logits, const float* bias, size_t T, size_t E, size_t k,
                      float route_scale, int score, uint32_t* idx, float* weights);
int vlo_route_hash(const float* logits, const uint32_t* token_ids, const uint32_t* table,
                   size_t T, size_t V, size_t E, size_t k, float route_scale, int score,
                   uint32_t* idx, float* weights);
int vlo_route_softmax(const float* logits, size_t T, size_t E, size_t k, uint32_t* idx,
                      float* weights);
int vlo_route_softmax_f64(const float* logits, size_t T, size_t E, size_t k, int norm,
                          uint32_t* idx, float* weights);
/* deepseek_v4_expert_swiglu on float weights (gate/up [inter x width], down [width x inter]). */
int vlo_expert_swiglu(const float* x, const float* gate_w, const float* down_w, const float* up_w,
                      const float* routing_weights, size_t T, size_t width, size_t inter,
                      float limit, float* out);
/* Stable counting sort of (token, slot) pairs by expert: offsets[E+1], pair_token/pair_slot[T*k]
 * ordered by expert ascending, then token, then slot. */
void vlo_dispatch(const uint32_t* idx, size_t T, size_t k, size_t E, uint32_t* offsets,
                  uint32_t* pair_token, uint32_t* pair_slot);
int vlo_hc_split_sinkhorn(const float* mixes, const float* scale, const float* base, size_t T, size_t m,
                          size_t iters, float eps, float* pre, float* post, float* comb);
int vlo_hc_pre(const float* x, const float* fn, const float* scale, const float* base, size_t T, size_t m,
               size_t W, size_t iters, float norm_eps, float hc_eps, float* reduced, float* pre, float* post,
               float* comb);
int vlo_hc_post(const float* sub, const float* residual, const float* post, const float* comb, size_t T,
                size_t m, size_t W, float* out);
int vlo_rms_norm(const float* x, const float* w, size_t rows, size_t width, float eps,
                 float* out);

typedef struct vlo_matrix {
    uint32_t type;
    size_t rows;
    size_t cols;
    const uint8_t* data;
} vlo_matrix;

typedef struct vlo_moe_layer {
    size_t hidden;        /* H */
    size_t intermediate;  /* I */
    size_t experts;       /* E */
    size_t top_k;         /* k */
    int score;            /* VLO_SCORE_* */
    int hash_routing;     /* 1: tid2eid table gather */
    int weight_after_down;/* 1: OLMoE (rank-order combine, float SwiGLU); 0: DeepSeek V4 */
    float route_scale;
    float routed_swiglu_limit;
    float shared_swiglu_limit;
    const float* router;  /* f32 [E x H] */
    const float* bias;    /* f32 [E] (learned routing) */
    const uint32_t* tid2eid; /* u32 [V x k] (hash routing) */
    size_t vocab;
    const vlo_matrix* w1; /* [E] gate, I x H */
    const vlo_matrix* w3; /* [E] up,   I x H */
    const vlo_matrix* w2; /* [E] down, H x I */
    const vlo_matrix* shared_w1; /* NULL: no shared expert */
    const vlo_matrix* shared_w3;
    const vlo_matrix* shared_w2;
    const void* grid_iq1_s;
    const void* grid_iq2_xxs;
    const void* grid_iq3_xxs;
    const void* grid_iq2_s;
} vlo_moe_layer;

/* The down-projection input of one DeepSeek V4 expert for one token (gate/up matvecs of type
 * `type`, I x H each; clamp at `limit` when positive; route weight when route_w is not NULL). */
int vlo_v4_expert_activation(uint32_t type, const uint8_t* w1, const uint8_t* w3, size_t I, size_t H,
                             const float* x, const float* route_w, float limit, const void* grid,
                             float* act);

/* One MoE layer over T tokens: out f32[T x H]; idx/weights [T x k] receive the route. Optional
 * logits_in (f32 [T x E]) replaces the router projection (config 3 feeds logits directly). */
int vlo_moe_forward(const vlo_moe_layer* layer, const float* x, const uint32_t* token_ids,
                    size_t T, const float* logits_in, float* out, uint32_t* idx,
                    float* weights);

#ifdef __cplusplus
}
#endif
#endif
