/*
 * vlb200 - C ABI of the B200 (sm_100a) MoE routed-expert library.
 *
 * This is the boundary that replaces vastloom's CUDA driver / matvec-accelerator seam:
 *   - src/cuda/cuda_driver.cpp (DynamicCudaBackend: dlopen of libcuda, embedded scalar PTX,
 *     *_with_transfer launches; include/vastloom/cuda/cuda_driver.hpp:41-344), and
 *   - src/cuda/cuda_matvec_accelerator.cpp (CudaMatvecAccelerator, the implementation of
 *     DeepseekV4MatvecAccelerator, include/vastloom/inference/deepseek_v4_reference.hpp:440-451).
 * A C++ adapter (vastloom_b200/host/b200_matvec_accelerator.hpp) implements the reference's
 * DeepseekV4MatvecAccelerator interface on top of these entry points.
 *
 * Conventions (mirroring include/vastloom/core/status.hpp:10-21 and cuda_driver.cpp:2727-2738):
 *   - every entry point returns an int status: VLB_OK (0) or VLB_ERR_* = vastloom ErrorCode + 1;
 *   - VLB_DECLINED is the accelerator's "false": the call was refused, outputs are untouched and
 *     the caller runs its CPU path (deepseek_v4_reference.hpp:440-451);
 *   - the message of the last failure is kept per handle (vlb_last_error) and per thread
 *     (vlb_thread_error) for calls that have no handle yet;
 *   - nothing aborts or throws across this boundary; device-side waits are bounded and surface as
 *     VLB_ERR_IO_ERROR.
 * Threading: calls on one handle are serialised by the handle's mutex; each handle owns one CUDA
 * stream on one device (the reference serialises its backend the same way, cuda_driver.cpp:2093).
 * A call on a handle makes the handle's device current on the calling thread and leaves it
 * current.
 * Memory: every device allocation the library makes is first reserved through the caller's
 * governor callbacks (CudaDriver::allocate reserves before cuMemAlloc, cuda_driver.cpp:2929-3005).
 */
#ifndef VLB200_H
#define VLB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VLB_ABI_VERSION 2

/* Status codes: 0 = success; 1..10 = vastloom::ErrorCode + 1 (status.hpp:10-21). */
enum {
    VLB_OK = 0,
    VLB_ERR_INVALID_ARGUMENT = 1,
    VLB_ERR_INVALID_FORMAT = 2,
    VLB_ERR_NOT_FOUND = 3,
    VLB_ERR_PERMISSION_DENIED = 4,
    VLB_ERR_IO_ERROR = 5,
    VLB_ERR_INTEGRITY_ERROR = 6,
    VLB_ERR_UNSAFE_PATH = 7,
    VLB_ERR_UNSUPPORTED = 8,
    VLB_ERR_RESOURCE_EXHAUSTED = 9,
    VLB_ERR_INTERNAL_ERROR = 10,
    VLB_DECLINED = 100
};

/* ggml storage types the device path accepts (ggml_quantization.hpp:35-46). */
enum {
    VLB_TYPE_F32 = 0,
    VLB_TYPE_Q8_0 = 8,
    VLB_TYPE_IQ2_XXS = 16,
    VLB_TYPE_IQ3_XXS = 18,
    VLB_TYPE_IQ1_S = 19,
    /* served on the CUDA cores (the per-row seam, dequantize and the expert kernels) */
    VLB_TYPE_Q4_K = 12,
    VLB_TYPE_Q5_K = 13,
    VLB_TYPE_Q6_K = 14,
    VLB_TYPE_IQ2_S = 22,
    VLB_TYPE_MXFP4 = 39
};

/* Router scoring:
 *   VLB_SCORE_SQRT_SOFTPLUS   sqrt_softplus scores, bias-selected top-k, renormalised weights times
 *                             route_scale (deepseek_v4_reference.cpp:65-69, 80-121, 223-307);
 *   VLB_SCORE_SIGMOID         the same with a sigmoid score (no reference router: an extra mode);
 *   VLB_SCORE_SOFTMAX         OLMoE: f32 softmax probabilities, top-k, no renormalisation
 *                             (olmoe_runtime.cpp:1120-1137);
 *   VLB_SCORE_SOFTMAX_F64     Qwen: f64 softmax, top-k by probability, weights f32(prob)
 *                             (qwen38_moe_route, qwen3_8_flash_next_reference.cpp:1186-1239 with
 *                             norm_topk_prob = false);
 *   VLB_SCORE_SOFTMAX_F64_NORM the same with norm_topk_prob = true (weights rescaled by the inverse
 *                             of the selected probabilities' sum).
 * The softmax modes ignore bias and route_scale. */
enum {
    VLB_SCORE_SQRT_SOFTPLUS = 0,
    VLB_SCORE_SIGMOID = 1,
    VLB_SCORE_SOFTMAX = 2,
    VLB_SCORE_SOFTMAX_F64 = 3,
    VLB_SCORE_SOFTMAX_F64_NORM = 4
};

typedef struct vlb_handle vlb_handle;
typedef struct vlb_matrix vlb_matrix;
typedef struct vlb_layer vlb_layer;

/* Governor hooks (include/vastloom/safety/resource_governor.hpp:60-113). reserve() is called with
 * the exact byte count BEFORE each device allocation and must return 0 to allow it; release() is
 * called after the matching free, or when the allocation failed after a successful reserve. A
 * NULL governor means "no accounting" (tests only). */
typedef struct vlb_governor {
    void* ctx;
    int (*reserve)(void* ctx, uint64_t bytes, const char* tag);
    void (*release)(void* ctx, uint64_t bytes, const char* tag);
} vlb_governor;

typedef struct vlb_device_info {
    int ordinal;
    int sm_count;
    int cc_major;
    int cc_minor;
    uint64_t total_bytes;
    uint64_t free_bytes;
    char name[96];
} vlb_device_info;

/* ---- library / device ------------------------------------------------------------------- */
int vlb_abi_version(void);
/* Thread-local message of the last failure of a call that had no handle (e.g. vlb_open). */
int vlb_thread_error(char* buf, size_t cap);
/* CudaDriverBackend::probe (cuda_driver.hpp:41-60): device count and one device's properties. */
int vlb_device_count(int* count);
int vlb_probe(int ordinal, vlb_device_info* info);

/* Opens a handle on one device with its own stream. min_free_after: allocations that would
 * leave less than this many free bytes on the device are refused (CudaMatvecAcceleratorOptions::
 * minimum_free_vram_after, cuda_matvec_accelerator.hpp:17-30). */
int vlb_open(int ordinal, const vlb_governor* governor, uint64_t min_free_after,
             vlb_handle** out);
void vlb_close(vlb_handle* h);
int vlb_last_error(const vlb_handle* h, char* buf, size_t cap);
/* The handle's CUDA stream (a cudaStream_t), for callers that enqueue their own work on it. */
void* vlb_stream(vlb_handle* h);
int vlb_synchronize(vlb_handle* h);

/* ---- codebooks -------------------------------------------------------------------------- */
/* Installs the IQ codebook for one type from the caller's table (the reference passes
 * iq1_s_grid_table() / iq2_xxs_grid_table() / iq3_xxs_grid_table(), ggml_quantization.hpp:
 * 63-76). The table's FNV-1a fingerprint must equal the reference's pinned value
 * (ggml_quantization.cpp:60,73,99) or VLB_ERR_INTEGRITY_ERROR is returned. */
int vlb_set_codebook(vlb_handle* h, uint32_t ggml_type, const void* table, size_t bytes);

/* ---- governed device buffers (CudaDriver::allocate / CudaAllocation) ---------------------- */
int vlb_alloc(vlb_handle* h, size_t bytes, const char* tag, void** dev_ptr);
int vlb_free(vlb_handle* h, void* dev_ptr);
int vlb_memcpy_h2d(vlb_handle* h, void* dst_dev, const void* src_host, size_t bytes);
int vlb_memcpy_d2h(vlb_handle* h, void* dst_host, const void* src_dev, size_t bytes);
/* Bytes currently allocated by this handle (resident matrices, layers, scratch). */
uint64_t vlb_allocated_bytes(const vlb_handle* h);

/* ---- resident packed matrices (DeepseekV4PackedMatrix, deepseek_v4_reference.hpp:104-141) --
 * Uploads one ggml matrix (rows x storage_cols, consecutive little-endian blocks, exactly the
 * reference's payload bytes) into device memory under its cache identity (never a host address;
 * deepseek_v4_reference.hpp:125-132). The device copy is re-laid out for the kernels (per-block
 * fp16 scales split from 16-byte-aligned block bodies); bytes per weight are unchanged. Every
 * block scale must be finite (validate_block_scales, ggml_quantization.cpp:205-215). */
int vlb_upload_matrix(vlb_handle* h, uint64_t cache_identity, uint32_t ggml_type, size_t rows,
                      size_t storage_cols, const void* payload, size_t payload_bytes,
                      vlb_matrix** out);
int vlb_release_matrix(vlb_handle* h, vlb_matrix* m);
/* Resident bytes of a matrix (scales + bodies). */
uint64_t vlb_matrix_bytes(const vlb_matrix* m);

/* ---- expert records to device (DeepseekV4ExpertPackRecord, include/vastloom/inference/
 * deepseek_v4_expert_pack.hpp:24-41; the VRAM half of ResidencyObject, include/vastloom/model/
 * residency.hpp:114-145, src/model/residency.cpp:183-212) ----------------------------------
 * One expert's record is one contiguous span of ggml bytes holding its tensors back to back
 * (`offset` = the tensor's packed_offset inside the record). vlb_upload_record_async copies the
 * whole span to the device in ONE host-to-device copy on the handle's upload stream (a stream of
 * its own, so the copy overlaps the handle's compute) and re-lays every block out on the device;
 * the matrices come out identical to vlb_upload_matrix's. It returns once the work is enqueued:
 * the record's host bytes must stay unchanged until vlb_upload_finish returns, and the copy is
 * asynchronous only from page-locked memory (vlb_host_alloc). reserved_bytes: VRAM the caller
 * already holds in its governor for these matrices (ResidencyObject::begin_vram_copy reserves
 * the record's bytes); the governor hooks are charged only for the device bytes above it, in
 * tensor order, and for the device copy of the record ("vlb-upload-staging", kept and grown
 * for later records). At most 64 tensors per record and 256 records in flight per handle. */
typedef struct vlb_upload vlb_upload;
typedef struct vlb_record_tensor {
    uint64_t cache_identity; /* deepseek_v4_expert_provider.cpp:75-90 for routed experts */
    uint32_t ggml_type;
    uint32_t reserved0;
    uint64_t rows;           /* shape[1] */
    uint64_t storage_cols;   /* shape[0] */
    uint64_t offset;         /* packed_offset within the record */
    uint64_t bytes;          /* rows x blocks per row x block bytes */
} vlb_record_tensor;
int vlb_upload_record_async(vlb_handle* h, const void* record_host, size_t record_bytes,
                            const vlb_record_tensor* tensors, uint32_t n_tensors,
                            uint64_t reserved_bytes, vlb_upload** out);
/* *done = 1 once the copy and the re-layout have finished (never blocks). */
int vlb_upload_query(vlb_handle* h, vlb_upload* u, int* done);
/* Waits for the upload, checks every block as the reference's decoders do, and hands out one
 * matrix per tensor (out[n_tensors], record order). On any failure (a block scale that is not
 * finite: VLB_ERR_INVALID_FORMAT naming the tensor) every matrix of the record is released.
 * Either way the upload object is consumed. */
int vlb_upload_finish(vlb_handle* h, vlb_upload* u, vlb_matrix** out, uint32_t n_tensors);
/* Page-locked host memory for records (cudaHostAlloc); freed with vlb_host_free. */
int vlb_host_alloc(vlb_handle* h, size_t bytes, void** out);
int vlb_host_free(vlb_handle* h, void* p);

/* The per-row operator seam: DeepseekV4MatvecAccelerator::matvec (deepseek_v4_reference.hpp:
 * 440-451) for a resident matrix, host input (storage_cols floats, zero-padded by the caller)
 * and host output (rows floats). Synchronous, like matvec_*_with_transfer
 * (cuda_driver.cpp:2083-2171). */
int vlb_matvec(vlb_handle* h, const vlb_matrix* m, const float* x_host, float* y_host);
/* Device form over n_tokens rows of x (row stride x_stride floats) into y (n_tokens x rows,
 * row stride y_stride floats), enqueued on `stream` (NULL = the handle's stream). */
int vlb_matvec_device(vlb_handle* h, const vlb_matrix* m, const float* x_dev, size_t n_tokens,
                      size_t x_stride, float* y_dev, size_t y_stride, void* stream);
/* Dequantizes the whole matrix to f32 rows x storage_cols on the device (bit-exact with the
 * reference's dequantize_*; ggml_quantization.cpp:217-435). */
int vlb_dequantize_device(vlb_handle* h, const vlb_matrix* m, float* out_dev, void* stream);

/* ---- the batched MoE layer (moe_forward, deepseek_v4_graph.cpp:1902-2274; OLMoE forward,
 * olmoe_runtime.cpp:1119-1290) ------------------------------------------------------------ */
typedef struct vlb_moe_layer_desc {
    uint32_t hidden;        /* H */
    uint32_t intermediate;  /* I */
    uint32_t experts;       /* E routed experts */
    uint32_t top_k;         /* k */
    int score;              /* VLB_SCORE_* */
    int hash_routing;       /* 1: experts from tid2eid[token*k + slot] */
    int weight_after_down;  /* 1: OLMoE semantics (float SwiGLU, rank-order combine w*down) */
    float route_scale;
    float routed_swiglu_limit;
    float shared_swiglu_limit;
    uint32_t max_tokens;    /* workspace bound for one forward call */
    uint32_t vocab;         /* rows of tid2eid */
    const float* router;    /* host f32 [E x H], copied at create */
    const float* bias;      /* host f32 [E] (learned routing) or NULL */
    const uint32_t* tid2eid;/* host u32 [vocab x k] (hash routing) or NULL */
    vlb_matrix* const* w1;  /* [E] gate (I x H) */
    vlb_matrix* const* w3;  /* [E] up   (I x H) */
    vlb_matrix* const* w2;  /* [E] down (H x I) */
    vlb_matrix* shared_w1;  /* NULL: no shared expert */
    vlb_matrix* shared_w3;
    vlb_matrix* shared_w2;
} vlb_moe_layer_desc;

int vlb_layer_create(vlb_handle* h, const vlb_moe_layer_desc* desc, vlb_layer** out);
int vlb_layer_destroy(vlb_handle* h, vlb_layer* layer);

/* Device-resident forward: x_dev f32 [T x H], token_ids_dev u32 [T] (hash routing; may be NULL
 * otherwise), optional logits_dev f32 [T x E] replacing the router projection, out_dev f32
 * [T x H]. Enqueued on `stream` (NULL = handle stream); no host synchronisation. */
int vlb_layer_forward_device(vlb_handle* h, vlb_layer* layer, const float* x_dev,
                             const uint32_t* token_ids_dev, const float* logits_dev, uint32_t T,
                             float* out_dev, void* stream);
/* Host form (the end-to-end call): copies x / token ids / logits in, runs the layer, copies the
 * output back, synchronises. */
int vlb_layer_forward(vlb_handle* h, vlb_layer* layer, const float* x_host,
                      const uint32_t* token_ids_host, const float* logits_host, uint32_t T,
                      float* out_host);

/* Prefill mode. A forward of T >= min_tokens runs the expert products as grouped GEMMs on the
 * tensor cores (tcgen05, fp16 operands with per-matrix / per-token / per-pair power-of-two scales,
 * f32 accumulation): layer outputs then match the reference within 2e-2 relative (about 1e-3 in
 * practice) instead of the decode path's 1e-5. Routing, dispatch and the combine order are the
 * same on both paths; IQ3_XXS / IQ1_S experts stay on the CUDA-core kernels. min_tokens = 0
 * restores the default (16 pairs per routed expert on average, at least 256 tokens);
 * 0xFFFFFFFF keeps every forward on the decode path. vlb_layer_prefill_tokens returns the
 * threshold in force (0 for a null argument). The prefill pipeline's waits are time-bounded: a
 * wait that runs out makes vlb_layer_forward return VLB_ERR_INTERNAL_ERROR. */
int vlb_layer_set_prefill_tokens(vlb_handle* h, vlb_layer* layer, uint32_t min_tokens);

/* Residual-block entry and exit. With an input norm set (weight: host f32 [hidden], copied; eps >
 * 0), every forward of plain token rows computes
 *     out = x + MoE(RMSNorm(x))
 * RMSNorm is deepseek_v4_rms_norm (deepseek_v4_reference.cpp:170-206: sequential f64 sum of
 * squares, bit-identical) fused with the entry step of the layer, the router and the experts run
 * on the normalised rows, and the residual is one f32 addition fused into the combine - the
 * composition between the MoE layers of a hash-routed chain (configuration 2). weight = NULL
 * removes it. Rows must be 16-byte aligned; given-routes and half-row forwards are refused while
 * it is set. */
int vlb_layer_set_input_norm(vlb_handle* h, vlb_layer* layer, const float* weight, float eps);

/* Hyper-Connection entry and exit (the ffn half of a DeepSeek V4 block, deepseek_v4_graph.cpp:
 * 2391-2408 and 2452-2469):
 *     split, reduced = hc_pre(x)           deepseek_v4_hc_pre, deepseek_v4_reference.cpp:479-547
 *     moe            = MoE(RMSNorm(reduced, norm_weight))
 *     out            = hc_post(moe, x)     deepseek_v4_hc_post, :549-610
 * With it set, x and out of vlb_layer_forward / vlb_layer_forward_device hold `multiplier` copies
 * of each token's hidden state, [T x multiplier x hidden] f32. The entry is one kernel (the mixing
 * projection as sequential f64 chains, the Sinkhorn split, the reduced row, the norm: mixes,
 * reduced row and norm bit-identical with the reference, the split too except where CUDA's and the
 * host's double exp differ in the last bit); the exit is fused into the combine (f64 sums in the
 * reference's order). The mixing weight is the f32 `hc_ffn_fn` form (deepseek_v4_graph.cpp:
 * 2289-2295). It replaces an input norm; NULL removes both. Given-routes and half-row forwards
 * are refused while it is set. A reduced row that is not finite fails the forward with
 * VLB_ERR_INVALID_FORMAT. */
typedef struct vlb_hc_desc {
    uint32_t multiplier;          /* m, 1..16 (config.hyper_multiplier); m x hidden <= 24576 */
    uint32_t sinkhorn_iterations; /* >= 1 (config.sinkhorn_iterations) */
    float norm_epsilon;           /* config.norm_epsilon: the mixing RMS and the ffn norm */
    float hc_epsilon;             /* config.hyper_epsilon */
    const float* mixing_weight;   /* hc_ffn_fn [(2+m)m x m*hidden] */
    const float* scale;           /* hc_ffn_scale [3] */
    const float* base;            /* hc_ffn_base [(2+m)m] */
    const float* norm_weight;     /* ffn_norm.weight [hidden] */
} vlb_hc_desc;
int vlb_layer_set_hyper_connection(vlb_handle* h, vlb_layer* layer, const vlb_hc_desc* desc);
/* The split of the last forward's first T tokens (host arrays; any may be NULL): pre and post
 * [T x m], combination [T x m x m] ([source][destination]). */
int vlb_layer_last_hyper_split(vlb_handle* h, vlb_layer* layer, uint32_t T, float* pre, float* post,
                               float* combination);
uint32_t vlb_layer_prefill_tokens(vlb_handle* h, vlb_layer* layer);

/* Given-routes forward (an expert-parallel group): idx_dev u32 [T x k] expert ids of this layer
 * (< experts), weights_dev f32 [T x k]; the router and top-k are skipped, everything else is the
 * layer forward (dispatch, experts, combine; the shared expert if the layer has one). An id out of
 * range is reported by vlb_layer_status (VLB_ERR_INVALID_FORMAT) and never indexes past the
 * expert table. Enqueued on `stream`. */
int vlb_layer_forward_routes_device(vlb_handle* h, vlb_layer* layer, const float* x_dev,
                                    const uint32_t* idx_dev, const float* weights_dev, uint32_t T,
                                    float* out_dev, void* stream);
/* Forward of half rows with one route each (a layer of top_k 1 whose experts are IQ2_XXS /
 * Q8_0, hidden % 8 == 0): rows_dev fp16 [T x H] = fp16(x * 2^e) with 2^e the power of two that
 * brings the row's max|x| into [2^14, 2^15), meta_dev u32 [T x 3] = (expert id, route weight as
 * f32 bits, max|x| as f32 bits), as vlb_ep_plan_half_device produces them. Always the tensor-core
 * prefill path (its operands are these rows; 2e-2 contract); out_dev f32 [T x H]. No counterpart
 * in the reference, whose expert-parallel exchange is not part of this path: it is the receiving
 * side of the half-row exchange below. Enqueued on `stream`. */
int vlb_layer_forward_rows_half_device(vlb_handle* h, vlb_layer* layer, const uint16_t* rows_dev,
                                       const uint32_t* meta_dev, uint32_t T, float* out_dev,
                                       void* stream);
/* Synchronises `stream` and reports the error bits the layer's last device forward left (hash
 * token id out of its table, out-of-range expert, unnormalisable weights, expert-kernel pipeline
 * timeout), as vlb_layer_forward does for the host form. */
int vlb_layer_status(vlb_handle* h, vlb_layer* layer, void* stream);

/* ---- expert parallelism (configuration 4: experts sharded over GPUs, all-to-all exchange) ----
 * Plan on the source rank: the T*k (token, slot) elements of idx_dev (global expert ids < E) in the
 * dispatch's stable order (expert ascending, then token, then slot) - with experts sharded in
 * contiguous ranges of experts_per_rank that is also destination-rank order; send_x_dev f32
 * [T*k x H] their x rows, send_expert_dev their expert id local to the owning rank
 * (id % experts_per_rank), send_weight_dev their route weight, elem_row_dev [T*k] element
 * (t * k + slot) -> send row, offsets_dev u32 [E + 2] device and offsets_host [E + 1] host copies
 * of the per-expert starts. ws_dev: vlb_ep_workspace_bytes(T, k, E) bytes of device scratch.
 * Synchronises `stream` (the host offsets size the exchange). */
size_t vlb_ep_workspace_bytes(uint32_t T, uint32_t k, uint32_t E);
int vlb_ep_plan_device(vlb_handle* h, const uint32_t* idx_dev, const float* weights_dev, uint32_t T,
                       uint32_t k, uint32_t E, uint32_t experts_per_rank, const float* x_dev, uint32_t H,
                       void* ws_dev,
                       uint32_t* offsets_dev, uint32_t* offsets_host, float* send_x_dev,
                       uint32_t* send_expert_dev, float* send_weight_dev, uint32_t* elem_row_dev,
                       void* stream);
/* The same plan with half rows for the exchange (half the bytes of f32 rows): send_rows_dev fp16
 * [T*k x H] in plan order, send_meta_dev u32 [T*k x 3] = (local expert id, route weight bits,
 * token max|x| bits), and the rank's own tokens for its shared expert, own_rows_dev fp16 [T x H]
 * with own_meta_dev [T x 3] = (experts_per_rank, 1.0f bits, max|x| bits): the inputs of
 * vlb_layer_forward_rows_half_device on the receiving rank. H % 8 == 0. expert_slot_dev (u32 [E],
 * NULL = identity) places the experts on the ranks: expert e is local expert slot % epr of rank
 * slot / epr, slot = expert_slot_dev[e], a permutation of [0, E) - a placement balanced by expert
 * load instead of contiguous ranges. The pairs are ordered by slot (expert order within a rank)
 * and offsets are per slot. An expert id >= E returns VLB_ERR_INVALID_FORMAT. One host
 * synchronisation (the offsets size the exchange). */
int vlb_ep_plan_half_device(vlb_handle* h, const uint32_t* idx_dev, const float* weights_dev, uint32_t T,
                            uint32_t k, uint32_t E, uint32_t experts_per_rank, const uint32_t* expert_slot_dev,
                            const float* x_dev, uint32_t H, void* ws_dev, uint32_t* offsets_dev,
                            uint32_t* offsets_host, uint16_t* send_rows_dev, uint32_t* send_meta_dev,
                            uint32_t* elem_row_dev, uint16_t* own_rows_dev, uint32_t* own_meta_dev, void* stream);
/* Expert outputs as fp16 rows for the return exchange: half_rows_dev [rows x H] = fp16(y * 2^e_r),
 * 2^e_r the power of two bringing row r's max|y| into [2^14, 2^15), row_scale_dev[r] = 2^-e_r.
 * Half the bytes of the f32 rows; each element keeps 11 significant bits. H % 8 == 0. */
int vlb_ep_pack_half_device(vlb_handle* h, const float* y_rows_dev, uint32_t rows, uint32_t H,
                            uint16_t* half_rows_dev, float* row_scale_dev, void* stream);
/* vlb_ep_combine_device on returned half rows: out[t] = sum over its k slots of
 * half_rows_dev[elem_row] * row_scale_dev[elem_row] (slot order) + shared_rows_dev[t] (f32; NULL:
 * none). */
int vlb_ep_combine_half_device(vlb_handle* h, const uint16_t* half_rows_dev, const float* row_scale_dev,
                               const uint32_t* elem_row_dev, uint32_t T, uint32_t k, const float* shared_rows_dev,
                               uint32_t H, float* out_dev, void* stream);
/* Combine on the source rank after the return exchange: out[t] = sum over its k slots of
 * y_rows_dev[elem_row_dev[t * k + slot]] (slot order) + shared_rows_dev[t] (NULL: none). */
int vlb_ep_combine_device(vlb_handle* h, const float* y_rows_dev, const uint32_t* elem_row_dev,
                          uint32_t T, uint32_t k, const float* shared_rows_dev, uint32_t H,
                          float* out_dev, void* stream);

/* ---- expert-parallel driver over NCCL -------------------------------------------------------
 * The whole configuration-4 step of one rank in one call, for a C or C++ host with one process
 * (or host thread) and one handle per GPU. Communicator set-up from an ncclUniqueId that rank 0
 * creates and the caller distributes (MPI, a key-value store, a file); then per step: route, plan,
 * counts all-to-all, half-row dispatch, the rank's expert group (its routed experts and the shared
 * expert) on the tensor-core path, fp16 results back, combine - grouped ncclSend/ncclRecv on the
 * step's stream. NCCL (>= 2.18) is loaded when first needed: $VLB_NCCL_LIBRARY, else
 * libnccl.so.2 (the copy the process has already loaded, if any); without it these entry points
 * return VLB_ERR_UNSUPPORTED and the rest of the library is unaffected. A process holds one
 * libnccl.so.2: one that also uses another NCCL user (PyTorch) loads that user first, so that the
 * driver binds its copy.
 *
 * Waits are bounded: the communicator is non-blocking and every host wait (set-up, the count
 * read-back, the end of a step) gives up after timeout_ms, aborts the communicator (ending this
 * rank's NCCL kernels) and returns VLB_ERR_IO_ERROR naming the exchange ("counts", "dispatch",
 * "return"). A layer whose exchange failed refuses every later forward; rebuild the communicator
 * and the layer. Failure messages are read with vlb_thread_error. The reference has no
 * expert-parallel exchange on this path, so none of these has a reference counterpart. */
#define VLB_EP_UNIQUE_ID_BYTES 128
typedef struct vlb_ep_comm vlb_ep_comm;
typedef struct vlb_ep_layer vlb_ep_layer;

/* NCCL's version code (e.g. 22703) of the library the driver loaded. */
int vlb_ep_nccl_version(int* version);
/* ncclGetUniqueId: rank 0 creates the id, every rank passes the same bytes to vlb_ep_comm_init. */
int vlb_ep_unique_id(uint8_t* id /* [VLB_EP_UNIQUE_ID_BYTES] */);
/* One rank's communicator on the handle's device (world ranks, ranks 0..world-1). Returns when
 * every rank has joined, or VLB_ERR_IO_ERROR after timeout_ms. */
int vlb_ep_comm_init(vlb_handle* h, const uint8_t* id, int rank, int world, uint32_t timeout_ms,
                     vlb_ep_comm** out);
/* Finalizes (bounded) and frees the communicator; an aborted one is only freed. */
int vlb_ep_comm_destroy(vlb_ep_comm* comm);
/* Aborts the communicator (a host-side decision that a peer is gone); later exchanges fail. */
int vlb_ep_comm_abort(vlb_ep_comm* comm);
/* Plain all-to-all of bytes: send_bytes[p] bytes to rank p from send_dev (peers in rank order),
 * recv_bytes[p] from rank p into recv_dev; both arrays host [world]. Enqueued on `stream` (NULL =
 * the handle's); returns once NCCL has issued it. The exchange the driver's steps use, exposed
 * for measuring the link (an NVLink all-to-all microbenchmark) and for callers' own exchanges. */
int vlb_ep_all_to_all_device(vlb_ep_comm* comm, const void* send_dev, const uint64_t* send_bytes,
                             void* recv_dev, const uint64_t* recv_bytes, void* stream);

typedef struct vlb_ep_layer_desc {
    uint32_t hidden, intermediate;
    uint32_t experts;           /* E routed experts over all ranks (a multiple of world) */
    uint32_t top_k;
    int score;                  /* VLB_SCORE_* (learned routing from given logits) */
    int weight_after_down;
    float route_scale;
    float routed_swiglu_limit;  /* must equal shared_swiglu_limit (one limit per group layer) */
    float shared_swiglu_limit;
    uint32_t max_tokens;        /* tokens of this rank per step */
    const float* bias;          /* host f32 [E] or NULL */
    const uint32_t* expert_slot;/* host u32 [E], a permutation of [0, E): expert e lives on rank
                                   slot / (E / world) as its local expert slot % (E / world);
                                   NULL = contiguous ranges of ids */
    /* this rank's E / world routed experts in local-slot order, then the shared expert: E/world+1
     * matrices each (IQ2_XXS or Q8_0, the tensor-core types) */
    vlb_matrix* const* w1;
    vlb_matrix* const* w3;
    vlb_matrix* const* w2;
} vlb_ep_layer_desc;

int vlb_ep_layer_create(vlb_handle* h, vlb_ep_comm* comm, const vlb_ep_layer_desc* desc,
                        vlb_ep_layer** out);
int vlb_ep_layer_destroy(vlb_handle* h, vlb_ep_layer* layer);
/* One step: x_dev f32 [T x H] and logits_dev f32 [T x E] of this rank's tokens, out_dev f32
 * [T x H] = its MoE output (routed experts wherever they live + the shared expert). Every rank
 * calls it once per step (T may differ between ranks). Synchronises `stream` at the count
 * read-back and at the end (the step's status). */
int vlb_ep_forward_device(vlb_handle* h, vlb_ep_layer* layer, const float* x_dev,
                          const float* logits_dev, uint32_t T, float* out_dev, void* stream);
/* Device times (ms) of the last completed step: plan, dispatch, experts, return, combine;
 * rows[0] = rows received for this rank's experts, rows[1] = rows sent (T * k). */
int vlb_ep_last_phases(vlb_ep_layer* layer, float* ms /* [5] */, uint64_t* rows /* [2] or NULL */);

/* Route of the last forward on this layer, for parity checks: idx / weights [T x k] in rank
 * order; offsets [E + 1]; pair_token / pair_slot [T x k] = the dispatch permutation (pairs
 * sorted by expert ascending, then token, then slot - the reference's visit order,
 * deepseek_v4_graph.cpp:2134-2223). Any pointer may be NULL. */
int vlb_layer_last_route(vlb_handle* h, vlb_layer* layer, uint32_t T, uint32_t* idx,
                         float* weights, uint32_t* offsets, uint32_t* pair_token,
                         uint32_t* pair_slot);

/* Bytes of weights a forward of the last route read (router + every selected expert's three
 * matrices + the shared expert), the algorithmic numerator of the HBM roofline. */
uint64_t vlb_layer_last_weight_bytes(vlb_handle* h, vlb_layer* layer);

/* Phase timing of the layer forward (CUDA events on the launching stream, recorded only while
 * enabled): ms[0] routing (router projection, scores, top-k), ms[1] dispatch, ms[2] gate/up +
 * SwiGLU, ms[3] down, ms[4] combine, for the last forward. n must be >= 5. */
int vlb_layer_set_profiling(vlb_handle* h, vlb_layer* layer, int enable);
int vlb_layer_phase_times(vlb_handle* h, vlb_layer* layer, float* ms, int n);

/* ---- standalone routing operators (deepseek_v4_route_*_logits, deepseek_v4_reference.hpp:
 * 634-650) on device buffers ----------------------------------------------------------------
 * Both are synchronous (they synchronise `stream` to report errors) and keep their scratch in a
 * grow-only buffer of the handle (released by vlb_close), so repeated calls allocate nothing. */
int vlb_route_device(vlb_handle* h, int score, int hash_routing, const float* logits_dev,
                     const float* bias_dev, const uint32_t* token_ids_dev,
                     const uint32_t* tid2eid_dev, uint32_t vocab, uint32_t T, uint32_t E,
                     uint32_t k, float route_scale, uint32_t* idx_dev, float* weights_dev,
                     void* stream);
/* The same router as vlb_route_device for callers that cannot allocate device memory: a runtime
 * whose ResourceGovernor is refusing new reservations under memory pressure, callers that may not
 * call cudaMalloc at all, and decode loops that cannot take the synchronisation cudaMalloc/cudaFree
 * may cause (vlb_route_device grows its handle's scratch with cudaMalloc when a call needs more).
 * This entry point has no counterpart in the reference. It allocates nothing: its score scratch
 * is a fixed 1 MiB array inside the library, present on every GPU that loads the library until
 * the process exits, so T*E may be at most 262,080 (larger requests return
 * VLB_ERR_RESOURCE_EXHAUSTED). The caller passes device inputs and outputs as for
 * vlb_route_device and the device ordinal to run on (made current for the call, the caller's
 * device restored after). The first call on each device also performs a one-time set-up (it
 * looks up the array's device address). Every call uses the same array: calls that overlap on
 * the GPU (other streams, other host threads) race on it; serialise them. It is ordinary host
 * code: it synchronises `stream` before returning (the route is written then), so it must not be
 * called from a CUDA host callback or while a stream capture is open. */
int vlb_route_device_noalloc(int ordinal, int score, int hash_routing, const float* logits_dev,
                             const float* bias_dev, const uint32_t* token_ids_dev,
                             const uint32_t* tid2eid_dev, uint32_t vocab, uint32_t T, uint32_t E,
                             uint32_t k, float route_scale, uint32_t* idx_dev,
                             float* weights_dev, void* stream);
/* Router projection logits[T x E] = f32(sum double(x) double(w)) (deepseek_v4_graph.cpp:
 * 735-767). */
int vlb_router_logits_device(vlb_handle* h, const float* x_dev, const float* w_dev, uint32_t T,
                             uint32_t H, uint32_t E, float* logits_dev, void* stream);
/* deepseek_v4_rms_norm (deepseek_v4_reference.cpp:170-206) on device rows. */
int vlb_rms_norm_device(vlb_handle* h, const float* x_dev, const float* w_dev, uint32_t rows,
                        uint32_t width, float eps, float* out_dev, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* VLB200_H */
