// Host side of the vlb200 C ABI (include/vlb200.h): device handles, governed allocations,
// codebook installation, resident matrices, MoE layer objects and their forward calls.
//
// Replaces the reference's driver boundary (src/cuda/cuda_driver.cpp) and the device half of
// its accelerator (src/cuda/cuda_matvec_accelerator.cpp); see the header for the contract.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "vlb_encode.cuh"
#include "vlb_launch.h"

using namespace vlb;

namespace {

thread_local std::string t_error;

int copy_message(const std::string& msg, char* buf, size_t cap) {
    if (!buf || cap == 0) return VLB_ERR_INVALID_ARGUMENT;
    const size_t n = msg.size() < cap - 1 ? msg.size() : cap - 1;
    std::memcpy(buf, msg.data(), n);
    buf[n] = '\0';
    return VLB_OK;
}

// Pinned codebook fingerprints: FNV-1a over the table bytes, ggml_quantization.cpp:49-99.
constexpr uint64_t kFpIq1S = 0x6703ed863501ae2eull;
constexpr uint64_t kFpIq2Xxs = 0xbb4ee025b5ac6e8eull;
constexpr uint64_t kFpIq3Xxs = 0xdfa5dc83d6a155d5ull;
constexpr uint64_t kFpIq2S = 0x123edd38a3b62b90ull;  // ggml_quantization.cpp:86

uint64_t fnv1a(const void* p, size_t n) {
    const uint8_t* b = static_cast<const uint8_t*>(p);
    uint64_t h = 14695981039346656037ull;
    for (size_t i = 0; i < n; ++i) {
        h ^= b[i];
        h *= 1099511628211ull;
    }
    return h;
}

// CUDA failures become io_error with the call and CUDA's own description (the reference's
// cuda_error, cuda_driver.cpp:2727-2738).
std::string cuda_msg(const char* op, cudaError_t e) {
    return std::string("CUDA call failed: ") + op + " (status=" + std::to_string((int)e) + ", " +
           cudaGetErrorName(e) + ": " + cudaGetErrorString(e) + ")";
}

}  // namespace

namespace vlb {
// Lets other sources of the library report a failure through vlb_thread_error.
void set_thread_error(const std::string& msg) { t_error = msg; }
}  // namespace vlb

// Record uploads: tensors per record, and records in flight per handle.
constexpr uint32_t kUploadMaxTensors = 64;
constexpr uint32_t kUploadSlots = 256;

// Frees the host records of an upload the handle is closing under (its memory goes with the
// handle's allocations).
static void delete_unfinished_upload(vlb_upload* u);

struct vlb_handle {
    int device = 0;
    cudaStream_t stream = nullptr;
    vlb_governor gov{};
    bool has_gov = false;
    uint64_t min_free_after = 0;
    std::mutex mu;
    std::string err;
    uint64_t* grid_iq1s = nullptr;
    uint64_t* grid_iq2xxs = nullptr;
    uint32_t* grid_iq3xxs = nullptr;
    uint64_t* grid_iq2s = nullptr;
    struct Alloc {
        size_t bytes;
        size_t hooked;  // the part reserved through the governor hooks (the rest the caller holds)
        std::string tag;
    };
    std::unordered_map<void*, Alloc> allocs;
    uint64_t allocated = 0;
    // record uploads (vlb_upload_record_async): their own stream, the device copy of the record
    // (grown only), a pinned arena of per-upload result words and the uploads in flight
    cudaStream_t upload_stream = nullptr;
    uint8_t* upload_stage = nullptr;
    size_t upload_stage_cap = 0;
    uint32_t* upload_results = nullptr;
    std::vector<uint32_t> upload_slots;
    std::unordered_set<vlb_upload*> uploads;
    // a record's matrices share one allocation (a device allocation costs ~0.4 ms of host time):
    // live matrices per shared allocation, freed with the last of them
    std::unordered_map<void*, uint32_t> block_refs;
    float* seam_x = nullptr;
    float* seam_y = nullptr;
    size_t seam_x_cap = 0, seam_y_cap = 0;
    // grow-only scratch of the synchronous helper entry points (routing, router logits): a
    // device allocation per call would cost more than the kernels themselves
    char* scratch = nullptr;
    size_t scratch_cap = 0;

    int fail(int code, std::string msg) {
        err = std::move(msg);
        return code;
    }
    // At least `bytes` of the helper scratch (callers hold the handle lock and synchronise their
    // stream before returning, so the previous user is done with it).
    int scratch_at_least(size_t bytes, char** out) {
        if (scratch_cap < bytes) {
            if (scratch) gfree(scratch);
            scratch = nullptr;
            scratch_cap = 0;
            const int st = galloc(bytes, "vlb-call-scratch", reinterpret_cast<void**>(&scratch));
            if (st != VLB_OK) return st;
            scratch_cap = bytes;
        }
        *out = scratch;
        return VLB_OK;
    }
    int cuda_fail(const char* op, cudaError_t e) {
        (void)cudaGetLastError();  // clear a sticky launch error so the handle stays usable
        return fail(VLB_ERR_IO_ERROR, cuda_msg(op, e));
    }
    Grids grids() const { return Grids{grid_iq1s, grid_iq2xxs, grid_iq3xxs, grid_iq2s}; }
    cudaStream_t pick(void* s) const { return s ? static_cast<cudaStream_t>(s) : stream; }

    // Governor-first allocation (CudaDriver::allocate, cuda_driver.cpp:2929-3005): reserve the
    // exact bytes, check live free memory against the configured floor, then allocate; every
    // failure after a successful reserve releases it again. `covered`: bytes of this allocation
    // the caller already holds a reservation for (a residency object's VRAM destination), which
    // the hooks are not charged for.
    int galloc(size_t bytes, const char* tag, void** out, size_t covered = 0) {
        *out = nullptr;
        if (bytes == 0) return fail(VLB_ERR_INVALID_ARGUMENT, "zero-byte device allocation");
        const size_t hooked = bytes - std::min(bytes, covered);
        const bool charge = has_gov && hooked != 0;
        if (charge && gov.reserve && gov.reserve(gov.ctx, hooked, tag) != 0)
            return fail(VLB_ERR_RESOURCE_EXHAUSTED,
                        std::string("governor refused the device reservation: ") + tag);
        size_t free_b = 0, total_b = 0;
        cudaError_t e = cudaMemGetInfo(&free_b, &total_b);
        if (e != cudaSuccess) {
            if (charge && gov.release) gov.release(gov.ctx, hooked, tag);
            return cuda_fail("cudaMemGetInfo", e);
        }
        if ((uint64_t)free_b < (uint64_t)bytes + min_free_after) {
            if (charge && gov.release) gov.release(gov.ctx, hooked, tag);
            return fail(VLB_ERR_RESOURCE_EXHAUSTED,
                        std::string("device allocation would cross the free-memory floor: ") + tag);
        }
        e = cudaMalloc(out, bytes);
        if (e != cudaSuccess) {
            *out = nullptr;
            if (charge && gov.release) gov.release(gov.ctx, hooked, tag);
            return cuda_fail("cudaMalloc", e);
        }
        allocs[*out] = Alloc{bytes, hooked, tag};
        allocated += bytes;
        return VLB_OK;
    }
    int gfree(void* p) {
        if (!p) return VLB_OK;
        auto it = allocs.find(p);
        if (it == allocs.end()) return fail(VLB_ERR_NOT_FOUND, "pointer is not a live allocation");
        cudaError_t e = cudaFree(p);
        if (e != cudaSuccess) {
            // Keep it accounted: a failed release must not hand the bytes back
            // (cuda_driver.cpp:2881-2894).
            return cuda_fail("cudaFree", e);
        }
        if (has_gov && gov.release && it->second.hooked)
            gov.release(gov.ctx, it->second.hooked, it->second.tag.c_str());
        allocated -= it->second.bytes;
        allocs.erase(it);
        return VLB_OK;
    }
};

struct vlb_matrix {
    vlb_handle* owner = nullptr;
    uint64_t identity = 0;
    uint32_t type = 0;
    size_t rows = 0, cols = 0;
    uint32_t bpr = 0;
    void* mem = nullptr;
    void* block = nullptr;  // the allocation it shares with the other matrices of one record
    size_t bytes = 0;  // resident bytes (scales + bodies)
    size_t payload_bytes = 0;
    DevMat dm{};
};

struct vlb_layer {
    vlb_moe_layer_desc desc{};
    bool has_shared = false;
    double* router = nullptr;  // f64 widening of the f32 router weights
    float* bias = nullptr;
    uint32_t* tid2eid = nullptr;
    DevMat* mats = nullptr;
    std::vector<const vlb_matrix*> host_mats;  // [3 x (E+1)]
    // residual block entry (vlb_layer_set_input_norm): RMSNorm weight [H] and epsilon
    float* norm_w = nullptr;
    float norm_eps = 0.f;
    // Hyper-Connection block (vlb_layer_set_hyper_connection): its parameters and split buffers in
    // one allocation; x_dev / out_dev then hold m copies per token
    void* hc_mem = nullptr;
    uint32_t hc_m = 0;
    // workspace
    void* ws = nullptr;
    MoeParams p{};
    uint32_t last_T = 0;
    bool last_logits_given = false;
    // forwards of at least this many tokens run the expert products on the prefill kernels
    uint32_t prefill_min_tokens = 0;
    // staging for the host-memory forward
    float* x_dev = nullptr;
    uint32_t* tok_dev = nullptr;
    float* logits_dev = nullptr;
    float* out_dev = nullptr;
    // the forward captured as a CUDA graph for one input binding, replayed while it matches
    cudaGraphExec_t gexec = nullptr;
    const void* gkey[7] = {nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
    uint32_t gkey_T = 0;
    // optional phase timing (vlb_layer_set_profiling)
    bool profiling = false;
    cudaEvent_t ev[kMoePhases + 1] = {};
};

#define VLB_LOCK(h)                                                                     \
    if (!(h)) {                                                                          \
        t_error = "null handle";                                                         \
        return VLB_ERR_INVALID_ARGUMENT;                                                 \
    }                                                                                    \
    std::lock_guard<std::mutex> _vlb_lock((h)->mu);                                      \
    {                                                                                    \
        cudaError_t _e = cudaSetDevice((h)->device);                                     \
        if (_e != cudaSuccess) return (h)->cuda_fail("cudaSetDevice", _e);               \
    }

#define VLB_CUDA(h, call)                                    \
    do {                                                     \
        cudaError_t _e = (call);                             \
        if (_e != cudaSuccess) return (h)->cuda_fail(#call, _e); \
    } while (0)

extern "C" {

int vlb_abi_version(void) { return VLB_ABI_VERSION; }

int vlb_thread_error(char* buf, size_t cap) { return copy_message(t_error, buf, cap); }

int vlb_device_count(int* count) {
    if (!count) return VLB_ERR_INVALID_ARGUMENT;
    *count = 0;
    cudaError_t e = cudaGetDeviceCount(count);
    if (e != cudaSuccess) {
        *count = 0;
        (void)cudaGetLastError();
        t_error = cuda_msg("cudaGetDeviceCount", e);
        return VLB_ERR_NOT_FOUND;
    }
    return VLB_OK;
}

int vlb_probe(int ordinal, vlb_device_info* info) {
    if (!info) return VLB_ERR_INVALID_ARGUMENT;
    int n = 0;
    if (vlb_device_count(&n) != VLB_OK || ordinal < 0 || ordinal >= n) {
        t_error = "CUDA device ordinal is not present";
        return VLB_ERR_NOT_FOUND;
    }
    cudaDeviceProp prop{};
    cudaError_t e = cudaGetDeviceProperties(&prop, ordinal);
    if (e != cudaSuccess) {
        t_error = cuda_msg("cudaGetDeviceProperties", e);
        return VLB_ERR_IO_ERROR;
    }
    std::memset(info, 0, sizeof(*info));
    info->ordinal = ordinal;
    info->sm_count = prop.multiProcessorCount;
    info->cc_major = prop.major;
    info->cc_minor = prop.minor;
    info->total_bytes = prop.totalGlobalMem;
    std::snprintf(info->name, sizeof(info->name), "%s", prop.name);
    int prev = 0;
    cudaGetDevice(&prev);
    if (cudaSetDevice(ordinal) == cudaSuccess) {
        size_t f = 0, t = 0;
        if (cudaMemGetInfo(&f, &t) == cudaSuccess) info->free_bytes = f;
        cudaSetDevice(prev);
    }
    return VLB_OK;
}

int vlb_open(int ordinal, const vlb_governor* governor, uint64_t min_free_after,
             vlb_handle** out) {
    if (!out) {
        t_error = "null output handle";
        return VLB_ERR_INVALID_ARGUMENT;
    }
    *out = nullptr;
    vlb_device_info info{};
    int st = vlb_probe(ordinal, &info);
    if (st != VLB_OK) return st;
    if (info.cc_major != 10) {
        t_error = "this library is built for sm_100a (B200); device compute capability is " +
                  std::to_string(info.cc_major) + "." + std::to_string(info.cc_minor);
        return VLB_ERR_UNSUPPORTED;
    }
    vlb_handle* h = new (std::nothrow) vlb_handle();
    if (!h) {
        t_error = "unable to allocate the handle";
        return VLB_ERR_RESOURCE_EXHAUSTED;
    }
    h->device = ordinal;
    h->min_free_after = min_free_after;
    if (governor) {
        h->gov = *governor;
        h->has_gov = true;
    }
    cudaError_t e = cudaSetDevice(ordinal);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        t_error = cuda_msg("cudaStreamCreate", e);
        delete h;
        return VLB_ERR_IO_ERROR;
    }
    *out = h;
    return VLB_OK;
}

void vlb_close(vlb_handle* h) {
    if (!h) return;
    {
        std::lock_guard<std::mutex> lock(h->mu);
        cudaSetDevice(h->device);
        cudaStreamSynchronize(h->stream);
        if (h->upload_stream) cudaStreamSynchronize(h->upload_stream);
        for (vlb_upload* u : h->uploads) delete_unfinished_upload(u);
        h->uploads.clear();
        for (auto& kv : h->allocs) {
            cudaFree(kv.first);
            if (h->has_gov && h->gov.release && kv.second.hooked)
                h->gov.release(h->gov.ctx, kv.second.hooked, kv.second.tag.c_str());
        }
        h->allocs.clear();
        if (h->upload_stream) cudaStreamDestroy(h->upload_stream);
        if (h->upload_results) cudaFreeHost(h->upload_results);
        cudaStreamDestroy(h->stream);
    }
    delete h;
}

int vlb_last_error(const vlb_handle* h, char* buf, size_t cap) {
    if (!h) return copy_message(t_error, buf, cap);
    return copy_message(h->err, buf, cap);
}

void* vlb_stream(vlb_handle* h) { return h ? (void*)h->stream : nullptr; }

int vlb_synchronize(vlb_handle* h) {
    VLB_LOCK(h);
    VLB_CUDA(h, cudaStreamSynchronize(h->stream));
    return VLB_OK;
}

int vlb_set_codebook(vlb_handle* h, uint32_t type, const void* table, size_t bytes) {
    VLB_LOCK(h);
    if (!table) return h->fail(VLB_ERR_INVALID_ARGUMENT, "null codebook");
    size_t want = 0;
    uint64_t fp = 0;
    void** slot = nullptr;
    switch (type) {
        case VLB_TYPE_IQ1_S: want = 2048 * 8; fp = kFpIq1S; slot = (void**)&h->grid_iq1s; break;
        case VLB_TYPE_IQ2_XXS: want = 256 * 8; fp = kFpIq2Xxs; slot = (void**)&h->grid_iq2xxs; break;
        case VLB_TYPE_IQ3_XXS: want = 256 * 4; fp = kFpIq3Xxs; slot = (void**)&h->grid_iq3xxs; break;
        case VLB_TYPE_IQ2_S: want = 1024 * 8; fp = kFpIq2S; slot = (void**)&h->grid_iq2s; break;
        default: return h->fail(VLB_ERR_UNSUPPORTED, "storage type has no codebook");
    }
    if (bytes != want) return h->fail(VLB_ERR_INVALID_FORMAT, "codebook has the wrong size");
    if (fnv1a(table, bytes) != fp)
        return h->fail(VLB_ERR_INTEGRITY_ERROR, "codebook fingerprint does not match the pinned ggml table");
    if (!*slot) {
        int st = h->galloc(bytes, "vlb-codebook", slot);
        if (st != VLB_OK) return st;
    }
    VLB_CUDA(h, cudaMemcpy(*slot, table, bytes, cudaMemcpyHostToDevice));
    return VLB_OK;
}

int vlb_alloc(vlb_handle* h, size_t bytes, const char* tag, void** dev_ptr) {
    VLB_LOCK(h);
    if (!dev_ptr) return h->fail(VLB_ERR_INVALID_ARGUMENT, "null output pointer");
    return h->galloc(bytes, tag ? tag : "vlb-buffer", dev_ptr);
}

int vlb_free(vlb_handle* h, void* p) {
    VLB_LOCK(h);
    return h->gfree(p);
}

int vlb_memcpy_h2d(vlb_handle* h, void* dst, const void* src, size_t bytes) {
    VLB_LOCK(h);
    VLB_CUDA(h, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, h->stream));
    VLB_CUDA(h, cudaStreamSynchronize(h->stream));
    return VLB_OK;
}

int vlb_memcpy_d2h(vlb_handle* h, void* dst, const void* src, size_t bytes) {
    VLB_LOCK(h);
    VLB_CUDA(h, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, h->stream));
    VLB_CUDA(h, cudaStreamSynchronize(h->stream));
    return VLB_OK;
}

uint64_t vlb_allocated_bytes(const vlb_handle* h) { return h ? h->allocated : 0; }

// ---- matrices -------------------------------------------------------------------------------

static float half_bits_to_float(uint16_t bits) {
    const uint32_t e = (bits >> 10) & 0x1fu, m = bits & 0x3ffu;
    const float mag = e == 0 ? std::ldexp((float)m, -24) : std::ldexp((float)(m | 0x400u), (int)e - 25);
    return (bits & 0x8000u) ? -mag : mag;
}

// TMA descriptor of a row-major fp16 matrix [rows x cols] read as boxes of 64 columns x
// prefill_box_rows() rows with the 128-byte swizzle of the UMMA K-major operand layout
// (cuTensorMapEncodeTiled, resolved through the runtime so the library does not link the driver
// API).
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(f);
    });
    return fn;
}

static bool encode_rows_fp16(CUtensorMap* map, void* base, size_t rows, size_t cols) {
    EncodeTiledFn fn = encode_tiled();
    if (!fn) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * 2};
    const cuuint32_t box[2] = {64, prefill_box_rows()};
    const cuuint32_t estr[2] = {1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The power of two the prefill kernels scale a matrix's weights by before rounding them to fp16:
// the largest possible |weight| (largest block scale x the format's largest factor: 128 for a
// Q8_0 quant, 15.5 / 4 x 43 for an IQ2_XXS grid value) lands in [2^13, 2^14).
static float prefill_scale(uint32_t type, float dmax) {
    const float factor = type == VLB_TYPE_Q8_0 ? 128.f : type == VLB_TYPE_IQ2_XXS ? 167.f : 0.f;
    const float bound = dmax * factor;
    if (!(bound > 0.f)) return 1.f;
    int e = 0;
    std::frexp(bound, &e);  // bound = f * 2^e, f in [0.5, 1)
    return std::ldexp(1.f, 14 - e);
}

// Checks one matrix's type, shape and payload size (both upload paths).
static int check_matrix(vlb_handle* h, uint32_t type, size_t rows, size_t cols, size_t payload_bytes,
                        TypeLayout* L) {
    if (!type_layout(type, L)) return h->fail(VLB_ERR_UNSUPPORTED, "storage type has no device kernel");
    if ((type == VLB_TYPE_IQ1_S && !h->grid_iq1s) || (type == VLB_TYPE_IQ2_XXS && !h->grid_iq2xxs) ||
        (type == VLB_TYPE_IQ3_XXS && !h->grid_iq3xxs) || (type == VLB_TYPE_IQ2_S && !h->grid_iq2s))
        return h->fail(VLB_ERR_NOT_FOUND, "the codebook for this storage type is not installed");
    if (rows == 0 || cols == 0 || cols % L->block_elems != 0 || rows > 0xffffffffu ||
        cols > 0xffffffffu || cols % 32 != 0)
        return h->fail(VLB_ERR_INVALID_ARGUMENT, "matrix dimensions are invalid");
    if (payload_bytes != rows * (cols / L->block_elems) * L->block_bytes)
        return h->fail(VLB_ERR_INVALID_FORMAT, "matrix payload size does not match its shape");
    return VLB_OK;
}

// The record of a matrix whose image (matrix_image) sits at m->mem. dmag: the largest |d| of a
// split-format matrix as fp16 bits (fp16 magnitudes order as integers).
static void describe_matrix(vlb_matrix* m, vlb_handle* h, uint64_t identity, uint32_t type, const TypeLayout& L,
                            const MatrixImage& img, size_t rows, size_t cols, size_t payload_bytes, uint16_t dmag) {
    const uint32_t bpr = (uint32_t)(cols / L.block_elems);
    const uint8_t* mem = reinterpret_cast<const uint8_t*>(m->mem);
    m->owner = h;
    m->identity = identity;
    m->type = type;
    m->rows = rows;
    m->cols = cols;
    m->bpr = bpr;
    m->bytes = img.resident;
    m->payload_bytes = payload_bytes;
    if (raw_type(type)) {
        m->dm = DevMat{type, (uint32_t)rows, (uint32_t)cols, bpr, nullptr, mem, nullptr, 1.f};
    } else {
        m->dm = DevMat{type, (uint32_t)rows, (uint32_t)cols, bpr, reinterpret_cast<const uint16_t*>(mem),
                       mem + img.d_bytes + img.sc_bytes,
                       img.sc_bytes ? reinterpret_cast<const uint32_t*>(mem + img.d_bytes) : nullptr,
                       prefill_scale(type, half_bits_to_float(dmag))};
    }
}

int vlb_upload_matrix(vlb_handle* h, uint64_t identity, uint32_t type, size_t rows,
                      size_t cols, const void* payload, size_t payload_bytes, vlb_matrix** out) {
    VLB_LOCK(h);
    if (!out || !payload) return h->fail(VLB_ERR_INVALID_ARGUMENT, "null matrix argument");
    *out = nullptr;
    TypeLayout L{};
    int st = check_matrix(h, type, rows, cols, payload_bytes, &L);
    if (st != VLB_OK) return st;
    const uint8_t* src = static_cast<const uint8_t*>(payload);
    const size_t bpr = cols / L.block_elems, nblocks = rows * bpr;
    uint16_t dmag = 0;
    for (size_t b = 0; b < nblocks; ++b) {
        const uint8_t* blk = src + b * L.block_bytes;
        if (!block_finite(type, blk)) return h->fail(VLB_ERR_INVALID_FORMAT, "quantized block scale is not finite");
        if (!raw_type(type)) dmag = std::max<uint16_t>(dmag, ld_u16(blk) & 0x7fffu);
    }
    const MatrixImage img = matrix_image(type, L, rows, cols);
    std::vector<uint8_t> staged;
    try {
        staged.assign(img.total, 0);
    } catch (const std::bad_alloc&) {
        return h->fail(VLB_ERR_RESOURCE_EXHAUSTED, "unable to stage the matrix on the host");
    }
    for (size_t r = 0; r < rows; ++r)
        for (size_t c = 0; c < bpr; ++c)
            encode_block(type, L, img, src + (r * bpr + c) * L.block_bytes,
                         blk_index((uint32_t)bpr, (uint32_t)r, (uint32_t)c), staged.data());
    vlb_matrix* m = new (std::nothrow) vlb_matrix();
    if (!m) return h->fail(VLB_ERR_RESOURCE_EXHAUSTED, "unable to allocate the matrix record");
    st = h->galloc(staged.size(), "vlb-resident-matrix", &m->mem);
    if (st != VLB_OK) {
        delete m;
        return st;
    }
    cudaError_t e = cudaMemcpy(m->mem, staged.data(), staged.size(), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        h->gfree(m->mem);
        delete m;
        return h->cuda_fail("cudaMemcpy(matrix)", e);
    }
    describe_matrix(m, h, identity, type, L, img, rows, cols, payload_bytes, dmag);
    *out = m;
    return VLB_OK;
}

// ---- expert records: one host-to-device copy, the re-layout on the device ------------------

}  // extern "C"

namespace {

// One tensor of a record for encode_record_kernel.
struct RecordJob {
    const uint8_t* src;  // its ggml bytes in the device copy of the record
    uint8_t* img;        // its matrix image
    uint32_t* result;    // [0] nonzero = a block the reference rejects, [1] largest |d| (fp16 bits)
    MatrixImage m;
    TypeLayout L;
    uint32_t type, bpr;
    size_t nblocks;
};

__global__ void __launch_bounds__(256) encode_record_kernel(RecordJob j) {
    uint32_t bad = 0, dmag = 0;
    const bool split = !raw_type(j.type);
    for (size_t b = (size_t)blockIdx.x * blockDim.x + threadIdx.x; b < j.nblocks; b += (size_t)gridDim.x * blockDim.x) {
        const uint8_t* blk = j.src + b * j.L.block_bytes;
        if (!block_finite(j.type, blk)) bad = 1u;
        if (split) dmag = max(dmag, (uint32_t)(ld_u16(blk) & 0x7fffu));
        const uint32_t r = (uint32_t)(b / j.bpr), c = (uint32_t)(b % j.bpr);
        encode_block(j.type, j.L, j.m, blk, blk_index(j.bpr, r, c), j.img);
    }
    bad = __reduce_or_sync(0xffffffffu, bad);
    dmag = __reduce_max_sync(0xffffffffu, dmag);
    if ((threadIdx.x & 31u) == 0u) {
        if (bad) atomicOr(j.result, 1u);
        if (dmag) atomicMax(j.result + 1, dmag);
    }
}

}  // namespace

struct vlb_upload {
    vlb_handle* owner = nullptr;
    std::vector<vlb_record_tensor> tensors;
    std::vector<vlb_matrix*> mats;
    uint32_t slot = 0;  // its results in the handle's pinned arena
    cudaEvent_t done = nullptr;
};

static void delete_unfinished_upload(vlb_upload* u) {
    for (vlb_matrix* m : u->mats) delete m;
    if (u->done) cudaEventDestroy(u->done);
    delete u;
}

// Releases an upload's matrices and its results slot (stream work on them has finished or was
// never enqueued).
// Frees a matrix's device image: its own allocation, or its share of a record's allocation (freed
// with the last matrix that uses it).
static int release_image(vlb_handle* h, vlb_matrix* m) {
    if (!m->block) return h->gfree(m->mem);
    auto it = h->block_refs.find(m->block);
    if (it == h->block_refs.end()) return h->fail(VLB_ERR_NOT_FOUND, "matrix block is not live");
    if (it->second > 1u) {
        --it->second;
        return VLB_OK;
    }
    const int st = h->gfree(m->block);
    if (st == VLB_OK) h->block_refs.erase(it);
    return st;
}

static void drop_upload(vlb_handle* h, vlb_upload* u) {
    for (vlb_matrix* m : u->mats) {
        if (!m) continue;
        release_image(h, m);
        delete m;
    }
    u->mats.clear();
    if (u->done) cudaEventDestroy(u->done);
    h->upload_slots.push_back(u->slot);
    h->uploads.erase(u);
    delete u;
}

extern "C" {

int vlb_upload_record_async(vlb_handle* h, const void* record, size_t record_bytes,
                            const vlb_record_tensor* tensors, uint32_t n, uint64_t reserved_bytes,
                            vlb_upload** out) {
    VLB_LOCK(h);
    if (!out || !record || !tensors || record_bytes == 0)
        return h->fail(VLB_ERR_INVALID_ARGUMENT, "null record argument");
    *out = nullptr;
    if (n == 0 || n > kUploadMaxTensors)
        return h->fail(VLB_ERR_INVALID_ARGUMENT, "a record holds 1 to 64 tensors");
    std::vector<TypeLayout> layouts(n);
    for (uint32_t i = 0; i < n; ++i) {
        const vlb_record_tensor& t = tensors[i];
        const int st = check_matrix(h, t.ggml_type, t.rows, t.storage_cols, t.bytes, &layouts[i]);
        if (st != VLB_OK) return h->fail(st, "record tensor " + std::to_string(i) + ": " + h->err);
        if (t.offset > record_bytes || t.bytes > record_bytes - t.offset)
            return h->fail(VLB_ERR_INVALID_FORMAT, "record tensor " + std::to_string(i) + " lies outside the record");
    }
    if (!h->upload_stream) {
        VLB_CUDA(h, cudaStreamCreateWithFlags(&h->upload_stream, cudaStreamNonBlocking));
        void* arena = nullptr;
        VLB_CUDA(h, cudaHostAlloc(&arena, (size_t)kUploadSlots * kUploadMaxTensors * 8, cudaHostAllocPortable));
        h->upload_results = static_cast<uint32_t*>(arena);
        for (uint32_t s = kUploadSlots; s-- > 0;) h->upload_slots.push_back(s);
    }
    if (h->upload_slots.empty())
        return h->fail(VLB_ERR_RESOURCE_EXHAUSTED, "too many record uploads in flight");
    // the device copy of the record, then the results words; grown only, reused in stream order
    const size_t res_off = (record_bytes + 255) / 256 * 256;
    const size_t stage_need = res_off + (size_t)kUploadMaxTensors * 8;
    if (h->upload_stage_cap < stage_need) {
        if (h->upload_stage) {
            VLB_CUDA(h, cudaStreamSynchronize(h->upload_stream));
            h->gfree(h->upload_stage);
        }
        h->upload_stage = nullptr;
        h->upload_stage_cap = 0;
        const int st = h->galloc(stage_need, "vlb-upload-staging", reinterpret_cast<void**>(&h->upload_stage));
        if (st != VLB_OK) return st;
        h->upload_stage_cap = stage_need;
    }
    vlb_upload* u = new (std::nothrow) vlb_upload();
    if (!u) return h->fail(VLB_ERR_RESOURCE_EXHAUSTED, "unable to allocate the upload record");
    u->owner = h;
    u->slot = h->upload_slots.back();
    h->upload_slots.pop_back();
    h->uploads.insert(u);
    u->tensors.assign(tensors, tensors + n);
    u->mats.assign(n, nullptr);
    // device images, 256-byte aligned in one allocation; the caller's VRAM reservation covers the
    // first reserved_bytes of it
    std::vector<size_t> at(n);
    size_t total = 0;
    for (uint32_t i = 0; i < n; ++i) {
        at[i] = total;
        total += (matrix_image(tensors[i].ggml_type, layouts[i], tensors[i].rows, tensors[i].storage_cols).total + 255) /
                 256 * 256;
    }
    void* block = nullptr;
    {
        const int st = h->galloc(total, "vlb-resident-matrix", &block, std::min<uint64_t>(reserved_bytes, total));
        if (st != VLB_OK) {
            const std::string msg = h->err;
            drop_upload(h, u);
            return h->fail(st, msg);
        }
    }
    h->block_refs[block] = 0;
    for (uint32_t i = 0; i < n; ++i) {
        vlb_matrix* m = new (std::nothrow) vlb_matrix();
        if (!m) {
            if (h->block_refs[block] == 0) {
                h->block_refs.erase(block);
                h->gfree(block);
            }
            drop_upload(h, u);
            return h->fail(VLB_ERR_RESOURCE_EXHAUSTED, "unable to allocate the matrix record");
        }
        m->mem = static_cast<char*>(block) + at[i];
        m->block = block;
        ++h->block_refs[block];
        u->mats[i] = m;
    }
    cudaStream_t s = h->upload_stream;
    uint32_t* res_dev = reinterpret_cast<uint32_t*>(h->upload_stage + res_off);
    uint32_t* res_host = h->upload_results + (size_t)u->slot * kUploadMaxTensors * 2;
    cudaError_t e = cudaEventCreateWithFlags(&u->done, cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaMemsetAsync(res_dev, 0, (size_t)n * 8, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(h->upload_stage, record, record_bytes, cudaMemcpyHostToDevice, s);
    for (uint32_t i = 0; i < n && e == cudaSuccess; ++i) {
        const vlb_record_tensor& t = tensors[i];
        RecordJob j{};
        j.src = h->upload_stage + t.offset;
        j.img = static_cast<uint8_t*>(u->mats[i]->mem);
        j.result = res_dev + 2 * i;
        j.L = layouts[i];
        j.m = matrix_image(t.ggml_type, j.L, t.rows, t.storage_cols);
        j.type = t.ggml_type;
        j.bpr = (uint32_t)(t.storage_cols / j.L.block_elems);
        j.nblocks = (size_t)t.rows * j.bpr;
        e = cudaMemsetAsync(j.img, 0, j.m.total, s);
        if (e != cudaSuccess) break;
        const size_t want = (j.nblocks + 255) / 256;
        const unsigned grid = (unsigned)std::max<size_t>(1, std::min<size_t>(want, 148u * 8u));
        encode_record_kernel<<<grid, 256, 0, s>>>(j);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpyAsync(res_host, res_dev, (size_t)n * 8, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaEventRecord(u->done, s);
    if (e != cudaSuccess) {
        cudaStreamSynchronize(s);
        drop_upload(h, u);
        return h->cuda_fail("record upload", e);
    }
    *out = u;
    return VLB_OK;
}

int vlb_upload_query(vlb_handle* h, vlb_upload* u, int* done) {
    VLB_LOCK(h);
    if (!u || !done || u->owner != h || !h->uploads.count(u))
        return h->fail(VLB_ERR_INVALID_ARGUMENT, "upload does not belong to this handle");
    const cudaError_t e = cudaEventQuery(u->done);
    if (e == cudaErrorNotReady) {
        *done = 0;
        return VLB_OK;
    }
    if (e != cudaSuccess) return h->cuda_fail("cudaEventQuery(upload)", e);
    *done = 1;
    return VLB_OK;
}

int vlb_upload_finish(vlb_handle* h, vlb_upload* u, vlb_matrix** out, uint32_t n) {
    VLB_LOCK(h);
    if (!u || u->owner != h || !h->uploads.count(u))
        return h->fail(VLB_ERR_INVALID_ARGUMENT, "upload does not belong to this handle");
    // the copy and the re-layout kernels wait on nothing, so this wait ends
    const cudaError_t e = cudaEventSynchronize(u->done);
    if (e != cudaSuccess) {
        cudaStreamSynchronize(h->upload_stream);
        drop_upload(h, u);
        return h->cuda_fail("record upload", e);
    }
    const uint32_t* res = h->upload_results + (size_t)u->slot * kUploadMaxTensors * 2;
    const uint32_t count = (uint32_t)u->tensors.size();
    for (uint32_t i = 0; i < count; ++i)
        if (res[2 * i]) {
            drop_upload(h, u);
            return h->fail(VLB_ERR_INVALID_FORMAT,
                           "record tensor " + std::to_string(i) + ": quantized block scale is not finite");
        }
    if (!out || n != count) {
        drop_upload(h, u);
        return h->fail(VLB_ERR_INVALID_ARGUMENT, "the output array must hold one matrix per record tensor");
    }
    for (uint32_t i = 0; i < count; ++i) {
        const vlb_record_tensor& t = u->tensors[i];
        TypeLayout L{};
        type_layout(t.ggml_type, &L);
        describe_matrix(u->mats[i], h, t.cache_identity, t.ggml_type, L,
                        matrix_image(t.ggml_type, L, t.rows, t.storage_cols), t.rows, t.storage_cols, t.bytes,
                        (uint16_t)res[2 * i + 1]);
        out[i] = u->mats[i];
    }
    u->mats.clear();
    drop_upload(h, u);
    return VLB_OK;
}

int vlb_host_alloc(vlb_handle* h, size_t bytes, void** out) {
    VLB_LOCK(h);
    if (!out || bytes == 0) return h->fail(VLB_ERR_INVALID_ARGUMENT, "invalid pinned allocation");
    *out = nullptr;
    const cudaError_t e = cudaHostAlloc(out, bytes, cudaHostAllocPortable);
    if (e != cudaSuccess) {
        *out = nullptr;
        (void)cudaGetLastError();
        return h->fail(VLB_ERR_RESOURCE_EXHAUSTED, cuda_msg("cudaHostAlloc", e));
    }
    return VLB_OK;
}

int vlb_host_free(vlb_handle* h, void* p) {
    VLB_LOCK(h);
    if (!p) return VLB_OK;
    VLB_CUDA(h, cudaFreeHost(p));
    return VLB_OK;
}


int vlb_release_matrix(vlb_handle* h, vlb_matrix* m) {
    VLB_LOCK(h);
    if (!m || m->owner != h) return h->fail(VLB_ERR_INVALID_ARGUMENT, "matrix does not belong to this handle");
    int st = release_image(h, m);
    if (st != VLB_OK) return st;
    delete m;
    return VLB_OK;
}

uint64_t vlb_matrix_bytes(const vlb_matrix* m) { return m ? m->payload_bytes : 0; }

int vlb_matvec(vlb_handle* h, const vlb_matrix* m, const float* x, float* y) {
    VLB_LOCK(h);
    if (!m || m->owner != h || !x || !y) return h->fail(VLB_ERR_INVALID_ARGUMENT, "invalid matvec argument");
    if (h->seam_x_cap < m->cols) {
        if (h->seam_x) h->gfree(h->seam_x);
        h->seam_x = nullptr;
        h->seam_x_cap = 0;
        int st = h->galloc(m->cols * sizeof(float), "vlb-seam-input", (void**)&h->seam_x);
        if (st != VLB_OK) return st;
        h->seam_x_cap = m->cols;
    }
    if (h->seam_y_cap < m->rows) {
        if (h->seam_y) h->gfree(h->seam_y);
        h->seam_y = nullptr;
        h->seam_y_cap = 0;
        int st = h->galloc(m->rows * sizeof(float), "vlb-seam-output", (void**)&h->seam_y);
        if (st != VLB_OK) return st;
        h->seam_y_cap = m->rows;
    }
    VLB_CUDA(h, cudaMemcpyAsync(h->seam_x, x, m->cols * sizeof(float), cudaMemcpyHostToDevice, h->stream));
    VLB_CUDA(h, launch_gemv(m->dm, h->grids(), h->seam_x, 1, (uint32_t)m->cols, h->seam_y, (uint32_t)m->rows, h->stream));
    VLB_CUDA(h, cudaMemcpyAsync(y, h->seam_y, m->rows * sizeof(float), cudaMemcpyDeviceToHost, h->stream));
    VLB_CUDA(h, cudaStreamSynchronize(h->stream));
    return VLB_OK;
}

int vlb_matvec_device(vlb_handle* h, const vlb_matrix* m, const float* x, size_t ntok,
                      size_t xstride, float* y, size_t ystride, void* stream) {
    VLB_LOCK(h);
    if (!m || m->owner != h || !x || !y || xstride < m->cols || ystride < m->rows)
        return h->fail(VLB_ERR_INVALID_ARGUMENT, "invalid matvec argument");
    VLB_CUDA(h, launch_gemv(m->dm, h->grids(), x, (uint32_t)ntok, (uint32_t)xstride, y, (uint32_t)ystride, h->pick(stream)));
    return VLB_OK;
}

int vlb_dequantize_device(vlb_handle* h, const vlb_matrix* m, float* out, void* stream) {
    VLB_LOCK(h);
    if (!m || m->owner != h || !out) return h->fail(VLB_ERR_INVALID_ARGUMENT, "invalid dequantize argument");
    VLB_CUDA(h, launch_dequant(m->dm, h->grids(), out, h->pick(stream)));
    return VLB_OK;
}

// ---- layers ---------------------------------------------------------------------------------

// K-split items the decode kernels' scratch holds per layer (16 KB each): enough for about four
// items per SM at decode sizes where the (unit, row group) items alone are too few.
constexpr uint32_t kSplitItems = 640;

static uint32_t max_units_for(uint32_t T, uint32_t k, uint32_t E) {
    return T * k / (uint32_t)kUnitTokens + E + T / (uint32_t)kUnitTokens + 8u;
}

static void free_layer(vlb_handle* h, vlb_layer* L) {
    if (L->gexec) cudaGraphExecDestroy(L->gexec);
    for (auto& e : L->ev)
        if (e) cudaEventDestroy(e);
    void* ptrs[] = {L->router, L->bias, L->tid2eid, L->mats, L->ws,
                    L->x_dev, L->tok_dev, L->logits_dev, L->out_dev, L->norm_w, L->hc_mem};
    for (void* p : ptrs)
        if (p) h->gfree(p);
    delete L;
}

int vlb_layer_create(vlb_handle* h, const vlb_moe_layer_desc* d, vlb_layer** out) {
    VLB_LOCK(h);
    if (!d || !out) return h->fail(VLB_ERR_INVALID_ARGUMENT, "null layer argument");
    *out = nullptr;
    const uint32_t H = d->hidden, I = d->intermediate, E = d->experts, k = d->top_k;
    if (H == 0 || I == 0 || E == 0 || k == 0 || k > E || k > 16 || E > 512 || H % 256 ||
        I % 256 || d->max_tokens == 0 || !d->w1 || !d->w3 || !d->w2)
        return h->fail(VLB_ERR_INVALID_ARGUMENT, "MoE layer dimensions are invalid");
    if (d->score < VLB_SCORE_SQRT_SOFTPLUS || d->score > VLB_SCORE_SOFTMAX_F64_NORM)
        return h->fail(VLB_ERR_INVALID_ARGUMENT, "unknown router score mode");
    if (d->score <= VLB_SCORE_SIGMOID && !(d->route_scale > 0.f && std::isfinite(d->route_scale)))
        return h->fail(VLB_ERR_INVALID_ARGUMENT, "route scale must be finite and positive");
    if (d->hash_routing && (!d->tid2eid || d->vocab == 0))
        return h->fail(VLB_ERR_INVALID_ARGUMENT, "hash routing needs a token-to-expert table");
    if (!d->router) return h->fail(VLB_ERR_INVALID_ARGUMENT, "the router weight is required");
    const bool has_shared = d->shared_w1 && d->shared_w3 && d->shared_w2;
    std::vector<const vlb_matrix*> hm(3 * (E + 1), nullptr);
    for (uint32_t e = 0; e < E; ++e) {
        hm[e] = d->w1[e];
        hm[(E + 1) + e] = d->w3[e];
        hm[2 * (E + 1) + e] = d->w2[e];
    }
    if (has_shared) {
        hm[E] = d->shared_w1;
        hm[(E + 1) + E] = d->shared_w3;
        hm[2 * (E + 1) + E] = d->shared_w2;
    }
    for (uint32_t e = 0; e < E + (has_shared ? 1u : 0u); ++e) {
        const vlb_matrix* a = hm[e];
        const vlb_matrix* b = hm[(E + 1) + e];
        const vlb_matrix* c = hm[2 * (E + 1) + e];
        if (!a || !b || !c || a->owner != h || b->owner != h || c->owner != h)
            return h->fail(VLB_ERR_INVALID_ARGUMENT, "an expert matrix is missing or foreign");
        if (a->rows != I || a->cols != H || b->rows != I || b->cols != H || c->rows != H ||
            c->cols != I || a->type != b->type)
            return h->fail(VLB_ERR_INVALID_FORMAT, "an expert matrix shape does not match the layer");
    }
    vlb_layer* L = new (std::nothrow) vlb_layer();
    if (!L) return h->fail(VLB_ERR_RESOURCE_EXHAUSTED, "unable to allocate the layer record");
    L->desc = *d;
    L->has_shared = has_shared;
    L->host_mats = hm;
    int st = VLB_OK;
#define TRY(expr)                 \
    do {                          \
        st = (expr);              \
        if (st != VLB_OK) {       \
            free_layer(h, L);     \
            return st;            \
        }                         \
    } while (0)
#define TRY_CUDA(call)                          \
    do {                                        \
        const cudaError_t e_ = (call);          \
        if (e_ != cudaSuccess) {                \
            free_layer(h, L);                   \
            return h->cuda_fail(#call, e_);     \
        }                                       \
    } while (0)
    {  // the router's f32 weights as f64: the sequential router chains consume f64 operands
        std::vector<double> wd;
        try {
            wd.assign(d->router, d->router + (size_t)E * H);
        } catch (const std::bad_alloc&) {
            free_layer(h, L);
            return h->fail(VLB_ERR_RESOURCE_EXHAUSTED, "unable to stage the router weights");
        }
        TRY(h->galloc((size_t)E * H * 8, "vlb-router", (void**)&L->router));
        TRY_CUDA(cudaMemcpy(L->router, wd.data(), (size_t)E * H * 8, cudaMemcpyHostToDevice));
    }
    if (d->bias) {
        TRY(h->galloc((size_t)E * 4, "vlb-router-bias", (void**)&L->bias));
        TRY_CUDA(cudaMemcpy(L->bias, d->bias, (size_t)E * 4, cudaMemcpyHostToDevice));
    }
    if (d->hash_routing) {
        TRY(h->galloc((size_t)d->vocab * k * 4, "vlb-tid2eid", (void**)&L->tid2eid));
        TRY_CUDA(cudaMemcpy(L->tid2eid, d->tid2eid, (size_t)d->vocab * k * 4, cudaMemcpyHostToDevice));
    }
    std::vector<DevMat> dm(3 * (E + 1));
    for (size_t i = 0; i < dm.size(); ++i) dm[i] = hm[i] ? hm[i]->dm : DevMat{};
    TRY(h->galloc(dm.size() * sizeof(DevMat), "vlb-expert-table", (void**)&L->mats));
    TRY_CUDA(cudaMemcpy(L->mats, dm.data(), dm.size() * sizeof(DevMat), cudaMemcpyHostToDevice));
    // workspace
    const size_t T = d->max_tokens, P = T * k + T;
    const uint32_t mu = max_units_for((uint32_t)T, k, E);
    size_t off = 0;
    auto carve = [&](size_t bytes) {
        const size_t at = off;
        off += (bytes + 255) / 256 * 256;
        return at;
    };
    const size_t o_logits = carve(T * E * 4), o_scores = carve(T * E * 4), o_idx = carve(T * k * 4),
                 o_w = carve(T * k * 4), o_off = carve((E + 2) * 4), o_pt = carve(P * 4),
                 o_ps = carve(P * 4), o_pw = carve(P * 4), o_units = carve((size_t)mu * sizeof(Unit)),
                 o_cnt = carve(32 + T * 4 + (size_t)kSplitItems * 16 * 4), o_cp = carve(T * k * 4),
                 o_act = carve(P * I * 4), o_sp = carve((size_t)kSplitItems * 16 * 32 * 8 * 4),
                 o_y = carve(P * H * 4), o_xs = carve(T * 4), o_am = carve(P * 4),
                 o_xn = carve(T * H * 4), o_xd = carve(T * H * 8);
    const uint32_t mpt = prefill_max_tiles((uint32_t)T, k, E);
    // xperm (prefill operand rows, P x H fp16) doubles as the decode kernels' gate/up activation
    // image (T rows of 4 H bytes) in a decode forward: room for the larger of the two
    const size_t o_xh = carve(P * H * 2 > T * H * 4 ? P * H * 2 : T * H * 4), o_acth = carve(P * I * 2),
                 o_pt2 = carve((size_t)mpt * sizeof(Unit));
    const size_t o_dc = carve(((T * k + 1023) / 1024) * E * 4);
    TRY(h->galloc(off, "vlb-layer-workspace", &L->ws));
    TRY(h->galloc(T * H * 4, "vlb-layer-x", (void**)&L->x_dev));
    TRY(h->galloc(T * 4, "vlb-layer-tokens", (void**)&L->tok_dev));
    TRY(h->galloc(T * E * 4, "vlb-layer-logits", (void**)&L->logits_dev));
    TRY(h->galloc(T * H * 4, "vlb-layer-out", (void**)&L->out_dev));
#undef TRY
#undef TRY_CUDA
    char* ws = static_cast<char*>(L->ws);
    MoeParams& p = L->p;
    p.H = H; p.I = I; p.E = E; p.k = k; p.T = 0;
    p.score = d->score;
    p.hash_routing = d->hash_routing;
    p.weight_after_down = d->weight_after_down;
    p.route_scale = d->route_scale;
    p.routed_limit = d->routed_swiglu_limit;
    p.shared_limit = d->shared_swiglu_limit;
    p.vocab = d->vocab;
    p.has_shared = has_shared ? 1 : 0;
    p.has_legacy = 0;
    p.has_mma = 0;
    p.fmt_gu = p.fmt_dn = 0;
    for (size_t i = 0; i < hm.size(); ++i) {
        const vlb_matrix* m = hm[i];
        if (!m) continue;
        if (m->type == VLB_TYPE_IQ2_XXS || m->type == VLB_TYPE_Q8_0) p.has_mma = 1;
        else p.has_legacy = 1;
        if (i < 2 * (size_t)(E + 1)) p.fmt_gu |= fmt_bit(m->type);
        else p.fmt_dn |= fmt_bit(m->type);
    }
    p.router = L->router;
    p.bias = L->bias;
    p.tid2eid = L->tid2eid;
    p.mats = L->mats;
    p.grids = h->grids();
    p.logits = reinterpret_cast<float*>(ws + o_logits);
    p.scores = reinterpret_cast<float*>(ws + o_scores);
    p.idx = reinterpret_cast<uint32_t*>(ws + o_idx);
    p.weights = reinterpret_cast<float*>(ws + o_w);
    p.offsets = reinterpret_cast<uint32_t*>(ws + o_off);
    p.pair_token = reinterpret_cast<uint32_t*>(ws + o_pt);
    p.pair_slot = reinterpret_cast<uint32_t*>(ws + o_ps);
    p.pair_weight = reinterpret_cast<float*>(ws + o_pw);
    p.units = reinterpret_cast<Unit*>(ws + o_units);
    p.counters = reinterpret_cast<uint32_t*>(ws + o_cnt);
    p.split_cnt = reinterpret_cast<uint32_t*>(ws + o_cnt + 32 + T * 4);
    p.split_part = reinterpret_cast<float*>(ws + o_sp);
    p.split_items = kSplitItems;
    p.combine_pairs = reinterpret_cast<uint32_t*>(ws + o_cp);
    p.act = reinterpret_cast<float*>(ws + o_act);
    p.y = reinterpret_cast<float*>(ws + o_y);
    p.xmax = reinterpret_cast<uint32_t*>(ws + o_cnt + 32);
    p.act_max = reinterpret_cast<uint32_t*>(ws + o_am);
    p.x_norm = reinterpret_cast<float*>(ws + o_xn);
    p.xd = reinterpret_cast<double*>(ws + o_xd);
    p.max_units = mu;
    p.prefill = 0;
    p.xperm = reinterpret_cast<__half*>(ws + o_xh);
    p.act_h = reinterpret_cast<__half*>(ws + o_acth);
    p.ptiles = reinterpret_cast<Unit*>(ws + o_pt2);
    p.max_ptiles = mpt;
    p.disp_counts = reinterpret_cast<uint32_t*>(ws + o_dc);
    if (!encode_rows_fp16(&p.bmap_x, p.xperm, P, H) || !encode_rows_fp16(&p.bmap_act, p.act_h, P, I)) {
        free_layer(h, L);
        return h->fail(VLB_ERR_INTERNAL_ERROR, "unable to encode the prefill TMA descriptors");
    }
    *out = L;
    return VLB_OK;
}

int vlb_layer_destroy(vlb_handle* h, vlb_layer* L) {
    VLB_LOCK(h);
    if (!L) return VLB_OK;
    VLB_CUDA(h, cudaStreamSynchronize(h->stream));
    free_layer(h, L);
    return VLB_OK;
}

// Error bits a layer forward leaves in its counters (route, given routes, prefill pipeline).
static int check_layer_flags(vlb_handle* h, uint32_t flags) {
    if (flags & 1u) return h->fail(VLB_ERR_INVALID_ARGUMENT, "hash route token id exceeds its table");
    if (flags & 2u) return h->fail(VLB_ERR_INVALID_FORMAT, "a route selects an out-of-range expert");
    if (flags & 4u) return h->fail(VLB_ERR_INVALID_ARGUMENT, "selected route weights cannot be normalized");
    if (flags & 8u) return h->fail(VLB_ERR_INTERNAL_ERROR, "an expert-kernel pipeline wait ran out of time");
    if (flags & 16u) return h->fail(VLB_ERR_INTERNAL_ERROR, "prefill shared memory is not 1 KB aligned");
    if (flags & kLayerErrHcTimeout)
        return h->fail(VLB_ERR_INTERNAL_ERROR, "a Hyper-Connection entry wait ran out of time");
    if (flags & kLayerErrHcNonFinite)
        return h->fail(VLB_ERR_INVALID_FORMAT, "Hyper-Connection reduced output is not finite");
    return VLB_OK;
}

// Default prefill threshold: 16 pairs per routed expert on average, and never below 256 tokens.
static uint32_t prefill_threshold(const vlb_layer* L) {
    if (L->prefill_min_tokens) return L->prefill_min_tokens;
    const uint32_t E = L->desc.experts, k = L->desc.top_k;
    const uint32_t per_expert = (16u * E + k - 1u) / k;
    return per_expert > 256u ? per_expert : 256u;
}

// One layer forward on stream s. Without profiling the whole launch sequence (a memset and seven
// kernels) is captured once as a CUDA graph for this exact input binding and replayed afterwards:
// at decode sizes the GPU work is short enough that per-kernel host submission would otherwise
// leave the device idle between kernels. A stream that cannot be captured (the legacy default
// stream) gets the same kernels launched directly.
static int forward_locked(vlb_handle* h, vlb_layer* L, const float* x, const uint32_t* tok,
                          const float* logits, uint32_t T, float* out, cudaStream_t s,
                          const uint32_t* routes_idx = nullptr, const float* routes_w = nullptr,
                          const uint16_t* x_half = nullptr, const uint32_t* routes_meta = nullptr) {
    if (T == 0 || T > L->desc.max_tokens)
        return h->fail(VLB_ERR_INVALID_ARGUMENT, "token count is zero or above the layer's max_tokens");
    if (L->desc.hash_routing && !tok && !routes_idx && !x_half)
        return h->fail(VLB_ERR_INVALID_ARGUMENT, "hash routing needs token ids");
    MoeParams p = L->p;
    p.T = T;
    p.x = x;
    p.token_ids = tok;
    p.logits_in = logits;
    p.routes_idx = routes_idx;
    p.routes_w = routes_w;
    p.x_half = reinterpret_cast<const __half*>(x_half);
    p.routes_meta = routes_meta;
    p.out = out;
    p.grids = h->grids();
    if (L->norm_w && (routes_idx || x_half))
        return h->fail(VLB_ERR_UNSUPPORTED, "a layer with an input norm takes plain token rows only");
    p.norm_w = L->norm_w;
    p.norm_eps = L->norm_eps;
    p.hc_m = L->hc_m;
    if (L->norm_w && ((reinterpret_cast<uintptr_t>(x) % 16u) || L->desc.hidden > kRmsMaxWidth))
        return h->fail(VLB_ERR_INVALID_ARGUMENT, "input rows of a normed layer must be 16-byte aligned");
    // half rows carry fp16 operands already: only the tensor-core prefill path consumes them
    p.prefill = (x_half || T >= prefill_threshold(L)) ? 1 : 0;
    const bool one_route = (routes_idx || x_half) && p.k == 1;
    p.direct_out = one_route && !p.has_shared && !p.weight_after_down && !p.has_legacy ? 1 : 0;
    // counters, per-token max|x| (the layer's max_tokens of them) and the K-split arrival counters
    const size_t zero_bytes = 32 + (size_t)L->desc.max_tokens * 4 + (size_t)kSplitItems * 16 * 4;
    L->last_T = T;
    L->last_logits_given = logits != nullptr;
    // prefill-size forwards are long enough that launching directly costs nothing, and their
    // token counts vary from call to call (a graph is keyed by T): no capture for them
    if (L->profiling || p.prefill) {
        VLB_CUDA(h, cudaMemsetAsync(p.counters, 0, zero_bytes, s));
        VLB_CUDA(h, launch_moe(p, s, L->profiling ? L->ev : nullptr));
        return VLB_OK;
    }
    const void* key[7] = {x, tok, logits, out, s, routes_idx, routes_w};
    bool same = L->gexec && L->gkey_T == T;
    for (int i = 0; same && i < 7; ++i) same = L->gkey[i] == key[i];
    if (!same) {
        if (L->gexec) {
            cudaGraphExecDestroy(L->gexec);
            L->gexec = nullptr;
        }
        cudaGraph_t graph = nullptr;
        cudaError_t e = cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal);
        if (e == cudaSuccess) {
            cudaError_t e1 = cudaMemsetAsync(p.counters, 0, zero_bytes, s);
            cudaError_t e2 = e1 == cudaSuccess ? launch_moe(p, s) : e1;
            e = cudaStreamEndCapture(s, &graph);
            if (e2 != cudaSuccess) e = e2;
        }
        if (e == cudaSuccess) e = cudaGraphInstantiate(&L->gexec, graph, 0);
        if (graph) cudaGraphDestroy(graph);
        if (e != cudaSuccess) {
            // not capturable here: launch directly
            (void)cudaGetLastError();
            L->gexec = nullptr;
            VLB_CUDA(h, cudaMemsetAsync(p.counters, 0, zero_bytes, s));
            VLB_CUDA(h, launch_moe(p, s));
            return VLB_OK;
        }
        for (int i = 0; i < 7; ++i) L->gkey[i] = key[i];
        L->gkey_T = T;
    }
    VLB_CUDA(h, cudaGraphLaunch(L->gexec, s));
    return VLB_OK;
}

int vlb_layer_forward_device(vlb_handle* h, vlb_layer* L, const float* x, const uint32_t* tok,
                             const float* logits, uint32_t T, float* out, void* stream) {
    VLB_LOCK(h);
    if (!L || !x || !out) return h->fail(VLB_ERR_INVALID_ARGUMENT, "invalid forward argument");
    return forward_locked(h, L, x, tok, logits, T, out, h->pick(stream));
}

int vlb_layer_forward_routes_device(vlb_handle* h, vlb_layer* L, const float* x, const uint32_t* idx,
                                    const float* weights, uint32_t T, float* out, void* stream) {
    VLB_LOCK(h);
    if (!L || !x || !out || !idx || !weights) return h->fail(VLB_ERR_INVALID_ARGUMENT, "invalid forward argument");
    return forward_locked(h, L, x, nullptr, nullptr, T, out, h->pick(stream), idx, weights);
}

int vlb_layer_forward_rows_half_device(vlb_handle* h, vlb_layer* L, const uint16_t* rows, const uint32_t* meta,
                                       uint32_t T, float* out, void* stream) {
    VLB_LOCK(h);
    if (!L || !rows || !meta || !out) return h->fail(VLB_ERR_INVALID_ARGUMENT, "invalid forward argument");
    if (L->desc.top_k != 1 || L->p.has_legacy || L->desc.hidden % 8)
        return h->fail(VLB_ERR_UNSUPPORTED,
                       "half-row forwards need one route per row, tensor-core expert formats and hidden % 8 == 0");
    return forward_locked(h, L, nullptr, nullptr, nullptr, T, out, h->pick(stream), nullptr, nullptr, rows, meta);
}

int vlb_layer_status(vlb_handle* h, vlb_layer* L, void* stream) {
    VLB_LOCK(h);
    if (!L) return h->fail(VLB_ERR_INVALID_ARGUMENT, "null layer");
    cudaStream_t s = h->pick(stream);
    uint32_t flags = 0;
    VLB_CUDA(h, cudaMemcpyAsync(&flags, L->p.counters + 3, 4, cudaMemcpyDeviceToHost, s));
    VLB_CUDA(h, cudaStreamSynchronize(s));
    return check_layer_flags(h, flags);
}

int vlb_layer_forward(vlb_handle* h, vlb_layer* L, const float* x, const uint32_t* tok,
                      const float* logits, uint32_t T, float* out) {
    VLB_LOCK(h);
    if (!L || !x || !out) return h->fail(VLB_ERR_INVALID_ARGUMENT, "invalid forward argument");
    if (T == 0 || T > L->desc.max_tokens)
        return h->fail(VLB_ERR_INVALID_ARGUMENT, "token count is zero or above the layer's max_tokens");
    const uint32_t H = L->desc.hidden * (L->hc_m ? L->hc_m : 1u), E = L->desc.experts;  // row width in and out
    cudaStream_t s = h->stream;
    VLB_CUDA(h, cudaMemcpyAsync(L->x_dev, x, (size_t)T * H * 4, cudaMemcpyHostToDevice, s));
    if (tok) VLB_CUDA(h, cudaMemcpyAsync(L->tok_dev, tok, (size_t)T * 4, cudaMemcpyHostToDevice, s));
    if (logits) VLB_CUDA(h, cudaMemcpyAsync(L->logits_dev, logits, (size_t)T * E * 4, cudaMemcpyHostToDevice, s));
    int st = forward_locked(h, L, L->x_dev, tok ? L->tok_dev : nullptr, logits ? L->logits_dev : nullptr,
                            T, L->out_dev, s);
    if (st != VLB_OK) return st;
    VLB_CUDA(h, cudaMemcpyAsync(out, L->out_dev, (size_t)T * H * 4, cudaMemcpyDeviceToHost, s));
    uint32_t flags = 0;
    VLB_CUDA(h, cudaMemcpyAsync(&flags, L->p.counters + 3, 4, cudaMemcpyDeviceToHost, s));
    VLB_CUDA(h, cudaStreamSynchronize(s));
    return check_layer_flags(h, flags);
}

int vlb_layer_set_input_norm(vlb_handle* h, vlb_layer* L, const float* weight, float eps) {
    VLB_LOCK(h);
    if (!L) return h->fail(VLB_ERR_INVALID_ARGUMENT, "null layer");
    if (L->hc_m)
        return h->fail(VLB_ERR_INVALID_ARGUMENT, "a Hyper-Connection layer takes its norm with its descriptor");
    const uint32_t H = L->desc.hidden;
    if (weight && !(eps > 0.f && std::isfinite(eps)))
        return h->fail(VLB_ERR_INVALID_ARGUMENT, "RMSNorm epsilon must be finite and positive");
    if (weight && H > kRmsMaxWidth) return h->fail(VLB_ERR_UNSUPPORTED, "hidden size too large for the input norm");
    if (weight)
        for (uint32_t c = 0; c < H; ++c)
            if (!std::isfinite(weight[c])) return h->fail(VLB_ERR_INVALID_ARGUMENT, "RMSNorm weight is not finite");
    VLB_CUDA(h, cudaStreamSynchronize(h->stream));
    if (L->gexec) {  // the captured forward does not have the new entry step
        cudaGraphExecDestroy(L->gexec);
        L->gexec = nullptr;
    }
    if (!weight) {
        if (L->norm_w) h->gfree(L->norm_w);
        L->norm_w = nullptr;
        return VLB_OK;
    }
    if (!L->norm_w) {
        int st = h->galloc((size_t)H * 4, "vlb-input-norm", (void**)&L->norm_w);
        if (st != VLB_OK) return st;
    }
    VLB_CUDA(h, cudaMemcpy(L->norm_w, weight, (size_t)H * 4, cudaMemcpyHostToDevice));
    L->norm_eps = eps;
    return VLB_OK;
}

int vlb_layer_set_hyper_connection(vlb_handle* h, vlb_layer* L, const vlb_hc_desc* d) {
    VLB_LOCK(h);
    if (!L) return h->fail(VLB_ERR_INVALID_ARGUMENT, "null layer");
    const uint32_t H = L->desc.hidden, T = L->desc.max_tokens;
    if (d) {
        const uint32_t m = d->multiplier;
        if (m == 0 || m > 16 || d->sinkhorn_iterations == 0 || !d->mixing_weight || !d->scale || !d->base ||
            !d->norm_weight)
            return h->fail(VLB_ERR_INVALID_ARGUMENT, "Hyper-Connection dimensions are invalid");
        if (!(d->norm_epsilon > 0.f && std::isfinite(d->norm_epsilon)) ||
            !(d->hc_epsilon > 0.f && std::isfinite(d->hc_epsilon)))
            return h->fail(VLB_ERR_INVALID_ARGUMENT, "Hyper-Connection epsilons must be finite and positive");
        if (!hc_entry_fits(m, H))
            return h->fail(VLB_ERR_UNSUPPORTED, "multiplier x hidden is too large for the Hyper-Connection entry");
        const size_t mw = (size_t)(2 + m) * m, fw = (size_t)m * H;
        for (size_t i = 0; i < mw * fw; ++i)
            if (!std::isfinite(d->mixing_weight[i]))
                return h->fail(VLB_ERR_INVALID_ARGUMENT, "Hyper-Connection mixing weight is not finite");
        for (size_t i = 0; i < mw; ++i)
            if (!std::isfinite(d->base[i])) return h->fail(VLB_ERR_INVALID_ARGUMENT, "Hyper-Connection base is not finite");
        for (size_t i = 0; i < 3; ++i)
            if (!std::isfinite(d->scale[i])) return h->fail(VLB_ERR_INVALID_ARGUMENT, "Hyper-Connection scale is not finite");
        for (uint32_t c = 0; c < H; ++c)
            if (!std::isfinite(d->norm_weight[c])) return h->fail(VLB_ERR_INVALID_ARGUMENT, "RMSNorm weight is not finite");
    }
    VLB_CUDA(h, cudaStreamSynchronize(h->stream));
    if (L->gexec) {  // the captured forward does not have the new entry and exit
        cudaGraphExecDestroy(L->gexec);
        L->gexec = nullptr;
    }
    // the host-memory forward's staging: m copies per token with the Hyper-Connection, one without
    const uint32_t m_new = d ? d->multiplier : 0u, rows_new = m_new ? m_new : 1u, rows_old = L->hc_m ? L->hc_m : 1u;
    if (rows_new != rows_old) {
        h->gfree(L->x_dev);
        h->gfree(L->out_dev);
        L->x_dev = L->out_dev = nullptr;
        int st = h->galloc((size_t)T * rows_new * H * 4, "vlb-layer-x", (void**)&L->x_dev);
        if (st == VLB_OK) st = h->galloc((size_t)T * rows_new * H * 4, "vlb-layer-out", (void**)&L->out_dev);
        if (st != VLB_OK) {
            L->hc_m = 0;  // the layer stays usable only after a successful set
            return st;
        }
    }
    if (L->hc_mem) h->gfree(L->hc_mem);
    L->hc_mem = nullptr;
    L->hc_m = 0;
    if (!d) {
        if (L->norm_w) h->gfree(L->norm_w);
        L->norm_w = nullptr;
        L->p.hc_m = 0;
        return VLB_OK;
    }
    const uint32_t m = d->multiplier;
    const size_t mw = (size_t)(2 + m) * m, fw = (size_t)m * H;
    auto up = [](size_t b) { return (b + 255) / 256 * 256; };
    const size_t o_fn = 0, o_scale = up(mw * fw * 8), o_base = o_scale + 256, o_pre = o_base + up(mw * 4);
    const size_t o_post = o_pre + up((size_t)T * m * 4), o_comb = o_post + up((size_t)T * m * 4);
    const size_t total = o_comb + up((size_t)T * m * m * 4);
    int st = h->galloc(total, "vlb-hyper-connection", &L->hc_mem);
    if (st != VLB_OK) return st;
    char* b = static_cast<char*>(L->hc_mem);
    {
        // the entry's chains read f64 operands (a widening per step would cost more than the step)
        std::vector<double> fnd;
        try {
            fnd.assign(d->mixing_weight, d->mixing_weight + mw * fw);
        } catch (const std::bad_alloc&) {
            return h->fail(VLB_ERR_RESOURCE_EXHAUSTED, "unable to stage the mixing weight");
        }
        VLB_CUDA(h, cudaMemcpy(b + o_fn, fnd.data(), mw * fw * 8, cudaMemcpyHostToDevice));
    }
    VLB_CUDA(h, cudaMemcpy(b + o_scale, d->scale, 12, cudaMemcpyHostToDevice));
    VLB_CUDA(h, cudaMemcpy(b + o_base, d->base, mw * 4, cudaMemcpyHostToDevice));
    if (!L->norm_w) {
        st = h->galloc((size_t)H * 4, "vlb-input-norm", (void**)&L->norm_w);
        if (st != VLB_OK) return st;
    }
    VLB_CUDA(h, cudaMemcpy(L->norm_w, d->norm_weight, (size_t)H * 4, cudaMemcpyHostToDevice));
    L->norm_eps = d->norm_epsilon;
    MoeParams& p = L->p;
    p.hc_iters = d->sinkhorn_iterations;
    p.hc_eps = d->hc_epsilon;
    p.hc_fn = reinterpret_cast<const double*>(b + o_fn);
    p.hc_scale = reinterpret_cast<const float*>(b + o_scale);
    p.hc_base = reinterpret_cast<const float*>(b + o_base);
    p.hc_pre = reinterpret_cast<float*>(b + o_pre);
    p.hc_post = reinterpret_cast<float*>(b + o_post);
    p.hc_comb = reinterpret_cast<float*>(b + o_comb);
    L->hc_m = m;
    return VLB_OK;
}

int vlb_layer_last_hyper_split(vlb_handle* h, vlb_layer* L, uint32_t T, float* pre, float* post, float* comb) {
    VLB_LOCK(h);
    if (!L || !L->hc_m) return h->fail(VLB_ERR_INVALID_ARGUMENT, "the layer has no Hyper-Connection");
    if (T == 0 || T > L->last_T) return h->fail(VLB_ERR_INVALID_ARGUMENT, "more tokens than the last forward had");
    const size_t m = L->hc_m;
    cudaStream_t s = h->stream;
    if (pre) VLB_CUDA(h, cudaMemcpyAsync(pre, L->p.hc_pre, T * m * 4, cudaMemcpyDeviceToHost, s));
    if (post) VLB_CUDA(h, cudaMemcpyAsync(post, L->p.hc_post, T * m * 4, cudaMemcpyDeviceToHost, s));
    if (comb) VLB_CUDA(h, cudaMemcpyAsync(comb, L->p.hc_comb, T * m * m * 4, cudaMemcpyDeviceToHost, s));
    VLB_CUDA(h, cudaStreamSynchronize(s));
    return VLB_OK;
}

int vlb_layer_set_prefill_tokens(vlb_handle* h, vlb_layer* L, uint32_t min_tokens) {
    VLB_LOCK(h);
    if (!L) return h->fail(VLB_ERR_INVALID_ARGUMENT, "null layer");
    if (L->prefill_min_tokens != min_tokens && L->gexec) {
        VLB_CUDA(h, cudaStreamSynchronize(h->stream));
        cudaGraphExecDestroy(L->gexec);
        L->gexec = nullptr;
    }
    L->prefill_min_tokens = min_tokens;
    return VLB_OK;
}

uint32_t vlb_layer_prefill_tokens(vlb_handle* h, vlb_layer* L) {
    if (!h || !L) return 0;
    std::lock_guard<std::mutex> lock(h->mu);
    return prefill_threshold(L);
}

int vlb_layer_last_route(vlb_handle* h, vlb_layer* L, uint32_t T, uint32_t* idx, float* w,
                         uint32_t* offsets, uint32_t* pt, uint32_t* ps) {
    VLB_LOCK(h);
    if (!L || T != L->last_T || T == 0) return h->fail(VLB_ERR_INVALID_ARGUMENT, "no route of that size");
    const size_t n = (size_t)T * L->desc.top_k;
    cudaStream_t s = h->stream;
    if (idx) VLB_CUDA(h, cudaMemcpyAsync(idx, L->p.idx, n * 4, cudaMemcpyDeviceToHost, s));
    if (w) VLB_CUDA(h, cudaMemcpyAsync(w, L->p.weights, n * 4, cudaMemcpyDeviceToHost, s));
    if (offsets) VLB_CUDA(h, cudaMemcpyAsync(offsets, L->p.offsets, (L->desc.experts + 1) * 4, cudaMemcpyDeviceToHost, s));
    if (pt) VLB_CUDA(h, cudaMemcpyAsync(pt, L->p.pair_token, n * 4, cudaMemcpyDeviceToHost, s));
    if (ps) VLB_CUDA(h, cudaMemcpyAsync(ps, L->p.pair_slot, n * 4, cudaMemcpyDeviceToHost, s));
    VLB_CUDA(h, cudaStreamSynchronize(s));
    return VLB_OK;
}

uint64_t vlb_layer_last_weight_bytes(vlb_handle* h, vlb_layer* L) {
    if (!h || !L || L->last_T == 0) return 0;
    std::lock_guard<std::mutex> lock(h->mu);
    cudaSetDevice(h->device);
    const uint32_t E = L->desc.experts;
    std::vector<uint32_t> off(E + 1);
    if (cudaMemcpyAsync(off.data(), L->p.offsets, (E + 1) * 4, cudaMemcpyDeviceToHost, h->stream) != cudaSuccess ||
        cudaStreamSynchronize(h->stream) != cudaSuccess)
        return 0;
    uint64_t bytes = L->last_logits_given ? 0 : (uint64_t)E * L->desc.hidden * 4;
    for (uint32_t e = 0; e < E; ++e)
        if (off[e + 1] > off[e])
            bytes += L->host_mats[e]->payload_bytes + L->host_mats[(E + 1) + e]->payload_bytes +
                     L->host_mats[2 * (E + 1) + e]->payload_bytes;
    if (L->has_shared)
        bytes += L->host_mats[E]->payload_bytes + L->host_mats[(E + 1) + E]->payload_bytes +
                 L->host_mats[2 * (E + 1) + E]->payload_bytes;
    return bytes;
}

int vlb_layer_set_profiling(vlb_handle* h, vlb_layer* L, int enable) {
    VLB_LOCK(h);
    if (!L) return h->fail(VLB_ERR_INVALID_ARGUMENT, "null layer");
    if (enable && !L->ev[0])
        for (auto& e : L->ev) VLB_CUDA(h, cudaEventCreate(&e));
    L->profiling = enable != 0;
    return VLB_OK;
}

int vlb_layer_phase_times(vlb_handle* h, vlb_layer* L, float* ms, int n) {
    VLB_LOCK(h);
    if (!L || !ms || n < kMoePhases || !L->profiling || L->last_T == 0)
        return h->fail(VLB_ERR_INVALID_ARGUMENT, "profiling is off or there is no forward to report");
    VLB_CUDA(h, cudaEventSynchronize(L->ev[kMoePhases]));
    for (int i = 0; i < kMoePhases; ++i) VLB_CUDA(h, cudaEventElapsedTime(&ms[i], L->ev[i], L->ev[i + 1]));
    return VLB_OK;
}

int vlb_route_device(vlb_handle* h, int score, int hash_routing, const float* logits,
                     const float* bias, const uint32_t* tok, const uint32_t* tid2eid,
                     uint32_t vocab, uint32_t T, uint32_t E, uint32_t k, float route_scale,
                     uint32_t* idx, float* weights, void* stream) {
    VLB_LOCK(h);
    if (!logits || !idx || !weights || T == 0 || E == 0 || k == 0 || k > E || k > 16 || E > 512 ||
        score < VLB_SCORE_SQRT_SOFTPLUS || score > VLB_SCORE_SOFTMAX_F64_NORM)
        return h->fail(VLB_ERR_INVALID_ARGUMENT, "invalid route argument");
    if (hash_routing && (!tok || !tid2eid || vocab == 0))
        return h->fail(VLB_ERR_INVALID_ARGUMENT, "hash routing needs token ids and a table");
    cudaStream_t s = h->pick(stream);
    char* scratch = nullptr;
    int st = h->scratch_at_least((size_t)T * E * 4 + 256, &scratch);
    if (st != VLB_OK) return st;
    float* scores = reinterpret_cast<float*>(scratch);
    uint32_t* flag = reinterpret_cast<uint32_t*>(scratch + (size_t)T * E * 4);
    cudaError_t e = cudaMemsetAsync(flag, 0, 4, s);
    if (e == cudaSuccess) e = launch_scores(logits, (size_t)T * E, score, scores, s);
    if (e == cudaSuccess)
        e = launch_route(scores, bias, tok, tid2eid, vocab, T, E, k, score, hash_routing,
                         route_scale, idx, weights, flag, s);
    uint32_t flags = 0;
    if (e == cudaSuccess) e = cudaMemcpyAsync(&flags, flag, 4, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return h->cuda_fail("route", e);
    if (flags & 1u) return h->fail(VLB_ERR_INVALID_ARGUMENT, "hash route token id exceeds its table");
    if (flags & 2u) return h->fail(VLB_ERR_INVALID_FORMAT, "route selects an out-of-range expert");
    if (flags & 4u) return h->fail(VLB_ERR_INVALID_ARGUMENT, "selected route weights cannot be normalized");
    return VLB_OK;
}

int vlb_router_logits_device(vlb_handle* h, const float* x, const float* w, uint32_t T,
                             uint32_t H, uint32_t E, float* logits, void* stream) {
    VLB_LOCK(h);
    if (!x || !w || !logits || T == 0 || H == 0 || E == 0 || H % 4)
        return h->fail(VLB_ERR_INVALID_ARGUMENT, "invalid router argument");
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(w)) % 16u)
        return h->fail(VLB_ERR_INVALID_ARGUMENT, "router inputs must be 16-byte aligned");
    if ((T + 3u) / 4u > 65535u) return h->fail(VLB_ERR_INVALID_ARGUMENT, "too many router tokens for one call");
    // scratch: scores [T x E] f32 | x as f64 [T x H] | w as f64 [E x H]
    const size_t sbytes = ((size_t)T * E * 4 + 255) / 256 * 256, xbytes = (size_t)T * H * 8;
    char* scratch = nullptr;
    int st = h->scratch_at_least(sbytes + xbytes + (size_t)E * H * 8, &scratch);
    if (st != VLB_OK) return st;
    double* xd = reinterpret_cast<double*>(scratch + sbytes);
    double* wd = reinterpret_cast<double*>(scratch + sbytes + xbytes);
    cudaStream_t s = h->pick(stream);
    cudaError_t e = launch_widen(x, (size_t)T * H, xd, s);
    if (e == cudaSuccess) e = launch_widen(w, (size_t)E * H, wd, s);
    if (e == cudaSuccess)
        e = launch_router(xd, wd, T, H, E, VLB_SCORE_SOFTMAX, logits, reinterpret_cast<float*>(scratch), s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return h->cuda_fail("router", e);
    return VLB_OK;
}

int vlb_rms_norm_device(vlb_handle* h, const float* x, const float* w, uint32_t rows,
                        uint32_t width, float eps, float* out, void* stream) {
    VLB_LOCK(h);
    if (!x || !w || !out || rows == 0 || width == 0 || !(eps > 0.f) || !std::isfinite(eps))
        return h->fail(VLB_ERR_INVALID_ARGUMENT, "invalid RMSNorm argument");
    if (width % 4u || width > kRmsMaxWidth || reinterpret_cast<uintptr_t>(x) % 16u)
        return h->fail(VLB_ERR_UNSUPPORTED, "RMSNorm rows must be 16-byte aligned, width % 4 == 0 and width <= " +
                                                std::to_string(kRmsMaxWidth));
    VLB_CUDA(h, launch_rms_norm(x, w, rows, width, eps, out, nullptr, nullptr, h->pick(stream)));
    return VLB_OK;
}

// ---- expert parallelism (configuration 4) ------------------------------------------------------

// Plan workspace: flag | pair_token [n] | pair_slot [n] | per-chunk counts | sorted weights [n] |
// per-token max|x| [T] (the last two only used by the half-row plan).
static size_t ep_round(size_t b) { return (b + 255) / 256 * 256; }

size_t vlb_ep_workspace_bytes(uint32_t T, uint32_t k, uint32_t E) {
    const size_t n = (size_t)T * k, chunks = (n + 1023) / 1024;
    return 256 + 4 * ep_round(n * 4) + ep_round(chunks * E * 4) + ep_round((size_t)T * 4);
}

int vlb_ep_plan_device(vlb_handle* h, const uint32_t* idx, const float* weights, uint32_t T, uint32_t k,
                       uint32_t E, uint32_t experts_per_rank, const float* x, uint32_t H, void* ws, uint32_t* offsets,
                       uint32_t* offsets_host, float* send_x, uint32_t* send_expert, float* send_weight,
                       uint32_t* elem_row, void* stream) {
    VLB_LOCK(h);
    if (!idx || !weights || !x || !ws || !offsets || !offsets_host || !send_x || !send_expert || !send_weight ||
        !elem_row || k == 0 || E == 0 || E > 512 || H == 0 || H % 4 || experts_per_rank == 0 ||
        E % experts_per_rank)
        return h->fail(VLB_ERR_INVALID_ARGUMENT, "invalid expert-parallel plan argument");
    cudaStream_t s = h->pick(stream);
    const size_t n = (size_t)T * k;
    char* w = static_cast<char*>(ws);
    uint32_t* flag = reinterpret_cast<uint32_t*>(w);
    uint32_t* pair_token = reinterpret_cast<uint32_t*>(w + 256);
    uint32_t* pair_slot = reinterpret_cast<uint32_t*>(w + 256 + (n * 4 + 255) / 256 * 256);
    uint32_t* counts = reinterpret_cast<uint32_t*>(w + 256 + 2 * ((n * 4 + 255) / 256 * 256));
    // expert ids are validated before the counting sort indexes anything with them
    uint32_t bad = 0;
    VLB_CUDA(h, cudaMemsetAsync(flag, 0, 4, s));
    VLB_CUDA(h, launch_ep_validate(idx, n, E, flag, s));
    VLB_CUDA(h, cudaMemcpyAsync(&bad, flag, 4, cudaMemcpyDeviceToHost, s));
    VLB_CUDA(h, cudaStreamSynchronize(s));
    if (bad) return h->fail(VLB_ERR_INVALID_FORMAT, "a route selects an out-of-range expert");
    MoeParams p{};
    p.T = T;
    p.k = k;
    p.E = E;
    p.idx = const_cast<uint32_t*>(idx);
    p.weights = const_cast<float*>(weights);
    p.offsets = offsets;
    p.pair_token = pair_token;
    p.pair_slot = pair_slot;
    p.pair_weight = send_weight;
    p.combine_pairs = elem_row;
    p.disp_counts = counts;
    p.has_shared = 0;
    VLB_CUDA(h, launch_stable_sort(p, s));
    VLB_CUDA(h, launch_ep_gather(pair_token, pair_slot, idx, (uint32_t)n, k, experts_per_rank, x, H, send_x,
                                 send_expert, s));
    if (n == 0) VLB_CUDA(h, cudaMemsetAsync(offsets, 0, (E + 2) * 4, s));
    VLB_CUDA(h, cudaMemcpyAsync(offsets_host, offsets, (E + 1) * 4, cudaMemcpyDeviceToHost, s));
    VLB_CUDA(h, cudaStreamSynchronize(s));
    return VLB_OK;
}

int vlb_ep_plan_half_device(vlb_handle* h, const uint32_t* idx, const float* weights, uint32_t T, uint32_t k,
                            uint32_t E, uint32_t experts_per_rank, const uint32_t* expert_slot, const float* x,
                            uint32_t H, void* ws, uint32_t* offsets, uint32_t* offsets_host, uint16_t* send_rows,
                            uint32_t* send_meta, uint32_t* elem_row, uint16_t* own_rows, uint32_t* own_meta,
                            void* stream) {
    VLB_LOCK(h);
    if (!idx || !weights || !x || !ws || !offsets || !offsets_host || !send_rows || !send_meta || !elem_row ||
        !own_rows || !own_meta || k == 0 || E == 0 || E > 512 || H == 0 || H % 8 || experts_per_rank == 0 ||
        E % experts_per_rank)
        return h->fail(VLB_ERR_INVALID_ARGUMENT, "invalid expert-parallel plan argument");
    cudaStream_t s = h->pick(stream);
    const size_t n = (size_t)T * k, chunks = (n + 1023) / 1024;
    char* w = static_cast<char*>(ws);
    uint32_t* flag = reinterpret_cast<uint32_t*>(w);
    uint32_t* pair_token = reinterpret_cast<uint32_t*>(w + 256);
    uint32_t* pair_slot = reinterpret_cast<uint32_t*>(w + 256 + ep_round(n * 4));
    uint32_t* counts = reinterpret_cast<uint32_t*>(w + 256 + 2 * ep_round(n * 4));
    float* sorted_w = reinterpret_cast<float*>(w + 256 + 2 * ep_round(n * 4) + ep_round(chunks * E * 4));
    uint32_t* xmax = reinterpret_cast<uint32_t*>(w + 256 + 3 * ep_round(n * 4) + ep_round(chunks * E * 4));
    uint32_t* slots = reinterpret_cast<uint32_t*>(w + 256 + 3 * ep_round(n * 4) + ep_round(chunks * E * 4) +
                                                  ep_round((size_t)T * 4));
    // routes -> exchange slots (an out-of-range id is flagged and made harmless), then the stable
    // sort by slot = by destination rank; one host synchronisation at the end reads the offsets that
    // size the exchange, and the flag
    VLB_CUDA(h, cudaMemsetAsync(flag, 0, 4, s));
    VLB_CUDA(h, launch_ep_slots(idx, n, E, expert_slot, slots, flag, s));
    VLB_CUDA(h, launch_prescale(x, T, H, xmax, nullptr, s));
    MoeParams p{};
    p.T = T;
    p.k = k;
    p.E = E;
    p.idx = slots;
    p.weights = const_cast<float*>(weights);
    p.offsets = offsets;
    p.pair_token = pair_token;
    p.pair_slot = pair_slot;
    p.pair_weight = sorted_w;
    p.combine_pairs = elem_row;
    p.disp_counts = counts;
    p.has_shared = 0;
    VLB_CUDA(h, launch_stable_sort(p, s));
    VLB_CUDA(h, launch_ep_gather_half(pair_token, pair_slot, slots, sorted_w, (uint32_t)n, k, experts_per_rank, x,
                                      xmax, H, reinterpret_cast<__half*>(send_rows), send_meta, s));
    VLB_CUDA(h, launch_ep_own_rows(x, xmax, T, H, experts_per_rank, reinterpret_cast<__half*>(own_rows), own_meta,
                                   s));
    if (n == 0) VLB_CUDA(h, cudaMemsetAsync(offsets, 0, (E + 2) * 4, s));
    uint32_t bad = 0;
    VLB_CUDA(h, cudaMemcpyAsync(offsets_host, offsets, (E + 1) * 4, cudaMemcpyDeviceToHost, s));
    VLB_CUDA(h, cudaMemcpyAsync(&bad, flag, 4, cudaMemcpyDeviceToHost, s));
    VLB_CUDA(h, cudaStreamSynchronize(s));
    if (bad) return h->fail(VLB_ERR_INVALID_FORMAT, "a route selects an out-of-range expert");
    return VLB_OK;
}

int vlb_ep_pack_half_device(vlb_handle* h, const float* y_rows, uint32_t rows, uint32_t H, uint16_t* half_rows,
                            float* row_scale, void* stream) {
    VLB_LOCK(h);
    if ((rows && (!y_rows || !half_rows || !row_scale)) || H == 0 || H % 8)
        return h->fail(VLB_ERR_INVALID_ARGUMENT, "invalid expert-parallel pack argument");
    VLB_CUDA(h, launch_ep_pack_half(y_rows, rows, H, reinterpret_cast<__half*>(half_rows), row_scale, h->pick(stream)));
    return VLB_OK;
}

int vlb_ep_combine_half_device(vlb_handle* h, const uint16_t* half_rows, const float* row_scale,
                               const uint32_t* elem_row, uint32_t T, uint32_t k, const float* shared_rows, uint32_t H,
                               float* out, void* stream) {
    VLB_LOCK(h);
    if (!half_rows || !row_scale || !elem_row || !out || H == 0 || H % 4)
        return h->fail(VLB_ERR_INVALID_ARGUMENT, "invalid expert-parallel combine argument");
    VLB_CUDA(h, launch_ep_combine_half(reinterpret_cast<const __half*>(half_rows), row_scale, elem_row, T, k,
                                       shared_rows, H, out, h->pick(stream)));
    return VLB_OK;
}

int vlb_ep_combine_device(vlb_handle* h, const float* y_rows, const uint32_t* elem_row, uint32_t T, uint32_t k,
                          const float* shared_rows, uint32_t H, float* out, void* stream) {
    VLB_LOCK(h);
    if (!y_rows || !elem_row || !out || H == 0 || H % 4)
        return h->fail(VLB_ERR_INVALID_ARGUMENT, "invalid expert-parallel combine argument");
    VLB_CUDA(h, launch_ep_combine(y_rows, elem_row, T, k, shared_rows, H, out, h->pick(stream)));
    return VLB_OK;
}

}  // extern "C"
