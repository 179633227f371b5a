// vlb_route_device_noalloc: the device router (sqrt-softplus / sigmoid / softmax scores, top-k,
// route weights) for callers that cannot allocate device memory.
//
// Who cannot allocate: a runtime whose ResourceGovernor has entered its pressure or critical state
// and refuses every new reservation, yet must still route the tokens already in flight; callers
// that are not allowed to call cudaMalloc at all (an embedding application that owns the device
// memory budget); and decode loops that cannot afford the device-wide synchronisation
// cudaMalloc/cudaFree may perform. vlb_route_device keeps its score scratch in the handle and grows
// it with cudaMalloc when a call needs more than the handle holds; this variant never allocates:
// its scratch is a fixed array compiled into the library.
//
// The call is ordinary host code: it launches kernels and then synchronises the stream to read the
// route's error flag, so it must not be made from a CUDA host callback or while a stream capture
// is open.
//
// The scratch is one file-scope __device__ array of kNoAllocScratchBytes (1 MiB). Every GPU that
// loads the library holds it until the process exits. In host code the array's name is only a
// host-side stand-in, never a device address (a kernel handed it would fault or, where the GPU
// can reach host memory, silently use the wrong memory), so the device address is resolved with
// cudaGetSymbolAddress once per device, with that device current, and passed to the kernels.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "vlb_launch.h"

namespace vlb {
void set_thread_error(const std::string& msg);  // vlb_abi.cu
}

namespace {

constexpr size_t kNoAllocScratchBytes = size_t{1} << 20;
constexpr size_t kFlagBytes = 256;  // error flag, then the scores start 256-byte aligned
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_route_scratch[kNoAllocScratchBytes];

std::mutex g_setup_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// The device address of g_route_scratch on `ordinal` (which must be current); resolved on the
// first call for each device and reused afterwards.
cudaError_t scratch_for(int ordinal, void** out) {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (!g_scratch_ptr[ordinal]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_route_scratch);
        if (e != cudaSuccess) return e;
        g_scratch_ptr[ordinal] = p;
    }
    *out = g_scratch_ptr[ordinal];
    return cudaSuccess;
}

int fail(int code, const std::string& msg) {
    vlb::set_thread_error(msg);
    return code;
}

int cuda_fail(const char* op, cudaError_t e) {
    (void)cudaGetLastError();
    return fail(VLB_ERR_IO_ERROR, std::string("CUDA call failed: ") + op + " (" + cudaGetErrorName(e) +
                                      ": " + cudaGetErrorString(e) + ")");
}

}  // namespace

extern "C" int vlb_route_device_noalloc(int ordinal, int score, int hash_routing,
                                        const float* logits, const float* bias,
                                        const uint32_t* token_ids, const uint32_t* tid2eid,
                                        uint32_t vocab, uint32_t T, uint32_t E, uint32_t k,
                                        float route_scale, uint32_t* idx, float* weights,
                                        void* stream) {
    if (ordinal < 0 || ordinal >= kMaxDevices)
        return fail(VLB_ERR_INVALID_ARGUMENT, "device ordinal is out of range");
    if (!logits || !idx || !weights || T == 0 || E == 0 || k == 0 || k > E || k > 16 || E > 512 ||
        score < VLB_SCORE_SQRT_SOFTPLUS || score > VLB_SCORE_SOFTMAX_F64_NORM)
        return fail(VLB_ERR_INVALID_ARGUMENT, "invalid route argument");
    if (hash_routing && (!token_ids || !tid2eid || vocab == 0))
        return fail(VLB_ERR_INVALID_ARGUMENT, "hash routing needs token ids and a table");
    const size_t need = kFlagBytes + (size_t)T * E * sizeof(float);
    if (need > kNoAllocScratchBytes)
        return fail(VLB_ERR_RESOURCE_EXHAUSTED,
                    "route too large for the fixed no-allocation scratch: T*E must be at most " +
                        std::to_string((kNoAllocScratchBytes - kFlagBytes) / sizeof(float)) +
                        ", got " + std::to_string((size_t)T * E));
    int prev = 0;
    cudaError_t e = cudaGetDevice(&prev);
    if (e != cudaSuccess) return cuda_fail("cudaGetDevice", e);
    if (prev != ordinal && (e = cudaSetDevice(ordinal)) != cudaSuccess) return cuda_fail("cudaSetDevice", e);
    void* base = nullptr;
    e = scratch_for(ordinal, &base);
    int st = VLB_OK;
    if (e != cudaSuccess) {
        st = cuda_fail("cudaGetSymbolAddress", e);
    } else {
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        uint32_t* flag = static_cast<uint32_t*>(base);
        float* scores = reinterpret_cast<float*>(static_cast<unsigned char*>(base) + kFlagBytes);
        uint32_t flags = 0;
        // The array keeps the previous call's contents: the flag must start at zero; the scores
        // are overwritten in full before they are read.
        e = cudaMemsetAsync(flag, 0, sizeof(uint32_t), s);
        if (e == cudaSuccess) e = vlb::launch_scores(logits, (size_t)T * E, score, scores, s);
        if (e == cudaSuccess)
            e = vlb::launch_route(scores, bias, token_ids, tid2eid, vocab, T, E, k, score,
                                  hash_routing, route_scale, idx, weights, flag, s);
        if (e == cudaSuccess) e = cudaMemcpyAsync(&flags, flag, sizeof(flags), cudaMemcpyDeviceToHost, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) st = cuda_fail("route (no-allocation)", e);
        else if (flags & 1u) st = fail(VLB_ERR_INVALID_ARGUMENT, "hash route token id exceeds its table");
        else if (flags & 2u) st = fail(VLB_ERR_INVALID_FORMAT, "route selects an out-of-range expert");
        else if (flags & 4u) st = fail(VLB_ERR_INVALID_ARGUMENT, "selected route weights cannot be normalized");
    }
    if (prev != ordinal && (e = cudaSetDevice(prev)) != cudaSuccess && st == VLB_OK)
        st = cuda_fail("cudaSetDevice (restoring the caller's device)", e);
    return st;
}
