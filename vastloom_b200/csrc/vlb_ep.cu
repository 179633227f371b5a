// Expert-parallel helpers (configuration 4: experts sharded over GPUs, tokens exchanged by
// all-to-all). The layer loop is the reference's (deepseek_v4_graph.cpp:2134-2274); what changes
// is where each (token, slot) pair's expert product runs. The source rank orders its pairs by
// global expert id (== by destination rank, experts being sharded in contiguous ranges) with the
// same stable counting sort as the single-GPU dispatch, gathers their x rows, and after the
// return exchange sums each token's rows and its shared-expert row.
#include <cuda_runtime.h>

#include "vlb_launch.h"

namespace vlb {
namespace {

__global__ void ep_validate_kernel(const uint32_t* __restrict__ idx, size_t n, uint32_t E, uint32_t* flag) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n && idx[i] >= E) atomicOr(flag, 1u);
}

// One CTA per send row: x row of the pair's token, 4 floats a thread.
__global__ void __launch_bounds__(256) ep_gather_kernel(const uint32_t* __restrict__ pair_token,
                                                        const uint32_t* __restrict__ pair_slot,
                                                        const uint32_t* __restrict__ idx, uint32_t k, uint32_t epr,
                                                        const float* __restrict__ x, uint32_t H,
                                                        float* __restrict__ send_x, uint32_t* __restrict__ send_expert) {
    const uint32_t pos = blockIdx.x;
    const uint32_t t = pair_token[pos];
    if (threadIdx.x == 0) send_expert[pos] = idx[(size_t)t * k + pair_slot[pos]] % epr;
    const float4* src = reinterpret_cast<const float4*>(x + (size_t)t * H);
    float4* dst = reinterpret_cast<float4*>(send_x + (size_t)pos * H);
    for (uint32_t c = threadIdx.x; c < H / 4u; c += blockDim.x) dst[c] = src[c];
}

// out[t] = sum over slots of y[elem_row[t * k + slot]] (slot order), + shared[t]; rows strided over
// gridDim.y (limited to 65535).
__global__ void __launch_bounds__(256) ep_combine_kernel(const float* __restrict__ y,
                                                         const uint32_t* __restrict__ elem_row, uint32_t T, uint32_t k,
                                                         const float* __restrict__ shared, uint32_t H,
                                                         float* __restrict__ out) {
    const uint32_t c4 = (blockIdx.x * blockDim.x + threadIdx.x) * 4u;
    if (c4 >= H) return;
    for (uint32_t t = blockIdx.y; t < T; t += gridDim.y) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (uint32_t j = 0; j < k; ++j) {
            const float4 v = *reinterpret_cast<const float4*>(y + (size_t)elem_row[(size_t)t * k + j] * H + c4);
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        if (shared) {
            const float4 v = *reinterpret_cast<const float4*>(shared + (size_t)t * H + c4);
            acc.x += v.x;
            acc.y += v.y;
            acc.z += v.z;
            acc.w += v.w;
        }
        *reinterpret_cast<float4*>(out + (size_t)t * H + c4) = acc;
    }
}

}  // namespace

cudaError_t launch_ep_validate(const uint32_t* idx, size_t n, uint32_t E, uint32_t* flag, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    ep_validate_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(idx, n, E, flag);
    return cudaGetLastError();
}

cudaError_t launch_ep_gather(const uint32_t* pair_token, const uint32_t* pair_slot, const uint32_t* idx,
                             uint32_t n, uint32_t k, uint32_t epr, const float* x, uint32_t H, float* send_x,
                             uint32_t* send_expert, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    ep_gather_kernel<<<n, 256, 0, s>>>(pair_token, pair_slot, idx, k, epr, x, H, send_x, send_expert);
    return cudaGetLastError();
}

cudaError_t launch_ep_combine(const float* y, const uint32_t* elem_row, uint32_t T, uint32_t k,
                              const float* shared_rows, uint32_t H, float* out, cudaStream_t s) {
    if (T == 0) return cudaSuccess;
    ep_combine_kernel<<<dim3((H / 4 + 255) / 256, T < 65535u ? T : 65535u), 256, 0, s>>>(y, elem_row, T, k,
                                                                                       shared_rows, H, out);
    return cudaGetLastError();
}

}  // namespace vlb
