// Expert-parallel helpers (configuration 4: experts sharded over GPUs, tokens exchanged by
// all-to-all). The layer loop is the reference's (deepseek_v4_graph.cpp:2134-2274); what changes
// is where each (token, slot) pair's expert product runs. The source rank orders its pairs by
// global expert id (== by destination rank, experts being sharded in contiguous ranges) with the
// same stable counting sort as the single-GPU dispatch, gathers their x rows, and after the
// return exchange sums each token's rows and its shared-expert row.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "vlb_launch.h"
#include "vlb_mma.cuh"

namespace vlb {
namespace {

__global__ void ep_validate_kernel(const uint32_t* __restrict__ idx, size_t n, uint32_t E, uint32_t* flag) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n && idx[i] >= E) atomicOr(flag, 1u);
}

// Routes as the exchange orders them: each global expert id replaced by its slot (rank r holds the
// slots [r * epr, (r + 1) * epr), so a stable sort by slot is a sort by destination rank); an id out
// of range is flagged and replaced by slot 0, so nothing downstream indexes past a table.
__global__ void ep_slots_kernel(const uint32_t* __restrict__ idx, size_t n, uint32_t E,
                                const uint32_t* __restrict__ slot_of, uint32_t* __restrict__ out, uint32_t* flag) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const uint32_t e = idx[i];
    if (e >= E) {
        atomicOr(flag, 1u);
        out[i] = 0;
        return;
    }
    out[i] = slot_of ? slot_of[e] : e;
}

// Expert outputs for the return exchange as fp16 rows: row r = fp16(y[r] * 2^e_r) with 2^e_r the
// power of two that brings the row's max|y| into [2^14, 2^15) (no overflow, small values kept
// normal), its f32 inverse 2^-e_r in scale[r]. One CTA per row.
__global__ void __launch_bounds__(256) ep_pack_half_kernel(const float* __restrict__ y, uint32_t H,
                                                           __half* __restrict__ rows, float* __restrict__ scale) {
    __shared__ float wmax[8];
    const float* src = y + (size_t)blockIdx.x * H;
    float m = 0.f;
    for (uint32_t c = threadIdx.x * 4u; c < H; c += blockDim.x * 4u) {
        const float4 v = *reinterpret_cast<const float4*>(src + c);
        m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31u) == 0) wmax[threadIdx.x >> 5] = m;
    __syncthreads();
    float mm = 0.f;
    for (uint32_t i = 0; i < blockDim.x / 32u; ++i) mm = fmaxf(mm, wmax[i]);
    const float s = mma::prescale_for(mm);
    if (threadIdx.x == 0) scale[blockIdx.x] = 1.f / s;  // exact: a power of two
    __half* dst = rows + (size_t)blockIdx.x * H;
    for (uint32_t c = threadIdx.x * 8u; c < H; c += blockDim.x * 8u) {
        const float4 a = *reinterpret_cast<const float4*>(src + c);
        const float4 b = *reinterpret_cast<const float4*>(src + c + 4u);
        const __half2 h0 = __floats2half2_rn(a.x * s, a.y * s), h1 = __floats2half2_rn(a.z * s, a.w * s);
        const __half2 h2 = __floats2half2_rn(b.x * s, b.y * s), h3 = __floats2half2_rn(b.z * s, b.w * s);
        uint4 o;
        o.x = *reinterpret_cast<const uint32_t*>(&h0);
        o.y = *reinterpret_cast<const uint32_t*>(&h1);
        o.z = *reinterpret_cast<const uint32_t*>(&h2);
        o.w = *reinterpret_cast<const uint32_t*>(&h3);
        *reinterpret_cast<uint4*>(dst + c) = o;
    }
}

// Combine from returned fp16 rows: out[t] = sum over slots of fp16 row * its scale (slot order) +
// shared[t] (f32, this rank's own rows).
__global__ void __launch_bounds__(256) ep_combine_half_kernel(const __half* __restrict__ rows,
                                                              const float* __restrict__ scale,
                                                              const uint32_t* __restrict__ elem_row, uint32_t T,
                                                              uint32_t k, const float* __restrict__ shared, uint32_t H,
                                                              float* __restrict__ out) {
    const uint32_t c4 = (blockIdx.x * blockDim.x + threadIdx.x) * 4u;
    if (c4 >= H) return;
    for (uint32_t t = blockIdx.y; t < T; t += gridDim.y) {
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (uint32_t j = 0; j < k; ++j) {
            const uint32_t r = elem_row[(size_t)t * k + j];
            const float sc = scale[r];
            const uint2 u = *reinterpret_cast<const uint2*>(rows + (size_t)r * H + c4);
            const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
            const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
            acc.x += a.x * sc;
            acc.y += a.y * sc;
            acc.z += b.x * sc;
            acc.w += b.y * sc;
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

// fp16 rows for the exchange: send row pos = fp16(x[token] * s_token) (s the power of two of the
// token's max|x|: exactly the row the receiver's tensor-core path would build from the f32 row),
// meta = (local expert id, route weight bits, max|x| bits). One CTA per send row, 8 columns a
// thread.
__global__ void __launch_bounds__(256) ep_gather_half_kernel(const uint32_t* __restrict__ pair_token,
                                                             const uint32_t* __restrict__ pair_slot,
                                                             const uint32_t* __restrict__ idx,
                                                             const float* __restrict__ sorted_w, uint32_t k,
                                                             uint32_t epr, const float* __restrict__ x,
                                                             const uint32_t* __restrict__ xmax, uint32_t H,
                                                             __half* __restrict__ rows, uint32_t* __restrict__ meta) {
    const uint32_t pos = blockIdx.x;
    const uint32_t t = pair_token[pos];
    const uint32_t xm = xmax[t];
    if (threadIdx.x == 0) {
        meta[3u * pos] = idx[(size_t)t * k + pair_slot[pos]] % epr;
        meta[3u * pos + 1u] = __float_as_uint(sorted_w[pos]);
        meta[3u * pos + 2u] = xm;
    }
    const float s = mma::prescale_for(__uint_as_float(xm));
    const float* src = x + (size_t)t * H;
    __half* dst = rows + (size_t)pos * H;
    for (uint32_t c = threadIdx.x * 8u; c < H; c += blockDim.x * 8u) {
        const float4 a = *reinterpret_cast<const float4*>(src + c);
        const float4 b = *reinterpret_cast<const float4*>(src + c + 4u);
        const __half2 h0 = __floats2half2_rn(a.x * s, a.y * s), h1 = __floats2half2_rn(a.z * s, a.w * s);
        const __half2 h2 = __floats2half2_rn(b.x * s, b.y * s), h3 = __floats2half2_rn(b.z * s, b.w * s);
        uint4 o;
        o.x = *reinterpret_cast<const uint32_t*>(&h0);
        o.y = *reinterpret_cast<const uint32_t*>(&h1);
        o.z = *reinterpret_cast<const uint32_t*>(&h2);
        o.w = *reinterpret_cast<const uint32_t*>(&h3);
        *reinterpret_cast<uint4*>(dst + c) = o;
    }
}

// The rank's own tokens as fp16 rows for its shared expert (local expert `epr`, weight 1).
__global__ void __launch_bounds__(256) ep_own_rows_kernel(const float* __restrict__ x,
                                                          const uint32_t* __restrict__ xmax, uint32_t H,
                                                          uint32_t epr, __half* __restrict__ rows,
                                                          uint32_t* __restrict__ meta) {
    const uint32_t t = blockIdx.x;
    const uint32_t xm = xmax[t];
    if (threadIdx.x == 0) {
        meta[3u * t] = epr;
        meta[3u * t + 1u] = __float_as_uint(1.0f);
        meta[3u * t + 2u] = xm;
    }
    const float s = mma::prescale_for(__uint_as_float(xm));
    for (uint32_t c = threadIdx.x * 8u; c < H; c += blockDim.x * 8u) {
        const float4 a = *reinterpret_cast<const float4*>(x + (size_t)t * H + c);
        const float4 b = *reinterpret_cast<const float4*>(x + (size_t)t * H + c + 4u);
        const __half2 h0 = __floats2half2_rn(a.x * s, a.y * s), h1 = __floats2half2_rn(a.z * s, a.w * s);
        const __half2 h2 = __floats2half2_rn(b.x * s, b.y * s), h3 = __floats2half2_rn(b.z * s, b.w * s);
        uint4 o;
        o.x = *reinterpret_cast<const uint32_t*>(&h0);
        o.y = *reinterpret_cast<const uint32_t*>(&h1);
        o.z = *reinterpret_cast<const uint32_t*>(&h2);
        o.w = *reinterpret_cast<const uint32_t*>(&h3);
        *reinterpret_cast<uint4*>(rows + (size_t)t * H + c) = o;
    }
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

cudaError_t launch_ep_slots(const uint32_t* idx, size_t n, uint32_t E, const uint32_t* slot_of, uint32_t* out,
                            uint32_t* flag, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    ep_slots_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(idx, n, E, slot_of, out, flag);
    return cudaGetLastError();
}

cudaError_t launch_ep_pack_half(const float* y, uint32_t rows, uint32_t H, __half* out, float* scale, cudaStream_t s) {
    if (rows == 0) return cudaSuccess;
    ep_pack_half_kernel<<<rows, 256, 0, s>>>(y, H, out, scale);
    return cudaGetLastError();
}

cudaError_t launch_ep_combine_half(const __half* rows, const float* scale, const uint32_t* elem_row, uint32_t T,
                                   uint32_t k, const float* shared_rows, uint32_t H, float* out, cudaStream_t s) {
    if (T == 0) return cudaSuccess;
    ep_combine_half_kernel<<<dim3((H / 4 + 255) / 256, T < 65535u ? T : 65535u), 256, 0, s>>>(
        rows, scale, elem_row, T, k, shared_rows, H, out);
    return cudaGetLastError();
}

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

cudaError_t launch_ep_gather_half(const uint32_t* pair_token, const uint32_t* pair_slot, const uint32_t* idx,
                                  const float* sorted_w, uint32_t n, uint32_t k, uint32_t epr, const float* x,
                                  const uint32_t* xmax, uint32_t H, __half* rows, uint32_t* meta, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    ep_gather_half_kernel<<<n, 256, 0, s>>>(pair_token, pair_slot, idx, sorted_w, k, epr, x, xmax, H, rows, meta);
    return cudaGetLastError();
}

cudaError_t launch_ep_own_rows(const float* x, const uint32_t* xmax, uint32_t T, uint32_t H, uint32_t epr,
                               __half* rows, uint32_t* meta, cudaStream_t s) {
    if (T == 0) return cudaSuccess;
    ep_own_rows_kernel<<<T, 256, 0, s>>>(x, xmax, H, epr, rows, meta);
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
