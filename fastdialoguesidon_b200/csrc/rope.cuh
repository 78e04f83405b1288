// rope.cuh - rotary position embedding on the q / k column blocks of a fused
// qkv row (the DiT head's rotate-half RoPE):
//   d < 32:  y[d] = x[d] * cos[t][d] - x[d + 32] * sin[t][d]
//   d >= 32: y[d] = x[d] * cos[t][d] + x[d - 32] * sin[t][d]
// computed in fp32 from fp32 tables and rounded once to the operand type, as
// triton/src/fds_triton/kernels.py:448-473 (_rope_split_kernel) does; v is
// copied bit-exactly when a destination is given. t = row % seq_len.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

namespace fds {

template <typename T>
__device__ __forceinline__ float to_f32(T x);
template <>
__device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }

// One thread: one (row, head, part) and one 8-column chunk c of each half
// (columns [8c, 8c+8) and [32+8c, 32+8c+8)), i.e. 16 outputs from 32 B of x.
template <typename T>
__global__ void __launch_bounds__(256) rope_rotate_kernel(const T* __restrict__ qkv, int64_t qkv_stride,
                                                          const float* __restrict__ cos_t,
                                                          const float* __restrict__ sin_t, T* __restrict__ dst_q,
                                                          T* __restrict__ dst_k, T* __restrict__ dst_v,
                                                          int64_t dst_stride, int rows, int seq_len, int heads) {
    // programmatic dependent launch (see grid_dependency_wait)
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int parts = dst_v != nullptr ? 3 : 2;
    const int64_t gid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t total = static_cast<int64_t>(rows) * heads * parts * 4;
    if (gid >= total) return;
    const int c = static_cast<int>(gid & 3);
    int64_t t = gid >> 2;
    const int part = static_cast<int>(t % parts);
    t /= parts;
    const int hh = static_cast<int>(t % heads);
    const int64_t row = t / heads;
    const int hid = heads * 64;

    const T* src = qkv + row * qkv_stride + static_cast<int64_t>(part) * hid + hh * 64;
    T* dst = (part == 0 ? dst_q : (part == 1 ? dst_k : dst_v)) + row * dst_stride + hh * 64;
    const uint4 lo = *reinterpret_cast<const uint4*>(src + 8 * c);
    const uint4 hi = *reinterpret_cast<const uint4*>(src + 32 + 8 * c);
    if (part == 2) {
        *reinterpret_cast<uint4*>(dst + 8 * c) = lo;
        *reinterpret_cast<uint4*>(dst + 32 + 8 * c) = hi;
        return;
    }
    const int pos = static_cast<int>(row % seq_len);
    const float4* cr = reinterpret_cast<const float4*>(cos_t + static_cast<int64_t>(pos) * 64);
    const float4* sr = reinterpret_cast<const float4*>(sin_t + static_cast<int64_t>(pos) * 64);
    float cl[8], sl[8], ch[8], sh[8];
    *reinterpret_cast<float4*>(&cl[0]) = cr[2 * c];
    *reinterpret_cast<float4*>(&cl[4]) = cr[2 * c + 1];
    *reinterpret_cast<float4*>(&ch[0]) = cr[8 + 2 * c];
    *reinterpret_cast<float4*>(&ch[4]) = cr[8 + 2 * c + 1];
    *reinterpret_cast<float4*>(&sl[0]) = sr[2 * c];
    *reinterpret_cast<float4*>(&sl[4]) = sr[2 * c + 1];
    *reinterpret_cast<float4*>(&sh[0]) = sr[8 + 2 * c];
    *reinterpret_cast<float4*>(&sh[4]) = sr[8 + 2 * c + 1];
    const T* xl = reinterpret_cast<const T*>(&lo);
    const T* xh = reinterpret_cast<const T*>(&hi);
    uint4 ylo, yhi;
    T* yl = reinterpret_cast<T*>(&ylo);
    T* yh = reinterpret_cast<T*>(&yhi);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const float a = to_f32(xl[e]);
        const float bb = to_f32(xh[e]);
        yl[e] = from_f32<T>(a * cl[e] - bb * sl[e]);
        yh[e] = from_f32<T>(bb * ch[e] + a * sh[e]);
    }
    *reinterpret_cast<uint4*>(dst + 8 * c) = ylo;
    *reinterpret_cast<uint4*>(dst + 32 + 8 * c) = yhi;
}

}  // namespace fds
