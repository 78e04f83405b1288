// gemm_kernel.cuh - sm_100a linear layers either side of the attention:
//   D[M, N] = A[M, K] . W[N, K]^T   (W as nn.Linear stores it)
// with one of three epilogues:
//   kStore   out (operand type) = D + bias                   (F.linear)
//   kRope    out = D + bias rounded to the operand type, then, on the q | k
//            column blocks (columns < rope_cols), the rotate-half RoPE of each
//            64-column head at position row % seq_len in fp32, rounded again
//            (F.linear followed by rope_split, so the attention can read q / k
//            rotated straight from the GEMM output)
//   kAccum   out (fp32) += D (+ bias)                        (x += a W^T into
//            the fp32 residual stream, torch.addmm(out_dtype=fp32, out=x))
//
// Persistent CTAs, one per SM at most, walk the 128 x BN output tiles in a
// static stride. Warp roles (384 threads):
//   warp 0      TMA producer: A / W tiles of BK = 64 columns into a 4-stage ring
//   warp 1      MMA issuer (one elected lane): tcgen05.mma kind::f16, M = 128,
//               N = BN, K = 16, fp32 accumulators in TMEM
//   warp 2      TMEM owner (allocates / releases the 2 x BN columns)
//   warp 3      idle
//   warps 4-11  epilogue: thread = output row = TMEM lane; two warps per lane
//               quarter, each taking half of the tile's columns, the next
//               chunk's TMEM load and bias in flight while one is written out
// The accumulator is double-buffered in TMEM, so the epilogue of tile i runs
// under the MMAs of tile i + 1 (the epilogue is latency-bound: it needs the
// warps). Every wait is bounded (see attn_kernel.cuh).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "attn_kernel.cuh"

namespace fds {
namespace gemm {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kThreads = 384;
constexpr int kEpiWarp0 = 4;
constexpr int kEpiWarps = 8;

enum Epi : int { kStore = 0, kRope = 1, kAccum = 2 };

// The ring is as deep as shared memory allows (6 stages of 32 KB for 128-wide
// tiles, 4 of 48 KB for 256-wide ones): the copies in flight have to cover the
// L2 / HBM latency of a stage while the tensor cores eat one stage per
// 256 / 512 cycles.
template <int BN>
struct Smem {
    static constexpr int kStages = BN == 128 ? 6 : 4;
    static constexpr int a_bytes = kBM * kBK * 2;
    static constexpr int b_bytes = BN * kBK * 2;
    static constexpr int a = 0;
    static constexpr int b = a + kStages * a_bytes;
    static constexpr int bars = b + kStages * b_bytes;
    static constexpr int kFull = 0;                 // [stage] A and W tiles landed
    static constexpr int kEmpty = kFull + kStages;  // [stage] MMAs done with the stage
    static constexpr int kAccFull = kEmpty + kStages;    // [buffer] tile's accumulator complete
    static constexpr int kAccEmpty = kAccFull + 2;       // [buffer] epilogue read it out
    static constexpr int kDrain = kAccEmpty + 2;
    static constexpr int kNumBars = kDrain + 1;
    // misc block, same offsets as the attention kernel's (the bounded waits read
    // it): +0 TMEM base, +4 abort flag, +8 status pointer, +16 timeout, +32 mirror
    static constexpr int misc = bars + kNumBars * 8;
    static constexpr int total = misc + 48;
    static constexpr int alloc = total + 1024;
};

struct Params {
    void* out;
    int64_t out_stride;       // elements
    const void* bias;         // [N] operand type, or null
    const float* cos_t;       // kRope: fp32 [>= seq_len, 64]
    const float* sin_t;
    int32_t* status;
    int32_t* status_host;
    int64_t timeout_ns;
    int32_t m, n, k;
    int32_t seq_len;          // kRope: position = row % seq_len
    int32_t rope_cols;        // kRope: columns [0, rope_cols) are rotated
    int32_t tiles_n;          // N / BN
    int32_t tiles;            // ceil(M / 128) * tiles_n
};

template <typename T>
__device__ __forceinline__ float to_f(T x);
template <>
__device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

template <typename T>
__device__ __forceinline__ float round_t(float x);  // x rounded to T and back
template <>
__device__ __forceinline__ float round_t<__half>(float x) { return __half2float(__float2half_rn(x)); }
template <>
__device__ __forceinline__ float round_t<__nv_bfloat16>(float x) {
    return __bfloat162float(__float2bfloat16_rn(x));
}

// bias[n0 + c], c < 32, as raw 16-bit values (zeros without a bias), and
// converted to fp32
template <typename T>
__device__ __forceinline__ void fetch_bias32(const T* bias, int n0, uint4 (&raw)[4]) {
#pragma unroll
    for (int q = 0; q < 4; ++q)
        raw[q] = bias != nullptr ? __ldg(reinterpret_cast<const uint4*>(bias + n0) + q) : make_uint4(0, 0, 0, 0);
}
template <typename T>
__device__ __forceinline__ float bias_at(const uint4 (&raw)[4], int c) {
    return to_f<T>(reinterpret_cast<const T*>(&raw[c >> 3])[c & 7]);
}

template <typename T>
__device__ __forceinline__ void store32(T* dst, const float (&v)[32]) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        uint4 u;
        u.x = DTypeTraits<T>::pack(v[8 * q + 0], v[8 * q + 1]);
        u.y = DTypeTraits<T>::pack(v[8 * q + 2], v[8 * q + 3]);
        u.z = DTypeTraits<T>::pack(v[8 * q + 4], v[8 * q + 5]);
        u.w = DTypeTraits<T>::pack(v[8 * q + 6], v[8 * q + 7]);
        reinterpret_cast<uint4*>(dst)[q] = u;
    }
}

template <typename T, int BN, int kEpi>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b, const Params p) {
    using S = Smem<BN>;
    extern __shared__ uint8_t smem_raw[];
    const uint32_t raw_addr = smem_u32(smem_raw);
    const uint32_t sbase = (raw_addr + 1023u) & ~1023u;
    uint8_t* smem = smem_raw + (sbase - raw_addr);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::bars);
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + S::misc);
    const WaitCtl ctl{sbase + S::misc};
    const auto bar = [&](int idx) { return sbase + S::bars + 8u * idx; };
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int kb_n = p.k / kBK;

    grid_launch_dependents();
    if (threadIdx.x == 0) {
        for (int s = 0; s < S::kStages; ++s) {
            mbar_init(&bars[S::kFull + s], 1);
            mbar_init(&bars[S::kEmpty + s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&bars[S::kAccFull + b], 1);
            mbar_init(&bars[S::kAccEmpty + b], kEpiWarps);  // one arrival per epilogue warp
        }
        mbar_init(&bars[S::kDrain], 1);
        st_shared_volatile_u32(ctl.misc + 4, 0);
        st_shared_u64(ctl.misc + 8, reinterpret_cast<uint64_t>(p.status));
        st_shared_u64(ctl.misc + 16, static_cast<uint64_t>(p.timeout_ns > 0 ? p.timeout_ns : kDefaultTimeoutNs));
        st_shared_u64(ctl.misc + 32, reinterpret_cast<uint64_t>(p.status_host));
        fence_barrier_init();
        fence_proxy_async_smem();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tensormap(&map_a);
        prefetch_tensormap(&map_b);
    }
    if (warp == 2) {
        tmem_alloc(tmem_holder, 2 * BN);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    grid_dependency_wait();
    const uint32_t tmem = *tmem_holder;

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        int g = 0;  // k-blocks issued
        bool ok = true;
        for (int t = blockIdx.x; ok && t < p.tiles; t += gridDim.x) {
            const int m0 = (t / p.tiles_n) * kBM, n0 = (t % p.tiles_n) * BN;
            for (int kb = 0; kb < kb_n; ++kb, ++g) {
                const int st = g % S::kStages;
                if (g >= S::kStages) {
                    ok = warp_wait(bar(S::kEmpty + st), ((g / S::kStages) - 1) & 1, ctl, FDS_STATUS_TIMEOUT_LOAD);
                    if (!ok) break;
                }
                if (elect_one()) {
                    mbar_arrive_expect_tx(bar(S::kFull + st), S::a_bytes + S::b_bytes);
                    tma_load_2d(sbase + S::a + st * S::a_bytes, &map_a, bar(S::kFull + st), kb * kBK, m0);
                    tma_load_2d(sbase + S::b + st * S::b_bytes, &map_b, bar(S::kFull + st), kb * kBK, n0);
                }
                __syncwarp();
            }
        }
        if (!ok) {
            // aborted: let the copies already issued land before the CTA exits
            for (int s = 0; s < S::kStages; ++s) {
                const int n_is = g > s ? (g - s + S::kStages - 1) / S::kStages : 0;
                if (n_is > 0) wait_bounded(bar(S::kFull + s), (n_is - 1) & 1, ctl, FDS_STATUS_TIMEOUT_DRAIN, false);
            }
            __syncwarp();
        }
    } else if (warp == 1) {
        // ------------------------------------------------ MMA issuer
        constexpr uint32_t idesc = idesc_f16(kBM, BN, DTypeTraits<T>::kFormat, 0, 0);
        int g = 0, lt = 0;
        bool ok = true, issued = false;
        for (int t = blockIdx.x; ok && t < p.tiles; t += gridDim.x, ++lt) {
            const int buf = lt & 1;
            if (lt >= 2) {  // the epilogue has read this accumulator out
                ok = warp_wait(bar(S::kAccEmpty + buf), ((lt >> 1) - 1) & 1, ctl, FDS_STATUS_TIMEOUT_MMA);
                if (!ok) break;
            }
            tc_fence_after();
            for (int kb = 0; kb < kb_n; ++kb, ++g) {
                const int st = g % S::kStages;
                ok = warp_wait(bar(S::kFull + st), (g / S::kStages) & 1, ctl, FDS_STATUS_TIMEOUT_MMA);
                if (!ok) break;
                tc_fence_after();
                if (elect_one()) {
                    const uint64_t da = sw128_desc(sbase + S::a + st * S::a_bytes);
                    const uint64_t db = sw128_desc(sbase + S::b + st * S::b_bytes);
#pragma unroll
                    for (int k = 0; k < kBK / 16; ++k)
                        mma_ss(tmem + buf * BN, da + 2 * k, db + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
                    mma_commit(bar(S::kEmpty + st));
                    if (kb + 1 == kb_n) mma_commit(bar(S::kAccFull + buf));
                }
                __syncwarp();
                issued = true;
            }
        }
        if (issued) {
            if (elect_one()) mma_commit(bar(S::kDrain));
            __syncwarp();
            wait_bounded(bar(S::kDrain), 0, ctl, FDS_STATUS_TIMEOUT_DRAIN, false);
            __syncwarp();
        }
    } else if (warp >= kEpiWarp0) {
        // ------------------------------------------------ epilogue
        const int wq = warp & 3;                       // TMEM lane quarter
        const int c_begin = ((warp - kEpiWarp0) >> 2) * (BN / 2);  // this warp's column half
        const int row = wq * 32 + lane;
        const uint32_t lane_addr = static_cast<uint32_t>(wq * 32) << 16;
        const T* bias = static_cast<const T*>(p.bias);
        int lt = 0;
        bool ok = true;
        for (int t = blockIdx.x; ok && t < p.tiles; t += gridDim.x, ++lt) {
            const int buf = lt & 1;
            const int m0 = (t / p.tiles_n) * kBM, n0 = (t % p.tiles_n) * BN;
            const int m = m0 + row;
            const bool valid = m < p.m;
            // kAccum: the residual rows do not depend on the product, so the
            // first chunk's are read while the MMAs still run
            float4 xr[2][8];
            float* xrow = static_cast<float*>(p.out) + static_cast<int64_t>(m) * p.out_stride + n0;
            if constexpr (kEpi == kAccum) {
                if (valid) {
#pragma unroll
                    for (int r = 0; r < 8; ++r) xr[0][r] = reinterpret_cast<const float4*>(xrow + c_begin)[r];
                }
            }
            ok = warp_wait(bar(S::kAccFull + buf), (lt >> 1) & 1, ctl, FDS_STATUS_TIMEOUT_SOFTMAX);
            if (!ok) break;
            tc_fence_after();
            const uint32_t tacc = tmem + lane_addr + buf * BN;
            if constexpr (kEpi == kAccum) {
                // 32 columns at a time; the next chunk's residual rows in flight
#pragma unroll
                for (int q = 0; q < BN / 64; ++q) {
                    const int c = c_begin + 32 * q;
                    uint32_t acc[32];
                    uint4 braw[4];
                    tmem_ld32(tacc + c, acc);
                    fetch_bias32<T>(bias, n0 + c, braw);
                    if (q + 1 < BN / 64 && valid) {
#pragma unroll
                        for (int r = 0; r < 8; ++r)
                            xr[(q + 1) & 1][r] = reinterpret_cast<const float4*>(xrow + c + 32)[r];
                    }
                    tmem_wait_ld();
                    if (valid) {
                        float4* dst = reinterpret_cast<float4*>(xrow + c);
#pragma unroll
                        for (int r = 0; r < 8; ++r) {
                            float4 x = xr[q & 1][r];
                            x.x += __uint_as_float(acc[4 * r]) + bias_at<T>(braw, 4 * r);
                            x.y += __uint_as_float(acc[4 * r + 1]) + bias_at<T>(braw, 4 * r + 1);
                            x.z += __uint_as_float(acc[4 * r + 2]) + bias_at<T>(braw, 4 * r + 2);
                            x.w += __uint_as_float(acc[4 * r + 3]) + bias_at<T>(braw, 4 * r + 3);
                            dst[r] = x;
                        }
                    }
                }
            } else if constexpr (kEpi == kRope) {
                // one 64-column head at a time (both halves of the rotation);
                // cos / sin repeat every 32 columns (cat([f, f])): this row's 32
                // pairs are read once per tile and serve every head
                const bool rot = valid && n0 + c_begin < p.rope_cols;
                float cs[32], sn[32];
                if (rot) {
                    const int pos = m % p.seq_len;
                    const float4* cr = reinterpret_cast<const float4*>(p.cos_t + static_cast<int64_t>(pos) * 64);
                    const float4* sr = reinterpret_cast<const float4*>(p.sin_t + static_cast<int64_t>(pos) * 64);
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        const float4 c4 = __ldg(cr + q), s4 = __ldg(sr + q);
                        cs[4 * q] = c4.x, cs[4 * q + 1] = c4.y, cs[4 * q + 2] = c4.z, cs[4 * q + 3] = c4.w;
                        sn[4 * q] = s4.x, sn[4 * q + 1] = s4.y, sn[4 * q + 2] = s4.z, sn[4 * q + 3] = s4.w;
                    }
                }
#pragma unroll 1
                for (int c = c_begin; c < c_begin + BN / 2; c += 64) {
#pragma unroll
                    for (int d0 = 0; d0 < 32; d0 += 16) {  // pairs (d, d + 32), 16 at a time
                        uint32_t lo[16], hi[16];
                        uint4 bl[4], bh[4];
                        tmem_ld16(tacc + c + d0, lo);
                        tmem_ld16(tacc + c + 32 + d0, hi);
#pragma unroll
                        for (int q = 0; q < 2; ++q) {
                            bl[q] = bias != nullptr ? __ldg(reinterpret_cast<const uint4*>(bias + n0 + c + d0) + q)
                                                    : make_uint4(0, 0, 0, 0);
                            bh[q] = bias != nullptr
                                        ? __ldg(reinterpret_cast<const uint4*>(bias + n0 + c + 32 + d0) + q)
                                        : make_uint4(0, 0, 0, 0);
                        }
                        tmem_wait_ld();
                        float a[16], b[16];
#pragma unroll
                        for (int d = 0; d < 16; ++d) {
                            a[d] = round_t<T>(__uint_as_float(lo[d]) + bias_at<T>(bl, d));
                            b[d] = round_t<T>(__uint_as_float(hi[d]) + bias_at<T>(bh, d));
                        }
                        if (rot) {
#pragma unroll
                            for (int d = 0; d < 16; ++d) {
                                const float x1 = a[d], x2 = b[d];
                                a[d] = x1 * cs[d0 + d] - x2 * sn[d0 + d];
                                b[d] = x2 * cs[d0 + d] + x1 * sn[d0 + d];
                            }
                        }
                        if (valid) {
                            T* dst = static_cast<T*>(p.out) + static_cast<int64_t>(m) * p.out_stride + n0 + c + d0;
#pragma unroll
                            for (int q = 0; q < 2; ++q) {
                                uint4 u, w;
                                u.x = DTypeTraits<T>::pack(a[8 * q + 0], a[8 * q + 1]);
                                u.y = DTypeTraits<T>::pack(a[8 * q + 2], a[8 * q + 3]);
                                u.z = DTypeTraits<T>::pack(a[8 * q + 4], a[8 * q + 5]);
                                u.w = DTypeTraits<T>::pack(a[8 * q + 6], a[8 * q + 7]);
                                w.x = DTypeTraits<T>::pack(b[8 * q + 0], b[8 * q + 1]);
                                w.y = DTypeTraits<T>::pack(b[8 * q + 2], b[8 * q + 3]);
                                w.z = DTypeTraits<T>::pack(b[8 * q + 4], b[8 * q + 5]);
                                w.w = DTypeTraits<T>::pack(b[8 * q + 6], b[8 * q + 7]);
                                reinterpret_cast<uint4*>(dst)[q] = u;
                                reinterpret_cast<uint4*>(dst + 32)[q] = w;
                            }
                        }
                    }
                }
            } else {
                // kStore: 32 columns at a time, the next chunk's TMEM load and bias in flight
                uint32_t acc[2][32];
                uint4 braw[2][4];
                tmem_ld32(tacc + c_begin, acc[0]);
                fetch_bias32<T>(bias, n0 + c_begin, braw[0]);
#pragma unroll
                for (int q = 0; q < BN / 64; ++q) {
                    const int c = c_begin + 32 * q;
                    tmem_wait_ld();
                    if (q + 1 < BN / 64) {
                        tmem_ld32(tacc + c + 32, acc[(q + 1) & 1]);
                        fetch_bias32<T>(bias, n0 + c + 32, braw[(q + 1) & 1]);
                    }
                    float v[32];
#pragma unroll
                    for (int d = 0; d < 32; ++d) v[d] = __uint_as_float(acc[q & 1][d]) + bias_at<T>(braw[q & 1], d);
                    if (valid)
                        store32<T>(static_cast<T*>(p.out) + static_cast<int64_t>(m) * p.out_stride + n0 + c, v);
                }
            }
            warp_arrive(bar(S::kAccEmpty + buf), lane);  // the MMA warp may reuse this accumulator
        }
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    if (warp == 2) {
        tc_fence_after();
        tmem_dealloc(tmem, 2 * BN);
    }
}

}  // namespace gemm
}  // namespace fds
