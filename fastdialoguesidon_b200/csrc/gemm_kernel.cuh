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
// Persistent CTAs, one per SM at most, walk the output tiles in a static
// stride: 128 x BN tiles, one per CTA, or (kPair) 256 x BN tiles over a
// cluster of two CTAs that share each tensor-core operation (tcgen05
// cta_group::2: each CTA loads its own 128 rows of A and half of the tile's W
// rows, so a CTA moves 32 KB per 64-deep k-block of a 256-wide tile instead of
// 48 KB; the even CTA issues the MMAs, each CTA's TMEM holds its own 128 output
// rows). Warp roles (384 threads):
//   warp 0      TMA producer: A / W tiles of BK = 64 columns into a 4-stage ring
//   warp 1      MMA issuer (one elected lane; the even CTA of a pair):
//               tcgen05.mma kind::f16, M = 128 (256 for a pair), N = BN,
//               K = 16, fp32 accumulators in TMEM
//   warp 2      TMEM owner (allocates / releases the 2 x BN columns)
//   warp 3      idle
//   warps 4-11  epilogue: thread = output row = TMEM lane; two warps per lane
//               quarter, each taking half of the tile's columns. A warp turns
//               128 bytes of each of its 32 rows at a time into a swizzled
//               shared-memory box and one lane hands the box to TMA: a store
//               (kStore, kRope) or an add into the fp32 residual done in L2
//               (kAccum), so the SM writes whole lines and never reads x
// The accumulator is double-buffered in TMEM, so the epilogue of tile i runs
// under the MMAs of tile i + 1. Every wait is bounded (see attn_kernel.cuh).
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

// The ring is as deep as 192 KB allows (a stage is a 128 x 64 A tile and this
// CTA's W rows): the copies in flight have to cover the L2 / HBM latency of a
// stage while the tensor cores eat one stage per 256 / 512 cycles.
// kCs: the RoPE epilogue's cos / sin rows of the tile (128 rows x 32 fp32 of
// each table, 128-byte swizzle) take 32 KB from the ring.
template <int BN, bool kPair, bool kCs = false>
struct Smem {
    static constexpr int kBNc = kPair ? BN / 2 : BN;  // W rows this CTA loads per tile
    static constexpr int a_bytes = kBM * kBK * 2;
    static constexpr int b_bytes = kBNc * kBK * 2;
    static constexpr int kCsBytes = kCs ? 2 * kBM * 128 : 0;
    static constexpr int kStages = (192 * 1024 - kCsBytes) / (a_bytes + b_bytes);
    static constexpr int a = 0;
    static constexpr int b = a + kStages * a_bytes;
    // one staging box per epilogue warp: 32 rows x 128 bytes, 1024-aligned (the
    // 128-byte swizzle repeats every 8 rows)
    static constexpr int kStgBytes = 32 * 128;
    static constexpr int stg = b + kStages * b_bytes;
    static constexpr int cs = stg + kEpiWarps * kStgBytes;  // cos rows, then sin rows
    static constexpr int bars = cs + kCsBytes;
    static constexpr int kFull = 0;                 // [stage] A and W tiles landed (a pair: both CTAs', on the even CTA)
    static constexpr int kEmpty = kFull + kStages;  // [stage] MMAs done with the stage
    static constexpr int kAccFull = kEmpty + kStages;    // [buffer] tile's accumulator complete
    static constexpr int kAccEmpty = kAccFull + 2;       // [buffer] epilogue read it out (a pair: both CTAs', on the even CTA)
    static constexpr int kDrain = kAccEmpty + 2;
    static constexpr int kCsFull = kDrain + 1;   // the tile's cos / sin rows landed (or are not needed)
    static constexpr int kCsEmpty = kCsFull + 1; // every epilogue warp has its rows in registers
    static constexpr int kNumBars = kCsEmpty + 1;
    // misc block, same offsets as the attention kernel's (the bounded waits read
    // it): +0 TMEM base, +4 abort flag, +8 status pointer, +16 timeout, +32 mirror
    static constexpr int misc = bars + kNumBars * 8;
    static constexpr int total = misc + 48;
    static constexpr int alloc = total + 1024;
    static_assert(stg % 1024 == 0 && cs % 1024 == 0 && alloc <= 227 * 1024, "shared-memory layout");
};

struct Params {
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
    int32_t tiles;            // ceil(M / tile rows) * tiles_n
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

// This lane's 128-byte row of its warp's staging box (16-byte chunk j at chunk
// j ^ (row & 7): the tensor map's 128-byte swizzle, and no two lanes of a
// quarter-warp on the same banks), written once the box's previous contents
// have been read out by TMA (lane 0 issued those copies). The writes are then
// made visible to the async proxy for the copy lane 0 issues next.
__device__ __forceinline__ void stage_row(uint32_t srow, int lane, const uint32_t (&w)[32]) {
    if (lane == 0) bulk_wait_read_all();
    __syncwarp();
    const int sw = lane & 7;
#pragma unroll
    for (int j = 0; j < 8; ++j)
        st_shared_v4(srow + (static_cast<uint32_t>(j ^ sw) << 4),
                     make_int4(static_cast<int>(w[4 * j]), static_cast<int>(w[4 * j + 1]),
                               static_cast<int>(w[4 * j + 2]), static_cast<int>(w[4 * j + 3])));
    fence_proxy_async_smem();
    __syncwarp();
}

template <typename T, int BN, int kEpi, bool kPair>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                const __grid_constant__ CUtensorMap map_out, const __grid_constant__ CUtensorMap map_cos,
                const __grid_constant__ CUtensorMap map_sin, const Params p) {
    using S = Smem<BN, kPair, kEpi == kRope>;
    constexpr int kTileM = kPair ? 2 * kBM : kBM;
    const uint32_t rank = kPair ? cluster_ctarank() : 0u;  // 0: the CTA that issues the MMAs
    const int unit0 = kPair ? static_cast<int>(blockIdx.x >> 1) : static_cast<int>(blockIdx.x);
    const int units = kPair ? static_cast<int>(gridDim.x >> 1) : static_cast<int>(gridDim.x);
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
            mbar_init(&bars[S::kAccEmpty + b], kPair ? 2 * kEpiWarps : kEpiWarps);  // one per epilogue warp
        }
        mbar_init(&bars[S::kDrain], 1);
        mbar_init(&bars[S::kCsFull], 1);
        mbar_init(&bars[S::kCsEmpty], kEpiWarps);
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
        prefetch_tensormap(&map_out);
        if constexpr (kEpi == kRope) {
            prefetch_tensormap(&map_cos);
            prefetch_tensormap(&map_sin);
        }
    }
    if (warp == 2) {
        if constexpr (kPair) {
            tmem_alloc_pair(tmem_holder, 2 * BN);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(tmem_holder, 2 * BN);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    __syncthreads();
    if constexpr (kPair) cluster_sync_all();  // the other CTA's barriers are initialised
    tc_fence_after();
    grid_dependency_wait();
    const uint32_t tmem = *tmem_holder;
    // the pair's shared barriers live in the even CTA
    const auto bar0 = [&](int idx) { return kPair ? map_to_rank(bar(idx), 0) : bar(idx); };

    if (warp == 0) {
        // ------------------------------------------------ TMA producer
        int g = 0;  // k-blocks issued
        bool ok = true;
        for (int t = unit0; ok && t < p.tiles; t += units) {
            // this CTA's A rows and W rows of the tile
            const int m0 = (t / p.tiles_n) * kTileM + static_cast<int>(rank) * kBM;
            const int n0 = (t % p.tiles_n) * BN + static_cast<int>(rank) * S::kBNc;
            for (int kb = 0; kb < kb_n; ++kb, ++g) {
                const int st = g % S::kStages;
                if (g >= S::kStages) {
                    ok = warp_wait(bar(S::kEmpty + st), ((g / S::kStages) - 1) & 1, ctl, FDS_STATUS_TIMEOUT_LOAD);
                    if (!ok) break;
                }
                if (elect_one()) {
                    if constexpr (kPair) {
                        // the even CTA's full barrier counts both CTAs' bytes; only it arms
                        const uint32_t fb = map_to_rank(bar(S::kFull + st), 0);
                        if (rank == 0) mbar_arrive_expect_tx(bar(S::kFull + st), 2 * (S::a_bytes + S::b_bytes));
                        tma_load_2d_pair(sbase + S::a + st * S::a_bytes, &map_a, fb, kb * kBK, m0);
                        tma_load_2d_pair(sbase + S::b + st * S::b_bytes, &map_b, fb, kb * kBK, n0);
                    } else {
                        mbar_arrive_expect_tx(bar(S::kFull + st), S::a_bytes + S::b_bytes);
                        tma_load_2d(sbase + S::a + st * S::a_bytes, &map_a, bar(S::kFull + st), kb * kBK, m0);
                        tma_load_2d(sbase + S::b + st * S::b_bytes, &map_b, bar(S::kFull + st), kb * kBK, n0);
                    }
                }
                __syncwarp();
            }
        }
        if (!ok && rank == 0) {
            // aborted: let the copies already armed land before the CTA exits
            // (a pair's odd CTA has no barrier of its own to watch: its copies
            // were issued at least one timeout before it gets here, and both
            // CTAs meet at the cluster barrier before either exits)
            for (int s = 0; s < S::kStages; ++s) {
                const int n_is = g > s ? (g - s + S::kStages - 1) / S::kStages : 0;
                if (n_is > 0) wait_bounded(bar(S::kFull + s), (n_is - 1) & 1, ctl, FDS_STATUS_TIMEOUT_DRAIN, false);
            }
            __syncwarp();
        }
    } else if (warp == 1 && rank == 0) {
        // ------------------------------------------------ MMA issuer
        constexpr uint32_t idesc = idesc_f16(kTileM, BN, DTypeTraits<T>::kFormat, 0, 0);
        // completions go to both CTAs of a pair (their stages and accumulators)
        const auto commit = [&](int idx) {
            if constexpr (kPair) {
                mma_commit_pair(bar(idx));
                mma_commit_pair(map_to_rank(bar(idx), 1));
            } else {
                mma_commit(bar(idx));
            }
        };
        int g = 0, lt = 0;
        bool ok = true, issued = false;
        for (int t = unit0; ok && t < p.tiles; t += units, ++lt) {
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
                    for (int k = 0; k < kBK / 16; ++k) {
                        if constexpr (kPair)
                            mma_ss_pair(tmem + buf * BN, da + 2 * k, db + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
                        else
                            mma_ss(tmem + buf * BN, da + 2 * k, db + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
                    }
                    commit(S::kEmpty + st);
                    if (kb + 1 == kb_n) commit(S::kAccFull + buf);
                }
                __syncwarp();
                issued = true;
            }
        }
        if (issued) {
            if (elect_one()) {
                if constexpr (kPair)
                    mma_commit_pair(bar(S::kDrain));
                else
                    mma_commit(bar(S::kDrain));
            }
            __syncwarp();
            wait_bounded(bar(S::kDrain), 0, ctl, FDS_STATUS_TIMEOUT_DRAIN, false);
            __syncwarp();
        }
    } else if (warp == 3 && kEpi == kRope) {
        // ------------------------------------------------ cos / sin rows of each tile
        // (positions (m0 + r) % seq_len, r < 128: one TMA box of each table when
        // they do not wrap past seq_len; otherwise, or for tiles with no rotated
        // column, the epilogue reads global memory and the barrier completes empty)
        int lt = 0, armed = -1;
        bool ok = true;
        for (int t = unit0; ok && t < p.tiles; t += units, ++lt) {
            const int m0 = (t / p.tiles_n) * kTileM + static_cast<int>(rank) * kBM, n0 = (t % p.tiles_n) * BN;
            if (lt >= 1) {
                ok = warp_wait(bar(S::kCsEmpty), (lt - 1) & 1, ctl, FDS_STATUS_TIMEOUT_LOAD);
                if (!ok) break;
            }
            const int pos0 = m0 % p.seq_len;
            const bool tma = n0 < p.rope_cols && pos0 + kBM <= p.seq_len;
            if (elect_one()) {
                if (tma) {
                    mbar_arrive_expect_tx(bar(S::kCsFull), S::kCsBytes);
                    tma_load_2d(sbase + S::cs, &map_cos, bar(S::kCsFull), 0, pos0);
                    tma_load_2d(sbase + S::cs + kBM * 128, &map_sin, bar(S::kCsFull), 0, pos0);
                } else {
                    mbar_arrive(bar(S::kCsFull));
                }
            }
            __syncwarp();
            if (tma) armed = lt;
        }
        if (!ok && armed >= 0) {  // aborted: the last copies issued land before the CTA exits
            wait_bounded(bar(S::kCsFull), armed & 1, ctl, FDS_STATUS_TIMEOUT_DRAIN, false);
            __syncwarp();
        }
    } else if (warp >= kEpiWarp0) {
        // ------------------------------------------------ epilogue
        const int wq = warp & 3;                       // TMEM lane quarter
        const int c_begin = ((warp - kEpiWarp0) >> 2) * (BN / 2);  // this warp's column half
        const int row = wq * 32 + lane;
        const uint32_t lane_addr = static_cast<uint32_t>(wq * 32) << 16;
        const uint32_t stg = sbase + S::stg + (warp - kEpiWarp0) * S::kStgBytes;
        const uint32_t srow = stg + lane * 128;
        const T* bias = static_cast<const T*>(p.bias);
        int lt = 0;
        bool ok = true;
        // one arrival per warp on the (even CTA's) accumulator-empty barrier
        const auto acc_empty = [&](int b) {
            if constexpr (kPair) {
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(bar0(S::kAccEmpty + b));
            } else {
                warp_arrive(bar(S::kAccEmpty + b), lane);
            }
        };
        for (int t = unit0; ok && t < p.tiles; t += units, ++lt) {
            const int buf = lt & 1;
            const int m0 = (t / p.tiles_n) * kTileM + static_cast<int>(rank) * kBM, n0 = (t % p.tiles_n) * BN;
            const int y0 = m0 + wq * 32;     // the warp's first row; rows >= m are clipped by TMA
            const bool live = y0 < p.m;      // a box wholly past the last row is not copied
            ok = warp_wait(bar(S::kAccFull + buf), (lt >> 1) & 1, ctl, FDS_STATUS_TIMEOUT_SOFTMAX);
            if (!ok) break;
            tc_fence_after();
            const uint32_t tacc = tmem + lane_addr + buf * BN;
            if constexpr (kEpi == kAccum) {
                // fp32 boxes of 32 columns, added into the residual by TMA
#pragma unroll 1
                for (int q = 0; q < BN / 64; ++q) {
                    const int c = c_begin + 32 * q;
                    uint32_t acc[32];
                    uint4 braw[4];
                    tmem_ld32(tacc + c, acc);
                    fetch_bias32<T>(bias, n0 + c, braw);
                    tmem_wait_ld();
                    if (q + 1 == BN / 64) acc_empty(buf);  // accumulator read out
                    uint32_t w[32];
#pragma unroll
                    for (int d = 0; d < 32; ++d) w[d] = __float_as_uint(__uint_as_float(acc[d]) + bias_at<T>(braw, d));
                    stage_row(srow, lane, w);
                    if (lane == 0 && live) {
                        tma_reduce_add_2d(&map_out, stg, n0 + c, y0);
                        bulk_commit_group();
                    }
                }
            } else if constexpr (kEpi == kRope) {
                // one 64-column head per box (both halves of the rotation).
                // cos / sin repeat every 32 columns (cat([f, f])): the row's 32
                // pairs serve every head of the tile, so they are read once per
                // tile (uncoalesced: a warp's lanes are 32 rows) and kept in
                // registers; each 16-pair chunk goes straight into the staging
                // box, so no whole head row is held
                float cs[32], sn[32];
                ok = warp_wait(bar(S::kCsFull), lt & 1, ctl, FDS_STATUS_TIMEOUT_SOFTMAX);
                if (!ok) break;
                if (n0 + c_begin < p.rope_cols) {
                    const int pos0 = m0 % p.seq_len;
                    if (pos0 + kBM <= p.seq_len) {
                        // this row of the staged boxes (16-byte chunk j at j ^ (row & 7))
                        const uint32_t crow = sbase + S::cs + row * 128, srow_s = crow + kBM * 128;
#pragma unroll
                        for (int q = 0; q < 8; ++q) {
                            const uint32_t off = static_cast<uint32_t>(q ^ (row & 7)) << 4;
                            const float4 c4 = ld_shared_v4f32(crow + off), s4 = ld_shared_v4f32(srow_s + off);
                            cs[4 * q] = c4.x, cs[4 * q + 1] = c4.y, cs[4 * q + 2] = c4.z, cs[4 * q + 3] = c4.w;
                            sn[4 * q] = s4.x, sn[4 * q + 1] = s4.y, sn[4 * q + 2] = s4.z, sn[4 * q + 3] = s4.w;
                        }
                    } else {
                        const int pos = (m0 + row) % p.seq_len;
                        const float4* cr = reinterpret_cast<const float4*>(p.cos_t + static_cast<int64_t>(pos) * 64);
                        const float4* sr = reinterpret_cast<const float4*>(p.sin_t + static_cast<int64_t>(pos) * 64);
#pragma unroll
                        for (int q = 0; q < 8; ++q) {
                            const float4 c4 = __ldg(cr + q), s4 = __ldg(sr + q);
                            cs[4 * q] = c4.x, cs[4 * q + 1] = c4.y, cs[4 * q + 2] = c4.z, cs[4 * q + 3] = c4.w;
                            sn[4 * q] = s4.x, sn[4 * q + 1] = s4.y, sn[4 * q + 2] = s4.z, sn[4 * q + 3] = s4.w;
                        }
                    }
                }
                warp_arrive(bar(S::kCsEmpty), lane);  // the rows are in registers
                const int sw = lane & 7;
#pragma unroll 1
                for (int c = c_begin; c < c_begin + BN / 2; c += 64) {
                    const bool rot = n0 + c < p.rope_cols;
                    if (lane == 0) bulk_wait_read_all();  // the box's previous head has been copied out
                    __syncwarp();
#pragma unroll
                    for (int d0 = 0; d0 < 32; d0 += 16) {  // pairs (d, d + 32), 16 at a time
                        uint32_t lo[16], hi[16];
                        uint4 bl[2], bh[2];
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
                            a[d] = round_t<T>(__uint_as_float(lo[d]) + to_f<T>(reinterpret_cast<const T*>(bl)[d]));
                            b[d] = round_t<T>(__uint_as_float(hi[d]) + to_f<T>(reinterpret_cast<const T*>(bh)[d]));
                        }
                        if (rot) {
#pragma unroll
                            for (int d = 0; d < 16; ++d) {
                                const float x1 = a[d], x2 = b[d];
                                a[d] = x1 * cs[d0 + d] - x2 * sn[d0 + d];
                                b[d] = x2 * cs[d0 + d] + x1 * sn[d0 + d];
                            }
                        }
                        // columns d0 .. d0 + 15 are 16-byte chunks d0 / 8, d0 / 8 + 1 of
                        // the 128-byte row; columns 32 + d0 .. chunks 4 + d0 / 8, ..
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const float* v = h == 0 ? a : b;
#pragma unroll
                            for (int q = 0; q < 2; ++q) {
                                const int j = 4 * h + d0 / 8 + q;
                                st_shared_v4(srow + (static_cast<uint32_t>(j ^ sw) << 4),
                                             make_int4(static_cast<int>(DTypeTraits<T>::pack(v[8 * q], v[8 * q + 1])),
                                                       static_cast<int>(DTypeTraits<T>::pack(v[8 * q + 2], v[8 * q + 3])),
                                                       static_cast<int>(DTypeTraits<T>::pack(v[8 * q + 4], v[8 * q + 5])),
                                                       static_cast<int>(DTypeTraits<T>::pack(v[8 * q + 6], v[8 * q + 7]))));
                            }
                        }
                    }
                    if (c + 64 == c_begin + BN / 2) acc_empty(buf);
                    fence_proxy_async_smem();
                    __syncwarp();
                    if (lane == 0 && live) {
                        tma_store_2d(&map_out, stg, n0 + c, y0);
                        bulk_commit_group();
                    }
                }
            } else {
                // kStore: 64-column boxes
#pragma unroll 1
                for (int c = c_begin; c < c_begin + BN / 2; c += 64) {
                    uint32_t a0[32], a1[32];
                    uint4 b0[4], b1[4];
                    tmem_ld32(tacc + c, a0);
                    tmem_ld32(tacc + c + 32, a1);
                    fetch_bias32<T>(bias, n0 + c, b0);
                    fetch_bias32<T>(bias, n0 + c + 32, b1);
                    tmem_wait_ld();
                    if (c + 64 == c_begin + BN / 2) acc_empty(buf);
                    uint32_t w[32];
#pragma unroll
                    for (int q = 0; q < 16; ++q) {
                        w[q] = DTypeTraits<T>::pack(__uint_as_float(a0[2 * q]) + bias_at<T>(b0, 2 * q),
                                                    __uint_as_float(a0[2 * q + 1]) + bias_at<T>(b0, 2 * q + 1));
                        w[16 + q] = DTypeTraits<T>::pack(__uint_as_float(a1[2 * q]) + bias_at<T>(b1, 2 * q),
                                                         __uint_as_float(a1[2 * q + 1]) + bias_at<T>(b1, 2 * q + 1));
                    }
                    stage_row(srow, lane, w);
                    if (lane == 0 && live) {
                        tma_store_2d(&map_out, stg, n0 + c, y0);
                        bulk_commit_group();
                    }
                }
            }
        }
        // the copies out of the staging boxes have landed before the CTA exits
        if (lane == 0) bulk_wait_all();
        __syncwarp();
    }
    __syncwarp();
    tc_fence_before();
    __syncthreads();
    // a pair: the even CTA's MMAs into this CTA's TMEM are drained and every
    // cross-CTA arrival has landed before either CTA releases TMEM or exits
    if constexpr (kPair) cluster_sync_all();
    if (warp == 2) {
        tc_fence_after();
        if constexpr (kPair)
            tmem_dealloc_pair(tmem, 2 * BN);
        else
            tmem_dealloc(tmem, 2 * BN);
    }
}

}  // namespace gemm
}  // namespace fds
