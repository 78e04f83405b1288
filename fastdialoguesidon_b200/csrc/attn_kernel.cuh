// attn_kernel.cuh - sm_100a attention forward with an optional relative_key bias.
//
// One CTA owns 256 query rows of one (window, head): two 128-row query tiles
// (Q0, Q1) that share every K/V tile. Warp roles (384 threads, 3 warpgroups):
//   warp 0                   MMA issuer of query tile 0
//   warp 1                   TMA producer (K / V ring, Q, the rel table)
//   warp 2                   MMA issuer of query tile 1
//   warp 3                   TMEM owner (allocates / releases the 512 columns)
//   warpgroup 1 (warps 4-7)  softmax of query tile 0 (thread = query row = TMEM lane)
//   warpgroup 2 (warps 8-11) softmax of query tile 1
// The control warps are the lowest-numbered (oldest) warps, which the warp
// schedulers favour when several warps are ready: their few instructions
// are on every hand-off's path, while the softmax warps always have
// independent work to issue.
// Each query tile has its own MMA warp, which serves that tile's hand-offs in
// their natural order (S(j+1) once S(j) is read out, P(j) V(j) once P(j) is
// stored); one MMA warp serving both tiles in a fixed order made each tile
// wait on the other's progress.
// tcgen05.mma groups are issued by one elected lane of a converged warp, so
// the descriptors are warp-uniform and the tensor pipe is fed at full rate.
//
// TMEM (512 columns): S0 [0,128) S1 [128,256) P0 [256,320) P1 [320,384)
//                     O0 [384,448) O1 [448,512).
// P (the exponentiated scores, two 16-bit values per column) has its own
// columns, so S(j+1) = Q K(j+1)^T runs while the softmax warps exponentiate
// S(j), and P(j) V(j) runs under the next tile's softmax.
//
// Relative bias (encoder): bias(i, j) = q_i . rel[clamp(j - i, -64, 8) + 64].
// Per query tile the MMA computes QR = Q . rel^T (N = 80, rows 73..79 zero)
// into the S columns once; the softmax threads copy their row of QR (scaled to
// log2 units) into shared memory. A KV tile whose every (i, j) pair saturates
// the clamp adds a per-row constant (QR[i,0] on the left, QR[i,72] on the
// right), which folds into the exponent's FFMA offset at no per-score cost;
// only the (at most three) near-diagonal tiles gather the bias per score.
// This is the clamp-saturation property the reference exploits in
// triton/src/fds_triton/kernels.py:364-398 (its _flexrel_kernel), realised
// here as a per-tile offset instead of running-max shifts.
//
// Online softmax: log2 units, lazy rescaling (the running max used for the
// exponent only moves when a tile's max exceeds it by more than 8, i.e. P is
// bounded by 256), fp32 row sums, P rounded to the operand type.
//
// Registers: launched at 168 per thread; the control warpgroup gives back down
// to 40 and the two softmax warpgroups take 232 (256*232 + 128*40 = 384*168),
// enough to hold a row of S (128 fp32) and of P (64 packed pairs) at once.
//
// Every wait is bounded by a globaltimer deadline; an expired wait records a
// status bit, raises a CTA-wide abort flag, and every role then drains its
// in-flight copies / MMAs and exits so the context stays usable.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "fds_b200.h"
#include "fds_ptx.cuh"

namespace fds {

constexpr int kBlockM = 128;       // query rows per tile (= TMEM lanes)
constexpr int kQTiles = 2;         // query tiles per CTA
constexpr int kRowsPerCta = kBlockM * kQTiles;
constexpr int kBlockN = 128;       // keys per KV tile
constexpr int kHeadDim = 64;
constexpr int kStages = 3;         // K/V shared-memory ring depth
constexpr int kTileBytes = kBlockM * kHeadDim * 2;
constexpr int kNumPos = 73;        // relative-key table rows
constexpr int kClampLeft = 64;
constexpr int kClampRight = 8;
constexpr int kRelRows = 80;       // table rows padded to a multiple of 16 (MMA N)
constexpr int kQrStride = 74;      // floats per row of the shared QR copy (conflict-free gather)
constexpr int kMmaWarp0 = 0;       // MMA issuer of query tile 0 (tile 1: kMmaWarp0 + 2)
constexpr int kLoadWarp = 1;
constexpr int kTmemWarp = 3;
constexpr int kSoftmaxWarp0 = 4;   // first softmax warp (query tile 0: warps 4-7, tile 1: 8-11)
constexpr int kThreads = 384;
constexpr int kLaunchRegs = 168;   // per thread at launch (checked at build time)
constexpr int kSoftmaxRegs = 232;
constexpr int kControlRegs = 40;
static_assert(256 * kSoftmaxRegs + 128 * kControlRegs <= kThreads * kLaunchRegs,
              "register split exceeds the launch pool");
constexpr int kTmemCols = 512;
constexpr int kTmemS = 0;          // S_w at kTmemS + 128 w
constexpr int kTmemP = 256;        // P_w at kTmemP + 64 w
constexpr int kTmemO = 384;        // O_w at kTmemO + 64 w
constexpr float kRescaleThreshold = 8.0f;
constexpr int64_t kDefaultTimeoutNs = 2000000000LL;

struct Smem {
    static constexpr int q0 = 0;
    static constexpr int q1 = q0 + kTileBytes;
    static constexpr int rel = q1 + kTileBytes;
    static constexpr int k = rel + kRelRows * 128;            // 1024-aligned
    static constexpr int v = k + kStages * kTileBytes;
    static constexpr int qr = v + kStages * kTileBytes;
    static constexpr int bars = qr + kRowsPerCta * kQrStride * 4;
    // barrier indices
    static constexpr int kQ = 0;
    static constexpr int kKFull = 1;
    static constexpr int kVFull = kKFull + kStages;
    static constexpr int kKEmpty = kVFull + kStages;    // S MMAs of every query tile done with a K stage
    static constexpr int kVEmpty = kKEmpty + kStages;   // P V MMAs of every query tile done with a V stage
    static constexpr int kSFull = kVEmpty + kStages;    // S(j) (or QR) in TMEM          [per query tile]
    static constexpr int kSFree = kSFull + 2;           // all 4 warps read S(j) out     [per query tile]
    static constexpr int kPFull = kSFree + 2;           // all 4 warps stored P(j)       [per query tile]
    static constexpr int kPvDone = kPFull + 2;          // P(j) V(j) complete            [per query tile]
    static constexpr int kDrain = kPvDone + 2;          // per query tile: its MMA warp's drain
    static constexpr int kNever = kDrain + 2;
    static constexpr int kNumBars = kNever + 1;
    // misc block: +0 TMEM base, +4 abort flag, +8 status word pointer, +16 wait timeout (ns)
    static constexpr int misc = bars + kNumBars * 8;
    static constexpr int total = misc + 32;
    static constexpr int alloc = total + 1024;  // slack for 1024-byte alignment
};
static_assert(Smem::k % 1024 == 0 && Smem::v % 1024 == 0 && Smem::rel % 1024 == 0, "swizzle atoms");
static_assert(Smem::alloc <= 232448, "shared memory budget");

struct AttnParams {
    void* out;
    int64_t out_stride;       // elements
    const int32_t* kv_len;    // [batch] or null
    int32_t* status;          // or null
    int64_t timeout_ns;
    int32_t heads;
    int32_t seq_len;
    int32_t q_x0, k_x0, v_x0; // column (elements) of head 0's q / k / v in their maps
    float scale_log2;         // softmax scale * log2(e)
    int32_t debug_flags;
};

template <typename T>
struct DTypeTraits;
template <>
struct DTypeTraits<__half> {
    static constexpr int kFormat = 0;
    __device__ static __forceinline__ uint32_t pack(float lo, float hi) {
        __half2 v = __floats2half2_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&v);
    }
};
template <>
struct DTypeTraits<__nv_bfloat16> {
    static constexpr int kFormat = 1;
    __device__ static __forceinline__ uint32_t pack(float lo, float hi) {
        __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&v);
    }
};

// Where the bounded waits find the CTA's abort flag, status word pointer and
// timeout: the shared-memory misc block (one 32-bit address in registers; the
// rest is only read on the slow path).
struct WaitCtl {
    uint32_t misc;
};

// Wait for completion of phase `parity` of the mbarrier at shared address
// `bar`, for at most the CTA's timeout. Returns false (after recording
// `err_bit` and raising the abort flag) on expiry, or at once when another role
// has already aborted.
__device__ __forceinline__ bool wait_bounded(uint32_t bar, uint32_t parity, WaitCtl ctl, int err_bit,
                                             bool honour_abort = true) {
    if (mbar_try_wait(bar, parity)) return true;
    const int64_t timeout_ns = static_cast<int64_t>(ld_shared_u64(ctl.misc + 16));
    const uint64_t t0 = globaltimer_ns();
    // iteration cap: ends the wait even if the global timer were not advancing
    // (each outer round is 16 probes, well over 16 ns)
    const int64_t max_rounds = timeout_ns / 16 + 1024;
    for (int64_t round = 0;; ++round) {
#pragma unroll 1
        for (int i = 0; i < 16; ++i)
            if (mbar_try_wait(bar, parity)) return true;
        if (honour_abort && ld_shared_volatile_u32(ctl.misc + 4) != 0) return false;
        if (static_cast<int64_t>(globaltimer_ns() - t0) > timeout_ns || round > max_rounds) {
            st_shared_volatile_u32(ctl.misc + 4, 1);
            int* status = reinterpret_cast<int*>(ld_shared_u64(ctl.misc + 8));
            if (status) atomicOr(status, err_bit);
            return false;
        }
    }
}

// All 32 lanes wait; the warp proceeds only if every lane saw the phase. Both
// the first probe and the bounded loop end in a full-warp vote: lanes may reach
// this point unconverged (after a lane-0-only arrive), and a lane that left
// early would then sit in the caller's next .sync.aligned tcgen05 instruction
// while the others wait for it in the vote.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, WaitCtl ctl, int err_bit) {
    if (__all_sync(0xffffffffu, mbar_try_wait(bar, parity))) return true;
    const bool ok = wait_bounded(bar, parity, ctl, err_bit);
    return __all_sync(0xffffffffu, ok);
}

// Arrive once per warp on `bar` (initialised with count 4 for a warpgroup):
// every lane's prior tcgen05 traffic is ordered before the arrival.
__device__ __forceinline__ void warp_arrive(uint32_t bar, int lane) {
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(bar);
}

// Tensor-core work of one query tile (one elected lane of its MMA warp issues
// every MMA and every commit that tracks them).
template <typename T, bool kRelBias>
struct TileMma {
    static constexpr int fmt = DTypeTraits<T>::kFormat;
    static constexpr uint32_t kIdescQK = idesc_f16(kBlockM, kBlockN, fmt, 0, 0);
    static constexpr uint32_t kIdescQR = idesc_f16(kBlockM, kRelRows, fmt, 0, 0);
    static constexpr uint32_t kIdescPV = idesc_f16(kBlockM, kHeadDim, fmt, 0, 1);

    uint8_t* smem;
    uint32_t bars;  // shared address of the barrier array
    uint32_t tmem;
    int w;  // query tile

    __device__ __forceinline__ uint32_t bar(int idx) const { return bars + 8u * idx; }

    __device__ __forceinline__ uint64_t q_desc() const {
        return sw128_desc(smem_u32(smem + (w ? Smem::q1 : Smem::q0)));
    }

    __device__ __forceinline__ void qr() const {  // S_w columns <- Q_w rel^T
        if (elect_one()) {
            const uint64_t dq = q_desc();
            const uint64_t dr = sw128_desc(smem_u32(smem + Smem::rel));
#pragma unroll
            for (int k = 0; k < kHeadDim / 16; ++k)
                mma_ss(tmem + kTmemS + w * kBlockN, dq + 2 * k, dr + 2 * k, kIdescQR, k > 0);
            mma_commit(bar(Smem::kSFull + w));
        }
        __syncwarp();
    }

    __device__ __forceinline__ void s(int jn) const {  // S_w columns <- Q_w K(jn)^T
        if (elect_one()) {
            const int st = jn % kStages;
            const uint64_t dq = q_desc();
            const uint64_t dk = sw128_desc(smem_u32(smem + Smem::k + st * kTileBytes));
#pragma unroll
            for (int k = 0; k < kHeadDim / 16; ++k)
                mma_ss(tmem + kTmemS + w * kBlockN, dq + 2 * k, dk + 2 * k, kIdescQK, k > 0);
            mma_commit(bar(Smem::kSFull + w));
            mma_commit(bar(Smem::kKEmpty + st));
        }
        __syncwarp();
    }

    __device__ __forceinline__ void pv(int jp) const {  // O_w += P_w V(jp)
        if (elect_one()) {
            const int st = jp % kStages;
            const uint64_t dv = sw128_desc(smem_u32(smem + Smem::v + st * kTileBytes));
#pragma unroll
            for (int k = 0; k < kBlockN / 16; ++k)
                mma_ts(tmem + kTmemO + w * kHeadDim, tmem + kTmemP + w * (kBlockN / 2) + 8 * k, dv + 128 * k,
                       kIdescPV, (jp > 0 || k > 0) ? 1u : 0u);
            mma_commit(bar(Smem::kPvDone + w));
            mma_commit(bar(Smem::kVEmpty + st));
        }
        __syncwarp();
    }

    // every MMA this lane issued completes before TMEM can be released
    __device__ __forceinline__ void drain(WaitCtl ctl) const {
        if (elect_one()) mma_commit(bar(Smem::kDrain + w));
        __syncwarp();
        wait_bounded(bar(Smem::kDrain + w), 0, ctl, FDS_STATUS_TIMEOUT_DRAIN, false);
        __syncwarp();
    }
};

// The MMA warp of query tile w: QR (encoder), then per KV tile S(j+1) once the
// softmax warps have read S(j) out of TMEM and O += P(j) V(j) once they have
// stored P(j).
template <typename T, bool kRelBias>
__device__ __forceinline__ void mma_role(uint8_t* smem, uint32_t bars, uint32_t tmem, WaitCtl ctl, int w,
                                         int n_tiles, bool has_q1) {
    if (n_tiles == 0 || (w == 1 && !has_q1)) return;
    const TileMma<T, kRelBias> mma{smem, bars, tmem, w};
    constexpr int err = FDS_STATUS_TIMEOUT_MMA;
    const uint32_t s_free = mma.bar(Smem::kSFree + w);
    const uint32_t p_full = mma.bar(Smem::kPFull + w);
    uint32_t free_parity = 0;
    bool issued = false;
    bool ok = warp_wait(mma.bar(Smem::kQ), 0, ctl, err);
    if (ok && kRelBias) {
        tc_fence_after();
        mma.qr();
        issued = true;
        ok = warp_wait(s_free, free_parity, ctl, err);  // QR copied out of the S columns
        free_parity ^= 1;
    }
    if (ok) ok = warp_wait(mma.bar(Smem::kKFull + 0), 0, ctl, err);
    if (ok) {
        tc_fence_after();
        mma.s(0);
        issued = true;
    }
    for (int j = 0; ok && j < n_tiles; ++j) {
        if (j + 1 < n_tiles) {
            ok = warp_wait(s_free, free_parity, ctl, err);
            free_parity ^= 1;
            if (ok) ok = warp_wait(mma.bar(Smem::kKFull + (j + 1) % kStages), ((j + 1) / kStages) & 1, ctl, err);
            if (!ok) break;
            tc_fence_after();
            mma.s(j + 1);
        }
        ok = warp_wait(p_full, j & 1, ctl, err);
        if (ok) ok = warp_wait(mma.bar(Smem::kVFull + j % kStages), (j / kStages) & 1, ctl, err);
        if (!ok) break;
        tc_fence_after();
        mma.pv(j);
    }
    if (issued) mma.drain(ctl);
}

// O *= alpha for this thread's row (32 lanes of a warp, 64 columns). Rare (the
// running max moves by more than the lazy threshold), so it is kept out of line:
// its registers then never compete with the exponentials of the hot loop.
__device__ __noinline__ void rescale_o_row(uint32_t tO, float alpha) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
        uint32_t o[32];
        tmem_ld32(tO + 32 * half, o);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 32; ++c) o[c] = __float_as_uint(__uint_as_float(o[c]) * alpha);
        tmem_st32(tO + 32 * half, o);
    }
}

// Online softmax of one query row (this thread) over the KV tiles: per tile,
// read S out of TMEM, bias, max, exponentiate into P (TMEM), rescale O when the
// running max moves. One instance per softmax thread; step() handles tile j.
template <typename T, bool kRelBias>
struct RowSoftmax {
    static constexpr int err = FDS_STATUS_TIMEOUT_SOFTMAX;
    uint32_t tS, tP, tO;
    float sl;
    uint32_t qrow;  // shared address of this row's Q.rel^T in log2 units (encoder)
    uint32_t s_full, s_free, p_full, pv_done;  // barrier shared addresses
    WaitCtl ctl;
    int i, kv_end, lane;
    float m_run, l_run;
    uint32_t s_parity;

    // kBand: per-score relative bias gathered from qrow (any tile; needed for
    // the near-diagonal ones); otherwise the per-row constant cb (a tile whose
    // every pair saturates the clamp, or no bias). kMask: keys >= kv_end.
    template <bool kBand, bool kMask>
    __device__ __forceinline__ bool step(int j, float cb) {
        bool ok = warp_wait(s_full, s_parity, ctl, err);
        s_parity ^= 1;
        if (!ok) return false;
        tc_fence_after();

        uint32_t sr[128];
        tmem_ld64(tS + 0, *reinterpret_cast<uint32_t(*)[64]>(&sr[0]));
        tmem_ld64(tS + 64, *reinterpret_cast<uint32_t(*)[64]>(&sr[64]));
        tmem_wait_ld();
        warp_arrive(s_free, lane);  // the MMA warp may now compute S(j+1) into these columns
        float s[128];
#pragma unroll
        for (int c = 0; c < 128; ++c) s[c] = __uint_as_float(sr[c]);

        const int n0 = j * kBlockN;
        // score in log2 units = s * mult + cb
        float mult = sl;
        if constexpr (kBand) {
            const int d0 = n0 - i + kClampLeft;
#pragma unroll
            for (int c = 0; c < 128; ++c) {
                const int idx = min(max(d0 + c, 0), kClampLeft + kClampRight);
                s[c] = fmaf(s[c], sl, ld_shared_f32(qrow + 4u * idx));
            }
            mult = 1.f;
            cb = 0.f;
        }
        if constexpr (kMask) {
            const int lim = kv_end - n0;
#pragma unroll
            for (int c = 0; c < 128; ++c)
                if (c >= lim) s[c] = -INFINITY;
        }

        float mx[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) mx[u] = fmax3(s[u], s[8 + u], s[16 + u]);
#pragma unroll
        for (int c = 24; c < 120; c += 16) {
#pragma unroll
            for (int u = 0; u < 8; ++u) mx[u] = fmax3(mx[u], s[c + u], s[c + 8 + u]);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) mx[u] = fmaxf(mx[u], s[120 + u]);
        const float mxa = fmax3(fmax3(mx[0], mx[1], mx[2]), fmax3(mx[3], mx[4], mx[5]), fmaxf(mx[6], mx[7]));
        const float tile_max = fmaf(mxa, mult, cb);

        const bool rescale = tile_max > m_run + kRescaleThreshold;
        float alpha = 1.f;
        if (rescale) {
            alpha = ex2_approx(m_run - tile_max);  // 0 on the first tile
            m_run = tile_max;
        }
        const float add = cb - m_run;
        const float ky = mult * (1.0f / kPolySpan), kb = (add - kPolyLo) * (1.0f / kPolySpan);

        // exponentials into packed 16-bit pairs, held in registers; 3 of every
        // 10 pairs go through the FMA-pipe polynomial so that the MUFU and FMA
        // pipes carry similar loads
        uint32_t pk[64];
        float2 ls[4];
#pragma unroll
        for (int a = 0; a < 4; ++a) ls[a] = make_float2(0.f, 0.f);
        const float2 mult2 = make_float2(mult, mult), add2 = make_float2(add, add);
#pragma unroll
        for (int c = 0; c < 64; ++c) {
            float2 pp;
            if (c % 10 == 1 || c % 10 == 4 || c % 10 == 7) {
                pp = exp2_poly2(s[2 * c], s[2 * c + 1], ky, kb);
            } else {
                const float2 x = ffma2(make_float2(s[2 * c], s[2 * c + 1]), mult2, add2);
                pp.x = ex2_approx(x.x);
                pp.y = ex2_approx(x.y);
            }
            ls[c & 3] = fadd2(ls[c & 3], pp);
            pk[c] = DTypeTraits<T>::pack(pp.x, pp.y);
        }
        ls[0] = fadd2(fadd2(ls[0], ls[1]), fadd2(ls[2], ls[3]));
        l_run = l_run * alpha + (ls[0].x + ls[0].y);

        if (j > 0) {
            // P(j-1) V(j-1) must be complete before its P columns are rewritten
            // and before O is rescaled (its latency hides under the work above).
            ok = warp_wait(pv_done, (j - 1) & 1, ctl, err);
            if (!ok) return false;
            tc_fence_after();
        }
        tmem_st32(tP + 0, *reinterpret_cast<uint32_t(*)[32]>(&pk[0]));
        tmem_st32(tP + 32, *reinterpret_cast<uint32_t(*)[32]>(&pk[32]));
        if (j > 0 && __any_sync(0xffffffffu, rescale)) rescale_o_row(tO, alpha);
        tmem_wait_st();
        warp_arrive(p_full, lane);
        return true;
    }
};

template <typename T, bool kRelBias>
__device__ __forceinline__ void softmax_role(uint32_t sbase, uint32_t tmem, const AttnParams& p, WaitCtl ctl,
                                             int warp, int lane, int b, int h, int q_base, int kv_end, int n_tiles,
                                             bool has_q1) {
    const int wg = (warp - kSoftmaxWarp0) >> 2;  // query tile of this warpgroup
    const int wq = warp & 3;                     // warp within the warpgroup (= TMEM lane quarter)
    const int row = (wq << 5) + lane;            // row in tile == TMEM lane
    const int i = q_base + wg * kBlockM + row;   // query index in the window
    const int L = p.seq_len;
    if (wg == 1 && !has_q1) return;

    T* out_row = reinterpret_cast<T*>(p.out) + (static_cast<int64_t>(b) * L + i) * p.out_stride + h * kHeadDim;
    if (n_tiles == 0) {  // no valid key: the context row is defined as zero
        if (i < L) {
            const uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll
            for (int c = 0; c < 8; ++c) reinterpret_cast<uint4*>(out_row)[c] = z;
        }
        return;
    }

    constexpr int err = FDS_STATUS_TIMEOUT_SOFTMAX;
    const uint32_t lane_addr = static_cast<uint32_t>(wq * 32) << 16;
    RowSoftmax<T, kRelBias> rs;
    rs.tS = tmem + lane_addr + kTmemS + wg * kBlockN;
    rs.tP = tmem + lane_addr + kTmemP + wg * (kBlockN / 2);
    rs.tO = tmem + lane_addr + kTmemO + wg * kHeadDim;
    rs.sl = p.scale_log2;
    const uint32_t qrow = sbase + Smem::qr + 4u * ((wg * kBlockM + row) * kQrStride);
    rs.qrow = qrow;
    const uint32_t bars = sbase + Smem::bars;
    rs.s_full = bars + 8u * (Smem::kSFull + wg);
    rs.s_free = bars + 8u * (Smem::kSFree + wg);
    rs.p_full = bars + 8u * (Smem::kPFull + wg);
    rs.pv_done = bars + 8u * (Smem::kPvDone + wg);
    rs.ctl = ctl;
    rs.i = i;
    rs.kv_end = kv_end;
    rs.lane = lane;
    rs.m_run = -INFINITY;
    rs.l_run = 0.f;
    rs.s_parity = 0;
    const float sl = p.scale_log2;

    bool ok = true;
    float qr_left = 0.f, qr_right = 0.f;
    if constexpr (kRelBias) {
        ok = warp_wait(rs.s_full, rs.s_parity, ctl, err);
        rs.s_parity ^= 1;
        if (ok) {
            tc_fence_after();
            uint32_t a[32], c2[32], d[16];
            tmem_ld32(rs.tS, a);
            tmem_ld32(rs.tS + 32, c2);
            tmem_ld16(rs.tS + 64, d);
            tmem_wait_ld();
            warp_arrive(rs.s_free, lane);  // the S columns may now receive S(0)
#pragma unroll
            for (int c = 0; c < 32; ++c) st_shared_f32(qrow + 4u * c, __uint_as_float(a[c]) * sl);
#pragma unroll
            for (int c = 0; c < 32; ++c) st_shared_f32(qrow + 4u * (32 + c), __uint_as_float(c2[c]) * sl);
#pragma unroll
            for (int c = 0; c < kNumPos - 64; ++c) st_shared_f32(qrow + 4u * (64 + c), __uint_as_float(d[c]) * sl);
            qr_left = __uint_as_float(a[0]) * sl;
            qr_right = __uint_as_float(d[kNumPos - 1 - 64]) * sl;
        }
    }

    // Tiles in key order: [0, jb0) every pair left-saturated (bias QR[i,0]),
    // [jb0, jb1) near-diagonal (per-score gather), [jb1, ...) every pair
    // right-saturated (bias QR[i,72]). With t0 the tile's first query row, a KV
    // tile starting at key n0 is near-diagonal iff t0 - 190 <= n0 <= t0 + 134.
    // Each class runs its own copy of the tile step, so the hot loops carry no
    // gather code; the last tile (key padding) takes the general step.
    const int n_last = n_tiles - 1;
    int j = 0;
    if constexpr (kRelBias) {
        const int t0 = q_base + wg * kBlockM;
        const int jb0 = t0 >= 190 ? (t0 - 190 + kBlockN - 1) / kBlockN : 0;
        const int jb1 = (t0 + 135 + kBlockN - 1) / kBlockN;
        for (; ok && j < min(jb0, n_last); ++j) ok = rs.template step<false, false>(j, qr_left);
        for (; ok && j < min(jb1, n_last); ++j) ok = rs.template step<true, false>(j, 0.f);
        for (; ok && j < n_last; ++j) ok = rs.template step<false, false>(j, qr_right);
        if (ok) ok = rs.template step<true, true>(n_last, 0.f);
    } else {
        for (; ok && j < n_last; ++j) ok = rs.template step<false, false>(j, 0.f);
        if (ok) ok = rs.template step<false, true>(n_last, 0.f);
    }

    if (ok) ok = warp_wait(rs.pv_done, (n_tiles - 1) & 1, ctl, err);
    if (ok) {
        tc_fence_after();
        uint32_t o[64];
        tmem_ld32(rs.tO, *reinterpret_cast<uint32_t(*)[32]>(&o[0]));
        tmem_ld32(rs.tO + 32, *reinterpret_cast<uint32_t(*)[32]>(&o[32]));
        tmem_wait_ld();
        if (i < L) {
            const float inv = 1.f / rs.l_run;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                uint4 v;
                v.x = DTypeTraits<T>::pack(__uint_as_float(o[8 * c + 0]) * inv, __uint_as_float(o[8 * c + 1]) * inv);
                v.y = DTypeTraits<T>::pack(__uint_as_float(o[8 * c + 2]) * inv, __uint_as_float(o[8 * c + 3]) * inv);
                v.z = DTypeTraits<T>::pack(__uint_as_float(o[8 * c + 4]) * inv, __uint_as_float(o[8 * c + 5]) * inv);
                v.w = DTypeTraits<T>::pack(__uint_as_float(o[8 * c + 6]) * inv, __uint_as_float(o[8 * c + 7]) * inv);
                reinterpret_cast<uint4*>(out_row)[c] = v;
            }
        }
    }
}

template <bool kRelBias>
__device__ __forceinline__ void load_role(uint8_t* smem, uint64_t* bars, const CUtensorMap* map_q,
                                          const CUtensorMap* map_k, const CUtensorMap* map_v,
                                          const CUtensorMap* map_r, const AttnParams& p, WaitCtl ctl,
                                          int b, int h, int q_base, int n_tiles, bool has_q1) {
    if (n_tiles == 0) return;
    const auto bar = [&](int idx) { return smem_u32(&bars[idx]); };
    if (elect_one()) {
        const uint32_t q_bytes = (has_q1 ? 2 : 1) * kTileBytes + (kRelBias ? kRelRows * 128 : 0);
        mbar_arrive_expect_tx(&bars[Smem::kQ], q_bytes);
        tma_load_3d(smem + Smem::q0, map_q, &bars[Smem::kQ], p.q_x0 + h * kHeadDim, q_base, b);
        if (has_q1)
            tma_load_3d(smem + Smem::q1, map_q, &bars[Smem::kQ], p.q_x0 + h * kHeadDim, q_base + kBlockM, b);
        if constexpr (kRelBias) tma_load_2d(smem + Smem::rel, map_r, &bars[Smem::kQ], 0, 0);
    }
    __syncwarp();

    int issued_tiles = 0;
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
        const int st = j % kStages;
        const uint32_t par = ((j / kStages) - 1) & 1;
        if (j >= kStages) {
            ok = warp_wait(bar(Smem::kKEmpty + st), par, ctl, FDS_STATUS_TIMEOUT_LOAD);
            if (!ok) break;
        }
        if (elect_one()) {
            mbar_arrive_expect_tx(&bars[Smem::kKFull + st], kTileBytes);
            tma_load_3d(smem + Smem::k + st * kTileBytes, map_k, &bars[Smem::kKFull + st], p.k_x0 + h * kHeadDim,
                        j * kBlockN, b);
        }
        __syncwarp();
        if (j >= kStages) {
            ok = warp_wait(bar(Smem::kVEmpty + st), par, ctl, FDS_STATUS_TIMEOUT_LOAD);
            if (!ok) {
                // K(j) was issued but V(j) was not: drain K(j) here
                wait_bounded(bar(Smem::kKFull + st), (j / kStages) & 1, ctl, FDS_STATUS_TIMEOUT_DRAIN, false);
                break;
            }
        }
        if (elect_one()) {
            mbar_arrive_expect_tx(&bars[Smem::kVFull + st], kTileBytes);
            tma_load_3d(smem + Smem::v + st * kTileBytes, map_v, &bars[Smem::kVFull + st], p.v_x0 + h * kHeadDim,
                        j * kBlockN, b);
        }
        __syncwarp();
        ++issued_tiles;
    }
    if (!ok) {
        // aborted: let every copy already issued land before the CTA exits
        wait_bounded(bar(Smem::kQ), 0, ctl, FDS_STATUS_TIMEOUT_DRAIN, false);
        for (int s = 0; s < kStages; ++s) {
            // loads issued into stage s: tiles s, s + kStages, ... below issued_tiles
            const int n = issued_tiles > s ? (issued_tiles - s + kStages - 1) / kStages : 0;
            if (n == 0) continue;
            wait_bounded(bar(Smem::kKFull + s), (n - 1) & 1, ctl, FDS_STATUS_TIMEOUT_DRAIN, false);
            wait_bounded(bar(Smem::kVFull + s), (n - 1) & 1, ctl, FDS_STATUS_TIMEOUT_DRAIN, false);
        }
        __syncwarp();
    }
}

template <typename T, bool kRelBias>
__global__ void __launch_bounds__(kThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                    const __grid_constant__ CUtensorMap map_v, const __grid_constant__ CUtensorMap map_r,
                    const AttnParams p) {
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte aligned base (the swizzle atoms), as an offset into the shared
    // array so that every access derived from it stays a shared-window access
    const uint32_t raw_addr = smem_u32(smem_raw);
    const uint32_t sbase = (raw_addr + 1023u) & ~1023u;
    uint8_t* smem = smem_raw + (sbase - raw_addr);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Smem::bars);
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + Smem::misc);
    const WaitCtl ctl{sbase + Smem::misc};

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int b = blockIdx.y / p.heads;
    const int h = blockIdx.y % p.heads;
    const int q_base = blockIdx.x * kRowsPerCta;
    const int L = p.seq_len;
    const bool has_q1 = q_base + kBlockM < L;
    int kv_end = L;
    if (p.kv_len != nullptr) kv_end = min(max(p.kv_len[b], 0), L);
    const int n_tiles = (kv_end + kBlockN - 1) / kBlockN;

    if (threadIdx.x == 0) {
        const uint32_t nq = has_q1 ? 2 : 1;  // query tiles releasing each K / V stage
        mbar_init(&bars[Smem::kQ], 1);
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&bars[Smem::kKFull + s], 1);
            mbar_init(&bars[Smem::kVFull + s], 1);
            mbar_init(&bars[Smem::kKEmpty + s], nq);
            mbar_init(&bars[Smem::kVEmpty + s], nq);
        }
        for (int w = 0; w < 2; ++w) {
            mbar_init(&bars[Smem::kSFull + w], 1);
            mbar_init(&bars[Smem::kSFree + w], 4);   // one arrival per softmax warp
            mbar_init(&bars[Smem::kPFull + w], 4);
            mbar_init(&bars[Smem::kPvDone + w], 1);
        }
        for (int d = 0; d < 2; ++d) mbar_init(&bars[Smem::kDrain + d], 1);
        mbar_init(&bars[Smem::kNever], 1);
        st_shared_volatile_u32(ctl.misc + 4, 0);  // abort flag
        st_shared_u64(ctl.misc + 8, reinterpret_cast<uint64_t>(p.status));
        st_shared_u64(ctl.misc + 16, static_cast<uint64_t>(p.timeout_ns > 0 ? p.timeout_ns : kDefaultTimeoutNs));
        fence_barrier_init();
        fence_proxy_async_smem();
    }
    if (warp == kLoadWarp && lane == 0) {
        prefetch_tensormap(&map_q);
        prefetch_tensormap(&map_k);
        prefetch_tensormap(&map_v);
        if (kRelBias) prefetch_tensormap(&map_r);
    }
    if (warp == kTmemWarp) {
        tmem_alloc(tmem_holder, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_holder;

    // The two register classes never share code again: each branch ends with
    // its own arrival on the CTA-wide barrier (every thread of the CTA arrives
    // exactly once, so all roles have finished with TMEM when it opens).
    if (warp >= kSoftmaxWarp0) {
        setmaxnreg_inc<kSoftmaxRegs>();
        softmax_role<T, kRelBias>(sbase, tmem, p, ctl, warp, lane, b, h, q_base, kv_end, n_tiles, has_q1);
        __syncwarp();
        tc_fence_before();
        named_barrier_sync(1, kThreads);
    } else {
        setmaxnreg_dec<kControlRegs>();
        if (warp == kMmaWarp0 || warp == kMmaWarp0 + 2) {
            // test hook: a wait on a barrier that nothing arrives on, to exercise
            // the bounded-wait error path without a real hang
            bool go = true;
            if (p.debug_flags & FDS_DEBUG_FORCE_TIMEOUT)
                go = warp_wait(sbase + Smem::bars + 8u * Smem::kNever, 0, ctl, FDS_STATUS_TIMEOUT_MMA);
            if (go)
                mma_role<T, kRelBias>(smem, sbase + Smem::bars, tmem, ctl, (warp - kMmaWarp0) >> 1, n_tiles, has_q1);
        } else if (warp == kLoadWarp) {
            load_role<kRelBias>(smem, bars, &map_q, &map_k, &map_v, &map_r, p, ctl, b, h, q_base, n_tiles, has_q1);
        }
        __syncwarp();
        tc_fence_before();
        named_barrier_sync(1, kThreads);
        if (warp == kTmemWarp) {
            tc_fence_after();
            tmem_dealloc(tmem, kTmemCols);
        }
    }
}

}  // namespace fds
