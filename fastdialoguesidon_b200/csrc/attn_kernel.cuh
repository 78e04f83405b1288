// attn_kernel.cuh - sm_100a attention forward with an optional relative_key bias.
//
// A work unit is 256 query rows of one (window, head): two 128-row query tiles
// (Q0, Q1) that share every K/V tile. A CTA walks a short list of work items;
// an item is a unit's KV tiles [t_begin, t_end). Warp roles (384 threads,
// 3 warpgroups):
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
// Schedules (chosen by the host):
//  * one unit per CTA: the grid is the unit list, each CTA holds one item;
//  * split last wave: when whole units leave the last wave partly idle, the
//    first (waves - 1) x SMs units still run one per CTA, and the remaining
//    units are cut, by weight, into one contiguous piece of (unit, KV tile)
//    steps per SM; those piece CTAs come last in the grid, so the hardware
//    hands them out as the whole units finish. A piece may end in the middle
//    of one unit and start another, so a cut unit has 2..kMaxParts parts on
//    different CTAs. Each part leaves its unnormalised O, running max and row
//    sum in the workspace and counts itself in (per 32-row warp, atomically);
//    the part that completes the count merges them all and writes the output.
//    No CTA ever waits for another, so no co-residency is needed. The
//    merging part resets the count, leaving the workspace ready for the next
//    call (a call that reported a timeout may leave counts behind: zero the
//    workspace again after one).
// All barrier phases run on across items (a piece holds up to three): the next
// item's Q / K / V loads, Q.rel^T and first S overlap the current item's last
// tiles and epilogue.
//
// TMEM (512 columns): S0 [0,128) S1 [128,256) P0 [256,320) P1 [320,384)
//                     O0 [384,448) O1 [448,512).
// P (the exponentiated scores, two 16-bit values per column) has its own
// columns, so S(j+1) = Q K(j+1)^T runs while the softmax warps exponentiate
// S(j), and P(j) V(j) runs under the next tile's softmax.
//
// Relative bias (encoder): bias(i, j) = q_i . rel[clamp(j - i, -64, 8) + 64].
// Per query tile and item the MMA computes QR = Q . rel^T (N = 80, rows 73..79
// zero) into the S columns; the softmax threads copy their row of QR (scaled
// to log2 units) into shared memory as a padded table, T[m] = QR[clamp(m - 4 -
// (row & 3), 0, 72)] for m in [0, 84), so that the bias of four adjacent keys
// is one aligned 16-byte load at a clamped index that is a multiple of 4. A KV tile whose every (i, j) pair
// saturates the clamp adds a per-row constant (QR[i,0] on the left, QR[i,72]
// on the right), which folds into the exponent's FFMA offset at no per-score
// cost; only the (at most three) near-diagonal tiles gather the bias per
// score. This is the clamp-saturation property the reference exploits in
// triton/src/fds_triton/kernels.py:364-398 (its _flexrel_kernel), realised
// here as a per-tile offset instead of running-max shifts.
//
// Online softmax: log2 units, lazy rescaling (the running max used for the
// exponent only moves when a tile's max exceeds it by more than 8, i.e. P is
// bounded by 256), fp32 row sums, P rounded to the operand type.
//
// Registers: launched at 168 per thread; the control warpgroup gives some back
// and the two softmax warpgroups take the rest (RegSplit: 224 / 56 for the
// encoder, 208 / 88 for the DiT; 256*224 + 128*56 = 256*208 + 128*88 =
// 384*168), enough to hold a row of S (128 fp32) and of P (64 packed pairs) at
// once while the MMA warps keep their item loop in registers (below 56 they
// spill on the hand-off path; the DiT's split P V hand-off needs more than 72).
// The encoder's split is the measured best of 232 / 40, 224 / 56 and 216 / 72;
// the DiT's is the largest softmax share at which neither role spills.
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
constexpr int kQTiles = 2;         // query tiles per unit
constexpr int kRowsPerCta = kBlockM * kQTiles;
constexpr int kBlockN = 128;       // keys per KV tile
constexpr int kHeadDim = 64;
constexpr int kStages = 3;         // K/V shared-memory ring depth
constexpr int kTileBytes = kBlockM * kHeadDim * 2;
constexpr int kNumPos = 73;        // relative-key table rows
constexpr int kClampLeft = 64;
constexpr int kClampRight = 8;
constexpr int kRelRows = 80;       // table rows padded to a multiple of 16 (MMA N)
constexpr int kQrStride = 84;      // floats per row of the padded shared QR table (see the header)
constexpr int kMmaWarp0 = 0;       // MMA issuer of query tile 0 (tile 1: kMmaWarp0 + 2)
constexpr int kLoadWarp = 1;
constexpr int kTmemWarp = 3;
constexpr int kSoftmaxWarp0 = 4;   // first softmax warp (query tile 0: warps 4-7, tile 1: 8-11)
constexpr int kThreads = 384;
constexpr int kLaunchRegs = 168;   // per thread at launch (checked at build time)
template <bool kRelBias>
struct RegSplit {
    static constexpr int kSoftmax = kRelBias ? 224 : 208;
    static constexpr int kControl = kRelBias ? 56 : 88;
    static_assert(256 * kSoftmax + 128 * kControl <= kThreads * kLaunchRegs, "register split exceeds the launch pool");
    static_assert(kSoftmax % 8 == 0 && kControl % 8 == 0 && kControl >= 24, "setmaxnreg operand");
};
// P(j) handed to the MMA warp in two key halves (DiT): P(j) V(j) over keys
// 0..63 starts while the softmax warps still exponentiate keys 64..127. The
// encoder keeps one hand-off per tile: it measured slower with the split, on
// its bias-free tiles too (its near-diagonal gather leaves no registers for a
// mid-tile one).
template <bool kRelBias>
struct PvSplit {
    static constexpr bool kOn = !kRelBias;
};
constexpr int kTmemCols = 512;
constexpr int kTmemS = 0;          // S_w at kTmemS + 128 w
constexpr int kTmemP = 256;        // P_w at kTmemP + 64 w
constexpr int kTmemO = 384;        // O_w at kTmemO + 64 w
constexpr float kRescaleThreshold = 8.0f;
constexpr int64_t kDefaultTimeoutNs = 2000000000LL;

// Split last wave: items per piece at most, parts per cut unit at most, and
// the workspace slot of a part: per row [O (64 fp32, unnormalised) | running
// max | row sum | 2 pad], stored as 17 column blocks of 4 floats x 256 rows,
// so that the 32 rows of a warp read or write 512 contiguous bytes per access.
constexpr int kMaxItems = 3;
constexpr int kMaxParts = 4;
constexpr int kPartRowFloats = 68;
constexpr int kPartBlocks = kPartRowFloats / 4;
constexpr int kSoftmaxWarps = 8;   // one part count per softmax warp (32 rows) and cut unit

struct Smem {
    static constexpr int q0 = 0;
    static constexpr int q1 = q0 + kTileBytes;
    static constexpr int rel = q1 + kTileBytes;
    static constexpr int k = rel + kRelRows * 128;            // 1024-aligned
    static constexpr int v = k + kStages * kTileBytes;
    static constexpr int qr = v + kStages * kTileBytes;
    static constexpr int bars = qr + kRowsPerCta * kQrStride * 4;
    // barrier indices
    static constexpr int kQ = 0;                        // Q (and, first, rel) landed       [per item]
    static constexpr int kQEmpty = 1;                   // both tiles' S MMAs done with Q   [per item]
    static constexpr int kKFull = 2;
    static constexpr int kVFull = kKFull + kStages;
    static constexpr int kKEmpty = kVFull + kStages;    // S MMAs of both query tiles done with a K stage
    static constexpr int kVEmpty = kKEmpty + kStages;   // P V MMAs of both query tiles done with a V stage
    static constexpr int kSFull = kVEmpty + kStages;    // S(j) (or QR) in TMEM          [per query tile]
    static constexpr int kSFree = kSFull + 2;           // all 4 warps read S(j) out     [per query tile]
    static constexpr int kPFull = kSFree + 2;           // all 4 warps stored P(j)       [per query tile]
    static constexpr int kPvDone = kPFull + 2;          // P(j) V(j) complete            [per query tile]
    static constexpr int kPHalf = kPvDone + 2;          // all 4 warps stored P(j)'s keys 0..63 (split P V) [per query tile]
    static constexpr int kDrain = kPHalf + 2;          // per query tile: its MMA warp's drain
    static constexpr int kNever = kDrain + 2;
    static constexpr int kNumBars = kNever + 1;
    // misc block: +0 TMEM base, +4 abort flag, +8 status word pointer,
    // +16 wait timeout (ns), +28 item count, +32 host status mirror pointer
    static constexpr int misc = bars + kNumBars * 8;
    static constexpr int items = (misc + 40 + 15) / 16 * 16;  // kMaxItems x 2 int4
    static constexpr int total = items + kMaxItems * 32;
    static constexpr int alloc = total + 1024;  // slack for 1024-byte alignment
};
static_assert(Smem::k % 1024 == 0 && Smem::v % 1024 == 0 && Smem::rel % 1024 == 0, "swizzle atoms");
static_assert(Smem::items % 16 == 0, "item records");
static_assert(Smem::alloc <= 232448, "shared memory budget");

struct AttnParams {
    void* out;
    int64_t out_stride;       // elements
    const int32_t* kv_len;    // [batch] or null (always null when the last wave is split)
    int32_t* status;          // or null
    int32_t* status_host;     // mapped pinned host mirror of the status bits, or null
    int64_t timeout_ns;
    int32_t heads;
    int32_t seq_len;
    int32_t q_x0, k_x0, v_x0; // column (elements) of head 0's q / k / v in their maps
    float scale_log2;         // softmax scale * log2(e)
    int32_t debug_flags;
    int32_t row_blocks;       // ceil(seq_len / 256)
    int32_t n_units;          // batch * heads * row_blocks
    int32_t whole_ctas;       // CTAs [0, whole_ctas) hold one whole unit each
    int32_t pieces;           // CTAs [whole_ctas, whole_ctas + pieces) hold the cut last wave (0: none)
    float* parts;             // pieces: [pieces][kMaxItems] slots of 256 rows x kPartRowFloats
    uint32_t* counts;         // pieces: [units - whole_ctas][kSoftmaxWarps] parts counted in
    // relative bias given as q.rel^T rows in global memory (the TensorRT
    // plugin's layout: [batch, seq_len, heads, 73], or [batch, heads, seq_len, 73]
    // with heads_in_z) instead of the in-kernel Q.rel^T product; or null
    const void* qr;
    // q / k / v / out laid out [batch, heads, seq_len, 64]: the map's third
    // coordinate is batch * heads + head and the head's column offset is 0
    int32_t heads_in_z;
};

// Tensor-map coordinates of head h of window b: {column of head 0 + x, row, z}.
__device__ __forceinline__ int head_x(const AttnParams& p, int h) { return p.heads_in_z ? 0 : h * 64; }
__device__ __forceinline__ int head_z(const AttnParams& p, int b, int h) { return p.heads_in_z ? b * p.heads + h : b; }

template <typename T>
struct DTypeTraits;
template <>
struct DTypeTraits<__half> {
    static constexpr int kFormat = 0;
    __device__ static __forceinline__ uint32_t pack(float lo, float hi) {
        __half2 v = __floats2half2_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&v);
    }
    __device__ static __forceinline__ float load_f32(const __half* x) { return __half2float(__ldg(x)); }
};
template <>
struct DTypeTraits<__nv_bfloat16> {
    static constexpr int kFormat = 1;
    __device__ static __forceinline__ uint32_t pack(float lo, float hi) {
        __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<uint32_t*>(&v);
    }
    __device__ static __forceinline__ float load_f32(const __nv_bfloat16* x) { return __bfloat162float(__ldg(x)); }
};

// ---------------------------------------------------------------- work items

enum ItemKind : int { kWhole = 0, kPart = 1 };

// One work item: query rows [q_base, q_base + 256) of (window b, head h), KV
// tiles [t_begin, t_end). Stored in shared memory as two int4:
// {b, h, q_base, has_q1 | kind << 1} and {t_begin, t_end, 0, 0}.
struct Item {
    int b, h, q_base, t_begin, t_end, kind;
    bool has_q1;
};

__device__ __forceinline__ void store_item(uint32_t sbase, int idx, const Item& it) {
    const uint32_t a = sbase + Smem::items + 32u * idx;
    st_shared_v4(a, make_int4(it.b, it.h, it.q_base, (it.has_q1 ? 1 : 0) | (it.kind << 1)));
    st_shared_v4(a + 16, make_int4(it.t_begin, it.t_end, 0, 0));
}

__device__ __forceinline__ Item load_item(uint32_t sbase, int idx) {
    const uint32_t a = sbase + Smem::items + 32u * idx;
    const int4 x = ld_shared_v4(a), y = ld_shared_v4(a + 16);
    Item it;
    it.b = x.x;
    it.h = x.y;
    it.q_base = x.z;
    it.has_q1 = (x.w & 1) != 0;
    it.kind = x.w >> 1;
    it.t_begin = y.x;
    it.t_end = y.y;
    return it;
}

// The KV tile range {t_begin, t_end} and has_q1 of item idx (what the MMA warps need).
__device__ __forceinline__ int2 item_tiles(uint32_t sbase, int idx) {
    const int4 y = ld_shared_v4(sbase + Smem::items + 32u * idx + 16);
    return make_int2(y.x, y.y);
}
__device__ __forceinline__ bool item_has_q1(uint32_t sbase, int idx) {
    return (ld_shared_v4(sbase + Smem::items + 32u * idx).w & 1) != 0;
}


__device__ __forceinline__ int kv_end_of(const AttnParams& p, int b) {
    return p.kv_len != nullptr ? min(max(p.kv_len[b], 0), p.seq_len) : p.seq_len;
}

// Unit u = (b * heads + h) * row_blocks + r (row block fastest).
__device__ __forceinline__ Item unit_item(const AttnParams& p, int u) {
    Item it;
    const int r = u % p.row_blocks;
    const int bh = u / p.row_blocks;
    it.h = bh % p.heads;
    it.b = bh / p.heads;
    it.q_base = r * kRowsPerCta;
    it.has_q1 = it.q_base + kBlockM < p.seq_len;
    it.t_begin = 0;
    it.t_end = 0;
    it.kind = kWhole;
    return it;
}

// Relative cost of one KV tile step of a unit with two / one query tiles (the
// last wave is cut by these weights; one-tile units run one softmax warpgroup
// and take about 3/5 of the time), and of starting a unit's item: its Q load,
// Q.rel^T and table fill, pipeline ramp and part epilogue, so that a piece
// that starts a second unit gets fewer tiles. An extra item cost a piece ~10 us
// on a B200 (7 tile steps of a two-tile unit); as a weight, 4 tile steps (20)
// cut the encoder layer at L = 6000 best (0.2070 ms unweighted; 10: 0.2062,
// 15: 0.2059, 20: 0.2042-0.2051, 25: 0.2048-0.2051, 35: 0.2053, 50: 0.2052).
// The start weight is capped at a sixth of a unit's tile weight, so that short
// units still split into pieces.
constexpr uint32_t kWeightTwoTiles = 5;
constexpr uint32_t kWeightOneTile = 3;
constexpr uint32_t kWeightUnitStart = 20;
__host__ __device__ constexpr uint32_t unit_start_weight(uint32_t n_tiles) {
    return n_tiles * kWeightTwoTiles / 6 < kWeightUnitStart ? n_tiles * kWeightTwoTiles / 6 : kWeightUnitStart;
}

// Geometry of the (unit, KV tile) sequence: per (window, head) R units, each a
// start of weight c0 = unit_start_weight(n) then n tiles, the last unit weighted w_last
// per tile (a one-tile unit when the last row block holds at most 128 rows),
// the others kWeightTwoTiles. 32-bit arithmetic: the host splits the last wave
// only when the total weight times the piece count stays below 2^31.
struct TileSeq {
    uint32_t n, R, w_last, c0;
    __device__ __forceinline__ explicit TileSeq(const AttnParams& p) {
        n = (p.seq_len + kBlockN - 1) / kBlockN;
        R = p.row_blocks;
        w_last = (R - 1) * kRowsPerCta + kBlockM < static_cast<uint32_t>(p.seq_len) ? kWeightTwoTiles : kWeightOneTile;
        c0 = unit_start_weight(n);
    }
    __device__ __forceinline__ uint32_t unit_full() const { return c0 + n * kWeightTwoTiles; }
    __device__ __forceinline__ uint32_t per_bh() const { return (R - 1) * unit_full() + c0 + n * w_last; }
    // weight before unit u
    __device__ __forceinline__ uint32_t unit_pos(uint32_t u) const {
        const uint32_t bh = u / R;
        return bh * per_bh() + (u - bh * R) * unit_full();
    }
    // global tile step (unit * n + tile) at weight position x (a position in a
    // unit's start maps to its first tile)
    __device__ __forceinline__ uint32_t tile_at(uint32_t x) const {
        const uint32_t full = (R - 1) * unit_full();
        const uint32_t bh = x / per_bh();
        const uint32_t rem = x - bh * per_bh();
        uint32_t r, q, w;
        if (rem < full) {
            r = rem / unit_full();
            q = rem - r * unit_full();
            w = kWeightTwoTiles;
        } else {
            r = R - 1;
            q = rem - full;
            w = w_last;
        }
        const uint32_t t = q < c0 ? 0 : (q - c0) / w;
        return (bh * R + r) * n + t;
    }
};

// Tile steps [first, last) of piece k (of `pieces`) of the cut last wave:
// units [whole_ctas, n_units), split at equal weight.
__device__ __forceinline__ uint2 piece_range(const AttnParams& p, const TileSeq& ts, uint32_t k) {
    const uint32_t x0 = ts.unit_pos(p.whole_ctas);
    const uint32_t wt = ts.unit_pos(p.n_units) - x0;
    const uint32_t P = p.pieces;
    const uint32_t first = ts.tile_at(x0 + k * wt / P);
    const uint32_t last = k + 1 == P ? static_cast<uint32_t>(p.n_units) * ts.n : ts.tile_at(x0 + (k + 1) * wt / P);
    return make_uint2(first, last);
}

// Fills this CTA's item list (thread 0, before the CTA-wide barrier); returns
// the item count (the host guarantees that a piece is non-empty and touches at
// most kMaxItems units).
__device__ __forceinline__ int build_items(const AttnParams& p, uint32_t sbase) {
    const uint32_t x = blockIdx.x;
    if (x < static_cast<uint32_t>(p.whole_ctas)) {
        Item it = unit_item(p, static_cast<int>(x));
        it.t_end = (kv_end_of(p, it.b) + kBlockN - 1) / kBlockN;
        store_item(sbase, 0, it);
        return 1;
    }
    const TileSeq ts(p);
    const uint2 r = piece_range(p, ts, x - p.whole_ctas);
    int count = 0;
    for (uint32_t u = r.x / ts.n; u * ts.n < r.y && count < kMaxItems; ++u) {
        Item it = unit_item(p, static_cast<int>(u));
        it.t_begin = static_cast<int>(r.x > u * ts.n ? r.x - u * ts.n : 0);
        it.t_end = static_cast<int>(r.y - u * ts.n < ts.n ? r.y - u * ts.n : ts.n);
        it.kind = (it.t_begin == 0 && it.t_end == static_cast<int>(ts.n)) ? kWhole : kPart;
        store_item(sbase, count++, it);
    }
    return count;
}

// ---------------------------------------------------------------- waits

// Where the bounded waits find the CTA's abort flag, status word pointer and
// timeout: the shared-memory misc block (one 32-bit address in registers; the
// rest is only read on the slow path).
struct WaitCtl {
    uint32_t misc;
};

__device__ __forceinline__ void raise_abort(WaitCtl ctl, int err_bit) {
    st_shared_volatile_u32(ctl.misc + 4, 1);
    int* status = reinterpret_cast<int*>(ld_shared_u64(ctl.misc + 8));
    if (status) atomicOr(status, err_bit);
    // host-visible mirror: a plain read-modify-write of mapped host memory
    // (only on this error path), which the host can poll without a sync
    volatile int* mirror = reinterpret_cast<volatile int*>(ld_shared_u64(ctl.misc + 32));
    if (mirror) {
        *mirror = *mirror | err_bit;
        __threadfence_system();
    }
}

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
            raise_abort(ctl, err_bit);
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

// ---------------------------------------------------------------- tensor cores

// Tensor-core work of one query tile (one elected lane of its MMA warp issues
// every MMA and every commit that tracks them).
template <typename T, bool kRelBias>
struct TileMma {
    static constexpr int fmt = DTypeTraits<T>::kFormat;
    static constexpr uint32_t kIdescQK = idesc_f16(kBlockM, kBlockN, fmt, 0, 0);
    static constexpr uint32_t kIdescQR = idesc_f16(kBlockM, kRelRows, fmt, 0, 0);
    static constexpr uint32_t kIdescPV = idesc_f16(kBlockM, kHeadDim, fmt, 0, 1);

    uint32_t sbase;  // shared address of the (1024-aligned) layout base
    uint32_t tmem;
    int w;  // query tile

    __device__ __forceinline__ uint32_t bar(int idx) const { return sbase + Smem::bars + 8u * idx; }

    __device__ __forceinline__ uint64_t q_desc() const { return sw128_desc(sbase + (w ? Smem::q1 : Smem::q0)); }

    __device__ __forceinline__ void qr() const {  // S_w columns <- Q_w rel^T
        if (elect_one()) {
            const uint64_t dq = q_desc();
            const uint64_t dr = sw128_desc(sbase + Smem::rel);
#pragma unroll
            for (int k = 0; k < kHeadDim / 16; ++k)
                mma_ss(tmem + kTmemS + w * kBlockN, dq + 2 * k, dr + 2 * k, kIdescQR, k > 0);
            mma_commit(bar(Smem::kSFull + w));
        }
        __syncwarp();
    }

    // S_w columns <- Q_w K(stage st)^T; `last` (the item's last S) also releases Q
    __device__ __forceinline__ void s(int st, bool last) const {
        if (elect_one()) {
            const uint64_t dq = q_desc();
            const uint64_t dk = sw128_desc(sbase + Smem::k + st * kTileBytes);
#pragma unroll
            for (int k = 0; k < kHeadDim / 16; ++k)
                mma_ss(tmem + kTmemS + w * kBlockN, dq + 2 * k, dk + 2 * k, kIdescQK, k > 0);
            mma_commit(bar(Smem::kSFull + w));
            mma_commit(bar(Smem::kKEmpty + st));
            if (last) mma_commit(bar(Smem::kQEmpty));
        }
        __syncwarp();
    }

    // O_w (+)= P_w V(stage st) over keys [16 k0, 16 k1); the group that ends at
    // key 128 completes the tile (P V done, V stage released)
    template <int k0, int k1>
    __device__ __forceinline__ void pv(int st, bool accumulate) const {
        if (elect_one()) {
            const uint64_t dv = sw128_desc(sbase + Smem::v + st * kTileBytes);
#pragma unroll
            for (int k = k0; k < k1; ++k)
                mma_ts(tmem + kTmemO + w * kHeadDim, tmem + kTmemP + w * (kBlockN / 2) + 8 * k, dv + 128 * k,
                       kIdescPV, (accumulate || k > 0) ? 1u : 0u);
            if (k1 == kBlockN / 16) {
                mma_commit(bar(Smem::kPvDone + w));
                mma_commit(bar(Smem::kVEmpty + st));
            }
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

// The MMA warp of query tile w. Per item: QR (encoder), then per KV tile S(j+1)
// once the softmax warps have read S(j) out of TMEM and O += P(j) V(j) once
// they have stored P(j). Every S-column write after the first waits for the
// softmax warps to have read the previous one (QR or S) out. An item without a
// second query tile still takes part in the count-2 barriers of tile 1 (Q and
// stage releases), after seeing each copy land so that it cannot run ahead.
template <typename T, bool kRelBias>
__device__ __forceinline__ void mma_role(uint32_t sbase, uint32_t tmem, WaitCtl ctl, int w, int n_items,
                                         bool qr_mma) {
    const TileMma<T, kRelBias> mma{sbase, tmem, w};
    constexpr int err = FDS_STATUS_TIMEOUT_MMA;
    uint32_t nw = 0;   // S-column writes (QR or S) so far; write k > 0 first waits for read k - 1
    uint32_t npv = 0;  // P V groups so far (phase of p_full)
    int qi = 0;        // items with KV tiles so far (phase of kQ)
    int g = 0;         // KV tiles so far (stage and phase of the K / V ring)
    bool ok = true;
    // wait until the softmax warps have read the previous S-column write out
    const auto s_free_wait = [&]() {
        if (nw > 0) ok = warp_wait(mma.bar(Smem::kSFree + w), (nw - 1) & 1, ctl, err);
        ++nw;
        return ok;
    };
    for (int idx = 0; ok && idx < n_items; ++idx) {
        const int2 tr = item_tiles(sbase, idx);
        const int nt = tr.y - tr.x;
        if (nt <= 0) continue;
        ok = warp_wait(mma.bar(Smem::kQ), qi & 1, ctl, err);
        if (!ok) break;
        ++qi;
        if (w == 1 && !item_has_q1(sbase, idx)) {
            if (elect_one()) mbar_arrive(mma.bar(Smem::kQEmpty));
            __syncwarp();
            for (int j = 0; ok && j < nt; ++j, ++g) {
                const int st = g % kStages;
                ok = warp_wait(mma.bar(Smem::kKFull + st), (g / kStages) & 1, ctl, err);
                if (!ok) break;
                if (elect_one()) mbar_arrive(mma.bar(Smem::kKEmpty + st));
                __syncwarp();
                ok = warp_wait(mma.bar(Smem::kVFull + st), (g / kStages) & 1, ctl, err);
                if (!ok) break;
                if (elect_one()) mbar_arrive(mma.bar(Smem::kVEmpty + st));
                __syncwarp();
            }
            continue;
        }
        tc_fence_after();
        if (kRelBias && qr_mma) {
            if (!s_free_wait()) break;  // the previous item's last S read out
            tc_fence_after();
            mma.qr();
        }
        if (!s_free_wait()) break;  // QR (or the previous item's last S) read out
        ok = warp_wait(mma.bar(Smem::kKFull + g % kStages), (g / kStages) & 1, ctl, err);
        if (!ok) break;
        tc_fence_after();
        mma.s(g % kStages, nt == 1);
        for (int j = 0; ok && j < nt; ++j, ++g) {
            if (j + 1 < nt) {
                const int gn = g + 1;
                if (!s_free_wait()) break;
                ok = warp_wait(mma.bar(Smem::kKFull + gn % kStages), (gn / kStages) & 1, ctl, err);
                if (!ok) break;
                tc_fence_after();
                mma.s(gn % kStages, j + 2 == nt);
            }
            constexpr int kHalfSteps = kBlockN / 32;
            if constexpr (PvSplit<kRelBias>::kOn) {
                ok = warp_wait(mma.bar(Smem::kPHalf + w), npv & 1, ctl, err);
                if (ok) ok = warp_wait(mma.bar(Smem::kVFull + g % kStages), (g / kStages) & 1, ctl, err);
                if (!ok) break;
                tc_fence_after();
                mma.template pv<0, kHalfSteps>(g % kStages, j > 0);
                ok = warp_wait(mma.bar(Smem::kPFull + w), npv & 1, ctl, err);
                ++npv;
                if (!ok) break;
                tc_fence_after();
                mma.template pv<kHalfSteps, 2 * kHalfSteps>(g % kStages, true);
            } else {
                ok = warp_wait(mma.bar(Smem::kPFull + w), npv & 1, ctl, err);
                ++npv;
                if (ok) ok = warp_wait(mma.bar(Smem::kVFull + g % kStages), (g / kStages) & 1, ctl, err);
                if (!ok) break;
                tc_fence_after();
                mma.template pv<0, 2 * kHalfSteps>(g % kStages, j > 0);
            }
        }
    }
    if (nw > 0) mma.drain(ctl);  // something was issued
}

// ---------------------------------------------------------------- softmax

// Whether score pair c (of a tile's 64) is exponentiated by the FMA-pipe
// polynomial instead of MUFU ex2: pairs 1, 4, 7 of every 10 in both kernels
// (the measured best of 10-40 % and of where in the 10 they sit; the DiT's
// best moved from 2 in 10 to 3 in 10 with the warpgroups' start offset).
template <bool kRelBias>
__device__ __forceinline__ constexpr bool poly_pair(int c) {
    return c % 10 == 1 || c % 10 == 4 || c % 10 == 7;
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
    uint32_t s_full, s_free, p_half, p_full, pv_done;  // barrier shared addresses
    WaitCtl ctl;
    int i, kv_end, lane, t_begin;
    float m_run, l_run;
    uint32_t s_parity, pv_parity;

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
            // keys n0 + c .. n0 + c + 3 (c a multiple of 4) take QR[clamp(k)] ..
            // QR[clamp(k + 3)] with k = n0 + c - i + 64: the padded table's entries
            // m .. m + 3 for m = clamp(k + 4 + (i & 3), 0, 80), a multiple of 4
            // (k + (i & 3) is: n0, c, 64 and the tile's first row are)
            const int e0 = n0 - i + kClampLeft + 4 + (i & 3);
#pragma unroll
            for (int c = 0; c < 128; c += 4) {
                const int m = min(max(e0 + c, 0), kQrStride - 4);
                const float4 b = ld_shared_v4f32(qrow + 4u * m);
                s[c] = fmaf(s[c], sl, b.x);
                s[c + 1] = fmaf(s[c + 1], sl, b.y);
                s[c + 2] = fmaf(s[c + 2], sl, b.z);
                s[c + 3] = fmaf(s[c + 3], sl, b.w);
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
            alpha = ex2_approx(m_run - tile_max);  // 0 on the item's first tile
            m_run = tile_max;
        }
        const float add = cb - m_run;
        const float ky = mult * (1.0f / kPolySpan), kb = (add - kPolyLo) * (1.0f / kPolySpan);

        // exponentials into packed 16-bit pairs, held in registers; some pairs
        // go through the FMA-pipe polynomial so that the MUFU and FMA pipes
        // carry similar loads (poly_pair)
        uint32_t pk[64];
        float2 ls[4];
#pragma unroll
        for (int a = 0; a < 4; ++a) ls[a] = make_float2(0.f, 0.f);
        const float2 mult2 = make_float2(mult, mult), add2 = make_float2(add, add);
        const bool later = j > t_begin;
        constexpr bool kSplit = PvSplit<kRelBias>::kOn;
#pragma unroll
        for (int c = 0; c < 64; ++c) {
            if (kSplit && c == 32) {
                // keys 0..63 done: store them once P(j-1) V(j-1) is complete (it
                // reads these P columns), after O is rescaled if the max moved
                if (later) {
                    ok = warp_wait(pv_done, pv_parity, ctl, err);
                    pv_parity ^= 1;
                    if (!ok) return false;
                    tc_fence_after();
                    if (__any_sync(0xffffffffu, rescale)) rescale_o_row(tO, alpha);
                }
                tmem_st32(tP + 0, *reinterpret_cast<uint32_t(*)[32]>(&pk[0]));
            }
            if (kSplit && c == 40) {
                // the first half of P(j) V(j) may start (the store ran under 8 pairs;
                // measured best of pairs 34-56: earlier waits on the store, later
                // delays the MMA)
                tmem_wait_st();
                warp_arrive(p_half, lane);
            }
            float2 pp;
            if (poly_pair<kRelBias>(c)) {
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

        if constexpr (!kSplit) {
            if (later) {
                // P(j-1) V(j-1) must be complete before its P columns are rewritten
                // and before O is rescaled (its latency hides under the work above).
                ok = warp_wait(pv_done, pv_parity, ctl, err);
                pv_parity ^= 1;
                if (!ok) return false;
                tc_fence_after();
            }
            tmem_st32(tP + 0, *reinterpret_cast<uint32_t(*)[32]>(&pk[0]));
        }
        tmem_st32(tP + 32, *reinterpret_cast<uint32_t(*)[32]>(&pk[32]));
        if (!kSplit && later && __any_sync(0xffffffffu, rescale)) rescale_o_row(tO, alpha);
        tmem_wait_st();
        warp_arrive(p_full, lane);
        return true;
    }
};

template <typename T>
__device__ __forceinline__ void store_row(T* out_row, const float (&o)[64], float inv) {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        uint4 v;
        v.x = DTypeTraits<T>::pack(o[8 * c + 0] * inv, o[8 * c + 1] * inv);
        v.y = DTypeTraits<T>::pack(o[8 * c + 2] * inv, o[8 * c + 3] * inv);
        v.z = DTypeTraits<T>::pack(o[8 * c + 4] * inv, o[8 * c + 5] * inv);
        v.w = DTypeTraits<T>::pack(o[8 * c + 6] * inv, o[8 * c + 7] * inv);
        reinterpret_cast<uint4*>(out_row)[c] = v;
    }
}

// A part of a cut unit done for this thread's row: its (O, m, l) go to the
// part's workspace slot and the warp counts itself in; the warp whose count
// completes the unit (per 32-row group) reads every part's rows back (its own
// included), merges them in piece order (m = max m_k, O = sum O_k 2^(m_k - m),
// l = sum l_k 2^(m_k - m); the same order whichever part merges, so results are
// reproducible), writes the output rows and resets the count for the next call. The other
// parts are the neighbouring pieces that touch the unit (a cut unit has at most
// kMaxParts parts; the host guarantees it). Fences follow the last-block
// pattern: each lane's rows are visible device-wide before the count moves,
// and the merging warp fences after seeing the full count.
template <typename T>
__device__ __forceinline__ void finish_part(const AttnParams& p, const float (&o)[64], float m, float l, int u,
                                            int item_idx, int unit_row, int group, int lane, T* out_row,
                                            bool valid) {
    const TileSeq ts(p);
    const uint32_t k = blockIdx.x - p.whole_ctas;  // this piece
    const auto slot = [&](uint32_t piece, uint32_t item) {
        return reinterpret_cast<float4*>(p.parts) +
               static_cast<int64_t>(piece * kMaxItems + item) * kPartBlocks * kRowsPerCta + unit_row;
    };
    float4* mine = slot(k, item_idx);
#pragma unroll
    for (int c = 0; c < 16; ++c)
        mine[c * kRowsPerCta] = make_float4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
    mine[16 * kRowsPerCta] = make_float4(m, l, 0.f, 0.f);

    // pieces touching unit u: contiguous, around this one, at most kMaxParts - 1
    // on either side. Lane j evaluates piece k - (kMaxParts - 1) + j (its tile
    // range: a few integer divisions), so the warp searches all candidates at
    // once instead of every lane walking them one after another.
    const uint32_t lo_tile = static_cast<uint32_t>(u) * ts.n, hi_tile = lo_tile + ts.n;
    constexpr int kSide = kMaxParts - 1;
    const int kc = static_cast<int>(k) - kSide + lane;
    uint2 rg = make_uint2(0u, 0u);
    bool touch = false;
    if (lane <= 2 * kSide && kc >= 0 && kc < p.pieces) {
        rg = piece_range(p, ts, static_cast<uint32_t>(kc));
        touch = lane < kSide ? rg.y > lo_tile : (lane > kSide ? rg.x < hi_tile : true);
    }
    const uint32_t near = __ballot_sync(0xffffffffu, touch);
    uint32_t k_first = k, k_last = k;
#pragma unroll
    for (int d = 1; d <= kSide; ++d) {  // the runs of touching pieces below and above k
        if (k_first + d == k + 1 && ((near >> (kSide - d)) & 1u)) --k_first;
        if (k_last + 1 == k + d && ((near >> (kSide + d)) & 1u)) ++k_last;
    }
    const uint32_t nparts = k_last - k_first + 1;

    uint32_t* count = p.counts + static_cast<int64_t>(u - p.whole_ctas) * kSoftmaxWarps + group;
    __threadfence();
    __syncwarp();
    uint32_t done = 0;
    if (lane == 0) done = atomicAdd(count, 1u);
    done = __shfl_sync(0xffffffffu, done, 0);
    if (done + 1 != nparts) return;  // another part completes the count and merges
    __threadfence();

    // fold the parts in piece order, so the result does not depend on which
    // part merges (am = -inf makes the first fold take its part unchanged)
    float am = -INFINITY, al = 0.f;
    float acc[64];
#pragma unroll
    for (int c = 0; c < 64; ++c) acc[c] = 0.f;
    // (this part's own rows are read back from its slot too: no registers held)
    for (uint32_t kk = k_first; kk <= k_last; ++kk) {
        // piece kk's first tile, from the lane that evaluated it above
        const uint32_t first_unit = __shfl_sync(0xffffffffu, rg.x, static_cast<int>(kk - k) + kSide) / ts.n;
        const float4* part = slot(kk, static_cast<uint32_t>(u) - first_unit);
        const float4 ml = __ldcg(part + 16 * kRowsPerCta);
        float4 v[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) v[c] = __ldcg(part + c * kRowsPerCta);
        const float pm = ml.x, pl = ml.y;
        const float mm = fmaxf(am, pm);
        const float fa = ex2_approx(am - mm), fb = ex2_approx(pm - mm);
#pragma unroll
        for (int c = 0; c < 16; ++c) {
            acc[4 * c + 0] = fmaf(acc[4 * c + 0], fa, v[c].x * fb);
            acc[4 * c + 1] = fmaf(acc[4 * c + 1], fa, v[c].y * fb);
            acc[4 * c + 2] = fmaf(acc[4 * c + 2], fa, v[c].z * fb);
            acc[4 * c + 3] = fmaf(acc[4 * c + 3], fa, v[c].w * fb);
        }
        al = fmaf(al, fa, pl * fb);
        am = mm;
    }
    if (valid) store_row<T>(out_row, acc, 1.f / al);
    __syncwarp();
    if (lane == 0) *count = 0;
}

// The padded relative-bias row of query row i, T[m] = QR[clamp(m - 4 - R, 0, 72)]
// (scaled to log2 units) for m in [0, 84), R = i mod 4, as 21 aligned 16-byte
// stores. Every lane runs the same instructions: the shift by R is two levels
// of selects over the seven table entries a 16-byte group can draw on, so that
// each store has all 32 lanes (32 consecutive rows) active, and the row
// stride (84 words) keeps each quarter-warp's 16-byte accesses on distinct
// banks. (A branch per residue ran each store with the 8 lanes of one residue,
// rows 4 apart, whose 16-byte chunks fall on 2 bank groups: 4-way conflicts,
// and four times the instructions: 1.76 us per item on a B200.)
__device__ __forceinline__ void fill_qr_row(uint32_t qrow, const uint32_t (&a)[32], const uint32_t (&c2)[32],
                                            const uint32_t (&d)[16], float sl, int R) {
    const auto qr = [&](int k) {  // QR[clamp(k, 0, 72)], k known at compile time
        k = k < 0 ? 0 : (k > kNumPos - 1 ? kNumPos - 1 : k);
        return __uint_as_float(k < 32 ? a[k] : (k < 64 ? c2[k - 32] : d[k - 64]));
    };
    const bool odd = (R & 1) != 0, high = (R & 2) != 0;
#pragma unroll
    for (int q = 0; q < kQrStride / 4; ++q) {
        // group q takes QR[4q - 4 - R + e], e = 0..3, from w[t] = QR[4q - 7 + t]:
        // z[t] = w[t + 1 - (R & 1)], then v[e] = z[e + 2 - (R & 2)]
        float z[6];
#pragma unroll
        for (int t = 0; t < 6; ++t) z[t] = odd ? qr(4 * q - 7 + t) : qr(4 * q - 6 + t);
        float v[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) v[e] = (high ? z[e] : z[e + 2]) * sl;
        st_shared_v4(qrow + 16u * q, make_int4(__float_as_int(v[0]), __float_as_int(v[1]), __float_as_int(v[2]),
                                               __float_as_int(v[3])));
    }
}

template <typename T, bool kRelBias, bool kQrGlobal>
__device__ __forceinline__ void softmax_role(uint32_t sbase, uint32_t tmem, const AttnParams& p, WaitCtl ctl,
                                             int warp, int lane, int n_items) {
    const int wg = (warp - kSoftmaxWarp0) >> 2;  // query tile of this warpgroup
    const int wq = warp & 3;                     // warp within the warpgroup (= TMEM lane quarter)
    const int row = (wq << 5) + lane;            // row in tile == TMEM lane
    const int L = p.seq_len;
    constexpr int err = FDS_STATUS_TIMEOUT_SOFTMAX;
    const uint32_t lane_addr = static_cast<uint32_t>(wq * 32) << 16;
    const float sl = p.scale_log2;
    const uint32_t qrow = sbase + Smem::qr + 4u * ((wg * kBlockM + row) * kQrStride);
    const uint32_t bars = sbase + Smem::bars;

    RowSoftmax<T, kRelBias> rs;
    rs.tS = tmem + lane_addr + kTmemS + wg * kBlockN;
    rs.tP = tmem + lane_addr + kTmemP + wg * (kBlockN / 2);
    rs.tO = tmem + lane_addr + kTmemO + wg * kHeadDim;
    rs.sl = sl;
    rs.qrow = qrow;
    rs.s_full = bars + 8u * (Smem::kSFull + wg);
    rs.s_free = bars + 8u * (Smem::kSFree + wg);
    rs.p_full = bars + 8u * (Smem::kPFull + wg);
    rs.p_half = bars + 8u * (Smem::kPHalf + wg);
    rs.pv_done = bars + 8u * (Smem::kPvDone + wg);
    rs.ctl = ctl;
    rs.lane = lane;
    rs.s_parity = 0;
    rs.pv_parity = 0;

    // The second query tile's warpgroup starts 600 cycles after the first: in
    // lockstep both warpgroups of an SM sub-partition wait on their S loads and
    // the hand-offs at the same moments; offset, one warp's waits fall under the
    // other's exponentials, and the offset persists over the items (measured,
    // encoder layer at L = 6000: 0.2100 -> 0.2085 ms; 450-800 cycles alike; DiT
    // unchanged). A bounded spin on the SM clock.
    if (wg == 1) {
        const long long t_start = clock64();
        while (clock64() - t_start < 600) {
        }
    }

    bool ok = true;
    for (int idx = 0; ok && idx < n_items; ++idx) {
        const Item it = load_item(sbase, idx);
        if (wg == 1 && !it.has_q1) continue;  // this unit has no second query tile
        const int i = it.q_base + wg * kBlockM + row;  // query index in the window
        T* out_row = reinterpret_cast<T*>(p.out) +
                     (p.heads_in_z ? (static_cast<int64_t>(it.b) * p.heads + it.h) * L + i
                                   : static_cast<int64_t>(it.b) * L + i) * p.out_stride +
                     head_x(p, it.h);
        if (it.t_end <= it.t_begin) {  // no valid key: the context row is defined as zero
            if (i < L) {
                const uint4 z = make_uint4(0, 0, 0, 0);
#pragma unroll
                for (int c = 0; c < 8; ++c) reinterpret_cast<uint4*>(out_row)[c] = z;
            }
            continue;
        }
        rs.i = i;
        rs.kv_end = kv_end_of(p, it.b);
        rs.t_begin = it.t_begin;
        rs.m_run = -INFINITY;
        rs.l_run = 0.f;

        float qr_left = 0.f, qr_right = 0.f;
        if constexpr (kRelBias && kQrGlobal) {
            // this row's 73 relative-key projections from global memory (rows
            // past the window read as zero, like the Q rows the copies fill)
            const T* src = static_cast<const T*>(p.qr) +
                           (p.heads_in_z ? (static_cast<int64_t>(it.b) * p.heads + it.h) * L + i
                                         : (static_cast<int64_t>(it.b) * L + i) * p.heads + it.h) * kNumPos;
            const bool in = i < L;
            const auto qr_at = [&](int r) { return in ? DTypeTraits<T>::load_f32(src + r) * sl : 0.f; };
            qr_left = qr_at(0);
            qr_right = qr_at(kNumPos - 1);
            const uint32_t t = qrow + 4u * (4 + (i & 3));
#pragma unroll
            for (int m = 0; m < 7; ++m) st_shared_f32(qrow + 4u * m, qr_left);
#pragma unroll
            for (int m = kQrStride - 8; m < kQrStride; ++m) st_shared_f32(qrow + 4u * m, qr_right);
#pragma unroll 8
            for (int c = 0; c < kNumPos; ++c) st_shared_f32(t + 4u * c, qr_at(c));
        } else if constexpr (kRelBias) {
            ok = warp_wait(rs.s_full, rs.s_parity, ctl, err);
            rs.s_parity ^= 1;
            if (!ok) break;
            tc_fence_after();
            uint32_t a[32], c2[32], d[16];
            tmem_ld32(rs.tS, a);
            tmem_ld32(rs.tS + 32, c2);
            tmem_ld16(rs.tS + 64, d);
            tmem_wait_ld();
            warp_arrive(rs.s_free, lane);  // the S columns may now receive the item's first S
            qr_left = __uint_as_float(a[0]) * sl;
            qr_right = __uint_as_float(d[kNumPos - 1 - 64]) * sl;
            fill_qr_row(qrow, a, c2, d, sl, i & 3);
        }

        // Tiles in key order: [.., jb0) every pair left-saturated (bias QR[i,0]),
        // [jb0, jb1) near-diagonal (per-score gather), [jb1, ..) every pair
        // right-saturated (bias QR[i,72]). With t0 the tile's first query row, a
        // KV tile starting at key n0 is near-diagonal iff t0 - 190 <= n0 <= t0 + 134.
        // Each class runs its own copy of the tile step, so the hot loops carry
        // no gather code; the item's last tile (key padding) takes the general step.
        const int j_last = it.t_end - 1;
        int j = it.t_begin;
        if constexpr (kRelBias) {
            const int t0 = it.q_base + wg * kBlockM;
            const int jb0 = t0 >= 190 ? (t0 - 190 + kBlockN - 1) / kBlockN : 0;
            const int jb1 = (t0 + 135 + kBlockN - 1) / kBlockN;
            for (; ok && j < min(jb0, j_last); ++j) ok = rs.template step<false, false>(j, qr_left);
            for (; ok && j < min(jb1, j_last); ++j) ok = rs.template step<true, false>(j, 0.f);
            for (; ok && j < j_last; ++j) ok = rs.template step<false, false>(j, qr_right);
            if (ok) ok = rs.template step<true, true>(j_last, 0.f);
        } else {
            for (; ok && j < j_last; ++j) ok = rs.template step<false, false>(j, 0.f);
            if (ok) ok = rs.template step<false, true>(j_last, 0.f);
        }
        if (!ok) break;

        // epilogue: the last P V must be complete before O is read (the next
        // item's first P V overwrites O only after this warpgroup's next P
        // store, which follows this read in program order)
        ok = warp_wait(rs.pv_done, rs.pv_parity, ctl, err);
        rs.pv_parity ^= 1;
        if (!ok) break;
        tc_fence_after();
        uint32_t ou[64];
        tmem_ld32(rs.tO, *reinterpret_cast<uint32_t(*)[32]>(&ou[0]));
        tmem_ld32(rs.tO + 32, *reinterpret_cast<uint32_t(*)[32]>(&ou[32]));
        tmem_wait_ld();
        float o[64];
#pragma unroll
        for (int c = 0; c < 64; ++c) o[c] = __uint_as_float(ou[c]);
        if (it.kind == kWhole) {
            if (i < L) store_row<T>(out_row, o, 1.f / rs.l_run);
        } else {
            const int u = (it.b * p.heads + it.h) * p.row_blocks + it.q_base / kRowsPerCta;
            finish_part<T>(p, o, rs.m_run, rs.l_run, u, idx, wg * kBlockM + row, wg * 4 + wq, lane, out_row, i < L);
        }
    }
}

// ---------------------------------------------------------------- TMA producer

template <bool kRelBias, bool kQrGlobal>
__device__ __forceinline__ void load_role(uint32_t sbase, const CUtensorMap* map_q, const CUtensorMap* map_k,
                                          const CUtensorMap* map_v, const CUtensorMap* map_r, const AttnParams& p,
                                          WaitCtl ctl, int n_items) {
    const auto bar = [&](int idx) { return sbase + Smem::bars + 8u * idx; };
    int qi = 0;           // items loaded (Q copies issued)
    int g = 0;            // K/V tiles fully issued
    bool k_only = false;  // K(g) issued, V(g) not (abort between the two)
    bool ok = true;
    for (int idx = 0; ok && idx < n_items; ++idx) {
        const Item it = load_item(sbase, idx);
        if (it.t_end <= it.t_begin) continue;
        if (qi > 0) {
            ok = warp_wait(bar(Smem::kQEmpty), (qi - 1) & 1, ctl, FDS_STATUS_TIMEOUT_LOAD);
            if (!ok) break;
        }
        const int z = head_z(p, it.b, it.h);
        if (elect_one()) {
            const bool rel = kRelBias && !kQrGlobal && qi == 0;  // the table for the Q.rel^T MMA
            const uint32_t q_bytes = (it.has_q1 ? 2 : 1) * kTileBytes + (rel ? kRelRows * 128 : 0);
            const int qx = p.q_x0 + head_x(p, it.h);
            mbar_arrive_expect_tx(bar(Smem::kQ), q_bytes);
            tma_load_3d(sbase + Smem::q0, map_q, bar(Smem::kQ), qx, it.q_base, z);
            if (it.has_q1) tma_load_3d(sbase + Smem::q1, map_q, bar(Smem::kQ), qx, it.q_base + kBlockM, z);
            if (rel) tma_load_2d(sbase + Smem::rel, map_r, bar(Smem::kQ), 0, 0);
        }
        __syncwarp();
        ++qi;
        const int kx = p.k_x0 + head_x(p, it.h), vx = p.v_x0 + head_x(p, it.h);
        for (int j = it.t_begin; j < it.t_end; ++j) {
            const int st = g % kStages;
            const uint32_t par = ((g / kStages) - 1) & 1;
            if (g >= kStages) {
                ok = warp_wait(bar(Smem::kKEmpty + st), par, ctl, FDS_STATUS_TIMEOUT_LOAD);
                if (!ok) break;
            }
            if (elect_one()) {
                mbar_arrive_expect_tx(bar(Smem::kKFull + st), kTileBytes);
                tma_load_3d(sbase + Smem::k + st * kTileBytes, map_k, bar(Smem::kKFull + st), kx, j * kBlockN, z);
            }
            __syncwarp();
            if (g >= kStages) {
                ok = warp_wait(bar(Smem::kVEmpty + st), par, ctl, FDS_STATUS_TIMEOUT_LOAD);
                if (!ok) {
                    k_only = true;
                    break;
                }
            }
            if (elect_one()) {
                mbar_arrive_expect_tx(bar(Smem::kVFull + st), kTileBytes);
                tma_load_3d(sbase + Smem::v + st * kTileBytes, map_v, bar(Smem::kVFull + st), vx, j * kBlockN, z);
            }
            __syncwarp();
            ++g;
        }
    }
    if (!ok) {
        // aborted: let every copy already issued land before the CTA exits
        if (qi > 0) wait_bounded(bar(Smem::kQ), (qi - 1) & 1, ctl, FDS_STATUS_TIMEOUT_DRAIN, false);
        const int gk = g + (k_only ? 1 : 0);
        for (int s = 0; s < kStages; ++s) {
            // loads issued into stage s: tiles s, s + kStages, ... below g (plus K(g) alone)
            const int nk = gk > s ? (gk - s + kStages - 1) / kStages : 0;
            const int nv = g > s ? (g - s + kStages - 1) / kStages : 0;
            if (nk > 0) wait_bounded(bar(Smem::kKFull + s), (nk - 1) & 1, ctl, FDS_STATUS_TIMEOUT_DRAIN, false);
            if (nv > 0) wait_bounded(bar(Smem::kVFull + s), (nv - 1) & 1, ctl, FDS_STATUS_TIMEOUT_DRAIN, false);
        }
        __syncwarp();
    }
}

// ---------------------------------------------------------------- kernel

// kQrGlobal (with kRelBias): the relative-key projections come from global
// memory (p.qr, the TensorRT plugin's form) instead of the Q.rel^T MMA.
template <typename T, bool kRelBias, bool kQrGlobal = false>
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
    // Launched after the previous kernel in the stream is allowed to finish:
    // nothing below reads or writes global memory before grid_dependency_wait
    // (the set-up, TMEM allocation and tensor-map prefetch overlap its tail).
    grid_launch_dependents();

    if (threadIdx.x == 0) {
        mbar_init(&bars[Smem::kQ], 1);
        mbar_init(&bars[Smem::kQEmpty], 2);  // both query tiles' MMA warps
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&bars[Smem::kKFull + s], 1);
            mbar_init(&bars[Smem::kVFull + s], 1);
            mbar_init(&bars[Smem::kKEmpty + s], 2);
            mbar_init(&bars[Smem::kVEmpty + s], 2);
        }
        for (int w = 0; w < 2; ++w) {
            mbar_init(&bars[Smem::kSFull + w], 1);
            mbar_init(&bars[Smem::kSFree + w], 4);   // one arrival per softmax warp
            mbar_init(&bars[Smem::kPFull + w], 4);
            mbar_init(&bars[Smem::kPvDone + w], 1);
            mbar_init(&bars[Smem::kPHalf + w], 4);
        }
        for (int d = 0; d < 2; ++d) mbar_init(&bars[Smem::kDrain + d], 1);
        mbar_init(&bars[Smem::kNever], 1);
        st_shared_volatile_u32(ctl.misc + 4, 0);  // abort flag
        st_shared_u64(ctl.misc + 8, reinterpret_cast<uint64_t>(p.status));
        st_shared_u64(ctl.misc + 32, reinterpret_cast<uint64_t>(p.status_host));
        st_shared_u64(ctl.misc + 16, static_cast<uint64_t>(p.timeout_ns > 0 ? p.timeout_ns : kDefaultTimeoutNs));
        grid_dependency_wait();  // build_items reads kv_len
        st_shared_volatile_u32(ctl.misc + 28, static_cast<uint32_t>(build_items(p, sbase)));
        fence_barrier_init();
        fence_proxy_async_smem();
    }
    if (warp == kLoadWarp && lane == 0) {
        prefetch_tensormap(&map_q);
        prefetch_tensormap(&map_k);
        prefetch_tensormap(&map_v);
        if (kRelBias && !kQrGlobal) prefetch_tensormap(&map_r);
    }
    if (warp == kTmemWarp) {
        tmem_alloc(tmem_holder, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    grid_dependency_wait();
    const uint32_t tmem = *tmem_holder;
    const int n_items = static_cast<int>(ld_shared_volatile_u32(ctl.misc + 28));

    // The two register classes never share code again: each branch ends with
    // its own arrival on the CTA-wide barrier (every thread of the CTA arrives
    // exactly once, so all roles have finished with TMEM when it opens).
    if (warp >= kSoftmaxWarp0) {
        setmaxnreg_inc<RegSplit<kRelBias>::kSoftmax>();
        softmax_role<T, kRelBias, kQrGlobal>(sbase, tmem, p, ctl, warp, lane, n_items);
        __syncwarp();
        tc_fence_before();
        named_barrier_sync(1, kThreads);
    } else {
        setmaxnreg_dec<RegSplit<kRelBias>::kControl>();
        if (warp == kMmaWarp0 || warp == kMmaWarp0 + 2) {
            // test hook: a wait on a barrier that nothing arrives on, to exercise
            // the bounded-wait error path without a real hang
            bool go = true;
            if (p.debug_flags & FDS_DEBUG_FORCE_TIMEOUT)
                go = warp_wait(sbase + Smem::bars + 8u * Smem::kNever, 0, ctl, FDS_STATUS_TIMEOUT_MMA);
            if (go) mma_role<T, kRelBias>(sbase, tmem, ctl, (warp - kMmaWarp0) >> 1, n_items, !kQrGlobal);
        } else if (warp == kLoadWarp) {
            load_role<kRelBias, kQrGlobal>(sbase, &map_q, &map_k, &map_v, &map_r, p, ctl, n_items);
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
