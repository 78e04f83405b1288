// fds_capi.cu - the extern "C" entry points declared in include/fds_b200.h:
// argument checks, TMA tensor maps over the caller's buffers, and launches on
// the caller's stream. No device allocation, no synchronisation, no host work
// that depends on tensor contents (safe inside CUDA-graph stream capture).
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdarg>
#include <cstdlib>
#include <cstring>
#include <cstdio>
#include <mutex>
#include <string>
#include <utility>

#include "attn_kernel.cuh"
#include "capi_internal.h"
#include "fds_b200.h"
#include "gemm_kernel.cuh"
#include "rope.cuh"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int ok() {
    g_last_error.clear();
    return FDS_OK;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
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

// Device must be compute capability 10.0 (B200 / sm_100a). Cached per device;
// the entries are atomics so that first calls from several host threads do not
// race (every thread computes the same value).
int check_device() {
    static std::atomic<int> cached[64];  // 0 unknown, 1 ok, 2 unsupported
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(FDS_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= 64) return fail(FDS_ERR_UNSUPPORTED_DEVICE, "device index %d out of range", dev);
    int state = cached[dev].load(std::memory_order_relaxed);
    if (state == 0) {
        int major = 0, minor = 0;
        cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
        state = (major == 10 && minor == 0) ? 1 : 2;
        cached[dev].store(state, std::memory_order_relaxed);
    }
    if (state != 1)
        return fail(FDS_ERR_UNSUPPORTED_DEVICE, "device %d is not sm_100 (B200); this library is built for sm_100a",
                    dev);
    return FDS_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// 3-D map over a [batch, seq_len, width] view of rows with `row_stride` elements:
// box = 64 columns x `box_rows` rows x 1 window, 128-byte swizzle, zero fill
// past seq_len (so a tile never reads the next window's rows).
int make_rows_map(CUtensorMap* map, const void* base, int dtype, int64_t width, int64_t seq_len, int64_t batch,
                  int64_t row_stride, int box_rows) {
    EncodeTiledFn enc = encode_fn();
    if (enc == nullptr) return fail(FDS_ERR_TENSOR_MAP, "cuTensorMapEncodeTiled unavailable from the driver");
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(width), static_cast<cuuint64_t>(seq_len),
                                static_cast<cuuint64_t>(batch)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(row_stride * 2),
                                   static_cast<cuuint64_t>(row_stride * 2 * seq_len)};
    const cuuint32_t box[3] = {64, static_cast<cuuint32_t>(box_rows), 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUtensorMapDataType dt =
        dtype == FDS_DTYPE_FP16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    CUresult r = enc(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(FDS_ERR_TENSOR_MAP, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
    return FDS_OK;
}

// 2-D map over the [73, 64] relative-key table, box 64 x 80 (rows 73..79 read as zero).
int make_rel_map(CUtensorMap* map, const void* base, int dtype) {
    EncodeTiledFn enc = encode_fn();
    if (enc == nullptr) return fail(FDS_ERR_TENSOR_MAP, "cuTensorMapEncodeTiled unavailable from the driver");
    const cuuint64_t dims[2] = {64, fds::kNumPos};
    const cuuint64_t strides[1] = {128};
    const cuuint32_t box[2] = {64, fds::kRelRows};
    const cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType dt =
        dtype == FDS_DTYPE_FP16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(FDS_ERR_TENSOR_MAP, "cuTensorMapEncodeTiled(rel) failed (%d)", static_cast<int>(r));
    return FDS_OK;
}

// 2-D map over a [rows, cols] row-major matrix (row stride `row_stride`
// elements), box 64 columns x `box_rows` rows, 128-byte swizzle, zero fill
// past the last row.
int make_matrix_map(CUtensorMap* map, const void* base, int dtype, int64_t cols, int64_t rows, int64_t row_stride,
                    int box_rows) {
    EncodeTiledFn enc = encode_fn();
    if (enc == nullptr) return fail(FDS_ERR_TENSOR_MAP, "cuTensorMapEncodeTiled unavailable from the driver");
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride * 2)};
    const cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
    const cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType dt =
        dtype == FDS_DTYPE_FP16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    CUresult r = enc(map, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(FDS_ERR_TENSOR_MAP, "cuTensorMapEncodeTiled(matrix) failed (%d)", static_cast<int>(r));
    return FDS_OK;
}

// The linear layers' output for the epilogue's TMA copies: boxes of 32 rows x
// 128 bytes (64 fp16 / bf16 or 32 fp32 columns), 128-byte swizzle, the layout
// the epilogue stages each box in.
int make_out_map(CUtensorMap* map, void* base, bool f32, int dtype, int64_t cols, int64_t rows, int64_t row_stride) {
    EncodeTiledFn enc = encode_fn();
    if (enc == nullptr) return fail(FDS_ERR_TENSOR_MAP, "cuTensorMapEncodeTiled unavailable from the driver");
    const int esize = f32 ? 4 : 2;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride * esize)};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / esize), 32};
    const cuuint32_t estr[2] = {1, 1};
    const CUtensorMapDataType dt = f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                   : dtype == FDS_DTYPE_FP16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                             : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    CUresult r = enc(map, dt, 2, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(FDS_ERR_TENSOR_MAP, "cuTensorMapEncodeTiled(output) failed (%d)", static_cast<int>(r));
    return FDS_OK;
}

// A RoPE table (fp32 [>= seq_len, 64], rows of 256 bytes) for the linear
// layers' RoPE epilogue: boxes of 128 rows x the first 32 columns (the table is
// cat([f, f]): the second half repeats them), 128-byte swizzle.
int make_rope_table_map(CUtensorMap* map, const float* base, int64_t seq_len) {
    EncodeTiledFn enc = encode_fn();
    if (enc == nullptr) return fail(FDS_ERR_TENSOR_MAP, "cuTensorMapEncodeTiled unavailable from the driver");
    const cuuint64_t dims[2] = {64, static_cast<cuuint64_t>(seq_len)};
    const cuuint64_t strides[1] = {64 * 4};
    const cuuint32_t box[2] = {32, static_cast<cuuint32_t>(fds::gemm::kBM)};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(FDS_ERR_TENSOR_MAP, "cuTensorMapEncodeTiled(rope table) failed (%d)", static_cast<int>(r));
    return FDS_OK;
}

// Kernels are launched with programmatic stream serialization: a launch may
// start its CTAs while the previous kernel in the stream drains, and waits in
// the kernel (griddepcontrol.wait) before touching memory. FDS_PDL=0 in the
// environment turns this off (plain stream order).
bool pdl_enabled() {
    static const bool on = [] {
        const char* v = std::getenv("FDS_PDL");
        return v == nullptr || std::strcmp(v, "0") != 0;
    }();
    return on;
}

// cudaFuncSetAttribute(kern, MaxDynamicSharedMemorySize, bytes) once per
// kernel and device (it is per-device state, and a per-call driver round trip
// otherwise); `done` is the kernel's own set of devices already configured.
template <typename Kern>
cudaError_t set_smem_once(Kern kern, int bytes, std::atomic<uint64_t>& done) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const uint64_t bit = dev >= 0 && dev < 64 ? (uint64_t{1} << dev) : 0;
    if (bit != 0 && (done.load(std::memory_order_acquire) & bit) != 0) return cudaSuccess;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess && bit != 0) done.fetch_or(bit, std::memory_order_release);
    return e;
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                       Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// SMs of the current device (cached per device, atomically as above); 0 if it
// cannot be queried.
int sm_count() {
    static std::atomic<int> cached[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    int n = cached[dev].load(std::memory_order_relaxed);
    if (n == 0) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
        cached[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

// Workspace of the split last wave for up to G pieces: the part counts (one
// per cut unit and 32-row group; at most G <= kMaxPieces units are cut) in a
// fixed region, so that calls with different piece counts can share a
// workspace (the counts stay zero between calls), then G x kMaxItems slots of
// 256 rows x kPartRowFloats floats.
constexpr int64_t kMaxPieces = 1024;
constexpr int64_t kWsSlotsOffset = kMaxPieces * fds::kSoftmaxWarps * 4;
int64_t ws_bytes_for(int64_t G) {
    return kWsSlotsOffset + G * fds::kMaxItems * fds::kRowsPerCta * fds::kPartRowFloats * 4;
}

struct Workspace {
    void* ptr;
    int64_t bytes;
    int grid_ctas;
};

// How a launch is laid out: `grid` CTAs, the first `whole` of them one unit
// each, the last `pieces` the cut last wave (0: one unit per CTA).
struct Plan {
    int64_t grid, whole, pieces;
};

// The split last wave needs a workspace, no kv_len, and with G = grid_ctas
// (0: the SM count) waves = ceil(U / G), the (waves - 1) G whole units first
// and the remaining units cut by weight into G pieces such that every piece
// touches at most kMaxItems (3) units and every cut unit has at most kMaxParts
// (4) parts: the piece weight is between a third of a two-tile unit (and at
// least a unit start and one tile) and twice the lightest unit (units weighted
// with their start cost, attn_kernel.cuh TileSeq). With grid_ctas == 0 it is used only when whole units leave
// more than 3% of the SM time of the waves idle.
Plan plan_schedule(int64_t batch, int64_t heads, int64_t seq_len, bool has_kv_len, bool has_ws, int64_t ws_bytes,
                   int64_t grid_ctas, int64_t sms) {
    const int64_t R = (seq_len + fds::kRowsPerCta - 1) / fds::kRowsPerCta;
    const int64_t U = batch * heads * R;
    Plan plan{U, U, 0};
    const int64_t G = grid_ctas > 0 ? grid_ctas : sms;
    if (!has_ws || has_kv_len || G <= 0 || G > kMaxPieces) return plan;
    const int64_t waves = (U + G - 1) / G;
    if (grid_ctas == 0 && static_cast<double>(U) / static_cast<double>(waves * G) >= 0.97) return plan;
    const int64_t n = (seq_len + fds::kBlockN - 1) / fds::kBlockN;
    const int64_t w2 = fds::kWeightTwoTiles, c0 = fds::unit_start_weight(static_cast<uint32_t>(n));
    const int64_t w_last = (R - 1) * fds::kRowsPerCta + fds::kBlockM < seq_len ? w2 : fds::kWeightOneTile;
    const int64_t unit_full = c0 + n * w2, unit_last = c0 + n * w_last;  // unit weights (attn_kernel.cuh TileSeq)
    const int64_t per_bh = (R - 1) * unit_full + unit_last;
    const int64_t whole = (waves - 1) * G;
    const auto unit_pos = [&](int64_t u) { return (u / R) * per_bh + (u % R) * unit_full; };
    const int64_t total = unit_pos(U);
    const int64_t wt = total - unit_pos(whole);
    const int64_t w_min = wt / G, w_max = (wt + G - 1) / G;
    const bool ok = ws_bytes >= ws_bytes_for(G) && w_min >= c0 + w2 && 3 * w_min >= unit_full &&
                    w_max <= 2 * unit_last && G * total < (int64_t{1} << 31);
    if (ok) plan = Plan{whole + G, whole, G};
    return plan;
}

// Launches on `plan`; the workspace is split into counts and slots.
template <typename T, bool kRelBias, bool kQrGlobal = false>
int launch_attn(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mr,
                fds::AttnParams p, int batch, const Workspace& ws, cudaStream_t stream) {
    auto kern = fds::attn_fwd_kernel<T, kRelBias, kQrGlobal>;
    static std::atomic<uint64_t> smem_set{0};
    cudaError_t e = set_smem_once(kern, fds::Smem::alloc, smem_set);
    if (e != cudaSuccess) return fail(FDS_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    p.row_blocks = (p.seq_len + fds::kRowsPerCta - 1) / fds::kRowsPerCta;
    const int64_t U = static_cast<int64_t>(batch) * p.heads * p.row_blocks;
    if (U > 0x7fffffffLL) return fail(FDS_ERR_INVALID_ARGUMENT, "too many work units (%lld)", static_cast<long long>(U));
    const int sms = sm_count();
    if (ws.grid_ctas < 0 || (ws.grid_ctas > 0 && sms > 0 && ws.grid_ctas > sms))
        return fail(FDS_ERR_INVALID_ARGUMENT, "grid_ctas must be in [0, %d] (got %d)", sms, ws.grid_ctas);
    if (ws.ptr != nullptr && (reinterpret_cast<uintptr_t>(ws.ptr) & 255u) != 0)
        return fail(FDS_ERR_INVALID_ARGUMENT, "workspace must be 256-byte aligned");
    const Plan plan = plan_schedule(batch, p.heads, p.seq_len, p.kv_len != nullptr, ws.ptr != nullptr, ws.bytes,
                                    ws.grid_ctas, sms);
    p.n_units = static_cast<int32_t>(U);
    p.whole_ctas = static_cast<int32_t>(plan.whole);
    p.pieces = static_cast<int32_t>(plan.pieces);
    p.parts = nullptr;
    p.counts = nullptr;
    if (plan.pieces > 0) {
        char* base = static_cast<char*>(ws.ptr);
        p.counts = reinterpret_cast<uint32_t*>(base);
        p.parts = reinterpret_cast<float*>(base + kWsSlotsOffset);
    }
    e = launch_pdl(kern, dim3(static_cast<unsigned>(plan.grid)), dim3(fds::kThreads), fds::Smem::alloc, stream, mq, mk,
                   mv, mr, p);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return fail(FDS_ERR_CUDA, "attention launch: %s", cudaGetErrorString(e));
    return FDS_OK;
}

int check_common(const void* qkv, int64_t qkv_row_stride, const void* out, int64_t out_row_stride, int batch,
                 int heads, int seq_len, int head_dim, int dtype) {
    if (qkv == nullptr || out == nullptr) return fail(FDS_ERR_INVALID_ARGUMENT, "null qkv/out pointer");
    if (head_dim != 64) return fail(FDS_ERR_INVALID_ARGUMENT, "head_dim must be 64 (got %d)", head_dim);
    if (dtype != FDS_DTYPE_FP16 && dtype != FDS_DTYPE_BF16)
        return fail(FDS_ERR_INVALID_ARGUMENT, "dtype must be FDS_DTYPE_FP16 or FDS_DTYPE_BF16 (got %d)", dtype);
    if (batch < 1 || heads < 1 || seq_len < 1)
        return fail(FDS_ERR_INVALID_ARGUMENT, "batch, heads and seq_len must be >= 1 (got %d, %d, %d)", batch, heads,
                    seq_len);
    if (static_cast<int64_t>(batch) * heads > 65535)
        return fail(FDS_ERR_INVALID_ARGUMENT, "batch * heads must be <= 65535 (got %lld)",
                    static_cast<long long>(batch) * heads);
    const int64_t hid = static_cast<int64_t>(heads) * 64;
    if (qkv_row_stride < 3 * hid)
        return fail(FDS_ERR_INVALID_ARGUMENT, "qkv row stride %lld < 3*heads*64 = %lld",
                    static_cast<long long>(qkv_row_stride), static_cast<long long>(3 * hid));
    if (qkv_row_stride % 8 != 0)
        return fail(FDS_ERR_INVALID_ARGUMENT, "qkv row stride must be a multiple of 8 elements (16 bytes)");
    if (out_row_stride < hid)
        return fail(FDS_ERR_INVALID_ARGUMENT, "out row stride %lld < heads*64 = %lld",
                    static_cast<long long>(out_row_stride), static_cast<long long>(hid));
    if (out_row_stride % 8 != 0)
        return fail(FDS_ERR_INVALID_ARGUMENT, "out row stride must be a multiple of 8 elements (16 bytes)");
    if (!aligned16(qkv) || !aligned16(out))
        return fail(FDS_ERR_INVALID_ARGUMENT, "qkv and out must be 16-byte aligned");
    return FDS_OK;
}

}  // namespace

int fds_detail::set_error(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

namespace {

// Clusters of two CTAs (the pair GEMM), with PDL like launch_pdl.
template <typename... KArgs, typename... Args>
cudaError_t launch_pair(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                        Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// The linear layers' tensor maps: A, W, the output, and the RoPE epilogue's
// cos / sin tables (copies of the output map for the other epilogues).
struct GemmMaps {
    CUtensorMap a, b, out, cos, sin;
};

template <typename T, int BN, int kEpi, bool kPair>
int launch_gemm(const GemmMaps& m, const fds::gemm::Params& p, int grid, cudaStream_t stream) {
    auto kern = fds::gemm::gemm_kernel<T, BN, kEpi, kPair>;
    constexpr int smem = fds::gemm::Smem<BN, kPair, kEpi == fds::gemm::kRope>::alloc;
    static std::atomic<uint64_t> smem_set{0};
    cudaError_t e = set_smem_once(kern, smem, smem_set);
    if (e != cudaSuccess) return fail(FDS_ERR_CUDA, "cudaFuncSetAttribute(gemm): %s", cudaGetErrorString(e));
    const dim3 g(static_cast<unsigned>(grid)), b(fds::gemm::kThreads);
    e = kPair ? launch_pair(kern, g, b, smem, stream, m.a, m.b, m.out, m.cos, m.sin, p)
              : launch_pdl(kern, g, b, smem, stream, m.a, m.b, m.out, m.cos, m.sin, p);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return fail(FDS_ERR_CUDA, "linear launch: %s", cudaGetErrorString(e));
    return FDS_OK;
}

template <typename T, int BN, bool kPair>
int launch_gemm_epi(int epi, const GemmMaps& m, const fds::gemm::Params& p, int grid, cudaStream_t stream) {
    switch (epi) {
        case FDS_EPILOGUE_STORE: return launch_gemm<T, BN, fds::gemm::kStore, kPair>(m, p, grid, stream);
        case FDS_EPILOGUE_ROPE: return launch_gemm<T, BN, fds::gemm::kRope, kPair>(m, p, grid, stream);
        default: return launch_gemm<T, BN, fds::gemm::kAccum, kPair>(m, p, grid, stream);
    }
}

template <typename T>
int launch_gemm_shape(int bn, bool pair, int epi, const GemmMaps& m, const fds::gemm::Params& p, int grid,
                      cudaStream_t stream) {
    if (pair)
        return bn == 256 ? launch_gemm_epi<T, 256, true>(epi, m, p, grid, stream)
                         : launch_gemm_epi<T, 128, true>(epi, m, p, grid, stream);
    return bn == 256 ? launch_gemm_epi<T, 256, false>(epi, m, p, grid, stream)
                     : launch_gemm_epi<T, 128, false>(epi, m, p, grid, stream);
}

// How many CTA pairs of the pair GEMM can be resident at once on the current
// device (clusters must sit within one GPC, so this can be below SMs / 2);
// cached per device. 0 if it cannot be queried.
int max_pairs() {
    static std::atomic<int> cached[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    int n = cached[dev].load(std::memory_order_relaxed);
    if (n == 0) {
        auto kern = fds::gemm::gemm_kernel<__half, 256, fds::gemm::kStore, true>;
        constexpr int smem = fds::gemm::Smem<256, true>::alloc;
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return 0;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(2);
        cfg.blockDim = dim3(fds::gemm::kThreads);
        cfg.dynamicSmemBytes = smem;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
            cudaGetLastError();
            return 0;
        }
        cached[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

// Output tile width: 256 columns (more reuse of each A tile) unless n is not a
// multiple of 256 or 128-column tiles fill the last wave of tiles over the
// launched CTAs (pairs) clearly better (measured at n = 1024, m = 6000).
int choose_bn(int64_t m, int64_t n, int64_t units, int tile_m) {
    if (n % 256 != 0) return 128;
    const int64_t mt = (m + tile_m - 1) / tile_m;
    const auto fill = [&](int64_t bn) {
        const int64_t tiles = mt * (n / bn);
        const int64_t waves = (tiles + units - 1) / units;
        return static_cast<double>(tiles) / static_cast<double>(waves * units);
    };
    return fill(128) > fill(256) + 0.1 ? 128 : 256;
}

}  // namespace

extern "C" {

int fds_abi_version(void) { return FDS_ABI_VERSION; }

const char* fds_last_error(void) { return g_last_error.c_str(); }

int fds_attn_smem_bytes(void) { return fds::Smem::alloc; }

int64_t fds_attn_workspace_bytes(int32_t grid_ctas) {
    int64_t G = grid_ctas;
    if (G <= 0) {
        G = sm_count();
        if (G <= 0) {
            fail(FDS_ERR_CUDA, "cannot query the SM count of the current device");
            return 0;
        }
    }
    return ws_bytes_for(G);
}

int fds_attn_schedule(int32_t batch, int32_t heads, int32_t seq_len, int32_t has_kv_len, int64_t workspace_bytes,
                      int32_t grid_ctas, int64_t* out) {
    if (out == nullptr || batch < 1 || heads < 1 || seq_len < 1 || grid_ctas < 0)
        return fail(FDS_ERR_INVALID_ARGUMENT, "fds_attn_schedule: invalid arguments");
    int64_t sms = 0;
    if (grid_ctas == 0 && workspace_bytes > 0) {
        sms = sm_count();
        if (sms <= 0) return fail(FDS_ERR_CUDA, "cannot query the SM count of the current device");
    }
    const Plan plan = plan_schedule(batch, heads, seq_len, has_kv_len != 0, workspace_bytes > 0, workspace_bytes,
                                    grid_ctas, sms);
    out[0] = plan.grid;
    out[1] = plan.whole;
    out[2] = plan.pieces;
    return ok();
}

int fds_flexrel_attn_fwd(const FdsFlexRelArgs* a, void* stream) {
    if (a == nullptr) return fail(FDS_ERR_INVALID_ARGUMENT, "null args");
    int rc = check_common(a->qkv, a->qkv_row_stride, a->out, a->out_row_stride, a->batch, a->heads, a->seq_len,
                          a->head_dim, a->dtype);
    if (rc != FDS_OK) return rc;
    if (a->rel == nullptr || !aligned16(a->rel))
        return fail(FDS_ERR_INVALID_ARGUMENT, "rel must be a 16-byte aligned [73, 64] table");
    if (!(a->scale > 0.f)) return fail(FDS_ERR_INVALID_ARGUMENT, "scale must be > 0");
    if ((rc = check_device()) != FDS_OK) return rc;

    CUtensorMap mqkv, mrel;
    const int64_t hid = static_cast<int64_t>(a->heads) * 64;
    if ((rc = make_rows_map(&mqkv, a->qkv, a->dtype, 3 * hid, a->seq_len, a->batch, a->qkv_row_stride,
                            fds::kBlockM)) != FDS_OK)
        return rc;
    if ((rc = make_rel_map(&mrel, a->rel, a->dtype)) != FDS_OK) return rc;

    fds::AttnParams p{};
    p.out = a->out;
    p.out_stride = a->out_row_stride;
    p.kv_len = a->kv_len;
    p.status = a->status;
    p.status_host = a->status_host;
    p.timeout_ns = a->timeout_ns;
    p.heads = a->heads;
    p.seq_len = a->seq_len;
    p.q_x0 = 0;
    p.k_x0 = static_cast<int32_t>(hid);
    p.v_x0 = static_cast<int32_t>(2 * hid);
    p.scale_log2 = a->scale * 1.4426950408889634f;
    p.debug_flags = a->debug_flags;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const Workspace ws{a->workspace, a->workspace_bytes, a->grid_ctas};
    rc = a->dtype == FDS_DTYPE_FP16 ? launch_attn<__half, true>(mqkv, mqkv, mqkv, mrel, p, a->batch, ws, s)
                                    : launch_attn<__nv_bfloat16, true>(mqkv, mqkv, mqkv, mrel, p, a->batch, ws, s);
    return rc == FDS_OK ? ok() : rc;
}

int fds_flexrel_qr_attn_fwd(const FdsFlexRelQrArgs* a, void* stream) {
    if (a == nullptr) return fail(FDS_ERR_INVALID_ARGUMENT, "null args");
    if (a->q == nullptr || a->k == nullptr || a->v == nullptr || a->qr == nullptr || a->out == nullptr)
        return fail(FDS_ERR_INVALID_ARGUMENT, "null q/k/v/qr/out pointer");
    if (a->head_dim != 64) return fail(FDS_ERR_INVALID_ARGUMENT, "head_dim must be 64 (got %d)", a->head_dim);
    if (a->dtype != FDS_DTYPE_FP16 && a->dtype != FDS_DTYPE_BF16)
        return fail(FDS_ERR_INVALID_ARGUMENT, "dtype must be FDS_DTYPE_FP16 or FDS_DTYPE_BF16 (got %d)", a->dtype);
    if (a->batch < 1 || a->heads < 1 || a->seq_len < 1)
        return fail(FDS_ERR_INVALID_ARGUMENT, "batch, heads and seq_len must be >= 1 (got %d, %d, %d)", a->batch,
                    a->heads, a->seq_len);
    if (static_cast<int64_t>(a->batch) * a->heads > 65535)
        return fail(FDS_ERR_INVALID_ARGUMENT, "batch * heads must be <= 65535");
    if (!aligned16(a->q) || !aligned16(a->k) || !aligned16(a->v) || !aligned16(a->out))
        return fail(FDS_ERR_INVALID_ARGUMENT, "q, k, v and out must be 16-byte aligned");
    if ((reinterpret_cast<uintptr_t>(a->qr) & 1u) != 0)
        return fail(FDS_ERR_INVALID_ARGUMENT, "qr must be 2-byte aligned");
    if (!(a->scale > 0.f)) return fail(FDS_ERR_INVALID_ARGUMENT, "scale must be > 0");
    int rc = check_device();
    if (rc != FDS_OK) return rc;

    const int64_t hid = static_cast<int64_t>(a->heads) * 64;
    CUtensorMap mq, mk, mv;
    if (a->heads_last) {
        // rows (b, t) of heads * 64 columns
        if ((rc = make_rows_map(&mq, a->q, a->dtype, hid, a->seq_len, a->batch, hid, fds::kBlockM)) != FDS_OK) return rc;
        if ((rc = make_rows_map(&mk, a->k, a->dtype, hid, a->seq_len, a->batch, hid, fds::kBlockM)) != FDS_OK) return rc;
        if ((rc = make_rows_map(&mv, a->v, a->dtype, hid, a->seq_len, a->batch, hid, fds::kBlockM)) != FDS_OK) return rc;
    } else {
        // rows t of 64 columns per (b, h): the map's third coordinate is b * heads + h
        const int64_t bh = static_cast<int64_t>(a->batch) * a->heads;
        if ((rc = make_rows_map(&mq, a->q, a->dtype, 64, a->seq_len, bh, 64, fds::kBlockM)) != FDS_OK) return rc;
        if ((rc = make_rows_map(&mk, a->k, a->dtype, 64, a->seq_len, bh, 64, fds::kBlockM)) != FDS_OK) return rc;
        if ((rc = make_rows_map(&mv, a->v, a->dtype, 64, a->seq_len, bh, 64, fds::kBlockM)) != FDS_OK) return rc;
    }
    fds::AttnParams p{};
    p.out = a->out;
    p.out_stride = a->heads_last ? hid : 64;
    p.kv_len = a->kv_len;
    p.status = a->status;
    p.status_host = a->status_host;
    p.timeout_ns = a->timeout_ns;
    p.heads = a->heads;
    p.seq_len = a->seq_len;
    p.q_x0 = p.k_x0 = p.v_x0 = 0;
    p.scale_log2 = a->scale * 1.4426950408889634f;
    p.debug_flags = a->debug_flags;
    p.qr = a->qr;
    p.heads_in_z = a->heads_last ? 0 : 1;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const Workspace ws{a->workspace, a->workspace_bytes, a->grid_ctas};
    // map_r is not read when qr comes from global memory
    rc = a->dtype == FDS_DTYPE_FP16 ? launch_attn<__half, true, true>(mq, mk, mv, mq, p, a->batch, ws, s)
                                    : launch_attn<__nv_bfloat16, true, true>(mq, mk, mv, mq, p, a->batch, ws, s);
    return rc == FDS_OK ? ok() : rc;
}

static int launch_rope(const void* qkv, int64_t qkv_row_stride, const float* cos_t, const float* sin_t, void* dq,
                       void* dk, void* dv, int64_t dst_stride, int rows, int seq_len, int heads, int dtype,
                       cudaStream_t s) {
    const int parts = dv != nullptr ? 3 : 2;
    const int64_t total = static_cast<int64_t>(rows) * heads * parts * 4;
    const int threads = 256;
    const int64_t blocks = (total + threads - 1) / threads;
    if (blocks > 0x7fffffffLL) return fail(FDS_ERR_INVALID_ARGUMENT, "rope: too many rows");
    const dim3 grid(static_cast<unsigned>(blocks)), block(threads);
    cudaError_t e;
    if (dtype == FDS_DTYPE_FP16)
        e = launch_pdl(fds::rope_rotate_kernel<__half>, grid, block, 0, s, static_cast<const __half*>(qkv),
                       qkv_row_stride, cos_t, sin_t, static_cast<__half*>(dq), static_cast<__half*>(dk),
                       static_cast<__half*>(dv), dst_stride, rows, seq_len, heads);
    else
        e = launch_pdl(fds::rope_rotate_kernel<__nv_bfloat16>, grid, block, 0, s,
                       static_cast<const __nv_bfloat16*>(qkv), qkv_row_stride, cos_t, sin_t,
                       static_cast<__nv_bfloat16*>(dq), static_cast<__nv_bfloat16*>(dk),
                       static_cast<__nv_bfloat16*>(dv), dst_stride, rows, seq_len, heads);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) return fail(FDS_ERR_CUDA, "rope launch: %s", cudaGetErrorString(e));
    return FDS_OK;
}

int fds_rope_attn_fwd(const FdsRopeArgs* a, void* stream) {
    if (a == nullptr) return fail(FDS_ERR_INVALID_ARGUMENT, "null args");
    int rc = check_common(a->qkv, a->qkv_row_stride, a->out, a->out_row_stride, a->batch, a->heads, a->seq_len,
                          a->head_dim, a->dtype);
    if (rc != FDS_OK) return rc;
    if (!a->qk_rotated) {
        if (a->cos == nullptr || a->sin == nullptr || !aligned16(a->cos) || !aligned16(a->sin))
            return fail(FDS_ERR_INVALID_ARGUMENT, "cos/sin must be 16-byte aligned fp32 [>= seq_len, 64] tables");
        if (a->qk_scratch == nullptr || !aligned16(a->qk_scratch))
            return fail(FDS_ERR_INVALID_ARGUMENT,
                        "qk_scratch must be a 16-byte aligned [batch*seq_len, 2*heads*64] buffer");
    }
    if (!(a->scale > 0.f)) return fail(FDS_ERR_INVALID_ARGUMENT, "scale must be > 0");
    if ((rc = check_device()) != FDS_OK) return rc;

    const int64_t hid = static_cast<int64_t>(a->heads) * 64;
    const int64_t rows = static_cast<int64_t>(a->batch) * a->seq_len;
    if (rows > 0x7fffffffLL) return fail(FDS_ERR_INVALID_ARGUMENT, "batch*seq_len too large");
    CUtensorMap mqk, mv;
    if ((rc = make_rows_map(&mv, a->qkv, a->dtype, 3 * hid, a->seq_len, a->batch, a->qkv_row_stride, fds::kBlockM)) !=
        FDS_OK)
        return rc;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (a->qk_rotated) {
        mqk = mv;  // q | k read rotated straight from qkv
    } else {
        if ((rc = make_rows_map(&mqk, a->qk_scratch, a->dtype, 2 * hid, a->seq_len, a->batch, 2 * hid,
                                fds::kBlockM)) != FDS_OK)
            return rc;
        char* scratch = static_cast<char*>(a->qk_scratch);
        rc = launch_rope(a->qkv, a->qkv_row_stride, a->cos, a->sin, scratch, scratch + hid * 2, nullptr, 2 * hid,
                         static_cast<int>(rows), a->seq_len, a->heads, a->dtype, s);
        if (rc != FDS_OK) return rc;
    }

    fds::AttnParams p{};
    p.out = a->out;
    p.out_stride = a->out_row_stride;
    p.kv_len = nullptr;
    p.status = a->status;
    p.status_host = a->status_host;
    p.timeout_ns = a->timeout_ns;
    p.heads = a->heads;
    p.seq_len = a->seq_len;
    p.q_x0 = 0;
    p.k_x0 = static_cast<int32_t>(hid);
    p.v_x0 = static_cast<int32_t>(2 * hid);
    p.scale_log2 = a->scale * 1.4426950408889634f;
    p.debug_flags = a->debug_flags;
    const Workspace ws{a->workspace, a->workspace_bytes, a->grid_ctas};
    rc = a->dtype == FDS_DTYPE_FP16 ? launch_attn<__half, false>(mqk, mqk, mv, mqk, p, a->batch, ws, s)
                                    : launch_attn<__nv_bfloat16, false>(mqk, mqk, mv, mqk, p, a->batch, ws, s);
    return rc == FDS_OK ? ok() : rc;
}

int fds_linear_fwd(const FdsLinearArgs* a, void* stream) {
    if (a == nullptr) return fail(FDS_ERR_INVALID_ARGUMENT, "null args");
    if (a->a == nullptr || a->w == nullptr || a->out == nullptr)
        return fail(FDS_ERR_INVALID_ARGUMENT, "null a/w/out pointer");
    if (a->dtype != FDS_DTYPE_FP16 && a->dtype != FDS_DTYPE_BF16)
        return fail(FDS_ERR_INVALID_ARGUMENT, "dtype must be FDS_DTYPE_FP16 or FDS_DTYPE_BF16 (got %d)", a->dtype);
    if (a->epilogue < FDS_EPILOGUE_STORE || a->epilogue > FDS_EPILOGUE_ACCUMULATE_F32)
        return fail(FDS_ERR_INVALID_ARGUMENT, "unknown epilogue %d", a->epilogue);
    if (a->m < 1 || a->n < 1 || a->k < 1) return fail(FDS_ERR_INVALID_ARGUMENT, "m, n, k must be >= 1");
    if (a->k % 64 != 0) return fail(FDS_ERR_INVALID_ARGUMENT, "k must be a multiple of 64 (got %d)", a->k);
    if (a->n % 128 != 0) return fail(FDS_ERR_INVALID_ARGUMENT, "n must be a multiple of 128 (got %d)", a->n);
    if (a->a_row_stride < a->k || a->a_row_stride % 8 != 0 || a->w_row_stride < a->k || a->w_row_stride % 8 != 0)
        return fail(FDS_ERR_INVALID_ARGUMENT, "a / w row strides must be >= k and multiples of 8 elements");
    const bool f32_out = a->epilogue == FDS_EPILOGUE_ACCUMULATE_F32;
    if (a->out_row_stride < a->n || a->out_row_stride % (f32_out ? 4 : 8) != 0)
        return fail(FDS_ERR_INVALID_ARGUMENT, "out row stride must be >= n and 16-byte aligned rows");
    if (!aligned16(a->a) || !aligned16(a->w) || !aligned16(a->out) || (a->bias != nullptr && !aligned16(a->bias)))
        return fail(FDS_ERR_INVALID_ARGUMENT, "a, w, bias and out must be 16-byte aligned");
    if (a->epilogue == FDS_EPILOGUE_ROPE) {
        if (a->cos == nullptr || a->sin == nullptr || !aligned16(a->cos) || !aligned16(a->sin))
            return fail(FDS_ERR_INVALID_ARGUMENT, "cos/sin must be 16-byte aligned fp32 [>= seq_len, 64] tables");
        if (a->seq_len < 1) return fail(FDS_ERR_INVALID_ARGUMENT, "seq_len must be >= 1");
        if (a->rope_cols < 0 || a->rope_cols > a->n || a->rope_cols % 64 != 0)
            return fail(FDS_ERR_INVALID_ARGUMENT, "rope_cols must be a multiple of 64 in [0, n]");
    }
    int rc = check_device();
    if (rc != FDS_OK) return rc;
    const int sms = sm_count();
    if (a->grid_ctas < 0 || (a->grid_ctas > 0 && sms > 0 && a->grid_ctas > sms))
        return fail(FDS_ERR_INVALID_ARGUMENT, "grid_ctas must be in [0, %d] (got %d)", sms, a->grid_ctas);
    if (a->cta_pair < FDS_GEMM_AUTO || a->cta_pair > FDS_GEMM_PAIR)
        return fail(FDS_ERR_INVALID_ARGUMENT, "cta_pair must be FDS_GEMM_AUTO, FDS_GEMM_SINGLE or FDS_GEMM_PAIR");
    int64_t ctas = a->grid_ctas > 0 ? a->grid_ctas : (sms > 0 ? sms : 148);
    // CTA pairs (256-row tiles) unless asked otherwise, there is only one
    // 128-row tile of output rows, k is short (below 512 the pair's extra set-up
    // and cluster barriers are not repaid: measured at m = 6000), or no pair can
    // be placed
    bool pair = a->cta_pair == FDS_GEMM_PAIR || (a->cta_pair == FDS_GEMM_AUTO && a->m > fds::gemm::kBM && a->k >= 512);
    if (pair) {
        const int64_t pairs = std::min<int64_t>(ctas / 2, max_pairs());
        if (pairs < 1) {
            if (a->cta_pair == FDS_GEMM_PAIR)
                return fail(FDS_ERR_INVALID_ARGUMENT, "no CTA pair can be launched (grid_ctas %d)", a->grid_ctas);
            pair = false;
        } else {
            ctas = 2 * pairs;
        }
    }
    const int tile_m = pair ? 2 * fds::gemm::kBM : fds::gemm::kBM;
    const int64_t units = pair ? ctas / 2 : ctas;
    const int bn = choose_bn(a->m, a->n, units, tile_m);
    const int64_t tiles = static_cast<int64_t>((a->m + tile_m - 1) / tile_m) * (a->n / bn);
    if (tiles > 0x7fffffffLL) return fail(FDS_ERR_INVALID_ARGUMENT, "too many tiles");

    GemmMaps maps;
    if ((rc = make_matrix_map(&maps.a, a->a, a->dtype, a->k, a->m, a->a_row_stride, fds::gemm::kBM)) != FDS_OK)
        return rc;
    if ((rc = make_matrix_map(&maps.b, a->w, a->dtype, a->k, a->n, a->w_row_stride, pair ? bn / 2 : bn)) != FDS_OK)
        return rc;
    if ((rc = make_out_map(&maps.out, a->out, f32_out, a->dtype, a->n, a->m, a->out_row_stride)) != FDS_OK) return rc;
    if (a->epilogue == FDS_EPILOGUE_ROPE) {
        if ((rc = make_rope_table_map(&maps.cos, a->cos, a->seq_len)) != FDS_OK) return rc;
        if ((rc = make_rope_table_map(&maps.sin, a->sin, a->seq_len)) != FDS_OK) return rc;
    } else {
        maps.cos = maps.out;
        maps.sin = maps.out;
    }
    fds::gemm::Params p{};
    p.bias = a->bias;
    p.cos_t = a->cos;
    p.sin_t = a->sin;
    p.status = a->status;
    p.status_host = a->status_host;
    p.timeout_ns = a->timeout_ns;
    p.m = a->m;
    p.n = a->n;
    p.k = a->k;
    p.seq_len = a->seq_len;
    p.rope_cols = a->epilogue == FDS_EPILOGUE_ROPE ? a->rope_cols : 0;
    p.tiles_n = a->n / bn;
    p.tiles = static_cast<int32_t>(tiles);
    const int grid = static_cast<int>((tiles < units ? tiles : units) * (pair ? 2 : 1));
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    rc = a->dtype == FDS_DTYPE_FP16 ? launch_gemm_shape<__half>(bn, pair, a->epilogue, maps, p, grid, s)
                                    : launch_gemm_shape<__nv_bfloat16>(bn, pair, a->epilogue, maps, p, grid, s);
    return rc == FDS_OK ? ok() : rc;
}

int fds_rope_split(const void* qkv, int64_t qkv_row_stride, const float* cos_t, const float* sin_t, void* out,
                   int32_t rows, int32_t seq_len, int32_t heads, int32_t head_dim, int32_t dtype, void* stream) {
    if (qkv == nullptr || out == nullptr || cos_t == nullptr || sin_t == nullptr)
        return fail(FDS_ERR_INVALID_ARGUMENT, "null pointer");
    if (head_dim != 64) return fail(FDS_ERR_INVALID_ARGUMENT, "head_dim must be 64 (got %d)", head_dim);
    if (dtype != FDS_DTYPE_FP16 && dtype != FDS_DTYPE_BF16)
        return fail(FDS_ERR_INVALID_ARGUMENT, "dtype must be FDS_DTYPE_FP16 or FDS_DTYPE_BF16");
    if (rows < 0 || seq_len < 1 || heads < 1)
        return fail(FDS_ERR_INVALID_ARGUMENT, "rows >= 0, seq_len >= 1, heads >= 1 required");
    const int64_t hid = static_cast<int64_t>(heads) * 64;
    if (qkv_row_stride < 3 * hid || qkv_row_stride % 8 != 0)
        return fail(FDS_ERR_INVALID_ARGUMENT, "qkv row stride must be >= 3*heads*64 and a multiple of 8");
    if (!aligned16(qkv) || !aligned16(out) || !aligned16(cos_t) || !aligned16(sin_t))
        return fail(FDS_ERR_INVALID_ARGUMENT, "all buffers must be 16-byte aligned");
    if (rows == 0) return ok();
    int rc = check_device();
    if (rc != FDS_OK) return rc;
    char* o = static_cast<char*>(out);
    const int64_t plane = static_cast<int64_t>(rows) * hid * 2;
    rc = launch_rope(qkv, qkv_row_stride, cos_t, sin_t, o, o + plane, o + 2 * plane, hid, rows, seq_len, heads, dtype,
                     static_cast<cudaStream_t>(stream));
    return rc == FDS_OK ? ok() : rc;
}

}  // extern "C"
