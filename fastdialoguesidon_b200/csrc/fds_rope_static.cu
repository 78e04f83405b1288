// fds_rope_static.cu - fds_rope_attn_fwd_static: the DiT RoPE attention without
// any device allocation by the caller or by this library.
//
// Who needs it: callers that must not allocate device memory once they are
// running -- an inference-engine plugin's enqueue (it only gets the
// workspace it declared up front), a real-time audio callback, or a serving
// loop that fixes its memory plan at start-up. cudaMalloc can implicitly
// synchronise the device and can fail under fragmentation, which such callers
// cannot afford in their hot loop. The regular fds_rope_attn_fwd needs a
// caller-provided [rows, 2*heads*64] scratch buffer for the rotated q | k; this
// variant keeps that buffer in a statically sized device array instead.
//
// Limits and rules:
//   * The array holds FDS_ROPE_STATIC_SCRATCH_BYTES (20 MiB): rows * 2 * heads
//     * 64 elements of the operand type must fit (one 120 s window of the DiT
//     head, 6000 x 1536 fp16 = 18.4 MB, does). Larger calls are rejected with
//     FDS_ERR_INVALID_ARGUMENT before anything is launched.
//   * Every GPU that loads the array holds the 20 MiB until the process exits
//     (with CUDA's default lazy module loading, a GPU loads it on the first
//     fds_rope_attn_fwd_static call made on it).
//   * The first call on a device looks up the array's device address
//     (cudaGetSymbolAddress, with that device current) and caches it; make
//     that first call before any stream capture. The cached address does not
//     survive cudaDeviceReset (the device's module is unloaded with the
//     context); do not call this entry point again on a device after a reset.
//   * The stream must belong to the current device (checked).
//   * All calls share the one array and it keeps the previous call's contents:
//     calls whose kernels overlap on the GPU (different streams, or different
//     graphs replayed concurrently) race on it. Nothing in it needs clearing:
//     the RoPE pass overwrites every scratch element the attention then reads.
#include <cuda_runtime.h>

#include <mutex>

#include "capi_internal.h"
#include "fds_b200.h"

namespace {

// The host-side name of this array is only a stand-in: kernels receive the
// device address obtained from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_rope_scratch[FDS_ROPE_STATIC_SCRATCH_BYTES];

std::mutex g_lock;
void* g_scratch_ptr[64];  // per-device address of g_rope_scratch, filled on first use

}  // namespace

extern "C" FDS_API int fds_rope_attn_fwd_static(const FdsRopeArgs* args, void* stream) {
    using fds_detail::set_error;
    if (args == nullptr) return set_error(FDS_ERR_INVALID_ARGUMENT, "null args");
    if (args->qk_scratch != nullptr)
        return set_error(FDS_ERR_INVALID_ARGUMENT,
                         "fds_rope_attn_fwd_static uses its own static scratch: pass qk_scratch = NULL");
    if (args->dtype != FDS_DTYPE_FP16 && args->dtype != FDS_DTYPE_BF16)
        return set_error(FDS_ERR_INVALID_ARGUMENT, "dtype must be FDS_DTYPE_FP16 or FDS_DTYPE_BF16");
    if (args->batch < 1 || args->seq_len < 1 || args->heads < 1)
        return set_error(FDS_ERR_INVALID_ARGUMENT, "batch, heads and seq_len must be >= 1");
    const long long need = static_cast<long long>(args->batch) * args->seq_len * 2LL * args->heads * 64LL * 2LL;
    if (need > static_cast<long long>(FDS_ROPE_STATIC_SCRATCH_BYTES))
        return set_error(FDS_ERR_INVALID_ARGUMENT,
                         "rotated q|k needs %lld bytes (batch*seq_len*2*heads*64 x 2 B) but the static scratch "
                         "holds %lld; use fds_rope_attn_fwd with a caller-provided scratch",
                         need, static_cast<long long>(FDS_ROPE_STATIC_SCRATCH_BYTES));
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return set_error(FDS_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= 64) return set_error(FDS_ERR_UNSUPPORTED_DEVICE, "device index %d out of range", dev);
    // the array's address belongs to the current device: a stream of another
    // device would run the kernels against that device's memory
    if (stream != nullptr) {
        int stream_dev = -1;
        e = cudaStreamGetDevice(static_cast<cudaStream_t>(stream), &stream_dev);
        if (e != cudaSuccess) return set_error(FDS_ERR_CUDA, "cudaStreamGetDevice: %s", cudaGetErrorString(e));
        if (stream_dev != dev)
            return set_error(FDS_ERR_INVALID_ARGUMENT,
                             "the stream belongs to device %d but device %d is current; make the stream's device "
                             "current before calling fds_rope_attn_fwd_static",
                             stream_dev, dev);
    }
    void* ptr = nullptr;
    {
        std::lock_guard<std::mutex> guard(g_lock);
        if (g_scratch_ptr[dev] == nullptr) {
            void* p = nullptr;
            e = cudaGetSymbolAddress(&p, g_rope_scratch);
            if (e != cudaSuccess || p == nullptr)
                return set_error(FDS_ERR_CUDA, "cudaGetSymbolAddress(static scratch): %s", cudaGetErrorString(e));
            g_scratch_ptr[dev] = p;
        }
        ptr = g_scratch_ptr[dev];
    }
    FdsRopeArgs a = *args;
    a.qk_scratch = ptr;
    return fds_rope_attn_fwd(&a, stream);
}
