/*
 * fds_b200.h - C ABI of the B200 (sm_100a) attention hot path of FastDialogueSidon.
 *
 * Plain C: device pointers, sizes and a stream handle (a cudaStream_t passed as
 * void*), no torch or C++ types, so that ctypes / cffi / any FFI can bind it.
 * Every entry point launches on the given stream, never synchronises, never
 * allocates device memory, and returns FDS_OK or an error code before any
 * launch when an argument is invalid (fds_last_error() then holds a message).
 * Kernels are launched with programmatic stream serialization: a launch may
 * place its CTAs while the previous kernel in the stream drains, and they wait
 * for that kernel to complete before touching memory, so stream order holds.
 * FDS_PDL=0 in the environment launches in plain stream order instead.
 *
 * Numerics: fp16 or bf16 operands, fp32 accumulation, fp32 online softmax in
 * log2 units, P rounded to the operand type for the P.V product (the same
 * rounding points as the reference's Triton kernels).
 *
 * Work is cut into units of 256 query rows of one (window, head), one per CTA.
 * Workspace (optional, both attention entry points): with a workspace of at
 * least fds_attn_workspace_bytes(grid_ctas) bytes, zero-filled once before its
 * first use, the kernels may split the last wave: when whole units would leave
 * part of it idle, the units of the last wave are cut into one piece per SM
 * (grid_ctas = G pieces; 0 = one per SM), and the parts of a cut unit are
 * merged through the workspace by whichever part finishes last (no CTA waits
 * for another). Calls leave the workspace ready for the next call (no reset
 * between calls or graph replays; zero it again after a call that reported a
 * timeout); calls that may overlap on the GPU (different streams) need
 * different workspaces. NULL keeps one unit per CTA. The split is used only
 * without kv_len, and only where it shortens the launch (or always, when
 * grid_ctas > 0 asks for it and the shape allows it); fds_attn_schedule tells.
 *
 * Status mirror (optional): a kernel whose bounded wait expires ORs an
 * FDS_STATUS_* bit into the device word *status and also stores its bits into
 * *status_host, a word of mapped pinned host memory (cudaHostAlloc /
 * cudaMallocHost; with unified addressing its host pointer is also its device
 * address). The caller can then notice a timeout by reading that host word at
 * any time, e.g. before its next call, without synchronising the device. The
 * store is plain (not atomic across the PCIe link): concurrent failures may
 * leave only some of their bits, but never zero.
 *
 * Per-device state the library caches on first use (kernel shared-memory
 * limits, the co-resident CTA-pair count, the static scratch address) does
 * not survive cudaDeviceReset of that device.
 */
#ifndef FDS_B200_H
#define FDS_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FDS_ABI_VERSION 4

#if defined(_WIN32)
#define FDS_API __declspec(dllexport)
#else
#define FDS_API __attribute__((visibility("default")))
#endif

/* return codes */
#define FDS_OK 0
#define FDS_ERR_INVALID_ARGUMENT 1
#define FDS_ERR_UNSUPPORTED_DEVICE 2
#define FDS_ERR_CUDA 3
#define FDS_ERR_TENSOR_MAP 4

/* operand types */
#define FDS_DTYPE_FP16 0
#define FDS_DTYPE_BF16 1

/* bits written (atomicOr) into *status by a kernel whose bounded wait expired */
#define FDS_STATUS_TIMEOUT_LOAD 0x1    /* TMA producer waited too long for a free stage */
#define FDS_STATUS_TIMEOUT_MMA 0x2     /* MMA issuer waited too long for operands / P */
#define FDS_STATUS_TIMEOUT_SOFTMAX 0x4 /* softmax warps waited too long for S / O */
#define FDS_STATUS_TIMEOUT_DRAIN 0x8   /* in-flight copies or MMAs did not drain at exit */

/* debug flags (tests only): make the MMA issuer wait on a barrier that nothing
 * arrives on, so that the bounded-wait error path runs without a real hang. */
#define FDS_DEBUG_FORCE_TIMEOUT 0x1

/*
 * Encoder relative_key self-attention (w2v-BERT conformer layer):
 *   S[b,h,i,j] = (q_i . k_j + q_i . rel[clamp(j - i, -64, +8) + 64]) * scale
 *   O[b,i,h,:] = softmax_j(S[b,h,i,:]) . V        over keys j < kv_len[b]
 * qkv is [batch*seq_len, >= 3*heads*64] row-major, q | k | v column blocks at
 * column offsets 0, heads*64, 2*heads*64 (the fused QKV GEMM output).
 * Replaces: triton/src/fds_triton/kernels.py:422 flexrel_attention (and the
 * equivalent split path kernels.py:634 flexrel_attention_split).
 */
typedef struct FdsFlexRelArgs {
    const void* qkv;          /* device, dtype, [batch*seq_len, qkv_row_stride] */
    int64_t qkv_row_stride;   /* elements; multiple of 8, >= 3*heads*64 */
    const void* rel;          /* device, dtype, [73, 64] contiguous */
    void* out;                /* device, dtype, [batch*seq_len, out_row_stride] */
    int64_t out_row_stride;   /* elements; >= heads*64 */
    const int32_t* kv_len;    /* device [batch] valid key count per window, or NULL (= seq_len) */
    int32_t* status;          /* device word for bounded-wait errors, or NULL */
    int32_t batch;
    int32_t heads;
    int32_t seq_len;
    int32_t head_dim;         /* must be 64 */
    int32_t dtype;            /* FDS_DTYPE_* */
    float scale;              /* softmax scale on (qk + qr); the reference uses 1/sqrt(64) */
    int64_t timeout_ns;       /* bound on every in-kernel wait; <= 0 selects 2 s */
    int32_t debug_flags;      /* 0 in production */
    void* workspace;          /* device, zero-filled once; or NULL (see "Workspace" above) */
    int64_t workspace_bytes;
    int32_t grid_ctas;        /* pieces of a split last wave; 0 = one per SM */
    int32_t* status_host;     /* mapped pinned host word, or NULL (see "Status mirror" above) */
} FdsFlexRelArgs;

FDS_API int fds_flexrel_attn_fwd(const FdsFlexRelArgs* args, void* stream);

/*
 * The same relative_key attention in the TensorRT plugin's form: separate q, k,
 * v and the relative-key projections qr = q . rel^T (unscaled, as the graph's
 * MatMul produces them) as inputs, so the bias is read, not computed:
 *   S[b,h,i,j] = (q_i . k_j + qr[b,i,h,clamp(j - i, -64, +8) + 64]) * scale
 * Layouts (contiguous): heads_last = 1: q, k, v, out [batch, seq_len, heads, 64]
 * and qr [batch, seq_len, heads, 73] (the plugin's); heads_last = 0: [batch,
 * heads, seq_len, 64] and [batch, heads, seq_len, 73]. kv_len, scale, status,
 * timeout and workspace as in FdsFlexRelArgs.
 * Replaces: trt/src/fastdialoguesidon/flexrel_triton.py:749 flexrel_attention_qr
 * and the sidon::FlexRelAttnQR / FlexRelAttnQRD plugins (:902-1028), whose
 * kernel body is _flexrel_qr_body (:559).
 */
typedef struct FdsFlexRelQrArgs {
    const void* q;            /* device, dtype, see the layouts above */
    const void* k;
    const void* v;
    const void* qr;           /* device, dtype, [.., 73] */
    void* out;                /* device, dtype, q's layout */
    const int32_t* kv_len;    /* device [batch], or NULL */
    int32_t* status;          /* device word for bounded-wait errors, or NULL */
    int32_t* status_host;     /* mapped pinned host mirror, or NULL */
    int32_t batch;
    int32_t heads;
    int32_t seq_len;
    int32_t head_dim;         /* must be 64 */
    int32_t dtype;            /* FDS_DTYPE_* */
    int32_t heads_last;       /* 1: [batch, seq_len, heads, ..]; 0: [batch, heads, seq_len, ..] */
    float scale;              /* the plugin uses 1/sqrt(64) */
    int64_t timeout_ns;
    int32_t debug_flags;
    void* workspace;          /* as in FdsFlexRelArgs */
    int64_t workspace_bytes;
    int32_t grid_ctas;
} FdsFlexRelQrArgs;

FDS_API int fds_flexrel_qr_attn_fwd(const FdsFlexRelQrArgs* args, void* stream);

/*
 * DiT head RoPE self-attention (bidirectional, no bias, no mask):
 *   q' = q*cos[t] + rotate_half(q)*sin[t], k' likewise (rotate_half(x) = [-x2, x1]),
 *   O = softmax(q' k'^T * scale) V
 * cos/sin are fp32 tables [>= seq_len, 64] indexed by the frame index t.
 * qk_scratch receives the rotated q | k rows ([batch*seq_len, 2*heads*64], dtype):
 * K is reused by every query tile, so it is rotated once per call rather than
 * once per tile.
 * Replaces: triton/src/fds_triton/model.py:319-325 (kernels.py:476 rope_split +
 * F.scaled_dot_product_attention).
 */
typedef struct FdsRopeArgs {
    const void* qkv;          /* device, dtype, [batch*seq_len, qkv_row_stride] */
    int64_t qkv_row_stride;   /* elements; multiple of 8, >= 3*heads*64 */
    const float* cos;         /* device fp32 [>= seq_len, 64] contiguous */
    const float* sin;         /* device fp32 [>= seq_len, 64] contiguous */
    void* qk_scratch;         /* device, dtype, [batch*seq_len, 2*heads*64] contiguous */
    void* out;                /* device, dtype, [batch*seq_len, out_row_stride] */
    int64_t out_row_stride;   /* elements; >= heads*64 */
    int32_t* status;          /* device word for bounded-wait errors, or NULL */
    int32_t batch;
    int32_t heads;
    int32_t seq_len;
    int32_t head_dim;         /* must be 64 */
    int32_t dtype;            /* FDS_DTYPE_* */
    float scale;              /* the reference uses 1/sqrt(64) (SDPA default) */
    int64_t timeout_ns;
    int32_t debug_flags;
    void* workspace;          /* as in FdsFlexRelArgs */
    int64_t workspace_bytes;
    int32_t grid_ctas;
    int32_t* status_host;     /* as in FdsFlexRelArgs */
    int32_t qk_rotated;       /* non-zero: the q | k columns of qkv are rotated already (the
                                 FDS_EPILOGUE_ROPE output of fds_linear_fwd): no RoPE pass,
                                 cos / sin / qk_scratch unused (may be NULL) */
} FdsRopeArgs;

FDS_API int fds_rope_attn_fwd(const FdsRopeArgs* args, void* stream);

/*
 * RoPE split: out[0] = rot(q), out[1] = rot(k), out[2] = v as [3, batch*seq_len, heads*64].
 * Replaces: triton/src/fds_triton/kernels.py:476 rope_split (pos = token % seq_len).
 */
FDS_API int fds_rope_split(const void* qkv, int64_t qkv_row_stride, const float* cos, const float* sin,
                   void* out, int32_t rows, int32_t seq_len, int32_t heads, int32_t head_dim,
                   int32_t dtype, void* stream);

/*
 * Allocation-free variant of fds_rope_attn_fwd (no counterpart in the
 * reference): for callers that cannot allocate device memory while running
 * (an engine plugin's enqueue, a real-time callback, a serving loop with a
 * fixed memory plan). The rotated q | k live in a static device array of
 * FDS_ROPE_STATIC_SCRATCH_BYTES that every GPU loading it holds until exit
 * (lazy module loading: from the first call on that GPU); args->qk_scratch
 * must be NULL and batch*seq_len*2*heads*64
 * 16-bit values must fit in it (else FDS_ERR_INVALID_ARGUMENT). The first call
 * on a device resolves the array's address (make it before any stream
 * capture) and caches it; the cached address does not survive
 * cudaDeviceReset. The stream must belong to the current device. All calls
 * share the array: calls that overlap on the GPU race.
 */
#define FDS_ROPE_STATIC_SCRATCH_BYTES (20u * 1024u * 1024u)
FDS_API int fds_rope_attn_fwd_static(const FdsRopeArgs* args, void* stream);

/*
 * Linear layer on the tensor cores, D = A W^T with W in nn.Linear's [n, k]
 * layout, fp16 / bf16 operands, fp32 accumulation, and one epilogue:
 *   FDS_EPILOGUE_STORE          out[m, n] (dtype) = D + bias
 *   FDS_EPILOGUE_ROPE           out = D + bias rounded to dtype, then the DiT's
 *                               rotate-half RoPE (cos / sin fp32 [>= seq_len, 64],
 *                               position = row % seq_len) on every 64-column head
 *                               of columns [0, rope_cols), rounded again: the q | k
 *                               the attention reads, with no separate RoPE pass
 *   FDS_EPILOGUE_ACCUMULATE_F32 out[m, n] (fp32) += D (+ bias): the residual
 *                               update x += a W^T
 * k must be a multiple of 64 and n of 128; rows past m are not written.
 * Replaces: the projections around the attention, triton/src/fds_triton/model.py
 * :289 (qkv = linear(xn, qkv_w, qkv_b), encoder), :318 (DiT qkv, followed by
 * rope_split :319), :291 and accumulate :53-57 (x += ctx out_w^T into the fp32
 * residual).
 */
#define FDS_EPILOGUE_STORE 0
#define FDS_EPILOGUE_ROPE 1
#define FDS_EPILOGUE_ACCUMULATE_F32 2

/* FdsLinearArgs.cta_pair: AUTO uses 256-row tiles over clusters of two CTAs
 * when m > 128 and k >= 512 (each CTA loads its own 128 rows of a and half of
 * the tile's w rows; one tensor-core operation spans both SMs), else 128-row
 * tiles on one CTA each; SINGLE / PAIR force one of the two. Both give the
 * same result bit for bit. */
#define FDS_GEMM_AUTO 0
#define FDS_GEMM_SINGLE 1
#define FDS_GEMM_PAIR 2

typedef struct FdsLinearArgs {
    const void* a;            /* device, dtype, [m, a_row_stride] */
    int64_t a_row_stride;     /* elements; multiple of 8, >= k */
    const void* w;            /* device, dtype, [n, w_row_stride] */
    int64_t w_row_stride;     /* elements; multiple of 8, >= k */
    const void* bias;         /* device, dtype, [n], or NULL */
    void* out;                /* device, [m, out_row_stride]: dtype, or fp32 for ACCUMULATE_F32 */
    int64_t out_row_stride;   /* elements; multiple of 8 (4 for fp32), >= n */
    const float* cos;         /* FDS_EPILOGUE_ROPE only */
    const float* sin;
    int32_t* status;          /* device word for bounded-wait errors, or NULL */
    int32_t* status_host;     /* mapped pinned host mirror, or NULL */
    int32_t m;                /* rows of a and out */
    int32_t n;                /* rows of w, columns of out */
    int32_t k;                /* columns of a and w */
    int32_t dtype;            /* FDS_DTYPE_* of a, w, bias (and out, unless ACCUMULATE_F32) */
    int32_t epilogue;         /* FDS_EPILOGUE_* */
    int32_t seq_len;          /* FDS_EPILOGUE_ROPE: frames per window */
    int32_t rope_cols;        /* FDS_EPILOGUE_ROPE: multiple of 64, <= n */
    int64_t timeout_ns;       /* bound on every in-kernel wait; <= 0 selects 2 s */
    int32_t grid_ctas;        /* persistent CTAs; 0 = one per SM */
    int32_t cta_pair;         /* FDS_GEMM_*: tiles over CTA pairs (tcgen05 cta_group::2) or one CTA each */
} FdsLinearArgs;

FDS_API int fds_linear_fwd(const FdsLinearArgs* args, void* stream);

/* Version of this ABI (FDS_ABI_VERSION). */
FDS_API int fds_abi_version(void);

/* Message for the last error returned on this host thread ("" if none). */
FDS_API const char* fds_last_error(void);

/* Shared-memory bytes a CTA of the attention kernels requests (for diagnostics). */
FDS_API int fds_attn_smem_bytes(void);

/* Workspace bytes a split last wave of grid_ctas pieces needs (0 = one per SM
 * of the current device; returns 0 and sets the error message if the device
 * cannot be queried). */
FDS_API int64_t fds_attn_workspace_bytes(int32_t grid_ctas);

/* The launch layout the attention kernels would use (diagnostics, tests):
 * out[0] = CTAs, out[1] = CTAs holding one whole unit each, out[2] = pieces of
 * the split last wave (0: none). workspace_bytes = 0 means no workspace; the
 * device is queried only when grid_ctas = 0 and a workspace is given. */
FDS_API int fds_attn_schedule(int32_t batch, int32_t heads, int32_t seq_len, int32_t has_kv_len,
                              int64_t workspace_bytes, int32_t grid_ctas, int64_t* out);

#ifdef __cplusplus
}
#endif

#endif /* FDS_B200_H */
