"""Attention ops of the FastDialogueSidon hot path on B200 (sm_100a).

Drop-in for the attention half of ``triton/src/fds_triton/kernels.py``: the
same names, argument order, layouts, dtypes and "``out`` written in place when
given" contract, computed by the hand-written tcgen05 kernels behind the C ABI
in ``include/fds_b200.h``. There is one encoder kernel (no fused/split
dispatch), no autotuning, no host synchronisation and no allocation other than
``out`` (and the DiT's rotated-q|k scratch), so every call is safe inside
``torch.cuda.graph`` capture once the device has run one eager call.

Schedule: each (device, stream) gets one zero-filled workspace (about 31 MB on
a 148-SM B200) that lets the library split the last wave -- when whole
256-row units would leave part of it idle, its units are cut into one piece
per SM and the parts merged through the workspace. Calls on one stream are
ordered, so they share it safely. Workspaces are never allocated inside a CUDA
graph capture: the first eager call on a device also zero-fills two spare
workspaces (and waits for that fill once), and a capture on a stream that has
none takes a spare; with no spare left the captured call keeps one unit per
CTA. After a reported timeout (:func:`check_status`) the device's workspaces
are zero-filled again.

Errors: invalid arguments raise :class:`FdsError` before any launch. It
subclasses both ``AssertionError`` (what the reference's ``assert`` checks
raise, ``kernels.py:430, 641``) and ``RuntimeError``. A missing native library
or a non-CUDA tensor raises as well: there is no CPU fallback.

Bounded-wait timeouts: a kernel whose wait expires records status bits in a
device word and in a pinned host mirror of it. Every op call first reads the
mirror (host memory, no synchronisation) and raises :class:`FdsError` if a
previous call on that device timed out, so a drop-in caller that never calls
:func:`check_status` still sees the failure at its next call (at the latest
its next window). :func:`check_status` synchronises, reports and clears both
words and re-zeroes the workspaces; a caller that wants the error attributed
to its window calls it once per window.
"""

from __future__ import annotations

import contextlib
import ctypes
import math

import torch

from . import _native as N

LEFT, RIGHT = 64, 8          # kernels.py:298 clamp of j - i
NUM_POS = LEFT + RIGHT + 1   # 73 relative-key table rows
NUM_POS_PAD = 128            # kept for API parity with kernels.py:300
LOG2E = 1.4426950408889634
HEAD_DIM = 64


class FdsError(AssertionError, RuntimeError):
    """Invalid argument or failed launch of an FDS kernel."""


_DTYPES = {torch.float16: N.FDS_DTYPE_FP16, torch.bfloat16: N.FDS_DTYPE_BF16}
_status_words: dict[int, torch.Tensor] = {}
_status_mirrors: dict[int, torch.Tensor] = {}
_mirror_views: dict = {}
_workspaces: dict[tuple[int, int], torch.Tensor] = {}
_spare_workspaces: dict[int, list[torch.Tensor]] = {}
_SPARE_WORKSPACES = 2


def _check(cond: bool, msg) -> None:
    """Raise FdsError(msg) unless cond; msg may be a zero-argument callable,
    formatted only on failure (the checks run on every call)."""
    if not cond:
        raise FdsError(msg() if callable(msg) else msg)


def _dev_index(device: torch.device) -> int:
    return device.index if device.index is not None else torch.cuda.current_device()


def _status(device: torch.device) -> torch.Tensor:
    """Per-device int32 word the kernels OR their bounded-wait error bits into."""
    idx = _dev_index(device)
    st = _status_words.get(idx)
    if st is None:
        # library state outlives the caller's context: never an inference tensor
        # (the reference pipeline runs under torch.inference_mode)
        with torch.inference_mode(False):
            st = torch.zeros(4, dtype=torch.int32, device=torch.device("cuda", idx))
        _status_words[idx] = st
    return st


def _status_mirror(device: torch.device) -> torch.Tensor:
    """Per-device pinned (mapped) host word the kernels mirror their error bits
    into; read by the host without synchronising."""
    idx = _dev_index(device)
    m = _status_mirrors.get(idx)
    if m is None:
        with torch.inference_mode(False):
            m = torch.zeros(4, dtype=torch.int32).pin_memory()
        _status_mirrors[idx] = m
    return m


def _on_device(device: torch.device):
    """``torch.cuda.device(device)``, or nothing when it is already current."""
    if device.index is None or device.index == torch.cuda.current_device():
        return contextlib.nullcontext()
    return torch.cuda.device(device)


def _raise_if_timed_out(device: torch.device) -> None:
    """Raise (without a device sync) if a kernel on ``device`` reported a
    timeout that :func:`check_status` has not cleared yet."""
    idx = _dev_index(device)
    m = _status_mirrors.get(idx)
    if m is not None:
        view = _mirror_views.get(idx)
        if view is None or view[0] is not m:  # the same pinned words, read without torch indexing
            view = _mirror_views[idx] = (m, m.numpy())
        bits = int(view[1][0])
        if bits:
            raise FdsError(f"an earlier FDS kernel on cuda:{_dev_index(device)} reported a bounded-wait "
                           f"timeout (status bits 0x{bits:x}); call check_status() to clear it")


def check_status(device: torch.device | int | None = None, clear: bool = True) -> int:
    """Synchronise ``device`` and raise :class:`FdsError` if any kernel on it
    recorded an expired bounded wait since the last check. Returns the bits."""
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else
                       (device if isinstance(device, int) else device.index))
    st = _status(dev)
    mirror = _status_mirror(dev)
    torch.cuda.synchronize(dev)
    bits = int(st[0].item()) | int(mirror[0])
    if clear and bits:
        with torch.inference_mode(False):
            st.zero_()
            mirror.zero_()
            for (idx, _), ws in _workspaces.items():
                if idx == dev.index:
                    ws.zero_()  # an aborted split may leave part counts behind
            for ws in _spare_workspaces.get(dev.index, []):
                ws.zero_()
        torch.cuda.synchronize(dev)
    if bits:
        raise FdsError(f"FDS kernel on {dev} reported a bounded-wait timeout (status bits 0x{bits:x})")
    return bits


def _stream_ptr(device: torch.device) -> int:
    """The current stream of ``device`` as a raw ``cudaStream_t`` value."""
    if _raw_stream is not None:
        return _raw_stream(_dev_index(device))
    return torch.cuda.current_stream(device).cuda_stream


# torch's own accessor for the current raw stream (what its compiled kernels
# launch on), much cheaper than building a Stream object; the public call
# otherwise
_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _workspace(device: torch.device, lib) -> torch.Tensor | None:
    """The balanced-schedule workspace of ``device``'s current stream (the C
    library leaves it ready for the next call), or None inside a graph capture
    that finds neither one nor a spare (never allocated during capture: the
    graph pool would zero it only at replay)."""
    idx = _dev_index(device)
    key = (idx, _stream_ptr(device))
    ws = _workspaces.get(key)
    if ws is not None:
        return ws
    if torch.cuda.is_current_stream_capturing():
        spares = _spare_workspaces.get(idx)
        if not spares:
            return None
        ws = spares.pop()
    else:
        nbytes = int(lib.fds_attn_workspace_bytes(0))
        if nbytes <= 0:
            raise FdsError(f"fds_attn_workspace_bytes failed: {N.last_error()}")
        cuda = torch.device("cuda", idx)
        with torch.inference_mode(False):
            ws = torch.zeros(nbytes, dtype=torch.uint8, device=cuda)
            if idx not in _spare_workspaces:
                # zero-filled now, handed to the first captures on new streams;
                # the one-time wait makes the fill complete before any graph runs
                _spare_workspaces[idx] = [torch.zeros(nbytes, dtype=torch.uint8, device=cuda)
                                          for _ in range(_SPARE_WORKSPACES)]
                torch.cuda.current_stream(cuda).synchronize()
    _workspaces[key] = ws
    return ws


def _schedule(device: torch.device, lib, balanced: bool, grid_ctas: int) -> dict:
    _check(grid_ctas >= 0, "grid_ctas must be >= 0")
    ws = _workspace(device, lib) if balanced else None
    if ws is None:
        return dict(workspace=None, workspace_bytes=0, grid_ctas=0)
    return dict(workspace=ws.data_ptr(), workspace_bytes=ws.numel(), grid_ctas=int(grid_ctas))


def _rows_operand(t: torch.Tensor, name: str) -> None:
    _check(isinstance(t, torch.Tensor), lambda: f"{name} must be a torch.Tensor")
    _check(t.dim() == 2, lambda: f"{name} must be 2-D [rows, columns], got {tuple(t.shape)}")
    _check(t.dtype in _DTYPES, lambda: f"{name} must be float16 or bfloat16, got {t.dtype}")
    _check(t.stride(1) == 1, lambda: f"{name} columns must be contiguous (stride(1) == 1)")
    _check(t.shape[0] <= 1 or t.stride(0) % 8 == 0, lambda: f"{name} row stride must be a multiple of 8 elements")
    _check(t.data_ptr() % 16 == 0, lambda: f"{name} must be 16-byte aligned")


def _on_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        _check(t.is_cuda, "tensors must be on a CUDA device (there is no CPU fallback)")


def _raise_rc(rc: int, what: str) -> None:
    if rc != N.FDS_OK:
        raise FdsError(f"{what} failed (code {rc}): {N.last_error()}")


def flexrel_attention(qkv: torch.Tensor, batch: int, heads: int, rel: torch.Tensor,
                      out: torch.Tensor | None = None, kv_len: torch.Tensor | None = None,
                      *, timeout_ns: int = 0, debug_flags: int = 0, balanced: bool = True,
                      grid_ctas: int = 0) -> torch.Tensor:
    """Relative-key self-attention of one w2v-BERT layer.

    qkv [B*L, 3*H*64] fp16/bf16 (q | k | v column blocks, rows b*L + t),
    rel [73, 64] same dtype -> context [B*L, H*64] (qkv dtype), written into
    ``out`` when given. ``kv_len`` (int32 CUDA [B], optional) excludes keys
    t >= kv_len[b] -- the key-padding mask of a bucketed batch; every query row
    (padded ones included) attends over the valid keys, as with HF's additive
    mask. A window with kv_len 0 yields zeros.

    Same contract as the reference ``flexrel_attention``
    (triton/src/fds_triton/kernels.py:422-442); ``kv_len`` is an addition.
    ``balanced=False`` keeps one 256-row unit per CTA; ``grid_ctas > 0`` asks
    for a split last wave of that many pieces whenever the shape allows it
    (tests use it to cut units at small sizes).
    """
    _rows_operand(qkv, "qkv")
    rows, width = qkv.shape
    _check(batch >= 1 and heads >= 1, "batch and heads must be >= 1")
    _check(width % 3 == 0, lambda: f"qkv width {width} is not 3 * hidden")
    hidden = width // 3
    _check(hidden % heads == 0, lambda: f"hidden {hidden} not divisible by heads {heads}")
    dim = hidden // heads
    _check(dim == HEAD_DIM, lambda: f"head_dim must be 64, got {dim}")
    _check(rows % batch == 0 and rows > 0, lambda: f"rows {rows} not a positive multiple of batch {batch}")
    length = rows // batch
    _check(isinstance(rel, torch.Tensor) and rel.shape == (NUM_POS, dim) and rel.is_contiguous(),
           lambda: f"rel must be a contiguous [{NUM_POS}, {dim}] tensor")
    _check(rel.dtype == qkv.dtype and rel.device == qkv.device, "rel must match qkv's dtype and device")
    _check(rel.data_ptr() % 16 == 0, "rel must be 16-byte aligned")
    if out is None:
        out = torch.empty(rows, hidden, device=qkv.device, dtype=qkv.dtype)
    else:
        _rows_operand(out, "out")
        _check(out.shape == (rows, hidden), lambda: f"out must be [{rows}, {hidden}], got {tuple(out.shape)}")
        _check(out.dtype == qkv.dtype and out.device == qkv.device, "out must match qkv's dtype and device")
    kv_ptr = None
    if kv_len is not None:
        _check(isinstance(kv_len, torch.Tensor) and kv_len.dtype == torch.int32
               and kv_len.shape == (batch,) and kv_len.is_contiguous() and kv_len.device == qkv.device,
               lambda: f"kv_len must be a contiguous int32 CUDA tensor of shape [{batch}] on qkv's device")
        kv_ptr = kv_len.data_ptr()
    _on_cuda(qkv, rel, out)
    dev = qkv.device
    _raise_if_timed_out(dev)
    lib = N.load()
    with _on_device(dev):
        args = N.FdsFlexRelArgs(
            qkv=qkv.data_ptr(), qkv_row_stride=qkv.stride(0) if rows > 1 else width,
            rel=rel.data_ptr(), out=out.data_ptr(),
            out_row_stride=out.stride(0) if rows > 1 else hidden,
            kv_len=kv_ptr, status=_status(dev).data_ptr(), status_host=_status_mirror(dev).data_ptr(),
            batch=batch, heads=heads, seq_len=length, head_dim=dim, dtype=_DTYPES[qkv.dtype],
            scale=1.0 / math.sqrt(dim), timeout_ns=int(timeout_ns), debug_flags=int(debug_flags),
            **_schedule(dev, lib, balanced and kv_len is None, grid_ctas),
        )
        rc = lib.fds_flexrel_attn_fwd(ctypes.byref(args), _stream_ptr(dev))
    _raise_rc(rc, "fds_flexrel_attn_fwd")
    return out


def flexrel_attention_qr(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, qr: torch.Tensor,
                         out: torch.Tensor | None = None, heads_last: bool = True,
                         kv_len: torch.Tensor | None = None, *, timeout_ns: int = 0, debug_flags: int = 0,
                         balanced: bool = True, grid_ctas: int = 0) -> torch.Tensor:
    """Relative-key attention with the bias projections given: the TensorRT
    plugin's form (sidon::FlexRelAttnQR / QRD). q, k, v, out [B, L, H, 64]
    (``heads_last``) or [B, H, L, 64], qr = q . rel^T [B, L, H, 73] or
    [B, H, L, 73], all contiguous fp16 / bf16;
    S = (q k^T + qr[.., clamp(j - i, -64, 8) + 64]) / 8, softmax, V.
    Reference: ``flexrel_attention_qr`` (trt/src/fastdialoguesidon/
    flexrel_triton.py:749-780). ``kv_len`` as in :func:`flexrel_attention`."""
    for name, t in (("q", q), ("k", k), ("v", v), ("qr", qr)):
        _check(isinstance(t, torch.Tensor) and t.dim() == 4 and t.is_contiguous(),
               lambda: f"{name} must be a contiguous 4-D tensor")
        _check(t.dtype in _DTYPES and t.dtype == q.dtype and t.device == q.device,
               lambda: f"{name} must be float16 / bfloat16 like q, on q's device")
    _check(q.shape == k.shape == v.shape, "q, k and v must have the same shape")
    if heads_last:
        batch, length, heads, dim = q.shape
        _check(qr.shape == (batch, length, heads, NUM_POS), lambda: f"qr must be [{batch}, {length}, {heads}, {NUM_POS}]")
    else:
        batch, heads, length, dim = q.shape
        _check(qr.shape == (batch, heads, length, NUM_POS), lambda: f"qr must be [{batch}, {heads}, {length}, {NUM_POS}]")
    _check(dim == HEAD_DIM, lambda: f"head_dim must be 64, got {dim}")
    for name, t in (("q", q), ("k", k), ("v", v)):
        _check(t.data_ptr() % 16 == 0, lambda: f"{name} must be 16-byte aligned")
    if out is None:
        out = torch.empty_like(q)
    else:
        _check(out.shape == q.shape and out.dtype == q.dtype and out.device == q.device and out.is_contiguous()
               and out.data_ptr() % 16 == 0, lambda: f"out must be a contiguous {tuple(q.shape)} {q.dtype} tensor")
    kv_ptr = None
    if kv_len is not None:
        _check(isinstance(kv_len, torch.Tensor) and kv_len.dtype == torch.int32
               and kv_len.shape == (batch,) and kv_len.is_contiguous() and kv_len.device == q.device,
               lambda: f"kv_len must be a contiguous int32 CUDA tensor of shape [{batch}] on q's device")
        kv_ptr = kv_len.data_ptr()
    _on_cuda(q, k, v, qr, out)
    dev = q.device
    _raise_if_timed_out(dev)
    lib = N.load()
    with _on_device(dev):
        args = N.FdsFlexRelQrArgs(
            q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), qr=qr.data_ptr(), out=out.data_ptr(),
            kv_len=kv_ptr, status=_status(dev).data_ptr(), status_host=_status_mirror(dev).data_ptr(),
            batch=batch, heads=heads, seq_len=length, head_dim=dim, dtype=_DTYPES[q.dtype],
            heads_last=1 if heads_last else 0, scale=1.0 / math.sqrt(dim), timeout_ns=int(timeout_ns),
            debug_flags=int(debug_flags), **_schedule(dev, lib, balanced and kv_len is None, grid_ctas))
        rc = lib.fds_flexrel_qr_attn_fwd(ctypes.byref(args), _stream_ptr(dev))
    _raise_rc(rc, "fds_flexrel_qr_attn_fwd")
    return out


def flexrel_attention_split(qkv: torch.Tensor, batch: int, heads: int, rel: torch.Tensor,
                            out: torch.Tensor | None = None) -> torch.Tensor:
    """Same contract and result as :func:`flexrel_attention`
    (reference ``kernels.py:634``). The reference splits the work into two cuDNN
    causal passes plus a band merge; on B200 one kernel does all of it."""
    return flexrel_attention(qkv, batch, heads, rel, out)


def cudnn_attention_available(device=None) -> bool:
    """Same meaning as the reference (``kernels.py:667-671``): whether cuDNN
    SDPA (sm80+ with a cuDNN build) is available, which the reference's model
    uses to choose its split path (``model.py:89``). This library's attention
    does not use cuDNN; :func:`encoder_attention` ignores the choice."""
    if not torch.backends.cudnn.is_available():
        return False
    return torch.cuda.get_device_capability(device) >= (8, 0)


def encoder_attention(qkv, batch, heads, rel, impl: str = "split", kv_len=None):
    """Reference ``kernels.py:674``; ``impl`` ("split" / "fused" / "auto") is
    accepted and ignored: there is a single kernel."""
    _check(impl in ("split", "fused", "auto"), lambda: f"unknown impl {impl!r}")
    return flexrel_attention(qkv, batch, heads, rel, kv_len=kv_len)


def _rope_tables(cos: torch.Tensor, sin: torch.Tensor, length: int, ref: torch.Tensor) -> None:
    for name, t in (("cos", cos), ("sin", sin)):
        _check(isinstance(t, torch.Tensor) and t.dtype == torch.float32 and t.dim() == 2
               and t.shape[1] == HEAD_DIM and t.shape[0] >= length and t.is_contiguous()
               and t.device == ref.device and t.data_ptr() % 16 == 0,
               lambda: f"{name} must be a contiguous fp32 [>= {length}, 64] table on {ref.device}")


def rope_split(qkv: torch.Tensor, length: int, heads: int, cos: torch.Tensor,
               sin: torch.Tensor) -> torch.Tensor:
    """qkv [B*L, 3*HID] -> [3, B*L, HID]: rotated q, rotated k, v (bit-exact),
    position = row % length. Reference ``kernels.py:476-487``."""
    _rows_operand(qkv, "qkv")
    rows, width = qkv.shape
    _check(width % 3 == 0, "qkv width is not 3 * hidden")
    hid = width // 3
    _check(hid % heads == 0 and hid // heads == HEAD_DIM, "head_dim must be 64")
    _check(length >= 1, "length must be >= 1")
    _rope_tables(cos, sin, min(length, rows) if rows else 1, qkv)
    _on_cuda(qkv, cos, sin)
    out = torch.empty(3, rows, hid, device=qkv.device, dtype=qkv.dtype)
    lib = N.load()
    with torch.cuda.device(qkv.device):
        rc = lib.fds_rope_split(qkv.data_ptr(), qkv.stride(0) if rows > 1 else width, cos.data_ptr(),
                                sin.data_ptr(), out.data_ptr(), rows, length, heads, HEAD_DIM,
                                _DTYPES[qkv.dtype], _stream_ptr(qkv.device))
    _raise_rc(rc, "fds_rope_split")
    return out


def rope_attention(qkv: torch.Tensor, batch: int, heads: int, cos: torch.Tensor, sin: torch.Tensor,
                   out: torch.Tensor | None = None, scratch: torch.Tensor | None = None,
                   *, timeout_ns: int = 0, debug_flags: int = 0, balanced: bool = True,
                   grid_ctas: int = 0) -> torch.Tensor:
    """DiT head self-attention: RoPE on q and k (frame index t = row % L), then
    bidirectional softmax(q k^T / 8) v. qkv [B*L, 3*HID] -> [B*L, HID].

    Replaces ``K.rope_split`` + ``F.scaled_dot_product_attention`` at
    triton/src/fds_triton/model.py:319-325. ``scratch`` ([B*L, 2*HID], qkv
    dtype) receives the rotated q | k; it is allocated when not given.
    ``balanced`` / ``grid_ctas`` as in :func:`flexrel_attention`.
    """
    _rows_operand(qkv, "qkv")
    rows, width = qkv.shape
    _check(batch >= 1 and heads >= 1, "batch and heads must be >= 1")
    _check(width % 3 == 0, "qkv width is not 3 * hidden")
    hid = width // 3
    _check(hid % heads == 0 and hid // heads == HEAD_DIM, "head_dim must be 64")
    _check(rows % batch == 0 and rows > 0, lambda: f"rows {rows} not a positive multiple of batch {batch}")
    length = rows // batch
    _rope_tables(cos, sin, length, qkv)
    if out is None:
        out = torch.empty(rows, hid, device=qkv.device, dtype=qkv.dtype)
    else:
        _rows_operand(out, "out")
        _check(out.shape == (rows, hid) and out.dtype == qkv.dtype and out.device == qkv.device,
               lambda: f"out must be a [{rows}, {hid}] {qkv.dtype} tensor on {qkv.device}")
    if scratch is None:
        scratch = torch.empty(rows, 2 * hid, device=qkv.device, dtype=qkv.dtype)
    else:
        _check(scratch.shape == (rows, 2 * hid) and scratch.is_contiguous() and scratch.dtype == qkv.dtype
               and scratch.device == qkv.device and scratch.data_ptr() % 16 == 0,
               lambda: f"scratch must be a contiguous [{rows}, {2 * hid}] {qkv.dtype} tensor on {qkv.device}")
    _on_cuda(qkv, cos, sin, out, scratch)
    dev = qkv.device
    _raise_if_timed_out(dev)
    lib = N.load()
    with _on_device(dev):
        args = N.FdsRopeArgs(
            qkv=qkv.data_ptr(), qkv_row_stride=qkv.stride(0) if rows > 1 else width,
            cos=cos.data_ptr(), sin=sin.data_ptr(), qk_scratch=scratch.data_ptr(), out=out.data_ptr(),
            out_row_stride=out.stride(0) if rows > 1 else hid, status=_status(dev).data_ptr(),
            status_host=_status_mirror(dev).data_ptr(),
            batch=batch, heads=heads, seq_len=length, head_dim=HEAD_DIM, dtype=_DTYPES[qkv.dtype],
            scale=1.0 / math.sqrt(HEAD_DIM), timeout_ns=int(timeout_ns), debug_flags=int(debug_flags),
            **_schedule(dev, lib, balanced, grid_ctas),
        )
        rc = lib.fds_rope_attn_fwd(ctypes.byref(args), _stream_ptr(dev))
    _raise_rc(rc, "fds_rope_attn_fwd")
    return out


def rotated_attention(qkv: torch.Tensor, batch: int, heads: int, out: torch.Tensor | None = None,
                      *, timeout_ns: int = 0, debug_flags: int = 0, balanced: bool = True,
                      grid_ctas: int = 0) -> torch.Tensor:
    """Bidirectional softmax(q k^T / 8) v over a qkv [B*L, 3*HID] whose q | k
    column blocks are rotated already (the :func:`linear_rope` output): the DiT
    attention with no RoPE pass and no scratch. -> [B*L, HID]."""
    _rows_operand(qkv, "qkv")
    rows, width = qkv.shape
    _check(batch >= 1 and heads >= 1, "batch and heads must be >= 1")
    _check(width % 3 == 0, "qkv width is not 3 * hidden")
    hid = width // 3
    _check(hid % heads == 0 and hid // heads == HEAD_DIM, "head_dim must be 64")
    _check(rows % batch == 0 and rows > 0, lambda: f"rows {rows} not a positive multiple of batch {batch}")
    length = rows // batch
    if out is None:
        out = torch.empty(rows, hid, device=qkv.device, dtype=qkv.dtype)
    else:
        _rows_operand(out, "out")
        _check(out.shape == (rows, hid) and out.dtype == qkv.dtype and out.device == qkv.device,
               lambda: f"out must be a [{rows}, {hid}] {qkv.dtype} tensor on {qkv.device}")
    _on_cuda(qkv, out)
    dev = qkv.device
    _raise_if_timed_out(dev)
    lib = N.load()
    with _on_device(dev):
        args = N.FdsRopeArgs(
            qkv=qkv.data_ptr(), qkv_row_stride=qkv.stride(0) if rows > 1 else width,
            cos=None, sin=None, qk_scratch=None, out=out.data_ptr(),
            out_row_stride=out.stride(0) if rows > 1 else hid, status=_status(dev).data_ptr(),
            status_host=_status_mirror(dev).data_ptr(), qk_rotated=1,
            batch=batch, heads=heads, seq_len=length, head_dim=HEAD_DIM, dtype=_DTYPES[qkv.dtype],
            scale=1.0 / math.sqrt(HEAD_DIM), timeout_ns=int(timeout_ns), debug_flags=int(debug_flags),
            **_schedule(dev, lib, balanced, grid_ctas),
        )
        rc = lib.fds_rope_attn_fwd(ctypes.byref(args), _stream_ptr(dev))
    _raise_rc(rc, "fds_rope_attn_fwd")
    return out


def _linear_call(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None, out: torch.Tensor,
                 epilogue: int, cos=None, sin=None, seq_len: int = 0, rope_cols: int = 0,
                 timeout_ns: int = 0, grid_ctas: int = 0, pair: bool | None = None) -> torch.Tensor:
    _rows_operand(x, "x")
    _rows_operand(w, "w")
    m, k = x.shape
    n, kw = w.shape
    _check(kw == k, lambda: f"w is [{n}, {kw}] but x has {k} columns")
    _check(w.dtype == x.dtype and w.device == x.device, "w must match x's dtype and device")
    _check(k % 64 == 0, lambda: f"in_features must be a multiple of 64 (got {k})")
    _check(n % 128 == 0, lambda: f"out_features must be a multiple of 128 (got {n})")
    if bias is not None:
        _check(isinstance(bias, torch.Tensor) and bias.shape == (n,) and bias.is_contiguous()
               and bias.dtype == x.dtype and bias.device == x.device and bias.data_ptr() % 16 == 0,
               lambda: f"bias must be a contiguous [{n}] {x.dtype} tensor on {x.device}")
    _on_cuda(x, w, out)
    dev = x.device
    _raise_if_timed_out(dev)
    lib = N.load()
    with _on_device(dev):
        args = N.FdsLinearArgs(
            a=x.data_ptr(), a_row_stride=x.stride(0) if m > 1 else k, w=w.data_ptr(),
            w_row_stride=w.stride(0) if n > 1 else k, bias=None if bias is None else bias.data_ptr(),
            out=out.data_ptr(), out_row_stride=out.stride(0) if m > 1 else n,
            cos=None if cos is None else cos.data_ptr(), sin=None if sin is None else sin.data_ptr(),
            status=_status(dev).data_ptr(), status_host=_status_mirror(dev).data_ptr(),
            m=m, n=n, k=k, dtype=_DTYPES[x.dtype], epilogue=epilogue, seq_len=int(seq_len),
            rope_cols=int(rope_cols), timeout_ns=int(timeout_ns), grid_ctas=int(grid_ctas),
            cta_pair=N.FDS_GEMM_AUTO if pair is None else (N.FDS_GEMM_PAIR if pair else N.FDS_GEMM_SINGLE))
        rc = lib.fds_linear_fwd(ctypes.byref(args), _stream_ptr(dev))
    _raise_rc(rc, "fds_linear_fwd")
    return out


def _linear_out(x: torch.Tensor, n: int, out: torch.Tensor | None, dtype) -> torch.Tensor:
    m = x.shape[0]
    if out is None:
        return torch.empty(m, n, device=x.device, dtype=dtype)
    _rows_operand(out, "out") if dtype != torch.float32 else None
    _check(out.shape == (m, n) and out.dtype == dtype and out.device == x.device and out.stride(1) == 1,
           lambda: f"out must be a [{m}, {n}] {dtype} tensor on {x.device} with contiguous rows")
    return out


def linear(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None = None,
           out: torch.Tensor | None = None, *, grid_ctas: int = 0, pair: bool | None = None) -> torch.Tensor:
    """``F.linear(x, w, b)`` on the tensor cores: x [M, K], w [N, K] (nn.Linear
    layout), fp16 / bf16, fp32 accumulation, result rounded once to x's dtype.
    Reference: ``linear`` (triton/src/fds_triton/model.py:50-51), used for the
    QKV projection before the attention (model.py:289).

    ``pair``: None (default) runs 256-row tiles over CTA pairs when x has more
    than 128 rows and K >= 512; True / False force CTA pairs / one CTA per
    128-row tile (the same result bit for bit: each output element sums over K
    in the same order either way, ``tests/test_linear_gpu.py``).
    ``grid_ctas`` caps the persistent CTAs (0: one per SM)."""
    out = _linear_out(x, w.shape[0], out, x.dtype)
    return _linear_call(x, w, b, out, N.FDS_EPILOGUE_STORE, grid_ctas=grid_ctas, pair=pair)


def linear_rope(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None, cos: torch.Tensor,
                sin: torch.Tensor, length: int, heads: int, out: torch.Tensor | None = None,
                *, grid_ctas: int = 0, pair: bool | None = None) -> torch.Tensor:
    """The DiT's QKV projection with RoPE in its epilogue: ``F.linear(x, w, b)``
    (rounded to x's dtype) followed by ``rope_split``'s rotation of the q and k
    column blocks (position = row % length), written as one [M, 3*heads*64]
    tensor that :func:`rotated_attention` reads directly. Replaces
    triton/src/fds_triton/model.py:318-319 (linear + K.rope_split)."""
    n = w.shape[0]
    _check(n == 3 * heads * HEAD_DIM, lambda: f"w must have 3*heads*64 = {3 * heads * HEAD_DIM} rows (got {n})")
    _check(length >= 1, "length must be >= 1")
    _rope_tables(cos, sin, min(length, x.shape[0]), x)
    out = _linear_out(x, n, out, x.dtype)
    return _linear_call(x, w, b, out, N.FDS_EPILOGUE_ROPE, cos=cos, sin=sin, seq_len=length,
                        rope_cols=2 * heads * HEAD_DIM, grid_ctas=grid_ctas, pair=pair)


def accumulate(x: torch.Tensor, a: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None = None,
               *, grid_ctas: int = 0, pair: bool | None = None) -> None:
    """``x += a @ w.T`` in place: fp16 / bf16 operands, fp32 accumulation added
    straight into the fp32 residual x (no reduced-precision GEMM output, no
    separate add). Reference: ``accumulate`` (triton/src/fds_triton/model.py:
    53-57, ``torch.addmm(x, a, w.t(), out_dtype=torch.float32, out=x)``), the
    attention's out-projection (model.py:291)."""
    _check(isinstance(x, torch.Tensor) and x.dtype == torch.float32 and x.dim() == 2,
           "x must be a 2-D fp32 tensor (the residual stream)")
    _check(x.stride(1) == 1 and (x.shape[0] <= 1 or x.stride(0) % 4 == 0) and x.data_ptr() % 16 == 0,
           "x rows must be contiguous and 16-byte aligned")
    _check(x.shape == (a.shape[0], w.shape[0]), lambda: f"x must be [{a.shape[0]}, {w.shape[0]}], got {tuple(x.shape)}")
    _linear_call(a, w, b, x, N.FDS_EPILOGUE_ACCUMULATE_F32, grid_ctas=grid_ctas, pair=pair)


def rope_tables(max_seq: int, device=None, dim: int = HEAD_DIM, base: float = 10000.0):
    """fp32 cos/sin [max_seq, dim] tables as the reference builds them
    (model.py:201-205: inv_freq = base^(-arange(0, dim/2)/(dim/2)), cat([f, f]))."""
    half = dim // 2
    inv_freq = 1.0 / (base ** (torch.arange(0, half, dtype=torch.float32) / float(half)))
    freqs = torch.outer(torch.arange(max_seq, dtype=torch.float32), inv_freq)
    cos = torch.cat([freqs.cos(), freqs.cos()], -1).contiguous()
    sin = torch.cat([freqs.sin(), freqs.sin()], -1).contiguous()
    if device is not None:
        cos, sin = cos.to(device), sin.to(device)
    return cos, sin
