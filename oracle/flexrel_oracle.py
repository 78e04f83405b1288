"""CPU oracle for the FastDialogueSidon attention hot path -- TEST INFRASTRUCTURE.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this module, and only as the checker or the timed CPU
baseline. The product path (``fastdialoguesidon_b200``) never calls it.

Each function restates, in plain torch fp32 (or numpy fp64) on the CPU, the
reference algorithm it cites. Parity of this oracle with the reference itself
is pinned by ``tests/golden/*.npz``, produced by ``tests/golden/make_golden.py``
from the reference's own modules (``FlexRelSelfAttention`` with eager
flex_attention, ``explicit_core_fp32``, ``DiTBlock._apply_rope`` + SDPA).
"""

from __future__ import annotations

import math

import numpy as np
import torch

LEFT, RIGHT = 64, 8
NUM_POS = LEFT + RIGHT + 1


def rel_index(length: int, q_start: int = 0, q_stop: int | None = None) -> torch.Tensor:
    """clamp(j - i, -64, 8) + 64 for rows i in [q_start, q_stop), all keys j.
    (trt/src/fastdialoguesidon/flexrel_triton.py:289-290, :314-317)"""
    q_stop = length if q_stop is None else q_stop
    pos = torch.arange(length)
    return torch.clamp(pos[None, :] - pos[q_start:q_stop, None], -LEFT, RIGHT) + LEFT


def flexrel_core(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, rel: torch.Tensor,
                 kv_len=None, chunk: int = 512) -> torch.Tensor:
    """Relative-key attention core in fp32, rows in chunks.

    q, k, v [B, H, L, D]; rel [73, D] -> [B, H, L, D] fp32.
    S = (q.k^T + gather(q.rel^T, clamp(j - i, -64, 8) + 64)) / sqrt(D), softmax
    over keys, times V. Restates torch_core_chunked
    (trt/src/fastdialoguesidon/flexrel_triton.py:298-329) and _attn_ref
    (triton/tests/test_kernels.py:98-109). ``kv_len`` [B] excludes keys
    j >= kv_len[b] (the additive key-padding mask of FlexRelSelfAttention,
    triton/src/fds_triton/reference/modeling.py:107-118, for rows with a valid
    key); a window with kv_len 0 gives zeros.
    """
    q, k, v, rel = (t.float() for t in (q, k, v, rel))
    batch, heads, length, dim = q.shape
    scale = 1.0 / math.sqrt(dim)
    out = torch.empty(batch, heads, length, dim, dtype=torch.float32)
    kmask = None
    if kv_len is not None:
        kv = torch.as_tensor(kv_len).to(torch.int64).clamp(0, length)
        kmask = torch.arange(length)[None, :] >= kv[:, None]  # [B, L] True = excluded
    for start in range(0, length, chunk):
        stop = min(start + chunk, length)
        qc = q[:, :, start:stop]
        idx = rel_index(length, start, stop)
        qr = torch.einsum("bhld,rd->bhlr", qc, rel)
        bias = torch.gather(qr, 3, idx.view(1, 1, stop - start, length).expand(batch, heads, -1, -1))
        scores = (qc @ k.transpose(-2, -1) + bias) * scale
        if kmask is not None:
            scores = scores.masked_fill(kmask[:, None, None, :], float("-inf"))
        p = torch.softmax(scores, dim=-1)
        if kmask is not None:
            p = torch.nan_to_num(p, nan=0.0)  # windows without a valid key
        out[:, :, start:stop] = p @ v
    return out


def flexrel_core_qr(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, qr: torch.Tensor,
                    kv_len=None, chunk: int = 512) -> torch.Tensor:
    """Relative-key attention with the projections qr = q . rel^T given (the
    TensorRT plugin's form): q, k, v [B, H, L, D], qr [B, H, L, 73] -> [B, H, L, D]
    fp32, S = (q.k^T + qr[.., clamp(j - i, -64, 8) + 64]) / sqrt(D), softmax,
    times V. Restates _flexrel_qr_body (trt/src/fastdialoguesidon/
    flexrel_triton.py:559-700: qr_left / qr_right outside the band, the gathered
    qr inside it, all scaled like q.k). ``kv_len`` as in :func:`flexrel_core`."""
    q, k, v, qr = (t.float() for t in (q, k, v, qr))
    batch, heads, length, dim = q.shape
    scale = 1.0 / math.sqrt(dim)
    out = torch.empty(batch, heads, length, dim, dtype=torch.float32)
    kmask = None
    if kv_len is not None:
        kv = torch.as_tensor(kv_len).to(torch.int64).clamp(0, length)
        kmask = torch.arange(length)[None, :] >= kv[:, None]
    for start in range(0, length, chunk):
        stop = min(start + chunk, length)
        idx = rel_index(length, start, stop)
        bias = torch.gather(qr[:, :, start:stop], 3, idx.view(1, 1, stop - start, length).expand(batch, heads, -1, -1))
        scores = (q[:, :, start:stop] @ k.transpose(-2, -1) + bias) * scale
        if kmask is not None:
            scores = scores.masked_fill(kmask[:, None, None, :], float("-inf"))
        p = torch.softmax(scores, dim=-1)
        if kmask is not None:
            p = torch.nan_to_num(p, nan=0.0)
        out[:, :, start:stop] = p @ v
    return out


def flexrel_rows(q, k, v, rel, start: int, stop: int) -> torch.Tensor:
    """Rows [start, stop) of :func:`flexrel_core` (no mask): one chunk of
    torch_core_chunked (flexrel_triton.py:312-328). Used to time the CPU path."""
    batch, heads, length, dim = q.shape
    qc = q[:, :, start:stop].float()
    idx = rel_index(length, start, stop)
    qr = torch.einsum("bhld,rd->bhlr", qc, rel.float())
    bias = torch.gather(qr, 3, idx.view(1, 1, stop - start, length).expand(batch, heads, -1, -1))
    scores = (qc @ k.float().transpose(-2, -1) + bias) * (1.0 / math.sqrt(dim))
    return torch.softmax(scores, dim=-1) @ v.float()


def split_qkv(qkv: torch.Tensor, batch: int, heads: int):
    """[B*L, 3*H*D] (q | k | v column blocks) -> three [B, H, L, D] fp32 views."""
    rows, width = qkv.shape
    hid = width // 3
    dim = hid // heads
    length = rows // batch
    return tuple(qkv[:, i * hid:(i + 1) * hid].float().reshape(batch, length, heads, dim).transpose(1, 2)
                 for i in range(3))


def merge_heads(o: torch.Tensor) -> torch.Tensor:
    """[B, H, L, D] -> [B*L, H*D] (the kernels' context layout)."""
    batch, heads, length, dim = o.shape
    return o.transpose(1, 2).reshape(batch * length, heads * dim)


def flexrel_attention(qkv: torch.Tensor, batch: int, heads: int, rel: torch.Tensor,
                      kv_len=None, chunk: int = 512) -> torch.Tensor:
    """Oracle of ``flexrel_attention(qkv, batch, heads, rel)`` (same layouts), fp32."""
    q, k, v = split_qkv(qkv, batch, heads)
    return merge_heads(flexrel_core(q, k, v, rel, kv_len=kv_len, chunk=chunk))


def flexrel_core_f64(q: np.ndarray, k: np.ndarray, v: np.ndarray, rel: np.ndarray) -> np.ndarray:
    """numpy fp64 restatement of the same core (small sizes): q, k, v [B, H, L, D]."""
    q, k, v, rel = (np.asarray(t, dtype=np.float64) for t in (q, k, v, rel))
    length, dim = q.shape[2], q.shape[3]
    idx = rel_index(length).numpy()
    qr = np.einsum("bhld,rd->bhlr", q, rel)
    bias = np.take_along_axis(qr, np.broadcast_to(idx, q.shape[:2] + (length, length)), axis=3)
    s = (q @ np.swapaxes(k, -1, -2) + bias) / math.sqrt(dim)
    s -= s.max(-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(-1, keepdims=True)
    return p @ v


def flexrel_layer(x: torch.Tensor, wq, bq, wk, bk, wv, bv, wo, bo, rel: torch.Tensor,
                  heads: int, kv_len=None) -> torch.Tensor:
    """One FlexRelSelfAttention layer (modeling.py:81-122) in fp32:
    q/k/v projections, relative-key core, output projection. x [B, L, C]."""
    batch, length, hidden = x.shape
    dim = hidden // heads

    def proj(w, b):
        return torch.nn.functional.linear(x.float(), w.float(), b.float()).view(batch, length, heads, dim).transpose(1, 2)

    ctx = flexrel_core(proj(wq, bq), proj(wk, bk), proj(wv, bv), rel, kv_len=kv_len)
    ctx = ctx.transpose(1, 2).reshape(batch, length, hidden)
    return torch.nn.functional.linear(ctx, wo.float(), bo.float())


# ------------------------------------------------------------------ DiT RoPE


def rope_tables(length: int, dim: int = 64, base: float = 10000.0):
    """fp32 cos/sin [length, dim] (modeling.py:243-266, model.py:201-205)."""
    half = dim // 2
    inv_freq = 1.0 / (base ** (torch.arange(0, half, dtype=torch.float32) / float(half)))
    freqs = torch.outer(torch.arange(length, dtype=torch.float32), inv_freq)
    return torch.cat([freqs.cos(), freqs.cos()], -1), torch.cat([freqs.sin(), freqs.sin()], -1)


def rope_apply(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [B, L, H, D] fp32; x*cos + rotate_half(x)*sin, rotate_half = cat(-x2, x1)
    (modeling.py:238-241, :274-276)."""
    length, dim = x.shape[1], x.shape[3]
    half = dim // 2
    c = cos[:length].view(1, length, 1, dim)
    s = sin[:length].view(1, length, 1, dim)
    rot = torch.cat([-x[..., half:], x[..., :half]], -1)
    return x * c + rot * s


def rope_split(qkv: torch.Tensor, length: int, heads: int, cos: torch.Tensor, sin: torch.Tensor):
    """Oracle of ``rope_split``: [3, B*L, HID] fp32 (q, k rotated; v as is), position = row % length
    (triton/src/fds_triton/kernels.py:448-487)."""
    rows, width = qkv.shape
    hid = width // 3
    dim = hid // heads
    pos = torch.arange(rows) % length
    out = []
    for part in range(2):
        x = qkv[:, part * hid:(part + 1) * hid].float().view(rows, heads, dim)
        c = cos[pos].view(rows, 1, dim)
        s = sin[pos].view(rows, 1, dim)
        rot = torch.cat([-x[..., dim // 2:], x[..., :dim // 2]], -1)
        out.append((x * c + rot * s).reshape(rows, hid))
    out.append(qkv[:, 2 * hid:].float())
    return torch.stack(out)


def rope_attention(qkv: torch.Tensor, batch: int, heads: int, cos: torch.Tensor, sin: torch.Tensor,
                   round_qk_to=None, chunk: int = 1024) -> torch.Tensor:
    """Oracle of ``rope_attention``: DiTBlock's rope + bidirectional softmax attention
    (modeling.py:290-312) in fp32, [B*L, HID]. ``round_qk_to`` (a torch dtype)
    rounds the rotated q/k as the GPU path stores them (the reference's
    rope_split does the same, kernels.py:469)."""
    rows, width = qkv.shape
    hid = width // 3
    dim = hid // heads
    length = rows // batch
    q, k, v = (qkv[:, i * hid:(i + 1) * hid].float().view(batch, length, heads, dim) for i in range(3))
    q, k = rope_apply(q, cos, sin), rope_apply(k, cos, sin)
    if round_qk_to is not None:
        q, k = q.to(round_qk_to).float(), k.to(round_qk_to).float()
    q, k, v = (t.transpose(1, 2) for t in (q, k, v))
    out = torch.empty(batch, heads, length, dim)
    scale = 1.0 / math.sqrt(dim)
    for start in range(0, length, chunk):
        stop = min(start + chunk, length)
        s = (q[:, :, start:stop] @ k.transpose(-1, -2)) * scale
        out[:, :, start:stop] = torch.softmax(s, -1) @ v
    return merge_heads(out)


# ------------------------------------------------------------------ metrics


def snr_db(ref: torch.Tensor, act: torch.Tensor) -> float:
    """20 log10(|ref| / |ref - act|) (triton/tests/test_kernels.py:27-29)."""
    ref, act = ref.double(), act.double()
    return float(20 * torch.log10(ref.norm() / (ref - act).norm().clamp_min(1e-30)))


def max_abs(ref: torch.Tensor, act: torch.Tensor) -> float:
    return float((ref.double() - act.double()).abs().max())
