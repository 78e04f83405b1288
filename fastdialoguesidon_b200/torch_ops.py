"""``torch.ops.fds.*`` registrations of the hot-path ops (CUDA only).

They route to the same C-ABI calls as :mod:`.kernels`; the fake (meta)
implementations let ``torch.compile`` / export trace through them.
"""

from __future__ import annotations

import torch

from . import kernels as _k


@torch.library.custom_op("fds::flexrel_attention", mutates_args=(), device_types="cuda")
def flexrel_attention_op(qkv: torch.Tensor, batch: int, heads: int, rel: torch.Tensor,
                         kv_len: torch.Tensor | None = None) -> torch.Tensor:
    return _k.flexrel_attention(qkv, batch, heads, rel, kv_len=kv_len)


@flexrel_attention_op.register_fake
def _(qkv, batch, heads, rel, kv_len=None):
    return qkv.new_empty(qkv.shape[0], qkv.shape[1] // 3)


@torch.library.custom_op("fds::rope_attention", mutates_args=(), device_types="cuda")
def rope_attention_op(qkv: torch.Tensor, batch: int, heads: int, cos: torch.Tensor,
                      sin: torch.Tensor) -> torch.Tensor:
    return _k.rope_attention(qkv, batch, heads, cos, sin)


@rope_attention_op.register_fake
def _(qkv, batch, heads, cos, sin):
    return qkv.new_empty(qkv.shape[0], qkv.shape[1] // 3)
