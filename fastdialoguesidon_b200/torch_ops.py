"""``torch.ops.fds.*`` registrations of the hot-path ops (CUDA only).

Schemas (the reference op ``flexrel_attention(qkv, batch, heads, rel,
out=None)``, triton/src/fds_triton/kernels.py:422, as an operator with an
out= overload, the way ATen registers its out variants):

    fds::flexrel_attention(Tensor qkv, int batch, int heads, Tensor rel,
                           Tensor? kv_len=None) -> Tensor
    fds::flexrel_attention.out(Tensor qkv, int batch, int heads, Tensor rel,
                               Tensor? kv_len=None, *, Tensor(a!) out) -> Tensor(a!)
    fds::rope_attention(Tensor qkv, int batch, int heads, Tensor cos,
                        Tensor sin) -> Tensor
    fds::rope_attention.out(Tensor qkv, int batch, int heads, Tensor cos,
                            Tensor sin, *, Tensor(a!) out, Tensor(b!) scratch) -> Tensor(a!)

``torch.ops.fds.flexrel_attention(qkv, b, h, rel, out=buf)`` resolves to the
``.out`` overload, writes the context into ``buf`` and returns it: nothing is
allocated, so the call can sit inside a CUDA-graph capture with a fixed memory
plan. The functional overloads allocate their result. All of them route to the
same C-ABI calls as :mod:`.kernels`; the fake (meta) implementations let
``torch.compile`` / export trace through them.
"""

from __future__ import annotations

import torch

from . import kernels as _k

_lib = torch.library.Library("fds", "DEF")
_lib.define("flexrel_attention(Tensor qkv, int batch, int heads, Tensor rel, Tensor? kv_len=None) -> Tensor")
_lib.define("flexrel_attention.out(Tensor qkv, int batch, int heads, Tensor rel, Tensor? kv_len=None, *, "
            "Tensor(a!) out) -> Tensor(a!)")
_lib.define("rope_attention(Tensor qkv, int batch, int heads, Tensor cos, Tensor sin) -> Tensor")
_lib.define("rope_attention.out(Tensor qkv, int batch, int heads, Tensor cos, Tensor sin, *, "
            "Tensor(a!) out, Tensor(b!) scratch) -> Tensor(a!)")


def _flexrel(qkv, batch, heads, rel, kv_len=None):
    return _k.flexrel_attention(qkv, batch, heads, rel, kv_len=kv_len)


def _flexrel_out(qkv, batch, heads, rel, kv_len=None, *, out):
    return _k.flexrel_attention(qkv, batch, heads, rel, out=out, kv_len=kv_len)


def _rope(qkv, batch, heads, cos, sin):
    return _k.rope_attention(qkv, batch, heads, cos, sin)


def _rope_out(qkv, batch, heads, cos, sin, *, out, scratch):
    return _k.rope_attention(qkv, batch, heads, cos, sin, out=out, scratch=scratch)


_lib.impl("flexrel_attention", _flexrel, "CUDA")
_lib.impl("flexrel_attention.out", _flexrel_out, "CUDA")
_lib.impl("rope_attention", _rope, "CUDA")
_lib.impl("rope_attention.out", _rope_out, "CUDA")


def _context_like(qkv):
    return qkv.new_empty(qkv.shape[0], qkv.shape[1] // 3)


@torch.library.register_fake("fds::flexrel_attention", lib=_lib)
def _(qkv, batch, heads, rel, kv_len=None):
    return _context_like(qkv)


@torch.library.register_fake("fds::rope_attention", lib=_lib)
def _(qkv, batch, heads, cos, sin):
    return _context_like(qkv)


# the out= overloads return their (caller-owned) `out` argument
_lib.impl("flexrel_attention.out", lambda qkv, batch, heads, rel, kv_len=None, *, out: out, "Meta")
_lib.impl("rope_attention.out", lambda qkv, batch, heads, cos, sin, *, out, scratch: out, "Meta")

# kept as module attributes for callers of the earlier Python-level names
flexrel_attention_op = torch.ops.fds.flexrel_attention
rope_attention_op = torch.ops.fds.rope_attention
