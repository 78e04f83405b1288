"""The torch operator boundary (``torch.ops.fds.*``) as a drop-in for the
reference op ``flexrel_attention(qkv, batch, heads, rel, out=None)``
(triton/src/fds_triton/kernels.py:422): the out= overload writes in place and
allocates nothing, also inside CUDA-graph capture, and a bounded-wait timeout
reaches the caller at its next call without a device synchronisation.
"""

import pytest
import torch

import fastdialoguesidon_b200 as F
from fastdialoguesidon_b200 import _native as N

pytestmark = pytest.mark.gpu


def _capture(fn):
    """Captures fn() in a new graph; returns (graph, bytes torch.cuda.memory_allocated
    grew by during the capture)."""
    torch.cuda.synchronize()
    before = torch.cuda.memory_allocated()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    torch.cuda.synchronize()
    return g, torch.cuda.memory_allocated() - before


def _capture_overhead() -> int:
    """What a capture itself may allocate (torch registers the default
    generator's graph state, e.g.), measured on an empty graph."""
    g, grew = _capture(lambda: None)
    del g
    return grew


def _inputs(B, L, H, seed, device):
    g = torch.Generator().manual_seed(seed)
    qkv = torch.randn(B * L, 3 * H * 64, generator=g).half().to(device)
    rel = torch.randn(73, 64, generator=g).half().to(device)
    return qkv, rel


@pytest.mark.parametrize("L", [1000, 6000])
def test_flexrel_out_overload_in_graph_allocates_nothing(cuda_device, L):
    B, H = 1, 16
    qkv, rel = _inputs(B, L, H, seed=L, device=cuda_device)
    eager = torch.ops.fds.flexrel_attention(qkv, B, H, rel)           # functional overload
    buf = torch.empty_like(eager)
    ret = torch.ops.fds.flexrel_attention(qkv, B, H, rel, out=buf)    # .out overload, eager
    assert ret.data_ptr() == buf.data_ptr() and torch.equal(buf, eager)
    overhead = _capture_overhead()
    # its own capture stream: no workspace there yet, a pre-zeroed spare is taken
    g, grew = _capture(lambda: torch.ops.fds.flexrel_attention(qkv, B, H, rel, out=buf))
    assert grew <= overhead, (grew, overhead)
    buf.zero_()
    torch.cuda.synchronize()
    before = torch.cuda.memory_allocated(cuda_device)
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    assert torch.cuda.memory_allocated(cuda_device) == before
    F.check_status()
    assert torch.equal(buf, eager)
    del g


def test_rope_out_overload_in_graph_allocates_nothing(cuda_device):
    B, L, H = 1, 2000, 12
    g0 = torch.Generator().manual_seed(3)
    qkv = (torch.randn(B * L, 3 * H * 64, generator=g0) * 0.55).half().to(cuda_device)
    cos, sin = F.rope_tables(L, cuda_device)
    eager = torch.ops.fds.rope_attention(qkv, B, H, cos, sin)
    buf = torch.empty_like(eager)
    scratch = torch.empty(B * L, 2 * H * 64, dtype=qkv.dtype, device=cuda_device)
    torch.ops.fds.rope_attention(qkv, B, H, cos, sin, out=buf, scratch=scratch)
    assert torch.equal(buf, eager)
    overhead = _capture_overhead()
    rets = []
    g, grew = _capture(lambda: rets.append(
        torch.ops.fds.rope_attention(qkv, B, H, cos, sin, out=buf, scratch=scratch)))
    assert grew <= overhead, (grew, overhead)
    buf.zero_()
    torch.cuda.synchronize()
    before = torch.cuda.memory_allocated(cuda_device)
    g.replay()
    torch.cuda.synchronize()
    assert torch.cuda.memory_allocated(cuda_device) == before
    F.check_status()
    assert rets[0].data_ptr() == buf.data_ptr() and torch.equal(buf, eager)
    del g


def test_timeout_reaches_the_next_call_without_a_sync(cuda_device):
    """A forced bounded-wait timeout (a wait on a barrier nothing arrives on,
    2 ms limit) is mirrored into pinned host memory; the next op call reads it
    and raises, before check_status() is ever called."""
    qkv, rel = _inputs(1, 300, 2, seed=9, device=cuda_device)
    F.flexrel_attention(qkv, 1, 2, rel, timeout_ns=2_000_000, debug_flags=N.FDS_DEBUG_FORCE_TIMEOUT)
    torch.cuda.current_stream().synchronize()   # the kernel has finished; no FDS status read so far
    with pytest.raises(F.FdsError, match="earlier FDS kernel"):
        torch.ops.fds.flexrel_attention(qkv, 1, 2, rel)
    with pytest.raises(F.FdsError, match="timeout"):
        F.check_status()
    out = torch.ops.fds.flexrel_attention(qkv, 1, 2, rel)   # cleared: calls work again
    assert F.check_status() == 0
    assert torch.equal(out, F.flexrel_attention(qkv, 1, 2, rel))


def test_state_created_under_inference_mode(cuda_device):
    """The reference pipeline calls the ops under torch.inference_mode
    (runtime.py:135); the library's per-device state made there must stay
    usable outside it (check_status clears it in place)."""
    import fastdialoguesidon_b200.kernels as K

    qkv, rel = _inputs(1, 300, 2, seed=13, device=cuda_device)
    saved = dict(K._status_words), dict(K._status_mirrors)
    K._status_words.clear()
    K._status_mirrors.clear()
    try:
        with torch.inference_mode():
            F.flexrel_attention(qkv, 1, 2, rel, timeout_ns=2_000_000, debug_flags=N.FDS_DEBUG_FORCE_TIMEOUT)
        with pytest.raises(F.FdsError, match="timeout"):
            F.check_status()
        assert F.check_status() == 0
    finally:
        K._status_words.update(saved[0])
        K._status_mirrors.update(saved[1])
