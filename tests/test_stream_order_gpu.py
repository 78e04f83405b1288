"""Stream order under programmatic dependent launch: the attention and RoPE
kernels start their CTAs while the previous kernel in the stream drains, and
must not touch memory before it has completed. A chain of calls with no other
kernel in between -- each reading the previous call's output, the last one
overwriting an input the call before it read -- must give bit for bit the
results of the same calls run one at a time with a device synchronisation
after each (the kernels are deterministic). The one-at-a-time results are
also checked against the CPU oracle (fp16: max-abs <= 2e-3 and SNR >= 55 dB
vs fp32, as in test_flexrel_gpu.py).
"""

import pytest
import torch

import fastdialoguesidon_b200 as F
from fastdialoguesidon_b200 import _native as N
from oracle import flexrel_oracle as O

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-3
MIN_SNR = 55.0


def _check(exp: torch.Tensor, got: torch.Tensor):
    got = got.float().cpu()
    err, snr = O.max_abs(exp, got), O.snr_db(exp, got)
    assert err <= MAX_ABS and snr >= MIN_SNR, (err, snr)


def _qkv(rows, heads, seed):
    gen = torch.Generator().manual_seed(seed)
    return torch.randn(rows, 3 * heads * 64, generator=gen).half()


def _run(calls, sync_each: bool):
    for c in calls:
        c()
        if sync_each:
            torch.cuda.synchronize()
    torch.cuda.synchronize()
    F.check_status()


@pytest.mark.parametrize("balanced", [False, True])
def test_encoder_chain_matches_one_at_a_time(cuda_device, balanced):
    """12-head call -> its [rows, 768] context is the qkv of a 4-head call ->
    a second 12-head call (another input) overwrites that context. With
    `balanced`, every call splits its last wave and the stream's workspace is
    shared along the chain."""
    B, L = 1, 1000
    qkv_a, qkv_b = _qkv(B * L, 12, 41), _qkv(B * L, 12, 42)
    rel = (torch.randn(73, 64, generator=torch.Generator().manual_seed(43))).half()
    a, b, r = qkv_a.to(cuda_device), qkv_b.to(cuda_device), rel.to(cuda_device)
    mid = torch.empty(B * L, 12 * 64, dtype=torch.float16, device=cuda_device)
    out = torch.empty(B * L, 4 * 64, dtype=torch.float16, device=cuda_device)
    kw12 = dict(grid_ctas=7) if balanced else dict(balanced=False)
    kw4 = dict(grid_ctas=6) if balanced else dict(balanced=False)
    if balanced:
        ws = N.load().fds_attn_workspace_bytes(0)
        assert N.schedule(B, 12, L, False, ws, 7)[2] == 7 and N.schedule(B, 4, L, False, ws, 6)[2] == 6
    calls = [lambda: F.flexrel_attention(a, B, 12, r, out=mid, **kw12),
             lambda: F.flexrel_attention(mid, B, 4, r, out=out, **kw4),
             lambda: F.flexrel_attention(b, B, 12, r, out=mid, **kw12)]

    _run(calls[:2], sync_each=True)  # allocates the stream's workspace outside the chains
    mid_a = mid.clone()
    _run(calls, sync_each=True)
    ref_out, ref_mid = out.clone(), mid.clone()
    _check(O.flexrel_attention(qkv_a, B, 12, rel), mid_a)
    _check(O.flexrel_attention(mid_a.cpu(), B, 4, rel), ref_out)
    _check(O.flexrel_attention(qkv_b, B, 12, rel), ref_mid)
    for _ in range(4):
        mid.zero_()
        out.zero_()
        _run(calls, sync_each=False)
        assert torch.equal(out, ref_out)
        assert torch.equal(mid, ref_mid)


def test_rope_chain_matches_one_at_a_time(cuda_device):
    """DiT: RoPE pass + attention (12 heads) -> context [rows, 768] is the qkv
    of a 4-head call (its RoPE pass reads it) -> a second 12-head call
    overwrites it."""
    B, L = 2, 600
    qkv_a, qkv_b = _qkv(B * L, 12, 44), _qkv(B * L, 12, 45)
    cos, sin = O.rope_tables(L)
    dc, ds = cos.to(cuda_device), sin.to(cuda_device)
    a, b = qkv_a.to(cuda_device), qkv_b.to(cuda_device)
    mid = torch.empty(B * L, 12 * 64, dtype=torch.float16, device=cuda_device)
    out = torch.empty(B * L, 4 * 64, dtype=torch.float16, device=cuda_device)
    s12 = torch.empty(B * L, 2 * 12 * 64, dtype=torch.float16, device=cuda_device)
    s4 = torch.empty(B * L, 2 * 4 * 64, dtype=torch.float16, device=cuda_device)
    calls = [lambda: F.rope_attention(a, B, 12, dc, ds, out=mid, scratch=s12),
             lambda: F.rope_attention(mid, B, 4, dc, ds, out=out, scratch=s4),
             lambda: F.rope_attention(b, B, 12, dc, ds, out=mid, scratch=s12)]

    _run(calls[:2], sync_each=True)
    mid_a = mid.clone()
    _run(calls, sync_each=True)
    ref_out, ref_mid = out.clone(), mid.clone()
    _check(O.rope_attention(qkv_a, B, 12, cos, sin, round_qk_to=torch.float16), mid_a)
    _check(O.rope_attention(mid_a.cpu(), B, 4, cos, sin, round_qk_to=torch.float16), ref_out)
    _check(O.rope_attention(qkv_b, B, 12, cos, sin, round_qk_to=torch.float16), ref_mid)
    for _ in range(4):
        mid.zero_()
        out.zero_()
        _run(calls, sync_each=False)
        assert torch.equal(out, ref_out)
        assert torch.equal(mid, ref_mid)
