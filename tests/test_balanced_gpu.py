"""Split last wave on the B200: units of the last wave cut into pieces and
merged through the workspace (by whichever part finishes last) must match the
CPU oracle like whole units do, across repeated calls and CUDA-graph replays
(the part counts reset themselves), for both attention kernels.

Small problems are forced to split with an explicit piece count
(``grid_ctas``); every case checks with ``fds_attn_schedule`` that a split
actually happened. The full-size case uses the automatic choice.
Tolerances as in test_flexrel_gpu.py: fp16 max-abs <= 2e-3 and SNR >= 55 dB vs
the fp32 oracle; bf16 SNR > 40 dB.
"""

import pytest
import torch

import fastdialoguesidon_b200 as F
from fastdialoguesidon_b200 import _native as N
from oracle import flexrel_oracle as O

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-3
MIN_SNR = 55.0
BF16_MIN_SNR = 40.0


def _check(exp: torch.Tensor, got: torch.Tensor, dtype=torch.float16):
    got = got.float().cpu()
    snr = O.snr_db(exp, got)
    if dtype == torch.bfloat16:
        assert snr > BF16_MIN_SNR, snr
        return
    err = O.max_abs(exp, got)
    assert err <= MAX_ABS and snr >= MIN_SNR, (err, snr)


def _inputs(batch, length, heads, seed, dtype=torch.float16, std=1.0, rel_std=1.0):
    gen = torch.Generator().manual_seed(seed)
    qkv = (torch.randn(batch * length, 3 * heads * 64, generator=gen) * std).to(dtype)
    rel = (torch.randn(73, 64, generator=gen) * rel_std).to(dtype)
    return qkv, rel


def _assert_split(B, L, H, grid):
    ws = N.load().fds_attn_workspace_bytes(grid)
    ctas, whole, pieces = N.schedule(B, H, L, False, ws, grid)
    assert pieces == grid and ctas == whole + pieces, (ctas, whole, pieces)


@pytest.mark.parametrize("B,L,H,grid", [
    (1, 1000, 16, 5),     # 60 whole units, 4 units cut into 5 pieces
    (1, 1000, 16, 37),    # 37 whole, 27 units into 37 pieces (cuts at many tile offsets)
    (1, 1000, 16, 64),    # one wave: pieces are exactly the units
    (2, 333, 16, 13),     # 3-tile units, one-tile last row blocks, cuts across windows / heads
    (1, 1100, 8, 9),      # last row block holds one query tile (76 rows)
    (3, 129, 4, 7),       # 2-tile units of 129 rows
])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_split_small_grids_match_oracle(cuda_device, B, L, H, grid, dtype):
    _assert_split(B, L, H, grid)
    qkv, rel = _inputs(B, L, H, seed=L + grid, dtype=dtype)
    exp = O.flexrel_attention(qkv, B, H, rel)
    q, r = qkv.to(cuda_device), rel.to(cuda_device)
    out = F.flexrel_attention(q, B, H, r, grid_ctas=grid)
    whole = F.flexrel_attention(q, B, H, r, balanced=False)
    F.check_status()
    _check(exp, out, dtype)
    _check(exp, whole, dtype)


def test_split_repeated_calls(cuda_device):
    """The merging parts reset their counts: back-to-back calls on one
    workspace give identical results."""
    B, L, H, grid = 1, 1000, 16, 13
    _assert_split(B, L, H, grid)
    qkv, rel = _inputs(B, L, H, seed=3)
    q, r = qkv.to(cuda_device), rel.to(cuda_device)
    first = F.flexrel_attention(q, B, H, r, grid_ctas=grid)
    outs = [F.flexrel_attention(q, B, H, r, grid_ctas=grid) for _ in range(6)]
    F.check_status()
    for o in outs:
        assert torch.equal(o, first)
    _check(O.flexrel_attention(qkv, B, H, rel), first)


def test_split_graph_replays(cuda_device):
    B, L, H, grid = 1, 1000, 16, 17
    _assert_split(B, L, H, grid)
    qkv, rel = _inputs(B, L, H, seed=4)
    q, r = qkv.to(cuda_device), rel.to(cuda_device)
    eager = F.flexrel_attention(q, B, H, r, grid_ctas=grid)
    out = torch.empty_like(eager)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        F.flexrel_attention(q, B, H, r, out=out, grid_ctas=grid)
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(3):
            F.flexrel_attention(q, B, H, r, out=out, grid_ctas=grid)
    for _ in range(4):
        out.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, eager)
    F.check_status()


def test_split_full_size_auto(cuda_device):
    """L=6000, 16 heads: 384 units on 148 SMs; the automatic choice splits the
    last wave (296 whole units + 148 pieces)."""
    idx = cuda_device.index if cuda_device.index is not None else torch.cuda.current_device()
    sms = torch.cuda.get_device_properties(idx).multi_processor_count
    ws = N.load().fds_attn_workspace_bytes(0)
    ctas, whole, pieces = N.schedule(1, 16, 6000, False, ws, 0)
    if sms == 148:
        assert (ctas, whole, pieces) == (444, 296, 148)
    qkv, rel = _inputs(1, 6000, 16, seed=11, std=0.64, rel_std=0.02)
    q, r = qkv.to(cuda_device), rel.to(cuda_device)
    out = F.flexrel_attention(q, 1, 16, r)
    whole_out = F.flexrel_attention(q, 1, 16, r, balanced=False)
    F.check_status()
    exp = O.flexrel_attention(qkv, 1, 16, rel)
    _check(exp, out)
    _check(exp, whole_out)
    assert (out.float() - whole_out.float()).abs().max().item() <= 1e-3


@pytest.mark.parametrize("B,L,H,grid", [(1, 1000, 12, 7), (2, 600, 12, 20)])
def test_rope_split_small_grids(cuda_device, B, L, H, grid):
    _assert_split(B, L, H, grid)
    gen = torch.Generator().manual_seed(L)
    qkv = torch.randn(B * L, 3 * H * 64, generator=gen).half()
    cos, sin = O.rope_tables(L)
    exp = O.rope_attention(qkv, B, H, cos, sin, round_qk_to=torch.float16)
    dev_qkv = qkv.to(cuda_device)
    dc, ds = cos.to(cuda_device), sin.to(cuda_device)
    out = F.rope_attention(dev_qkv, B, H, dc, ds, grid_ctas=grid)
    whole = F.rope_attention(dev_qkv, B, H, dc, ds, balanced=False)
    F.check_status()
    _check(exp, out)
    _check(exp, whole)


def test_split_bounded_wait_reports_and_recovers(cuda_device):
    """A forced MMA-warp timeout in a split launch: every CTA reports and exits,
    parts of cut units may leave counts behind; check_status zero-fills the
    device's workspaces, and the next call is correct."""
    B, L, H, grid = 1, 1000, 4, 6
    _assert_split(B, L, H, grid)
    qkv, rel = _inputs(B, L, H, seed=5)
    q, r = qkv.to(cuda_device), rel.to(cuda_device)
    F.flexrel_attention(q, B, H, r, grid_ctas=grid, timeout_ns=2_000_000, debug_flags=N.FDS_DEBUG_FORCE_TIMEOUT)
    with pytest.raises(F.FdsError, match="timeout"):
        F.check_status()
    out = F.flexrel_attention(q, B, H, r, grid_ctas=grid)
    F.check_status()
    _check(O.flexrel_attention(qkv, B, H, rel), out)


def test_split_grids_share_one_workspace(cuda_device):
    """Calls with different piece counts on one stream share its workspace: the
    part counts live at fixed places, apart from the part slots, and stay zero
    between calls."""
    B, L, H = 1, 1000, 16
    qkv, rel = _inputs(B, L, H, seed=6)
    exp = O.flexrel_attention(qkv, B, H, rel)
    q, r = qkv.to(cuda_device), rel.to(cuda_device)
    for grid in (5, 37, 13, 64, 17, 5, 37):
        _assert_split(B, L, H, grid)
        out = F.flexrel_attention(q, B, H, r, grid_ctas=grid)
        F.check_status()
        _check(exp, out)
