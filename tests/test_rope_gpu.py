"""DiT RoPE attention and rope_split on the B200 vs the oracle and the
reference-generated golden fixture.

Tolerance: max-abs <= 2e-3 and SNR >= 55 dB vs fp32 for
the attention output; rope_split q/k SNR > 45 dB and v bit-exact, as the
reference's own test_rope_split (triton/tests/test_kernels.py:132-150).
"""

import pytest
import torch

import fastdialoguesidon_b200 as F
from oracle import flexrel_oracle as O
from conftest import golden_names, load_golden

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-3
MIN_SNR = 55.0


def _check(exp, got):
    got = got.float().cpu()
    err, snr = O.max_abs(exp, got), O.snr_db(exp, got)
    assert err <= MAX_ABS and snr >= MIN_SNR, (err, snr)


@pytest.mark.parametrize("name", golden_names("rope_"))
def test_golden_fixture(cuda_device, name):
    g = load_golden(name)
    m = g["meta"]
    B, L, H = m["batch"], m["length"], m["heads"]
    qkv = torch.from_numpy(g["qkv"]).to(cuda_device)
    cos, sin = F.rope_tables(L, cuda_device)
    split = F.rope_split(qkv, L, H, cos, sin)
    assert O.snr_db(torch.from_numpy(g["q_rot"]), split[0].float().cpu()) > 45
    assert O.snr_db(torch.from_numpy(g["k_rot"]), split[1].float().cpu()) > 45
    assert torch.equal(split[2], qkv[:, 2 * H * 64:])
    out = F.rope_attention(qkv, B, H, cos, sin)
    F.check_status()
    _check(torch.from_numpy(g["expected"]), out)


def test_reference_rope_split_shape(cuda_device):
    """triton/tests/test_kernels.py:132-150: B=2, L=97, H=12, tables of 200 rows, bf16."""
    torch.manual_seed(0)
    B, L, H = 2, 97, 12
    qkv = torch.randn(B * L, 3 * H * 64).bfloat16()
    cos, sin = F.rope_tables(200)
    out = F.rope_split(qkv.to(cuda_device), L, H, cos.to(cuda_device), sin.to(cuda_device))
    ref = O.rope_split(qkv, L, H, cos, sin)
    for part in range(2):
        assert O.snr_db(ref[part], out[part].float().cpu()) > 45
    assert torch.equal(out[2].cpu(), qkv[:, 2 * H * 64:])


@pytest.mark.parametrize("B,L", [(1, 1), (2, 97), (1, 129), (3, 300), (1, 1000)])
def test_rope_attention_shapes(cuda_device, B, L):
    H = 12
    gen = torch.Generator().manual_seed(L)
    qkv = torch.randn(B * L, 3 * H * 64, generator=gen).half()
    cos, sin = O.rope_tables(max(L, 8))
    exp = O.rope_attention(qkv, B, H, cos, sin, round_qk_to=torch.float16)
    out = F.rope_attention(qkv.to(cuda_device), B, H, cos.to(cuda_device), sin.to(cuda_device))
    F.check_status()
    _check(exp, out)


def test_config4_full_size(cuda_device):
    """BASELINE config 4 shape for one layer: L=6000, 12 x 64 heads, RoPE base 10000,
    q/k/v spread of x ~ N(0,1) projected by W ~ N(0, 0.02)."""
    B, L, H = 1, 6000, 12
    gen = torch.Generator().manual_seed(4)
    qkv = (torch.randn(B * L, 3 * H * 64, generator=gen) * 0.55).half()
    cos, sin = O.rope_tables(L)
    exp = O.rope_attention(qkv, B, H, cos, sin, round_qk_to=torch.float16)
    out = F.rope_attention(qkv.to(cuda_device), B, H, cos.to(cuda_device), sin.to(cuda_device))
    F.check_status()
    _check(exp, out)
    # against the unrounded fp32 reference too (the tolerance still holds)
    _check(O.rope_attention(qkv, B, H, cos, sin), out)


def test_torch_op_and_graph(cuda_device):
    B, L, H = 2, 500, 12
    gen = torch.Generator().manual_seed(5)
    qkv = torch.randn(B * L, 3 * H * 64, generator=gen).half().to(cuda_device)
    cos, sin = F.rope_tables(L, cuda_device)
    a = torch.ops.fds.rope_attention(qkv, B, H, cos, sin)
    out = torch.empty_like(a)
    scratch = torch.empty(B * L, 2 * H * 64, dtype=qkv.dtype, device=cuda_device)
    F.rope_attention(qkv, B, H, cos, sin, out=out, scratch=scratch)
    g = torch.cuda.CUDAGraph()
    out2 = torch.zeros_like(a)
    with torch.cuda.graph(g):
        F.rope_attention(qkv, B, H, cos, sin, out=out2, scratch=scratch)
    g.replay()
    torch.cuda.synchronize()
    F.check_status()
    assert torch.equal(a, out) and torch.equal(a, out2)
