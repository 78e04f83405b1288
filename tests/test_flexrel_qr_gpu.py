"""The TensorRT-plugin form of the relative-key attention (fds_flexrel_qr_attn_fwd,
flexrel_attention_qr): separate q, k, v and the given projections qr = q.rel^T
(rounded to the operand type, as the plugin's graph computes them), in the
plugin's [B, L, H, 64] / [B, L, H, 73] layout and in [B, H, L, ..], against the
CPU oracle of _flexrel_qr_body (trt/src/fastdialoguesidon/flexrel_triton.py:559).
Tolerance as the rest of the suite: max-abs <= 2e-3 and SNR >= 55 dB (fp16)."""

import pytest
import torch

import fastdialoguesidon_b200 as F
from oracle import flexrel_oracle as O

pytestmark = pytest.mark.gpu

MAX_ABS, MIN_SNR = 2e-3, 55.0


def _inputs(B, L, H, seed, std=0.64):
    g = torch.Generator().manual_seed(seed)
    q, k, v = ((torch.randn(B, L, H, 64, generator=g) * std).half() for _ in range(3))
    rel = (torch.randn(73, 64, generator=g) * 0.3).half()
    qr = torch.einsum("blhd,rd->blhr", q.float(), rel.float()).half()
    return q, k, v, rel, qr


def _check(exp, got):
    got = got.float().cpu()
    err, snr = O.max_abs(exp, got), O.snr_db(exp, got)
    assert err <= MAX_ABS and snr >= MIN_SNR, (err, snr)


@pytest.mark.parametrize("B,L,H", [(1, 500, 16), (2, 333, 16), (1, 6000, 16), (3, 130, 2)])
def test_heads_last_matches_oracle(cuda_device, B, L, H):
    q, k, v, rel, qr = _inputs(B, L, H, seed=L + B)
    d = cuda_device
    out = F.flexrel_attention_qr(q.to(d), k.to(d), v.to(d), qr.to(d))
    F.check_status()
    assert out.shape == (B, L, H, 64)
    t = (lambda x: x.permute(0, 2, 1, 3))  # [B, L, H, .] -> [B, H, L, .]
    exp = O.flexrel_core_qr(t(q), t(k), t(v), t(qr)).permute(0, 2, 1, 3)
    _check(exp, out)


def test_heads_first_layout_and_kv_len(cuda_device):
    B, L, H = 2, 1000, 4
    q, k, v, rel, qr = _inputs(B, L, H, seed=7)
    t = (lambda x: x.permute(0, 2, 1, 3).contiguous())
    d = cuda_device
    kv = torch.tensor([1000, 517], dtype=torch.int32)
    out = F.flexrel_attention_qr(t(q).to(d), t(k).to(d), t(v).to(d), t(qr).to(d), heads_last=False,
                                 kv_len=kv.to(d))
    F.check_status()
    exp = O.flexrel_core_qr(t(q), t(k), t(v), t(qr), kv_len=kv)
    _check(exp, out)


def test_agrees_with_the_fused_qkv_entry_point(cuda_device):
    """Given qr = q.rel^T, the plugin form and flexrel_attention on the fused
    qkv compute the same attention (up to qr's rounding to fp16)."""
    B, L, H = 1, 2000, 16
    q, k, v, rel, qr = _inputs(B, L, H, seed=11)
    d = cuda_device
    out = F.flexrel_attention_qr(q.to(d), k.to(d), v.to(d), qr.to(d)).reshape(B * L, H * 64)
    qkv = torch.cat([x.reshape(B * L, H * 64) for x in (q, k, v)], 1).to(d)
    ref = F.flexrel_attention(qkv, B, H, rel.to(d))
    F.check_status()
    assert O.max_abs(ref.float().cpu(), out.float().cpu()) <= MAX_ABS
    assert O.snr_db(ref.float().cpu(), out.float().cpu()) >= MIN_SNR


def test_bf16(cuda_device):
    """bf16 operands (the plugin accepts BF16|FP16): the reference's own bf16
    bar, SNR > 40 dB (triton/tests/test_kernels.py:119)."""
    B, L, H = 1, 700, 8
    g = torch.Generator().manual_seed(17)
    q, k, v = ((torch.randn(B, L, H, 64, generator=g) * 0.64).to(torch.bfloat16) for _ in range(3))
    rel = (torch.randn(73, 64, generator=g) * 0.3).to(torch.bfloat16)
    qr = torch.einsum("blhd,rd->blhr", q.float(), rel.float()).to(torch.bfloat16)
    d = cuda_device
    out = F.flexrel_attention_qr(q.to(d), k.to(d), v.to(d), qr.to(d))
    F.check_status()
    t = (lambda x: x.permute(0, 2, 1, 3))
    exp = O.flexrel_core_qr(t(q), t(k), t(v), t(qr)).permute(0, 2, 1, 3)
    assert O.snr_db(exp, out.float().cpu()) > 40.0
