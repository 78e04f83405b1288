"""The 13-layer config-2 window (L = 6000, 16 x 64 heads) built with the
stacking rule the benchmark uses: an fp32 residual stream, x_0 ~ N(0, 1),
per layer qkv_i = fp16(x_i W_qkv,i^T), ctx_i = Attn_i(qkv_i), y_i = ctx_i
W_out,i^T (linear_out) and x_{i+1} = x_i + y_i, weights ~ N(0, 0.02), zero
biases, rel ~ N(0, 0.02).

Every layer is checked on its own inputs against the fp32 CPU oracle, before
and after linear_out: max-abs <= 2e-3 and SNR >= 55 dB (the north-star
tolerance). The stack as a whole is also run twice -- once through this
library, once through the oracle only (qkv rounded to fp16 as the model's
GEMM does) -- and the accumulated attention updates x_13 - x_0 of the two are
compared.
"""

import pytest
import torch

import fastdialoguesidon_b200 as F
from oracle import flexrel_oracle as O

pytestmark = pytest.mark.gpu

LAYERS, HEADS, L = 13, 16, 6000
MAX_ABS, MIN_SNR = 2e-3, 55.0
STACK_MIN_SNR = 50.0


def _weights(seed):
    g = torch.Generator().manual_seed(seed)
    hid = HEADS * 64
    x0 = torch.randn(L, hid, generator=g)
    layers = []
    for _ in range(LAYERS):
        w_qkv = torch.randn(3 * hid, hid, generator=g) * 0.02
        w_out = torch.randn(hid, hid, generator=g) * 0.02
        rel = (torch.randn(73, 64, generator=g) * 0.02).half()
        layers.append((w_qkv, w_out, rel))
    return x0, layers


def test_stacked_config2_window(cuda_device):
    x0, layers = _weights(seed=1000)
    x = x0.to(cuda_device)
    x_ref = x0.clone()
    worst = []
    for i, (w_qkv, w_out, rel) in enumerate(layers):
        wq, wo, r = w_qkv.to(cuda_device), w_out.to(cuda_device), rel.to(cuda_device)
        qkv = (x @ wq.t()).half()
        ctx = F.flexrel_attention(qkv, 1, HEADS, r)
        F.check_status()
        # this layer, on its own inputs: before and after linear_out
        exp_ctx = O.flexrel_attention(qkv.cpu(), 1, HEADS, rel)
        got_ctx = ctx.float().cpu()
        exp_y, got_y = exp_ctx @ w_out.t(), got_ctx @ w_out.t()
        for what, e, g in (("ctx", exp_ctx, got_ctx), ("linear_out", exp_y, got_y)):
            err, snr = O.max_abs(e, g), O.snr_db(e, g)
            worst.append((snr, err, i, what))
            assert err <= MAX_ABS and snr >= MIN_SNR, (i, what, err, snr)
        x = x + ctx.float() @ wo.t()
        # the oracle-only stack (its own fp16-rounded qkv)
        qkv_ref = (x_ref @ w_qkv.t()).half()
        x_ref = x_ref + O.flexrel_attention(qkv_ref, 1, HEADS, rel) @ w_out.t()
    delta, delta_ref = (x.cpu() - x0), (x_ref - x0)
    stack_snr = O.snr_db(delta_ref, delta)
    print(f"worst per-layer: {min(worst)}; stacked update x13 - x0: {stack_snr:.1f} dB, "
          f"max-abs {O.max_abs(delta_ref, delta):.2e}")
    assert stack_snr >= STACK_MIN_SNR, stack_snr
