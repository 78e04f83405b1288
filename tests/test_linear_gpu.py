"""The tcgen05 linear layers either side of the attention (fds_linear_fwd):

* ``linear`` = F.linear (triton/src/fds_triton/model.py:50, the QKV projection
  at :289) against the fp32 product, at the encoder's and the DiT's shapes;
* ``linear_rope`` = F.linear followed by rope_split (model.py:318-319) against
  the CPU oracle's rope_split of the fp16-rounded product;
* ``accumulate`` = torch.addmm(x, a, w.t(), out_dtype=fp32, out=x)
  (model.py:53-57, the out-projection at :291) against the fp32 update;
* whole attention layers built from them (encoder: QKV -> relative-key
  attention -> out-projection into the residual; DiT: QKV with RoPE ->
  attention over the rotated qkv) against the fp32 oracle, max-abs <= 2e-3 and
  SNR >= 55 dB on the attention output as elsewhere in the suite.

GEMM tolerances: the kernel accumulates in fp32 like cuBLAS, in a different
order, and rounds once to fp16 / bf16: |ours - fp32| <= 1 ulp of the operand
type at the output's largest magnitude, SNR >= 60 dB (fp16) / 45 dB (bf16).
"""

import pytest
import torch

import fastdialoguesidon_b200 as F
from oracle import flexrel_oracle as O

pytestmark = pytest.mark.gpu

ULP = {torch.float16: 2.0 ** -10, torch.bfloat16: 2.0 ** -7}
MIN_SNR = {torch.float16: 60.0, torch.bfloat16: 45.0}


def _operands(m, k, n, seed, dtype=torch.float16, device="cuda", bias=True):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(m, k, generator=g).to(dtype)
    w = (torch.randn(n, k, generator=g) * 0.02).to(dtype)
    b = (torch.randn(n, generator=g) * 0.1).to(dtype) if bias else None
    to = (lambda t: None if t is None else t.to(device))
    return x, w, b, to(x), to(w), to(b)


def _ref(x, w, b):
    y = x.double() @ w.double().t()
    if b is not None:
        y = y + b.double()
    return y.float()


def _check_gemm(ref, got, dtype):
    got = got.float().cpu()
    bound = ULP[dtype] * float(ref.abs().max()) + 1e-6
    err = O.max_abs(ref, got)
    assert err <= bound, (err, bound)
    assert O.snr_db(ref, got) >= MIN_SNR[dtype]


@pytest.mark.parametrize("m,k,n", [(6000, 1024, 3072), (6000, 768, 2304), (1000, 1024, 1024), (333, 1024, 3072),
                                   (1, 768, 256), (129, 64, 128)])
def test_linear_matches_fp32(cuda_device, m, k, n):
    x, w, b, xd, wd, bd = _operands(m, k, n, seed=m + n)
    _check_gemm(_ref(x, w, b), F.linear(xd, wd, bd), torch.float16)
    F.check_status()


def test_linear_bf16_no_bias_and_small_grid(cuda_device):
    """bf16, no bias, and 3 persistent CTAs walking many tiles each (accumulator
    double buffer and stage ring wrap many times)."""
    x, w, b, xd, wd, bd = _operands(1000, 1024, 3072, seed=5, dtype=torch.bfloat16, bias=False)
    _check_gemm(_ref(x, w, None), F.linear(xd, wd, None, grid_ctas=3), torch.bfloat16)
    F.check_status()


def test_linear_out_and_strided_rows(cuda_device):
    """out= written in place; A taken as a column slice of a wider buffer."""
    g = torch.Generator().manual_seed(9)
    wide = torch.randn(500, 1024 + 64, generator=g).half().to(cuda_device)
    x = wide[:, 32:32 + 1024]
    w = (torch.randn(1024, 1024, generator=g) * 0.02).half().to(cuda_device)
    out = torch.full((500, 1024), 7.0, dtype=torch.float16, device=cuda_device)
    ret = F.linear(x, w, None, out=out)
    assert ret.data_ptr() == out.data_ptr()
    _check_gemm(_ref(x.cpu(), w.cpu(), None), out, torch.float16)


@pytest.mark.parametrize("B,L", [(1, 6000), (2, 333)])
def test_linear_rope_matches_rope_split(cuda_device, B, L):
    H = 12
    hid = H * 64
    x, w, b, xd, wd, bd = _operands(B * L, hid, 3 * hid, seed=L)
    cos, sin = F.rope_tables(L, cuda_device)
    got = F.linear_rope(xd, wd, bd, cos, sin, L, H).float().cpu()
    y16 = _ref(x, w, b).half()
    exp = O.rope_split(y16, L, H, cos.cpu(), sin.cpu())  # [3, rows, hid] fp32: rotate the rounded product
    bound = 2 * ULP[torch.float16] * float(exp.abs().max()) + 1e-6
    for part in range(3):
        e, g_ = exp[part], got[:, part * hid:(part + 1) * hid]
        assert O.max_abs(e, g_) <= bound, (part, O.max_abs(e, g_), bound)
        assert O.snr_db(e, g_) >= 60.0
    F.check_status()


def test_accumulate_into_fp32_residual(cuda_device):
    m, k, n = 6000, 1024, 1024
    g = torch.Generator().manual_seed(3)
    x = torch.randn(m, n, generator=g)
    a = torch.randn(m, k, generator=g).half()
    w = (torch.randn(n, k, generator=g) * 0.02).half()
    xd = x.to(cuda_device)
    F.accumulate(xd, a.to(cuda_device), w.to(cuda_device))
    F.check_status()
    delta = (a.double() @ w.double().t()).float()
    exp = x + delta
    err = O.max_abs(exp, xd.cpu())
    assert err <= 1e-4 * float(delta.abs().max()) + 1e-5, err
    assert O.snr_db(delta, xd.cpu() - x) >= 90.0


def test_linear_graph_replay_is_bit_equal(cuda_device):
    x, w, b, xd, wd, bd = _operands(6000, 1024, 3072, seed=11)
    eager = F.linear(xd, wd, bd)
    out = torch.empty_like(eager)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        F.linear(xd, wd, bd, out=out)
    torch.cuda.current_stream().wait_stream(s)
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr, stream=s):
        F.linear(xd, wd, bd, out=out)
    out.zero_()
    gr.replay()
    torch.cuda.synchronize()
    F.check_status()
    assert torch.equal(out, eager)
    del gr


def test_encoder_attention_layer(cuda_device):
    """QKV projection (with bias) -> relative-key attention -> out-projection
    accumulated into the fp32 residual, all on the library, against the fp32
    oracle layer on the same fp16 weights (the attention on this layer's own
    fp16 qkv)."""
    L, H = 2000, 16
    hid = H * 64
    g = torch.Generator().manual_seed(21)
    x = torch.randn(L, hid, generator=g)
    w_qkv = (torch.randn(3 * hid, hid, generator=g) * 0.02).half()
    b_qkv = (torch.randn(3 * hid, generator=g) * 0.02).half()
    w_out = (torch.randn(hid, hid, generator=g) * 0.02).half()
    rel = (torch.randn(73, 64, generator=g) * 0.02).half()
    d = cuda_device
    xd = x.to(d)
    qkv = F.linear(xd.half(), w_qkv.to(d), b_qkv.to(d))
    ctx = F.flexrel_attention(qkv, 1, H, rel.to(d))
    F.accumulate(xd, ctx, w_out.to(d))
    F.check_status()
    exp_ctx = O.flexrel_attention(qkv.cpu(), 1, H, rel)
    err, snr = O.max_abs(exp_ctx, ctx.float().cpu()), O.snr_db(exp_ctx, ctx.float().cpu())
    assert err <= 2e-3 and snr >= 55.0, (err, snr)
    exp_x = x + exp_ctx.double().__matmul__(w_out.double().t()).float()
    dx_exp, dx_got = exp_x - x, xd.cpu() - x
    assert O.snr_db(dx_exp, dx_got) >= 55.0


def test_dit_attention_layer_with_rope_epilogue(cuda_device):
    """linear_rope -> rotated_attention (no RoPE pass, no scratch) equals the
    separate linear -> rope_attention path within the suite tolerance, and both
    match the fp32 oracle of the rotated attention."""
    B, L, H = 1, 3000, 12
    hid = H * 64
    x, w, b, xd, wd, bd = _operands(B * L, hid, 3 * hid, seed=31)
    cos, sin = F.rope_tables(L, cuda_device)
    fused = F.rotated_attention(F.linear_rope(xd, wd, bd, cos, sin, L, H), B, H)
    qkv = F.linear(xd, wd, bd)
    separate = F.rope_attention(qkv, B, H, cos, sin)
    F.check_status()
    exp = O.rope_attention(qkv.cpu(), B, H, cos.cpu(), sin.cpu(), round_qk_to=torch.float16)
    for got in (fused, separate):
        err, snr = O.max_abs(exp, got.float().cpu()), O.snr_db(exp, got.float().cpu())
        assert err <= 2e-3 and snr >= 55.0, (err, snr)


def test_linear_rope_bf16(cuda_device):
    B, L, H = 1, 1000, 12
    hid = H * 64
    x, w, b, xd, wd, bd = _operands(B * L, hid, 3 * hid, seed=41, dtype=torch.bfloat16)
    cos, sin = F.rope_tables(L, cuda_device)
    got = F.linear_rope(xd, wd, bd, cos, sin, L, H).float().cpu()
    y = _ref(x, w, b).to(torch.bfloat16)
    exp = O.rope_split(y, L, H, cos.cpu(), sin.cpu())
    bound = 2 * ULP[torch.bfloat16] * float(exp.abs().max()) + 1e-6
    for part in range(3):
        e, g_ = exp[part], got[:, part * hid:(part + 1) * hid]
        assert O.max_abs(e, g_) <= bound and O.snr_db(e, g_) >= MIN_SNR[torch.bfloat16], part
    F.check_status()


def test_accumulate_bf16_with_bias(cuda_device):
    m, k, n = 700, 768, 768
    g = torch.Generator().manual_seed(43)
    x = torch.randn(m, n, generator=g)
    a = torch.randn(m, k, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    bias = (torch.randn(n, generator=g) * 0.1).to(torch.bfloat16)
    xd = x.to(cuda_device)
    F.accumulate(xd, a.to(cuda_device), w.to(cuda_device), bias.to(cuda_device))
    F.check_status()
    delta = (a.double() @ w.double().t() + bias.double()).float()
    assert O.max_abs(x + delta, xd.cpu()) <= 1e-4 * float(delta.abs().max()) + 1e-5


@pytest.mark.parametrize("m,k,n", [(6000, 1024, 3072), (6000, 1024, 1024), (129, 64, 128), (257, 128, 256),
                                   (1, 64, 128)])
def test_pair_and_single_cta_tiles(cuda_device, m, k, n):
    """256-row tiles over CTA pairs (tcgen05 cta_group::2, the default for more
    than 128 rows) and 128-row tiles on one CTA each, forced both ways, against
    the fp32 product (m = 1 and 129: a pair whose second CTA has no valid row)."""
    x, w, b, xd, wd, bd = _operands(m, k, n, seed=m + 3 * n)
    ref = _ref(x, w, b)
    for pair in (True, False):
        _check_gemm(ref, F.linear(xd, wd, bd, pair=pair), torch.float16)
    F.check_status()


@pytest.mark.parametrize("grid_ctas", [2, 3, 4])
def test_pair_tiles_on_few_ctas(cuda_device, grid_ctas):
    """1-2 CTA pairs walking 24-48 tiles each (stage ring and accumulator
    double buffer wrap many times across the pair's barriers)."""
    x, w, b, xd, wd, bd = _operands(3000, 512, 2304, seed=grid_ctas)
    _check_gemm(_ref(x, w, b), F.linear(xd, wd, bd, grid_ctas=grid_ctas, pair=True), torch.float16)
    F.check_status()


@pytest.mark.parametrize("pair", [True, False])
def test_rope_and_accumulate_both_tilings(cuda_device, pair):
    B, L, H = 2, 700, 12
    hid = H * 64
    x, w, b, xd, wd, bd = _operands(B * L, hid, 3 * hid, seed=51)
    cos, sin = F.rope_tables(L, cuda_device)
    got = F.linear_rope(xd, wd, bd, cos, sin, L, H, pair=pair).float().cpu()
    exp = O.rope_split(_ref(x, w, b).half(), L, H, cos.cpu(), sin.cpu())
    bound = 2 * ULP[torch.float16] * float(exp.abs().max()) + 1e-6
    for part in range(3):
        assert O.max_abs(exp[part], got[:, part * hid:(part + 1) * hid]) <= bound, part
    m, k, n = B * L, 1024, 1024
    g = torch.Generator().manual_seed(53)
    r = torch.randn(m, n, generator=g)
    a = torch.randn(m, k, generator=g).half()
    wo = (torch.randn(n, k, generator=g) * 0.02).half()
    rd = r.to(cuda_device)
    F.accumulate(rd, a.to(cuda_device), wo.to(cuda_device), pair=pair)
    F.check_status()
    delta = (a.double() @ wo.double().t()).float()
    assert O.max_abs(r + delta, rd.cpu()) <= 1e-4 * float(delta.abs().max()) + 1e-5


@pytest.mark.parametrize("pair", [True, False])
def test_rope_cols_not_a_multiple_of_the_tile_half(cuda_device, pair):
    """fds_linear_fwd's RoPE epilogue rotates exactly the 64-column heads below
    rope_cols, also when rope_cols (here 192 of 512) ends inside the 128-column
    half of a tile one epilogue warp writes."""
    from fastdialoguesidon_b200 import _native as N
    from fastdialoguesidon_b200.kernels import _linear_call
    L, n, k, rope_cols = 300, 512, 256, 192
    x, w, b, xd, wd, bd = _operands(2 * L, k, n, seed=61)
    cos, sin = F.rope_tables(L, cuda_device)
    out = torch.empty(2 * L, n, dtype=torch.float16, device=cuda_device)
    _linear_call(xd, wd, bd, out, N.FDS_EPILOGUE_ROPE, cos=cos, sin=sin, seq_len=L, rope_cols=rope_cols, pair=pair)
    F.check_status()
    y = _ref(x, w, b).half().float()                       # F.linear rounded to fp16
    pos = torch.arange(2 * L) % L
    c, s = cos.cpu()[pos], sin.cpu()[pos]                  # [rows, 64]
    exp = y.clone()
    for h in range(rope_cols // 64):
        blk = y[:, 64 * h:64 * (h + 1)]
        rot = torch.cat([-blk[:, 32:], blk[:, :32]], dim=1)
        exp[:, 64 * h:64 * (h + 1)] = blk * c + rot * s
    got = out.float().cpu()
    bound = 2 * ULP[torch.float16] * float(exp.abs().max()) + 1e-6
    assert O.max_abs(exp, got) <= bound  # a rotated head past rope_cols (or one left out) is far off
