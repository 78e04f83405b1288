"""The CPU oracle against the golden fixtures generated from the reference
(tests/golden/make_golden.py) and against its own fp64 restatement."""

import json

import numpy as np
import pytest
import torch

from oracle import flexrel_oracle as O
from conftest import golden_names, load_golden


@pytest.mark.parametrize("name", golden_names("core_"))
def test_core_matches_reference(name):
    g = load_golden(name)
    m = g["meta"]
    qkv = torch.from_numpy(g["qkv"])
    rel = torch.from_numpy(g["rel"])
    kv = g.get("kv_len")
    out = O.flexrel_attention(qkv, m["batch"], m["heads"], rel, kv_len=None if kv is None else torch.from_numpy(kv))
    exp = torch.from_numpy(g["expected"])
    assert O.max_abs(exp, out) < 2e-5, O.max_abs(exp, out)
    # the reference's own restatements agree exactly with its flex path
    for key in ("flex_vs_explicit_max_abs", "flex_vs_attn_ref_max_abs"):
        if key in m:
            assert m[key] < 1e-5


@pytest.mark.parametrize("name", ["core_b1_l160_h2", "core_b3_l7_h2", "core_b1_l73_h2"])
def test_core_fp32_vs_fp64(name):
    g = load_golden(name)
    m = g["meta"]
    qkv = torch.from_numpy(g["qkv"])
    rel = torch.from_numpy(g["rel"])
    q, k, v = O.split_qkv(qkv, m["batch"], m["heads"])
    ref64 = O.merge_heads(torch.from_numpy(O.flexrel_core_f64(q.numpy(), k.numpy(), v.numpy(), rel.float().numpy())))
    out = O.flexrel_attention(qkv, m["batch"], m["heads"], rel)
    assert O.max_abs(ref64, out) < 2e-5


def test_chunking_is_exact():
    g = load_golden("core_b1_l500_h2")
    qkv, rel = torch.from_numpy(g["qkv"]), torch.from_numpy(g["rel"])
    a = O.flexrel_attention(qkv, 1, 2, rel, chunk=512)
    b = O.flexrel_attention(qkv, 1, 2, rel, chunk=37)
    assert O.max_abs(a, b) < 1e-6


def test_config1_layer_matches_reference():
    """one full layer with projections, regenerated from the
    fixture's seed with the same recipe, against the reference module's output."""
    g = load_golden("layer_cfg1_l750")
    m = g["meta"]
    gen = torch.Generator().manual_seed(m["seed"])
    L, C = m["length"], m["hidden"]
    x = torch.randn(1, L, C, generator=gen)
    ws = [torch.randn(C, C, generator=gen) * 0.02 for _ in range(4)]
    rel = torch.randn(73, 64, generator=gen) * 0.02
    zero = torch.zeros(C)
    y = O.flexrel_layer(x, ws[0], zero, ws[1], zero, ws[2], zero, ws[3], zero, rel, m["heads"])[0]
    rows = torch.from_numpy(g["rows"])
    assert O.max_abs(torch.from_numpy(g["expected_rows"]), y[rows]) < 1e-5
    assert O.max_abs(torch.from_numpy(g["row_norms"]), y.norm(dim=1)) < 1e-4
    assert O.max_abs(torch.from_numpy(g["col_sums"]), y.sum(0)) < 1e-3


@pytest.mark.parametrize("name", golden_names("rope_"))
def test_rope_matches_reference(name):
    g = load_golden(name)
    m = g["meta"]
    B, L, H = m["batch"], m["length"], m["heads"]
    qkv = torch.from_numpy(g["qkv"])
    cos, sin = O.rope_tables(L)
    split = O.rope_split(qkv, L, H, cos, sin)
    assert O.max_abs(torch.from_numpy(g["q_rot"]), split[0]) < 1e-5
    assert O.max_abs(torch.from_numpy(g["k_rot"]), split[1]) < 1e-5
    out = O.rope_attention(qkv, B, H, cos, sin)
    assert O.max_abs(torch.from_numpy(g["expected"]), out) < 2e-5


def test_rope_tables_match_library_tables():
    """The library's fp32 tables (device path) are built the way the reference builds them."""
    import fastdialoguesidon_b200 as F

    c1, s1 = O.rope_tables(300)
    c2, s2 = F.rope_tables(300)
    assert torch.equal(c1, c2) and torch.equal(s1, s2)


def test_kv_len_semantics():
    """kv_len masks keys only; every row attends over the valid keys; 0 gives zeros."""
    gen = torch.Generator().manual_seed(0)
    qkv = torch.randn(2 * 50, 3 * 64, generator=gen)
    rel = torch.randn(73, 64, generator=gen)
    out = O.flexrel_attention(qkv, 2, 1, rel, kv_len=torch.tensor([0, 20]))
    assert torch.count_nonzero(out[:50]) == 0
    # window 1: the explicit formula with keys >= 20 excluded
    q, k, v = O.split_qkv(qkv[50:], 1, 1)
    s = (q @ k.transpose(-1, -2) + torch.gather(
        torch.einsum("bhld,rd->bhlr", q, rel), 3, O.rel_index(50).view(1, 1, 50, 50))) / 8.0
    s[..., 20:] = float("-inf")
    exp = O.merge_heads(torch.softmax(s, -1) @ v)
    assert O.max_abs(exp, out[50:]) < 1e-5


def test_exp2_polynomial_error_bound():
    """The kernels' software 2^x (fds_ptx.cuh exp2_poly2), evaluated here in
    fp32 with the same steps (each FMA with a single rounding), stays within
    1e-4 relative error of exp2 over the softmax's working range, gives tiny
    non-negative values below its clamp (-inf included) and huge finite values
    above it (no inf or NaN whatever the input)."""
    src = open(__import__("pathlib").Path(__file__).resolve().parents[1] /
               "fastdialoguesidon_b200" / "csrc" / "fds_ptx.cuh").read()
    import re
    body = src.split("float2 exp2_poly2(")[1]
    c3, c2, c1, c0 = [np.float32(v) for v in re.findall(r"make_float2\((0\.[0-9]+)f, 0\.[0-9]+f\)", body)[:4]]
    lo = np.float32(re.search(r"kPolyLo = (-?[0-9.]+)f", src).group(1))
    span = np.float32(re.search(r"kPolySpan = (-?[0-9.]+)f", src).group(1))

    def fma(a, b, c):  # one rounding (fp32 x fp32 products are exact in fp64)
        return (np.float64(1) * a * b + c).astype(np.float32)

    def exp2_poly(x):
        x = np.asarray(x, dtype=np.float32)
        ky, kb = np.float32(1 / span), np.float32(-lo / span)  # mult = 1, add = 0
        with np.errstate(invalid="ignore", over="ignore"):
            y = np.clip(np.nan_to_num(fma(x, ky, kb), nan=0.0, posinf=1.0, neginf=0.0), 0, 1).astype(np.float32)
        shift = np.float32(12582912.0) + lo
        t = fma(y, span, shift)
        r = fma(t, np.float32(-1), shift)
        f = fma(y, span, r)
        q = fma(fma(fma(c3, f, c2), f, c1), f, c0)
        return (q.view(np.int32) + (t.view(np.int32) << 23)).view(np.float32).astype(np.float64)

    x = np.linspace(-120.0, 60.0, 400001, dtype=np.float32)
    rel_err = np.abs(exp2_poly(x) / np.exp2(x.astype(np.float64)) - 1)
    assert rel_err.max() < 1e-4, rel_err.max()
    below = exp2_poly(np.array([-126.6, -127, -200, -1e6, -3e38, -np.inf], dtype=np.float32))
    assert np.all(below >= 0) and np.all(below <= 2.0 ** -124), below
    above = exp2_poly(np.array([66.4, 67, 100, 1e6, 3e38, np.inf], dtype=np.float32))
    assert np.all(np.isfinite(above)) and np.all(above >= 2.0 ** 65), above


def test_qr_form_matches_the_core():
    """flexrel_core_qr (the plugin form, qr given) equals flexrel_core when qr
    is q.rel^T in fp32: the QR-form oracle rests on the golden-pinned core."""
    gen = torch.Generator().manual_seed(12)
    q, k, v = (torch.randn(2, 3, 150, 64, generator=gen) for _ in range(3))
    rel = torch.randn(73, 64, generator=gen) * 0.3
    qr = torch.einsum("bhld,rd->bhlr", q, rel)
    for kv in (None, [150, 77]):
        a = O.flexrel_core(q, k, v, rel, kv_len=kv)
        b = O.flexrel_core_qr(q, k, v, qr, kv_len=kv)
        assert O.max_abs(a, b) < 1e-5
