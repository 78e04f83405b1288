"""Generate the golden fixtures in this directory from the REFERENCE itself.

Run once in a container where the reference checkout is importable:

    python tests/golden/make_golden.py /path/to/FastDialogueSidon
    (or FDS_REFERENCE_ROOT=/path/to/FastDialogueSidon python tests/golden/make_golden.py)

It imports the reference's own fp32 modules -- FlexRelSelfAttention with eager
flex_attention (triton/src/fds_triton/reference/modeling.py:33-122),
explicit_core_fp32 (trt/src/fastdialoguesidon/flexrel_triton.py:282-295),
_attn_ref (triton/tests/test_kernels.py:98-109) and DiTBlock._apply_rope +
F.scaled_dot_product_attention (modeling.py:243-312) -- on seeded inputs, and
writes inputs + outputs as .npz. The tests then pin the repository's oracle
against these files without needing the reference at run time.
"""

from __future__ import annotations

import json
import math
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _import_reference(root: Path):
    os.environ["FDS_FLEX_NO_COMPILE"] = "1"
    sys.path.insert(0, str(root / "triton" / "src"))
    sys.path.insert(0, str(root / "trt" / "src"))
    sys.path.insert(0, str(root / "triton" / "tests"))
    from fds_triton.reference import modeling  # noqa: E402
    from fastdialoguesidon import flexrel_triton  # noqa: E402
    import test_kernels  # noqa: E402
    return modeling, flexrel_triton, test_kernels


def _identity_attention(modeling, hidden: int, heads: int, rel: torch.Tensor):
    """FlexRelSelfAttention whose q/k/v/out projections are the identity, so the
    module output is exactly its attention core."""
    m = modeling.FlexRelSelfAttention(hidden, heads, 64, 8).eval()
    with torch.no_grad():
        eye = torch.eye(hidden)
        for lin in (m.linear_q, m.linear_k, m.linear_v, m.linear_out):
            lin.weight.copy_(eye)
            lin.bias.zero_()
        m.distance_embedding.weight.copy_(rel)
    return m


def _hf_additive_mask(batch: int, length: int, kv_len) -> torch.Tensor:
    """[B, 1, L, L] additive key-padding mask as transformers builds it for
    Wav2Vec2Bert (finfo.min on padded key columns)."""
    mask = torch.zeros(batch, 1, length, length)
    for b, n in enumerate(kv_len):
        mask[b, :, :, n:] = torch.finfo(torch.float32).min
    return mask


def core_case(refs, name: str, batch: int, length: int, heads: int, seed: int, kv_len=None) -> dict:
    modeling, ft, tk = refs
    gen = torch.Generator().manual_seed(seed)
    hid = heads * 64
    qkv = torch.randn(batch * length, 3 * hid, generator=gen).half()
    rel = torch.randn(73, 64, generator=gen).half()
    x = qkv.float()
    q, k, v = (x[:, i * hid:(i + 1) * hid].reshape(batch, length, hid) for i in range(3))
    # FlexRelSelfAttention projects one hidden tensor; feed q, k, v through
    # identity projections by running the core it builds (score_mod path).
    m = _identity_attention(modeling, hid, heads, rel.float())
    with torch.no_grad():
        shape = (batch, length, heads, 64)
        qh, kh, vh = (t.view(shape).transpose(1, 2) for t in (q, k, v))
        query_rel = torch.einsum("bhld,rd->bhlr", qh, m.distance_embedding.weight) / math.sqrt(64)
        mask = None if kv_len is None else _hf_additive_mask(batch, length, kv_len)[:, 0]

        def score_mod(score, b, h, qi, kj):
            s = score + query_rel[b, h, qi, torch.clamp(kj - qi, -64, 8) + 64]
            return s if mask is None else s + mask[b, qi, kj]

        flex = m._flex()(qh, kh, vh, score_mod=score_mod)
        flex = flex.transpose(1, 2).reshape(batch * length, hid)
        extra = {}
        if kv_len is None:
            exp = ft.explicit_core_fp32(qh, kh, vh, rel.float()).transpose(1, 2).reshape(batch * length, hid)
            tref = tk._attn_ref(qkv.float(), batch, heads, rel.float())
            # the module forward on identity projections must agree too
            if batch * length <= 4096:
                mod = m(x[:, :hid].reshape(batch, length, hid))[0]  # q = k = v = x_q here
                extra["module_self_check"] = float(
                    (mod.reshape(batch * length, hid) - ft.explicit_core_fp32(
                        *(x[:, :hid].reshape(batch, length, heads, 64).transpose(1, 2),) * 3,
                        rel.float()).transpose(1, 2).reshape(batch * length, hid)).abs().max())
            extra["flex_vs_explicit_max_abs"] = float((flex - exp).abs().max())
            extra["flex_vs_attn_ref_max_abs"] = float((flex - tref).abs().max())
    out = {"qkv": qkv.numpy(), "rel": rel.numpy(), "expected": flex.numpy().astype(np.float32)}
    if kv_len is not None:
        out["kv_len"] = np.asarray(kv_len, dtype=np.int32)
    meta = {"name": name, "batch": batch, "length": length, "heads": heads, "seed": seed,
            "source": "FlexRelSelfAttention score_mod + flex_attention (eager, fp32)", **extra}
    np.savez_compressed(HERE / f"{name}.npz", meta=json.dumps(meta), **out)
    return meta


def layer_case(refs, name: str, length: int, seed: int) -> dict:
    """one full FlexRelSelfAttention layer (with projections),
    B=1, hidden 1024 = 16 x 64, x ~ N(0,1), weights ~ N(0, 0.02), zero bias,
    rel ~ N(0, 0.02). The weights are regenerated from ``seed`` by the test
    (same recipe), so only summaries of the output are stored."""
    modeling, _, _ = refs
    gen = torch.Generator().manual_seed(seed)
    hidden, heads = 1024, 16
    x = torch.randn(1, length, hidden, generator=gen)
    ws = [torch.randn(hidden, hidden, generator=gen) * 0.02 for _ in range(4)]
    rel = torch.randn(73, 64, generator=gen) * 0.02
    m = modeling.FlexRelSelfAttention(hidden, heads, 64, 8).eval()
    with torch.no_grad():
        for lin, w in zip((m.linear_q, m.linear_k, m.linear_v, m.linear_out), ws):
            lin.weight.copy_(w)
            lin.bias.zero_()
        m.distance_embedding.weight.copy_(rel)
        y = m(x)[0][0]
    rows = np.array([0, 1, 63, 64, 71, 72, 73, 374, length - 9, length - 8, length - 1])
    meta = {"name": name, "length": length, "hidden": hidden, "heads": heads, "seed": seed,
            "recipe": "gen=Generator().manual_seed(seed); x=randn(1,L,1024); 4x W=randn(1024,1024)*0.02 "
                      "(q,k,v,out); rel=randn(73,64)*0.02; zero biases",
            "source": "FlexRelSelfAttention.forward (eager flex_attention, fp32)"}
    np.savez_compressed(HERE / f"{name}.npz", meta=json.dumps(meta), rows=rows,
                        expected_rows=y[rows].numpy(), row_norms=y.norm(dim=1).numpy(),
                        col_sums=y.sum(0).numpy())
    return meta


def rope_case(refs, name: str, batch: int, length: int, heads: int, seed: int) -> dict:
    modeling, _, _ = refs
    gen = torch.Generator().manual_seed(seed)
    hid = heads * 64
    qkv = torch.randn(batch * length, 3 * hid, generator=gen).half()
    blk = modeling.DiTBlock(hid, heads).eval()
    x = qkv.float()
    shape = (batch, length, heads, 64)
    q, k, v = (x[:, i * hid:(i + 1) * hid].reshape(shape) for i in range(3))
    with torch.no_grad():
        qr, kr = blk._apply_rope(q, k)
        att = torch.nn.functional.scaled_dot_product_attention(
            qr.permute(0, 2, 1, 3), kr.permute(0, 2, 1, 3), v.permute(0, 2, 1, 3))
        att = att.permute(0, 2, 1, 3).reshape(batch * length, hid)
    meta = {"name": name, "batch": batch, "length": length, "heads": heads, "seed": seed,
            "source": "DiTBlock._apply_rope + F.scaled_dot_product_attention (fp32)"}
    np.savez_compressed(HERE / f"{name}.npz", meta=json.dumps(meta), qkv=qkv.numpy(),
                        q_rot=qr.reshape(batch * length, hid).numpy(), k_rot=kr.reshape(batch * length, hid).numpy(),
                        expected=att.numpy().astype(np.float32))
    return meta


def main(root: str) -> None:
    refs = _import_reference(Path(root))
    metas = [
        core_case(refs, "core_b1_l64_h16", 1, 64, 16, seed=0),
        core_case(refs, "core_b1_l500_h2", 1, 500, 2, seed=1),
        core_case(refs, "core_b2_l333_h1", 2, 333, 1, seed=2),
        core_case(refs, "core_b1_l160_h2", 1, 160, 2, seed=3),
        core_case(refs, "core_b1_l1_h2", 1, 1, 2, seed=4),
        core_case(refs, "core_b3_l7_h2", 3, 7, 2, seed=5),
        core_case(refs, "core_b1_l73_h2", 1, 73, 2, seed=6),
        core_case(refs, "core_b2_l300_h1_masked", 2, 300, 1, seed=7, kv_len=[117, 300]),
        core_case(refs, "core_b3_l130_h1_masked", 3, 130, 1, seed=8, kv_len=[1, 64, 129]),
        layer_case(refs, "layer_cfg1_l750", 750, seed=0),
        rope_case(refs, "rope_b2_l97_h2", 2, 97, 2, seed=9),
    ]
    for m in metas:
        print(json.dumps(m))


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("FDS_REFERENCE_ROOT")
    if not root:
        raise SystemExit("usage: make_golden.py <reference checkout> (or set FDS_REFERENCE_ROOT)")
    main(root)
