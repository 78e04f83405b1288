"""The C ABI without a GPU: the library loads, exports every symbol the public
header declares, and rejects invalid arguments before touching any device;
the Python op layer validates shapes/dtypes like the reference's asserts."""

import ctypes
import re
from pathlib import Path

import pytest
import torch

import fastdialoguesidon_b200 as F
from fastdialoguesidon_b200 import _native as N

HEADER = Path(__file__).resolve().parents[1] / "include" / "fds_b200.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    return re.findall(r"FDS_API\s+[\w\s\*]+?\b(fds_\w+)\s*\(", text)


def test_header_and_binding_agree():
    names = declared_functions()
    assert sorted(names) == sorted(N.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol():
    lib = N.load()
    for name in declared_functions():
        assert hasattr(lib, name), name
    assert lib.fds_abi_version() == N.ABI_VERSION
    assert lib.fds_attn_smem_bytes() <= 232448  # fits one B200 CTA


def test_struct_layouts_match_header():
    text = HEADER.read_text()
    for struct, cls in (("FdsFlexRelArgs", N.FdsFlexRelArgs), ("FdsRopeArgs", N.FdsRopeArgs),
                        ("FdsLinearArgs", N.FdsLinearArgs), ("FdsFlexRelQrArgs", N.FdsFlexRelQrArgs)):
        body = re.search(r"typedef struct %s \{(.*?)\} %s;" % (struct, struct), text, re.S).group(1)
        fields = re.findall(r"^\s*[\w\s\*]+?\b(\w+);", body, re.M)
        assert fields == [f[0] for f in cls._fields_], (struct, fields)


def _flexrel_args(**kw):
    base = dict(qkv=16, qkv_row_stride=3072, rel=16, out=16, out_row_stride=1024, kv_len=None, status=None,
                batch=1, heads=16, seq_len=100, head_dim=64, dtype=N.FDS_DTYPE_FP16, scale=0.125,
                timeout_ns=0, debug_flags=0)
    base.update(kw)
    return N.FdsFlexRelArgs(**base)


@pytest.mark.parametrize("bad", [
    dict(head_dim=128), dict(dtype=7), dict(batch=0), dict(seq_len=0), dict(heads=0),
    dict(qkv_row_stride=3000), dict(qkv_row_stride=3076), dict(out_row_stride=1000),
    dict(qkv=0), dict(qkv=18), dict(rel=0), dict(scale=0.0), dict(batch=5000, heads=16),
])
def test_c_abi_rejects_invalid_arguments_before_launch(bad):
    lib = N.load()
    rc = lib.fds_flexrel_attn_fwd(ctypes.byref(_flexrel_args(**bad)), None)
    assert rc == N.FDS_ERR_INVALID_ARGUMENT
    assert lib.fds_last_error()  # a message explains it
    assert lib.fds_flexrel_attn_fwd(None, None) == N.FDS_ERR_INVALID_ARGUMENT


def test_c_abi_rope_split_rejects_invalid_arguments():
    lib = N.load()
    rc = lib.fds_rope_split(16, 2304, 16, 16, 16, 10, 10, 12, 32, N.FDS_DTYPE_FP16, None)
    assert rc == N.FDS_ERR_INVALID_ARGUMENT
    rc = lib.fds_rope_split(16, 2300, 16, 16, 16, 10, 10, 12, 64, N.FDS_DTYPE_FP16, None)
    assert rc == N.FDS_ERR_INVALID_ARGUMENT


def _linear_args(**kw):
    base = dict(a=16, a_row_stride=1024, w=16, w_row_stride=1024, bias=None, out=16, out_row_stride=3072,
                cos=None, sin=None, status=None, status_host=None, m=6000, n=3072, k=1024,
                dtype=N.FDS_DTYPE_FP16, epilogue=N.FDS_EPILOGUE_STORE, seq_len=0, rope_cols=0, timeout_ns=0,
                grid_ctas=0)
    base.update(kw)
    return N.FdsLinearArgs(**base)


@pytest.mark.parametrize("bad", [
    dict(k=1000, a_row_stride=1000, w_row_stride=1000), dict(n=3000, out_row_stride=3000), dict(m=0),
    dict(dtype=5), dict(epilogue=9), dict(a=0), dict(w=0), dict(out=0), dict(a=24), dict(bias=8),
    dict(a_row_stride=1000), dict(out_row_stride=3000), dict(epilogue=N.FDS_EPILOGUE_ROPE, seq_len=100),
    dict(epilogue=N.FDS_EPILOGUE_ROPE, cos=16, sin=16, seq_len=0, rope_cols=128),
    dict(epilogue=N.FDS_EPILOGUE_ROPE, cos=16, sin=16, seq_len=100, rope_cols=100),
    dict(epilogue=N.FDS_EPILOGUE_ROPE, cos=16, sin=16, seq_len=100, rope_cols=4096),
    dict(epilogue=N.FDS_EPILOGUE_ACCUMULATE_F32, out_row_stride=3070),
])
def test_c_abi_linear_rejects_invalid_arguments_before_launch(bad):
    lib = N.load()
    rc = lib.fds_linear_fwd(ctypes.byref(_linear_args(**bad)), None)
    assert rc == N.FDS_ERR_INVALID_ARGUMENT, bad
    assert lib.fds_last_error()
    assert lib.fds_linear_fwd(None, None) == N.FDS_ERR_INVALID_ARGUMENT


def _qr_args(**kw):
    base = dict(q=16, k=16, v=16, qr=16, out=16, kv_len=None, status=None, status_host=None, batch=1, heads=16,
                seq_len=100, head_dim=64, dtype=N.FDS_DTYPE_FP16, heads_last=1, scale=0.125, timeout_ns=0,
                debug_flags=0)
    base.update(kw)
    return N.FdsFlexRelQrArgs(**base)


@pytest.mark.parametrize("bad", [
    dict(head_dim=32), dict(dtype=4), dict(batch=0), dict(seq_len=0), dict(q=0), dict(qr=0), dict(k=24),
    dict(qr=17), dict(scale=-1.0), dict(batch=5000),
])
def test_c_abi_qr_rejects_invalid_arguments_before_launch(bad):
    lib = N.load()
    assert lib.fds_flexrel_qr_attn_fwd(ctypes.byref(_qr_args(**bad)), None) == N.FDS_ERR_INVALID_ARGUMENT
    assert lib.fds_last_error()


def test_linear_validation():
    x = torch.zeros(100, 1024, dtype=torch.float16)
    w = torch.zeros(3072, 1024, dtype=torch.float16)
    with pytest.raises(F.FdsError):
        F.linear(x, torch.zeros(3072, 1000, dtype=torch.float16))        # in_features mismatch
    with pytest.raises(F.FdsError):
        F.linear(x[:, :1000], torch.zeros(3072, 1000, dtype=torch.float16))  # k not a multiple of 64
    with pytest.raises(F.FdsError):
        F.linear(x, w, torch.zeros(3071, dtype=torch.float16))           # bias shape
    with pytest.raises(F.FdsError):
        F.accumulate(torch.zeros(100, 3072, dtype=torch.float16), x, w)  # residual must be fp32
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        F.linear(x, w)                                                  # valid shapes, CPU tensors


def test_op_validation_mirrors_reference_asserts():
    """Bad shapes raise FdsError, which is an AssertionError like the reference's checks."""
    qkv = torch.zeros(100, 3 * 1024, dtype=torch.float16)
    rel = torch.zeros(73, 64, dtype=torch.float16)
    with pytest.raises(AssertionError):
        F.flexrel_attention(qkv, 1, 8, rel)                       # head_dim 128
    with pytest.raises(AssertionError):
        F.flexrel_attention(qkv, 1, 16, torch.zeros(72, 64, dtype=torch.float16))
    with pytest.raises(F.FdsError):
        F.flexrel_attention(qkv.float(), 1, 16, rel.float())      # fp32 operands
    with pytest.raises(F.FdsError):
        F.flexrel_attention(qkv, 3, 16, rel)                      # rows not a multiple of batch
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        F.flexrel_attention(qkv, 1, 16, rel)                      # valid shapes, CPU tensors
    with pytest.raises(F.FdsError):
        F.encoder_attention(qkv, 1, 16, rel, impl="magic")
    with pytest.raises(F.FdsError):
        F.rope_attention(torch.zeros(10, 2304, dtype=torch.float16), 1, 12, torch.zeros(5, 64), torch.zeros(5, 64))


def test_no_cpu_fallback_in_product_path():
    """The package never imports the oracle."""
    import sys

    pkg = Path(F.__file__).resolve().parent
    for py in pkg.rglob("*.py"):
        assert "oracle" not in py.read_text().replace("oracles", ""), py
    assert all(not m.startswith("oracle") for m in sys.modules if m.startswith("fastdialoguesidon_b200"))
