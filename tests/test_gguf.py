"""GGUF reader (mb_gguf_inspect) on files written by the gguf 0.19.0 package; no GPU."""
import numpy as np
import pytest

import mold_b200 as mb
import oracle
from oracle import flux_ref as F
from tests.gguf_util import write_gguf


def test_inspect_lists_names_types_shapes(tmp_path):
    x = oracle.randn(1, (64, 512), 0.02)
    t = {
        "a.weight": F.QTensorRef(oracle.GGML_Q8_0, (64, 512), oracle.quantize(x, oracle.GGML_Q8_0)),
        "b.weight": F.QTensorRef(oracle.GGML_Q6_K, (64, 512), oracle.quantize(x, oracle.GGML_Q6_K)),
        "c.weight": F.QTensorRef(oracle.GGML_Q4_1, (64, 512), oracle.quantize(x, oracle.GGML_Q4_1)),
        "b.bias": F.QTensorRef(oracle.GGML_F32, (64,), oracle.quantize(x[0, :64], oracle.GGML_F32)),
    }
    p = tmp_path / "t.gguf"
    write_gguf(p, t)
    got = {n: (ty, sh) for n, ty, sh in mb.gguf_inspect(p)}
    assert got == {"a.weight": (8, (64, 512)), "b.weight": (14, (64, 512)), "c.weight": (3, (64, 512)),
                   "b.bias": (0, (64,))}


def test_inspect_rejects_bad_files(tmp_path):
    p = tmp_path / "bad.gguf"
    p.write_bytes(b"NOTGGUF" + bytes(64))
    with pytest.raises(mb.MoldError):
        mb.gguf_inspect(p)
    with pytest.raises(mb.MoldError):
        mb.gguf_inspect(tmp_path / "absent.gguf")
    # truncated tensor data
    x = oracle.randn(2, (32, 256), 0.02)
    q = tmp_path / "trunc.gguf"
    write_gguf(q, {"w": F.QTensorRef(oracle.GGML_Q8_0, (32, 256), oracle.quantize(x, oracle.GGML_Q8_0))})
    data = q.read_bytes()
    q.write_bytes(data[: len(data) - 100])
    with pytest.raises(mb.MoldError):
        mb.gguf_inspect(q)
