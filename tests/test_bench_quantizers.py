"""The benchmark's synthetic-weight quantizers (torch, run on the GPU in bench.py) produce valid
GGUF blocks: decoded by the oracle they reproduce the input to the type's precision."""
import numpy as np
import pytest
import torch

import bench
import oracle


@pytest.mark.parametrize("quant,tol", [("q4_k", 0.1), ("q8_0", 0.01), ("q4_1", 0.1), ("q6_k", 0.03)])
def test_quantizer_roundtrip(quant, tol):
    t, fn, _ = bench.quantizer(quant)
    x = torch.from_numpy(oracle.randn(41, (24, 1024), 0.02))
    raw = fn(x).numpy()
    assert raw.shape == (24, oracle.codec.row_bytes(t, 1024))
    y = oracle.dequantize(raw, t, (24, 1024))
    err = np.linalg.norm(y - x.numpy()) / np.linalg.norm(x.numpy())
    assert err < tol, err
