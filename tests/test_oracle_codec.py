"""The oracle's GGML codecs against golden vectors from the gguf 0.19.0 package."""
import os

import numpy as np
import pytest

import oracle

GOLD = os.path.join(os.path.dirname(__file__), "golden", "codec_golden.npz")


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD)


def test_q8_0_quantize_matches_gguf(gold):
    q = oracle.quantize(gold["q8_in"], oracle.GGML_Q8_0)
    assert np.array_equal(q.reshape(-1), gold["q8_blocks"].reshape(-1))


def test_q8_0_dequant_bit_exact(gold):
    d = oracle.dequantize(gold["q8_blocks"], oracle.GGML_Q8_0, gold["q8_in"].shape)
    assert np.array_equal(d.view(np.uint32), gold["q8_deq"].astype(np.float32).view(np.uint32))


def test_q4_k_dequant_bit_exact_random_blocks(gold):
    blocks = gold["q4k_blocks"]
    d = oracle.dequantize(blocks, oracle.GGML_Q4_K, (blocks.shape[0], 256))
    ref = gold["q4k_deq"].astype(np.float32)
    assert np.array_equal(d.view(np.uint32), ref.view(np.uint32))


def test_f16_conversion_matches_numpy():
    rng = np.random.default_rng(0)
    bits = rng.integers(0, 65536, size=200000, dtype=np.uint32).astype(np.uint16)
    bits = bits[~np.isnan(bits.view(np.float16))]
    lib = oracle.codec._load()
    out = np.empty(bits.size, dtype=np.float32)
    lib.or_f16_to_f32.argtypes = [oracle.codec.ctypes.c_void_p, oracle.codec.ctypes.c_int64, oracle.codec.ctypes.c_void_p]
    lib.or_f16_to_f32(bits.ctypes.data, bits.size, out.ctypes.data)
    assert np.array_equal(out, bits.view(np.float16).astype(np.float32))
    x = (rng.standard_normal(200000) * np.exp(rng.uniform(-20, 12, 200000))).astype(np.float32)
    h = np.empty(x.size, dtype=np.uint16)
    lib.or_f32_to_f16.argtypes = lib.or_f16_to_f32.argtypes
    lib.or_f32_to_f16(x.ctypes.data, x.size, h.ctypes.data)
    assert np.array_equal(h, x.astype(np.float16).view(np.uint16))


def test_q4_k_quantizer_roundtrip_error():
    x = oracle.randn(3, (64, 1024), 0.02)
    q = oracle.quantize(x, oracle.GGML_Q4_K)
    assert q.shape == (64, 1024 // 256 * 144)
    d = oracle.dequantize(q, oracle.GGML_Q4_K, x.shape)
    err = np.linalg.norm(d - x) / np.linalg.norm(x)
    assert err < 0.1


def test_q4_k_edge_blocks():
    # all-zero rows and constant rows decode exactly
    x = np.zeros((2, 256), np.float32)
    x[1] = 0.5
    d = oracle.dequantize(oracle.quantize(x, oracle.GGML_Q4_K), oracle.GGML_Q4_K, x.shape)
    assert np.all(d[0] == 0)
    assert np.allclose(d[1], 0.5, rtol=1e-3)


def test_randn_deterministic_and_normal():
    a = oracle.randn(42, (100000,))
    b = oracle.randn(42, (100000,))
    c = oracle.randn(43, (100000,))
    assert np.array_equal(a, b)
    assert not np.array_equal(a, c)
    assert abs(a.mean()) < 0.02 and abs(a.std() - 1) < 0.02


def test_bf16_rounding_rne():
    x = np.array([1.0, 1.00390625, 1.005859375, -2.5e-8, 3.4e38], np.float32)
    r = oracle.round_bf16(x)
    assert r[0] == 1.0 and r[1] == 1.0  # tie to even
    assert r[2] == np.float32(1.0078125)


NEW_TYPES = [("q4_0", oracle.GGML_Q4_0, 32), ("q4_1", oracle.GGML_Q4_1, 32), ("q5_0", oracle.GGML_Q5_0, 32),
             ("q5_1", oracle.GGML_Q5_1, 32), ("q5_k", oracle.GGML_Q5_K, 256), ("q6_k", oracle.GGML_Q6_K, 256)]


@pytest.mark.parametrize("name,t,be", NEW_TYPES)
def test_dequant_bit_exact_random_blocks(gold, name, t, be):
    blocks = gold[name + "_blocks"]
    d = oracle.dequantize(blocks, t, (blocks.shape[0], be))
    assert np.array_equal(d.view(np.uint32), gold[name + "_deq"].view(np.uint32))


@pytest.mark.parametrize("name,t,be", NEW_TYPES)
def test_quantizer_roundtrip_error(name, t, be):
    x = oracle.randn(21, (8, 1024), 0.02)
    err = np.linalg.norm(oracle.dequantize(oracle.quantize(x, t), t, x.shape) - x) / np.linalg.norm(x)
    assert err < (0.1 if name.startswith("q4") else 0.05), err
