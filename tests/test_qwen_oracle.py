"""Qwen-Image oracle and host logic on CPU: the scheduler against the reference's own
known answers (qwen_image/sampling.rs:136-240), RoPE positions, CFG, key order."""
import math

import numpy as np
import torch

from mold_b200 import sampling
from mold_b200.ops import key_order
from oracle import qwen_ref as Q


def test_calculate_shift_matches_qwen_defaults():
    assert abs(Q.calculate_shift(4096) - 0.6935483870967742) < 1e-9
    assert abs(sampling.qwen_calculate_shift(4096) - 0.6935483870967742) < 1e-9


def test_exponential_time_shift_is_monotonic():
    assert Q.time_shift_exponential(0.69, 1.0, 0.1) < Q.time_shift_exponential(0.69, 1.0, 0.9)


def test_image_seq_len_matches_patchified_latents():
    assert sampling.qwen_image_seq_len(128, 128, 2) == 4096
    assert sampling.qwen_image_seq_len(116, 208, 2) == 6032


def test_scheduler_descending_with_terminal_zero():
    s = Q.scheduler_sigmas(50, 4096)
    assert len(s) == 51 and s[-1] == 0.0
    assert all(a >= b for a, b in zip(s, s[1:]))
    assert abs(s[0] * Q.NUM_TRAIN_TIMESTEPS - 1000.0 * s[0]) < 1e-10
    assert abs(s[-2] - Q.SHIFT_TERMINAL) < 1e-10


def test_stretch_shift_known_answers():
    assert abs(Q.stretch_shift_to_terminal([1.0, 0.5])[1] - Q.SHIFT_TERMINAL) < 1e-10
    assert Q.stretch_shift_to_terminal([1.0]) == [1.0]
    assert Q.scheduler_sigmas(1, 4096) == [1.0, 0.0]


def test_host_sigmas_equal_oracle():
    for n, seq in ((30, 4096), (50, 4096), (8, 1024), (2, 6032)):
        assert sampling.qwen_sigmas(n, seq) == Q.scheduler_sigmas(n, seq)
    assert len(Q.scheduler_sigmas(30, 4096)) == 31


def test_rope_ids_centred():
    img, txt = Q.rope_ids(1, 64, 64, 5)
    assert img.shape == (4096, 3) and txt.shape == (5, 3)
    assert img[:, 1].min() == -32 and img[:, 1].max() == 31 and img[:, 2].min() == -32
    assert (img[:, 0] == 0).all()
    assert (txt[:, 0] == np.arange(32, 37)).all() and (txt[:, 0] == txt[:, 2]).all()
    odd, t2 = Q.rope_ids(1, 5, 3, 1)   # odd sizes: negative half is the larger one
    assert odd[:, 1].min() == -3 and odd[:, 1].max() == 1 and odd[:, 2].min() == -2 and odd[:, 2].max() == 0
    assert t2[0, 0] == 2


def test_cfg_combine_properties():
    rng = np.random.default_rng(0)
    c = rng.standard_normal((16, 6, 4)).astype(np.float32)
    u = rng.standard_normal((16, 6, 4)).astype(np.float32)
    assert np.allclose(Q.cfg_combine(c, u, 1.0), c, atol=1e-6)   # g = 1: comb = c, scale 1
    out = Q.cfg_combine(c, u, 4.0)
    assert np.allclose(np.linalg.norm(out, axis=0), np.linalg.norm(c, axis=0), rtol=1e-5)  # per-pixel norm kept


def test_key_order_permutation():
    mask = torch.tensor([1, 0, 1, 1, 0, 0, 1], dtype=torch.uint8)
    pos, nv = key_order(mask, 5)
    assert nv == 4 + 5
    assert sorted(pos.tolist()) == list(range(12))
    kept = pos[:7][mask.bool()]
    assert kept.tolist() == [0, 1, 2, 3]               # kept text keys first, in order
    assert pos[7:].tolist() == list(range(4, 9))       # then the image keys
    assert (pos[:7][~mask.bool()] >= nv).all()         # masked keys after the valid prefix
    pos, nv = key_order(torch.zeros(3, dtype=torch.uint8), 2)
    assert nv == 2 and pos.tolist() == [2, 3, 4, 0, 1]


def test_inpaint_blend_known_answers():
    """img2img.rs:346-362: mask 0 restores orig * (1 - sigma) + noise * sigma; mask 1 keeps the
    current latent (flux/transformer.rs:79-87 is the same blend)."""
    from oracle import flux_ref as F
    cur = np.array([100.0, 200.0], np.float32)
    orig = np.array([2.0, 4.0], np.float32)
    noise = np.array([10.0, 20.0], np.float32)
    assert F.inpaint_blend(cur, (np.zeros(2, np.float32), orig, noise), 0.25).tolist() == [4.0, 8.0]
    assert F.inpaint_blend(cur, (np.ones(2, np.float32), orig, noise), 0.25).tolist() == [100.0, 200.0]
    # flow_match_interpolate_blends_encoded_and_noise (img2img.rs:172-190): sigma 0 and 0.5
    assert F.inpaint_blend(cur, (np.zeros(2, np.float32), orig, noise), 0.0).tolist() == [2.0, 4.0]
    assert F.inpaint_blend(cur, (np.zeros(2, np.float32), orig, noise), 0.5).tolist() == [6.0, 12.0]
