"""Host sampling glue of the FLUX path (candle flux::sampling as called at
flux/pipeline.rs:2044-2048, 2129, 2158): the product's get_schedule, patchify, unpack,
img_ids and txt_ids against the oracle's restatements (oracle/flux_ref.py), plus
properties the reference's own tests state for the sibling flux2 sampler
(flux2/sampling.rs:161-226: endpoints, length N + 1, shift toward 1, patchify/unpack
round trip)."""
import math

import numpy as np
import pytest
import torch

from mold_b200 import sampling as S
from oracle import flux_ref as F


@pytest.mark.parametrize("n", [1, 4, 20, 28, 50])
@pytest.mark.parametrize("seq", [None, 256, 1024, 4096, 6144])
def test_get_schedule_matches_oracle(n, seq):
    a, b = S.get_schedule(n, seq), F.get_schedule(n, seq)
    assert len(a) == n + 1
    assert a == b  # same float64 arithmetic, bit for bit
    assert a[0] == pytest.approx(1.0, abs=1e-12) and a[-1] == 0.0
    assert all(x > y for x, y in zip(a, a[1:]))


def test_get_schedule_known_answer_1024():
    # mu at 4096 image tokens is max_shift = 1.15; t' = e^mu / (e^mu + 1/t - 1)
    s = S.get_schedule(4, 4096)
    e = math.exp(1.15)
    want = [1.0] + [e / (e + 1.0 / t - 1.0) for t in (0.75, 0.5, 0.25)] + [0.0]
    assert s == pytest.approx(want, abs=1e-12)
    assert s[1] > 0.9 and s[2] > 0.75  # shifted toward 1 (a linear schedule gives 0.75, 0.5)
    # mu at 256 tokens is base_shift = 0.5
    e = math.exp(0.5)
    assert S.get_schedule(2, 256)[1] == pytest.approx(e / (e + 1.0), abs=1e-12)


@pytest.mark.parametrize("c,h,w", [(16, 128, 128), (16, 64, 96), (32, 8, 4)])
def test_patchify_unpack_match_oracle(c, h, w):
    lat = np.random.default_rng(c * h + w).standard_normal((c, h, w)).astype(np.float32)
    p = S.patchify(torch.from_numpy(lat)).numpy()
    assert p.shape == (h // 2 * w // 2, 4 * c)
    assert np.array_equal(p, F.patchify(lat))
    # token (i, j) holds channel ch's 2x2 patch in (dy, dx) order at columns ch*4 + dy*2 + dx
    i, j, ch = h // 4, w // 4, c - 1
    assert np.array_equal(p[i * (w // 2) + j, ch * 4:ch * 4 + 4], lat[ch, 2 * i:2 * i + 2, 2 * j:2 * j + 2].ravel())
    back = S.unpack(torch.from_numpy(p), h, w).numpy()
    assert np.array_equal(back, lat)
    assert np.array_equal(F.unpack(p, h, w), lat)


@pytest.mark.parametrize("ht,wt", [(64, 64), (48, 32), (1, 5)])
def test_img_ids_txt_ids_match_oracle(ht, wt):
    a = S.img_ids(ht, wt).numpy()
    assert np.array_equal(a, F.img_ids(ht, wt))
    assert a.shape == (ht * wt, 3) and (a[:, 0] == 0).all()
    if ht > 1 and wt > 1:
        assert a[wt + 1].tolist() == [0.0, 1.0, 1.0]  # row-major: token wt + 1 is (row 1, col 1)
    t = S.txt_ids(7).numpy()
    assert t.shape == (7, 3) and not t.any()
