"""Generates the full-width oracle fixtures (FLUX.1-dev and Qwen-Image widths at the headline
1024x1024 token counts) in this directory, from the numpy oracle (oracle/flux_ref.py,
oracle/qwen_ref.py). Everything is seeded through the oracle's C generator and quantizers, so
the GPU tests rebuild the same GGUF bytes and inputs bit for bit on any host.

    python tests/golden/make_fullwidth.py [flux_q4_k] [flux_q8_0] [qwen_q4_k] [flux_full_q4_k] [qwen_full_q4_k]

It takes about half an hour of CPU per FLUX case (the 28-step denoise dominates).

Fixtures (fullwidth_<case>.npz). Residual-stream tensors are stored as the block's UPDATE
(output minus input, float16) on every ROW_STRIDE-th row, which keeps the files small and
measures the error relative to what the block adds:

flux_q4_k / flux_q8_0: FLUX.1-dev widths (hidden 3072, 24 heads x 128, MLP 12288, T5 width 4096,
  pooled 768) with 1 double + 1 single block, weights synth_weights(seed) in the case's GGUF type;
  512 text + 4096 image tokens (a 128 x 128 x 16 latent, 64 x 64 patches), guidance 3.5.
  d_img, d_txt    double block 0 update of the image / text stream; its inputs are the stems
                  (img_in, txt_in) and the vec embedding at t = T_BLOCK
  d_single        single block 0 update on the seeded input X_SINGLE [4608, 3072] ~ N(0, 1)
  pred            float16 [4096, 64]: the whole model's prediction at t = T_BLOCK
  denoise         float32 [4096, 64]: the latent after the 28-step schedule (get_schedule(28, 4096))
flux_full_q4_k: the full FLUX.1-dev architecture (19 double + 38 single blocks) in Q4_K, seed 14,
  the same token counts and guidance; one forward (about 25 min of CPU).
  pred            float16 [4096, 64]: the model's prediction at t = T_BLOCK
qwen_full_q4_k: the full Qwen-Image architecture (60 blocks) in Q4_K, seed 15, with the qwen_q4_k
  inputs; one forward with the conditional prompt (about 15 min of CPU).
  pred            float16 [4096, 64]: the prediction at t = 700
qwen_q4_k: Qwen-Image widths (hidden 3072, 24 heads, MLP 12288, text width 3584) with 1 block,
  4096 image + 256 text tokens, conditional mask keeping the first 200 text tokens,
  unconditional mask a seeded 60 % pattern.
  pred            float16 [4096, 64]: the forward at t = 700 with the conditional prompt
  d_cfg_step      float16 [16, 128, 128]: the update of the latent by one CFG Euler step
                  (guidance 4.0) over the first two sigmas of the 30-step schedule
"""
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle  # noqa: E402
from oracle import flux_ref as F  # noqa: E402
from oracle import qwen_ref as Q  # noqa: E402

ROW_STRIDE = 24
LT, HT, WT = 512, 64, 64          # FLUX: text tokens, image token grid
T_BLOCK = 0.8
GUIDANCE = 3.5
N_STEPS = 28
FLUX_CASES = {"flux_q4_k": (oracle.GGML_Q4_K, 11), "flux_q8_0": (oracle.GGML_Q8_0, 12)}
Q_LT, Q_T, Q_GUIDANCE, Q_STEPS = 256, 700.0, 4.0, 30


class _Cached(F.QTensorRef):
    """QTensorRef whose decode is computed once (the oracle decodes on every use)."""

    def f32(self):
        if not hasattr(self, "_f"):
            self._f = super().f32()
        return self._f


def cached(W):
    return {n: _Cached(q.ggml_type, q.shape, q.raw) for n, q in W.items()}


def flux_config():
    return F.FluxConfig(depth=1, depth_single_blocks=1)


def flux_inputs(seed):
    """Seeded inputs of a FLUX case (the GPU tests call this too)."""
    img = oracle.randn(seed * 100 + 1, (HT * WT, 64))
    txt = oracle.randn(seed * 100 + 2, (LT, 4096))
    y = oracle.randn(seed * 100 + 3, (768,))
    x_single = oracle.randn(seed * 100 + 4, (LT + HT * WT, 3072))
    return img, F.img_ids(HT, WT), txt, np.zeros((LT, 3), np.float32), y, x_single


def flux_block_inputs(W, cfg, img, ids, txt, tids, y):
    """The double block's inputs as the model forms them: stems, vec at T_BLOCK, RoPE table."""
    pe = F.embed_nd(np.concatenate([tids, ids], axis=0), cfg.axes_dim, cfg.theta)
    txt_h = F.linear(txt, W["txt_in.weight"], W["txt_in.bias"])
    img_h = F.linear(img, W["img_in.weight"], W["img_in.bias"])
    vec = F.vec_embedding(W, cfg, T_BLOCK, y, GUIDANCE)
    return img_h, txt_h, vec, pe


def qwen_config():
    return Q.QwenConfig(num_layers=1)


def qwen_inputs():
    x = oracle.randn(901, (HT * WT, 64))
    txt = oracle.randn(902, (2, Q_LT, 3584))
    mk = np.zeros((2, Q_LT), np.uint8)
    mk[0, :200] = 1
    mk[1] = (np.random.default_rng(903).random(Q_LT) < 0.6).astype(np.uint8)
    mk[1, 0] = 1
    latent = oracle.randn(904, (16, 2 * HT, 2 * WT))
    return x, txt, mk, latent


def make_flux(name):
    qt, seed = FLUX_CASES[name]
    cfg = flux_config()
    W = cached(F.synth_weights(cfg, seed=seed, qtype=qt))
    img, ids, txt, tids, y, xs = flux_inputs(seed)
    img_h, txt_h, vec, pe = flux_block_inputs(W, cfg, img, ids, txt, tids, y)
    t0 = time.time()
    img1, txt1 = F.double_block(W, "double_blocks.0.", cfg, img_h, txt_h, vec, pe)
    xs1 = F.single_block(W, "single_blocks.0.", cfg, xs, vec, pe)
    pred = F.forward(W, cfg, img, ids, txt, tids, T_BLOCK, y, GUIDANCE)
    print(f"{name}: blocks + forward {time.time() - t0:.0f} s", flush=True)
    den = F.denoise(W, cfg, img, ids, txt, tids, y, F.get_schedule(N_STEPS, HT * WT), GUIDANCE)
    print(f"{name}: denoise done {time.time() - t0:.0f} s", flush=True)
    s = slice(None, None, ROW_STRIDE)
    np.savez_compressed(os.path.join(HERE, f"fullwidth_{name}.npz"),
                        d_img=(img1 - img_h)[s].astype(np.float16), d_txt=(txt1 - txt_h)[s].astype(np.float16),
                        d_single=(xs1 - xs)[s].astype(np.float16), pred=pred.astype(np.float16),
                        denoise=den.astype(np.float32))


FULL_SEED = 14


def make_flux_full(name):
    """The full-depth model: one forward (decodes are not cached, so memory stays at the raw bytes)."""
    cfg = F.FluxConfig()
    W = F.synth_weights(cfg, seed=FULL_SEED, qtype=oracle.GGML_Q4_K)
    img, ids, txt, tids, y, _ = flux_inputs(FULL_SEED)
    t0 = time.time()
    pred = F.forward(W, cfg, img, ids, txt, tids, T_BLOCK, y, GUIDANCE)
    print(f"{name}: forward {time.time() - t0:.0f} s", flush=True)
    np.savez_compressed(os.path.join(HERE, f"fullwidth_{name}.npz"), pred=pred.astype(np.float16))


QWEN_FULL_SEED = 15


def make_qwen_full(name):
    """The full-depth Qwen-Image model: one forward (decodes not cached)."""
    cfg = Q.QwenConfig()
    W = Q.synth_weights(cfg, seed=QWEN_FULL_SEED, qtype=oracle.GGML_Q4_K)
    x, txt, mk, _ = qwen_inputs()
    t0 = time.time()
    pred = Q.forward(W, cfg, x, Q_T, txt[0], mk[0].astype(bool), HT, WT)
    print(f"{name}: forward {time.time() - t0:.0f} s", flush=True)
    np.savez_compressed(os.path.join(HERE, f"fullwidth_{name}.npz"), pred=pred.astype(np.float16))


def make_qwen(name):
    cfg = qwen_config()
    W = cached(Q.synth_weights(cfg, seed=13, qtype=oracle.GGML_Q4_K))
    x, txt, mk, latent = qwen_inputs()
    t0 = time.time()
    pred = Q.forward(W, cfg, x, Q_T, txt[0], mk[0].astype(bool), HT, WT)
    sig = Q.scheduler_sigmas(Q_STEPS, HT * WT)[:2]
    step = Q.denoise(W, cfg, latent, txt[0], mk[0].astype(bool), sig, txt[1], mk[1].astype(bool), Q_GUIDANCE)
    print(f"{name}: {time.time() - t0:.0f} s", flush=True)
    np.savez_compressed(os.path.join(HERE, f"fullwidth_{name}.npz"), pred=pred.astype(np.float16),
                        d_cfg_step=(step - latent).astype(np.float16))


def main(argv):
    todo = argv or list(FLUX_CASES) + ["qwen_q4_k", "flux_full_q4_k", "qwen_full_q4_k"]
    for name in todo:
        if name == "flux_full_q4_k":
            make_flux_full(name)
        elif name == "qwen_full_q4_k":
            make_qwen_full(name)
        else:
            (make_qwen if name.startswith("qwen") else make_flux)(name)


if __name__ == "__main__":
    main(sys.argv[1:])
