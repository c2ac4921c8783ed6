"""Host-side FLUX.1 sampling glue (candle flux::sampling as called at
crates/mold-inference/src/flux/pipeline.rs:2044-2048, 2129, 2158).

get_schedule: t_i = linspace(1, 0, N+1); with a shift, mu is linear in the
image sequence length through (256, 0.5) and (4096, 1.15) and
t' = e^mu / (e^mu + (1/t - 1)) (the same form as qwen_image/sampling.rs:19-27).
patchify / unpack: 2x2 patches, [C, H, W] <-> [(H/2)(W/2), 4C] (flux2/sampling.rs:45-48, 149-159).
img_ids: (0, row, col) per patch; txt ids are zeros (FLUX.1 uses 3 axes).
"""
import math

import torch


def get_schedule(num_steps, image_seq_len=None, base_shift=0.5, max_shift=1.15):
    ts = [v / num_steps for v in range(num_steps + 1)][::-1]
    if image_seq_len is None:
        return ts
    m = (max_shift - base_shift) / (4096.0 - 256.0)
    mu = m * image_seq_len + (base_shift - m * 256.0)
    e = math.exp(mu)
    return [0.0 if t <= 0.0 else e / (e + (1.0 / t - 1.0)) for t in ts]


def patchify(latent):
    c, h, w = latent.shape
    return latent.reshape(c, h // 2, 2, w // 2, 2).permute(1, 3, 0, 2, 4).reshape(h // 2 * w // 2, c * 4)


def unpack(x, h, w):
    c4 = x.shape[1]
    return x.reshape(h // 2, w // 2, c4 // 4, 2, 2).permute(2, 0, 3, 1, 4).reshape(c4 // 4, h, w)


def img_ids(h_tokens, w_tokens, device=None):
    r = torch.arange(h_tokens, dtype=torch.float32, device=device).repeat_interleave(w_tokens)
    c = torch.arange(w_tokens, dtype=torch.float32, device=device).repeat(h_tokens)
    return torch.stack([torch.zeros_like(r), r, c], dim=1)


def txt_ids(n, device=None):
    return torch.zeros((n, 3), dtype=torch.float32, device=device)
