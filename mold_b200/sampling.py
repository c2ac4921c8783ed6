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

# ---- Qwen-Image scheduler (qwen_image/sampling.rs:12-129): FlowMatchEulerDiscreteScheduler
# with exponential shift mu(seq_len) through (256, 0.5) and (8192, 0.9), shift_terminal 0.02.
QWEN_NUM_TRAIN_TIMESTEPS = 1000


def qwen_calculate_shift(image_seq_len, base_seq=256, max_seq=8192, base_shift=0.5, max_shift=0.9):
    m = (max_shift - base_shift) / (max_seq - base_seq)
    return image_seq_len * m + (base_shift - m * base_seq)


def qwen_sigmas(num_steps, image_seq_len, shift_terminal=0.02):
    """QwenImageScheduler::new: sigmas = linspace(1, 1/N, N) -> e^mu / (e^mu + (1/s - 1)) ->
    stretched so the last equals shift_terminal -> append 0. Length N + 1."""
    if num_steps == 1:
        s = [1.0]
    else:
        step = (1.0 / num_steps - 1.0) / (num_steps - 1)
        s = [1.0 + step * i for i in range(num_steps)]
    e = math.exp(qwen_calculate_shift(image_seq_len))
    s = [e / (e + (1.0 / x - 1.0)) for x in s]
    one_minus_z = 1.0 - s[-1]
    if abs(one_minus_z) >= 1e-12:
        scale = one_minus_z / (1.0 - shift_terminal)
        s = [1.0 - (1.0 - x) / scale for x in s]
    return s + [0.0]


def qwen_image_seq_len(latent_h, latent_w, patch_size=2):
    return (latent_h // patch_size) * (latent_w // patch_size)


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
