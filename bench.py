#!/usr/bin/env python
"""FLUX.1-dev Q4_K 1024x1024 denoising benchmark on B200 (steps/s; images/s at N GPUs).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference] [--quant q4_k|q8_0]

One process per GPU (torchrun for N > 1). Every rank holds a full replica of the
synthetic FLUX.1-dev transformer (random N(0, 0.02) weights quantized to GGUF
Q4_K on the device, seed 0) and denoises its own image (seed = rank): the work
shards by image, with no collective on the data path (weak scaling). A "step"
is one transformer forward over 512 text + 4096 image tokens plus the Euler
update, replayed from the library's captured CUDA graph.

Printed JSON line (rank 0): value = whole-job steps/s over the K timed steps
(max of per-rank CUDA-event times), e2e = the same metric through the public
denoise call with host<->device copies in the timed region, roofline of the
dominant kernel (the dequant-GEMM), cpu_baseline = the CPU oracle timed on this
host. --impl reference times the reference's CPU path (the oracle port; the Rust
reference cannot be built on this image) on the same metric.
"""
import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

L_TXT, LAT_H, LAT_W = 512, 128, 128          # 1024x1024 -> 128x128x16 latent -> 64x64 tokens
L_IMG = (LAT_H // 2) * (LAT_W // 2)
N_SCHEDULE = 28
GUIDANCE = 3.5


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=28)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--quant", default="q4_k", choices=["q4_k", "q8_0", "q4_1", "q6_k"],
                    help="GGUF type of the synthetic weights (the headline is q4_k)")
    ap.add_argument("--model", default="flux", choices=["flux", "qwen"],
                    help="flux: the headline FLUX.1-dev line; qwen: Qwen-Image 1024x1024 with CFG (config 5)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline sample")
    ap.add_argument("--kernels-only", action="store_true", help="only the standalone kernel timings (profiling)")
    ap.add_argument("--kernel", default="gemm,attention",
                    help="with --kernels-only: comma list of gemm, attention, gemm_qwen_mlp0, gemv, ln_modulate, "
                         "qk_norm_rope, dequant (the HBM-bound ones at the FLUX step's shapes, L2 flushed between "
                         "launches)")
    ap.add_argument("--sweep", action="store_true",
                    help="BASELINE config 2: the Q4_K dequant-GEMM over the ten FLUX linear shapes, one JSON line each")
    ap.add_argument("--sweep-only", default=None, metavar="LINEAR:M",
                    help="with --sweep: only this shape (e.g. attn_out:1536), for a profiler capture")
    return ap.parse_args()


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


# ------------------------------------------------------------------ clocks
class ClockSampler:
    FIELDS = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.idx), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 6:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for n, v in zip(names, parts[2:6]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------------ synthetic GGUF weights on the device
def q4k_quantize_torch(x):
    """f32 [N, K] (CUDA) -> Q4_K bytes [N, K/256*144]: per 32-value sub-block min/max,
    6-bit scales/mins relative to the super-block maxima (same method as the oracle's quantizer)."""
    import torch
    N, K = x.shape
    nb = K // 256
    xb = x.reshape(N, nb, 8, 32)
    mn = torch.clamp(xb.amin(-1), max=0.0)
    mx = torch.maximum(xb.amax(-1), mn)
    scale = (mx - mn) / 15.0
    mins = -mn
    d = (scale.amax(-1) / 63.0).half()
    dmin = (mins.amax(-1) / 63.0).half()
    df, dmf = d.float().unsqueeze(-1), dmin.float().unsqueeze(-1)
    sc = torch.where(df > 0, torch.clamp(torch.round(scale / df.clamp_min(1e-30)), 0, 63), torch.zeros_like(scale))
    m = torch.where(dmf > 0, torch.clamp(torch.round(mins / dmf.clamp_min(1e-30)), 0, 63), torch.zeros_like(mins))
    dl = (df * sc).unsqueeze(-1)
    ml = (dmf * m).unsqueeze(-1)
    q = torch.where(dl > 0, torch.clamp(torch.round((xb + ml) / dl.clamp_min(1e-30)), 0, 15), torch.zeros_like(xb))
    q = q.to(torch.uint8).reshape(N, nb, 4, 2, 32)
    qs = (q[:, :, :, 0, :] | (q[:, :, :, 1, :] << 4)).reshape(N, nb, 128)
    sc, m = sc.to(torch.int32), m.to(torch.int32)
    s = torch.empty((N, nb, 12), dtype=torch.int32, device=x.device)
    s[..., 0:4] = (sc[..., 0:4] & 63) | ((sc[..., 4:8] >> 4) << 6)
    s[..., 4:8] = (m[..., 0:4] & 63) | ((m[..., 4:8] >> 4) << 6)
    s[..., 8:12] = (sc[..., 4:8] & 0xF) | ((m[..., 4:8] & 0xF) << 4)
    head = torch.cat([d.view(torch.uint8).reshape(N, nb, 2), dmin.view(torch.uint8).reshape(N, nb, 2),
                      s.to(torch.uint8)], dim=-1)
    return torch.cat([head, qs], dim=-1).reshape(N, nb * 144).contiguous()


def q8_0_quantize_torch(x):
    import torch
    N, K = x.shape
    xb = x.reshape(N, K // 32, 32)
    d = xb.abs().amax(-1, keepdim=True) / 127.0
    idv = torch.where(d > 0, 1.0 / d.clamp_min(1e-30), torch.zeros_like(d))
    v = xb * idv
    q = (torch.sign(v) * torch.floor(v.abs() + 0.5)).to(torch.int8)
    return torch.cat([d.half().view(torch.uint8).reshape(N, K // 32, 2), q.view(torch.uint8)], -1).reshape(N, -1)


def q4_1_quantize_torch(x):
    """f32 [N, K] -> Q4_1 bytes [N, K/32*20]: per 32-value block d = (max - min)/15, m = min (f16)."""
    import torch
    N, K = x.shape
    xb = x.reshape(N, K // 32, 32)
    mn, mx = xb.amin(-1), xb.amax(-1)
    d = ((mx - mn) / 15.0).half()
    m = mn.half()
    df, mf = d.float().unsqueeze(-1), m.float().unsqueeze(-1)
    q = torch.where(df > 0, torch.clamp(torch.round((xb - mf) / df.clamp_min(1e-30)), 0, 15), torch.zeros_like(xb))
    q = q.to(torch.uint8)
    qs = q[..., :16] | (q[..., 16:] << 4)
    head = torch.cat([d.view(torch.uint8).reshape(N, K // 32, 2), m.view(torch.uint8).reshape(N, K // 32, 2)], -1)
    return torch.cat([head, qs], -1).reshape(N, -1).contiguous()


def q6_k_quantize_torch(x):
    """f32 [N, K] -> Q6_K bytes [N, K/256*210]: signed absmax scale per 16 values, int8 scales
    relative to the super-block's largest (f16 d), 6-bit quants."""
    import torch
    N, K = x.shape
    nb = K // 256
    xs = x.reshape(N, nb, 16, 16)
    idx = xs.abs().argmax(-1, keepdim=True)
    sv = torch.gather(xs, -1, idx).squeeze(-1) / -32.0
    d = (sv.abs().amax(-1) / 127.0).half()
    df = d.float().unsqueeze(-1)
    sc = torch.where(df > 0, torch.clamp(torch.round(sv / df.clamp_min(1e-30)), -127, 127), torch.zeros_like(sv))
    ds = (df * sc).unsqueeze(-1)
    q = torch.where(ds != 0, torch.clamp(torch.round(xs / torch.where(ds != 0, ds, torch.ones_like(ds))) + 32, 0, 63),
                    torch.full_like(xs, 32.0)).to(torch.int32).reshape(N, nb, 2, 4, 32)  # (n2, quarter g, l)
    ql0 = (q[:, :, :, 0] & 0xF) | ((q[:, :, :, 2] & 0xF) << 4)
    ql1 = (q[:, :, :, 1] & 0xF) | ((q[:, :, :, 3] & 0xF) << 4)
    ql = torch.stack([ql0, ql1], 3).reshape(N, nb, 128)
    qh = (((q[:, :, :, 0] >> 4) & 3) | (((q[:, :, :, 1] >> 4) & 3) << 2) | (((q[:, :, :, 2] >> 4) & 3) << 4) |
          (((q[:, :, :, 3] >> 4) & 3) << 6)).reshape(N, nb, 64)
    out = torch.cat([ql.to(torch.uint8), qh.to(torch.uint8), sc.to(torch.int8).view(torch.uint8),
                     d.view(torch.uint8).reshape(N, nb, 2)], -1)
    return out.reshape(N, nb * 210).contiguous()


def quantizer(quant):
    """(ggml type id, torch quantizer, values per block) of a --quant choice."""
    return {"q4_k": (12, q4k_quantize_torch, 256), "q8_0": (8, q8_0_quantize_torch, 32),
            "q4_1": (3, q4_1_quantize_torch, 32), "q6_k": (14, q6_k_quantize_torch, 256)}[quant]


def build_flux(quant, device, seed=0):
    import torch
    import mold_b200 as mb
    cfg = mb.FluxConfig()
    model = mb.FluxTransformer(cfg, max_txt=L_TXT, max_img=L_IMG, device=device)
    g = torch.Generator(device=f"cuda:{device}")
    keep = {}
    gtype, qfn, _ = quantizer(quant)
    for i, (name, shape) in enumerate(mb.flux.tensor_specs(cfg)):
        g.manual_seed(WEIGHT_SALT + seed * 1000003 + i)
        if len(shape) == 2:
            x = torch.randn(shape, generator=g, device=f"cuda:{device}") * 0.02
            if shape[1] % 256 == 0:
                raw = qfn(x)
                model.set_tensor(name, (raw, gtype, shape))
            else:  # rows shorter than a super-block (img_in [3072, 64]) stay BF16 as in GGUF files
                raw = x.bfloat16().view(torch.uint8).reshape(shape[0], -1).contiguous()
                model.set_tensor(name, (raw, mb.GGML_BF16, shape))
            if name == "single_blocks.0.linear1.weight":
                keep["linear1"] = (raw, gtype, shape)
            del x
        else:
            x = torch.randn(shape, generator=g, device=f"cuda:{device}") * 0.02
            if name.endswith(".scale"):
                x = x + 1.0
            model.set_tensor(name, (x.contiguous().view(torch.uint8), mb.GGML_F32, shape))
    assert model.missing() == []
    torch.cuda.synchronize()
    return model, cfg, keep


# ---- Qwen-Image (config 5): 60 dual-stream blocks, 4096 image + 256 text tokens, CFG batch 2, 30 steps
Q_TXT, Q_STEPS, Q_GUIDANCE = 256, 30, 4.0


def build_qwen(quant, device, seed=0):
    import torch
    import mold_b200 as mb
    cfg = mb.QwenConfig()
    model = mb.QwenTransformer(cfg, max_txt=Q_TXT, max_img=L_IMG, max_batch=2, device=device)
    g = torch.Generator(device=f"cuda:{device}")
    keep = {}
    gtype, qfn, _ = quantizer(quant)
    for i, (name, shape) in enumerate(mb.qwen.tensor_specs(cfg)):
        g.manual_seed(WEIGHT_SALT + seed * 1000003 + i)
        x = torch.randn(shape, generator=g, device=f"cuda:{device}") * 0.02
        if len(shape) == 2:
            if shape[1] % 256 == 0:
                raw = qfn(x)
                model.set_tensor(name, (raw, gtype, shape))
            else:
                raw = x.bfloat16().view(torch.uint8).reshape(shape[0], -1).contiguous()
                model.set_tensor(name, (raw, mb.GGML_BF16, shape))
            if name == "transformer_blocks.0.img_mlp.net.0.proj.weight":
                keep["mlp0"] = (raw, gtype, shape)
        else:
            if "norm" in name:
                x = x + 1.0
            model.set_tensor(name, (x.contiguous().view(torch.uint8), mb.GGML_F32, shape))
        del x
    assert model.missing() == []
    torch.cuda.synchronize()
    return model, cfg, keep


# ------------------------------------------------------------------ CPU oracle sample (cpu_baseline / reference arm)
class CpuSample:
    """One FLUX single-stream block (BASELINE config 1 shape: 512 txt + 1024 img tokens,
    hidden 3072) through the numpy oracle with the benchmark's GGUF type. A full step
    (19 double + 38 single blocks at 512 + 4096 tokens) is extrapolated from the block
    time by the ratio of algorithmic FLOPs (linears + attention)."""

    def __init__(self, quant, l_txt=512, l_img=1024):
        from oracle import flux_ref as F
        import oracle
        self.F = F
        self.cfg = F.FluxConfig(depth=0, depth_single_blocks=1)
        qt = quantizer(quant)[0]
        self.W = F.synth_weights(self.cfg, seed=0, qtype=qt, only=lambda n: n.startswith("single_blocks.0."))
        L = l_txt + l_img
        side = int(round(l_img ** 0.5))
        self.x = oracle.randn(1, (L, 3072))
        self.vec = oracle.randn(2, (3072,))
        ids = np.concatenate([np.zeros((l_txt, 3), np.float32), F.img_ids(side, l_img // side)])
        self.pe = F.embed_nd(ids, self.cfg.axes_dim, self.cfg.theta)
        import mold_b200.flux as mf
        full = mf.step_flops(mf.FluxConfig(), L_TXT, L_IMG)
        h, m = 3072, 12288
        blk = 2 * L * h * (3 * h + m) + 2 * L * (h + m) * h + 4 * L * L * h
        self.ratio = full / blk
        self.desc = f"1 single block at {l_txt}+{l_img} tokens"

    def run(self):
        t0 = time.perf_counter()
        self.F.single_block(self.W, "single_blocks.0.", self.cfg, self.x, self.vec, self.pe)
        return time.perf_counter() - t0

    @staticmethod
    def cores():
        try:
            return len(os.sched_getaffinity(0))
        except AttributeError:
            return os.cpu_count()


class QwenCpuSample:
    """One Qwen-Image block at 256 text + 1024 image tokens (hidden 3072) through the numpy
    oracle; a full CFG step (2 sequences x 60 blocks at 256 + 4096 tokens) is extrapolated by
    the ratio of algorithmic FLOPs."""

    def __init__(self, quant, l_txt=256, l_img=1024):
        from oracle import qwen_ref as Q
        from oracle import flux_ref as F
        import oracle
        self.Q = Q
        self.cfg = Q.QwenConfig(num_layers=1)
        qt = quantizer(quant)[0]
        self.W = Q.synth_weights(self.cfg, seed=0, qtype=qt, only=lambda n: n.startswith("transformer_blocks.0."))
        side = int(round(l_img ** 0.5))
        self.img = oracle.randn(1, (l_img, 3072))
        self.txt = oracle.randn(2, (l_txt, 3072))
        self.temb = oracle.randn(3, (3072,))
        self.mask = np.ones(l_txt, bool)
        ii, it = Q.rope_ids(1, side, l_img // side, l_txt)
        self.pe_i = F.embed_nd(ii, self.cfg.axes_dim, self.cfg.theta)
        self.pe_t = F.embed_nd(it, self.cfg.axes_dim, self.cfg.theta)
        import mold_b200.qwen as mq
        full = mq.step_flops(mq.QwenConfig(), Q_TXT, L_IMG, batch=2)
        L, h, m = l_txt + l_img, 3072, 12288
        self.ratio = full / (2 * L * h * 4 * h + 2 * L * 2 * h * m + 4 * L * L * h)
        self.desc = f"1 Qwen-Image block at {l_txt}+{l_img} tokens"

    def run(self):
        t0 = time.perf_counter()
        self.Q.block(self.W, "transformer_blocks.0.", self.cfg, self.img, self.txt, self.mask, self.temb,
                     self.pe_i, self.pe_t)
        return time.perf_counter() - t0

    cores = staticmethod(CpuSample.cores)


def cpu_sample(args):
    return QwenCpuSample(args.quant) if args.model == "qwen" else CpuSample(args.quant)


METRIC = {"flux": "flux_dev_1024_denoise_steps_per_s", "qwen": "qwen_image_1024_cfg_denoise_steps_per_s"}
WORKLOAD = {"flux": "FLUX.1-dev {q} 1024x1024 (4096 img + 512 txt tokens), 28-step schedule, guidance 3.5, batch 1",
            "qwen": "Qwen-Image {q} 1024x1024 (4096 img + 256 txt tokens), CFG batch 2 (cond + uncond), "
                    "30-step schedule, guidance 4.0"}


def all_host_threads():
    """Let the CPU sample use every host core: torchrun sets OMP_NUM_THREADS=1 in each rank's
    environment when it starts more than one process, which would leave BLAS single-threaded."""
    from threadpoolctl import threadpool_limits
    return threadpool_limits(limits=CpuSample.cores())


def reference_arm(args, rank):
    if rank != 0:
        return
    with all_host_threads():
        s = cpu_sample(args)
        for _ in range(max(args.warmup, 1)):
            s.run()
        times = [s.run() for _ in range(args.steps)]
    t_step = statistics.mean(times) * s.ratio
    v = 1.0 / t_step
    line = {"impl": "reference", "metric": METRIC[args.model], "value": v, "unit": "steps/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_step * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,0.02) weights quantized to GGUF, N(0,1) activations)",
            "config": {"workload": WORKLOAD[args.model].format(q=args.quant.upper()),
                       "sample": "%s per step, extrapolated x%.1f by FLOPs" % (s.desc, s.ratio)},
            "cpu_baseline": {"value": v, "unit": "steps/s", "cores": s.cores(), "kind": "port",
                             "sample": "numpy/OpenBLAS oracle, %s per step, extrapolated x%.1f by FLOPs to a "
                                       "full step; the Rust reference (candle CPU) cannot be built on this image"
                                       % (s.desc, s.ratio)},
            "e2e": {"value": v, "unit": "steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ kernel timings
def time_gemm(raw, gtype, shape, M, device, reps=20):
    """CUDA-event time of one dequant-GEMM launch shape (the weight `raw` [N, K] in GGUF bytes,
    M activation rows), timed alone on the launching stream after 3 warm-up launches."""
    import torch
    import mold_b200 as mb
    st = torch.cuda.current_stream()
    N, K = shape
    w = mb.QMatMul.from_device_bytes(raw, gtype, N, K, device)
    x = torch.randn((M, K), device=f"cuda:{device}").bfloat16()
    y = torch.empty((M, N), device=f"cuda:{device}", dtype=torch.bfloat16)
    for _ in range(3):
        w.forward(x, out=y)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(st)
    for _ in range(reps):
        w.forward(x, out=y)
    e1.record(st)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / reps
    flops = 2.0 * M * N * K
    del w
    return {"shape": [M, N, K], "ms": ms, "tflops": flops / ms / 1e9, "weight_bytes": raw.numel(),
            "act_bytes": 2 * M * K + 2 * M * N}


def time_attention(L, H, device, reps=20):
    """CUDA-event time of the joint attention over L tokens, H heads of 128."""
    import torch
    import mold_b200 as mb
    st = torch.cuda.current_stream()
    q = torch.randn((H, L, 128), device=f"cuda:{device}").bfloat16()
    k = torch.randn_like(q)
    v = torch.randn_like(q)
    o = torch.empty((L, H * 128), device=f"cuda:{device}", dtype=torch.bfloat16)
    for _ in range(3):
        mb.attention(q, k, v, out=o)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    e0.record(st)
    for _ in range(reps):
        mb.attention(q, k, v, out=o)
    e1.record(st)
    torch.cuda.synchronize()
    ams = e0.elapsed_time(e1) / reps
    return {"shape": [H, L, L, 128], "ms": ams, "tflops": 4.0 * L * L * 128 * H / ams / 1e9}


def _events_ms(fn, reps, flush, st):
    """Median CUDA-event time of fn() on stream st over `reps` launches, each preceded (outside the
    timed pair of events) by a read of `flush` (256 MB, larger than L2): the launch finds none of
    its inputs in L2, and no dirty lines of the flush are written back during it."""
    import torch
    for _ in range(3):
        fn()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    for e0, e1 in ev:
        flush.sum()
        e0.record(st)
        fn()
        e1.record(st)
    torch.cuda.synchronize()
    return statistics.median(e0.elapsed_time(e1) for e0, e1 in ev)


def time_hbm_kernels(want, raw, gtype, qfn, device, peaks, reps=10):
    """The HBM-bound kernels alone at the FLUX step's shapes, from a cold L2, with their
    algorithmic bytes (every input byte read once, every output byte written once):
      gemv          mb_qgemv over 264,192 x 3072 rows (a quarter of the step's 1,056,768
                    modulation rows; 456 MB in Q4_K), f32 x, silu, bias
      ln_modulate   4608 x 3072 f32 in -> bf16 out (+ 2 x 3072 f32 shift/scale)
      qk_norm_rope  4608 x 9216 bf16 qkv in -> q, k, v bf16 [24, 4608, 128] out, + the RoPE table
      dequant       the linear1 weight (21504 x 3072, GGUF) -> bf16"""
    import torch
    import mold_b200 as mb
    dev = f"cuda:{device}"
    st = torch.cuda.current_stream()
    flush = torch.empty(64 << 20, dtype=torch.float32, device=dev)
    out = {}
    g = torch.Generator(device=dev).manual_seed(11)
    hbm = peaks["hbm_gbs"]

    def rec(name, ms, nbytes, shape):
        out[name] = {"shape": shape, "ms": ms, "bytes": nbytes, "gbs": nbytes / ms / 1e6,
                     "frac_of_hbm": nbytes / ms / 1e6 / hbm}

    if "gemv" in want:
        N, K = 264192, 3072
        parts = [qfn(torch.randn((N // 8, K), generator=g, device=dev) * 0.02) for _ in range(8)]
        wr = torch.cat(parts)
        del parts
        w = mb.QMatMul.from_device_bytes(wr, gtype, N, K, device)
        del wr
        x = torch.randn(K, generator=g, device=dev)
        b = torch.randn(N, generator=g, device=dev) * 0.02
        ms = _events_ms(lambda: mb.qgemv(w, x, True, b), reps, flush, st)
        rec("gemv", ms, N * mb.ops.row_bytes(gtype, K) + 4 * (K + 2 * N), [N, K])
        del w
    L, C = L_TXT + L_IMG, 3072
    if "ln_modulate" in want:
        x = torch.randn((L, C), generator=g, device=dev)
        sh, sc = torch.randn(C, generator=g, device=dev), torch.randn(C, generator=g, device=dev)
        ms = _events_ms(lambda: mb.ln_modulate(x, sh, sc), reps, flush, st)
        rec("ln_modulate", ms, L * C * 6 + 8 * C, [L, C])
    if "qk_norm_rope" in want:
        qkv = torch.randn((L, 3 * C), generator=g, device=dev).bfloat16()
        qs, ks = torch.ones(128, device=dev), torch.ones(128, device=dev)
        pe = mb.rope_table(torch.cat([mb.sampling.txt_ids(L_TXT, device=dev),
                                      mb.sampling.img_ids(LAT_H // 2, LAT_W // 2, device=dev)]))
        q, k_, v = (torch.empty((24, L, 128), dtype=torch.bfloat16, device=dev) for _ in range(3))
        ms = _events_ms(lambda: mb.qk_norm_rope(qkv, 24, qs, ks, pe, q=q, k=k_, v=v), reps, flush, st)
        rec("qk_norm_rope", ms, L * 3 * C * 2 * 2 + pe.numel() * 4, [L, 3 * C])
    if "dequant" in want:
        N, K = 3 * 3072 + 12288, 3072
        w = mb.QMatMul.from_device_bytes(raw, gtype, N, K, device)
        o = torch.empty((N, K), dtype=torch.bfloat16, device=dev)
        ms = _events_ms(lambda: mb.lib().mb_dequant(w.handle, ctypes.c_void_p(o.data_ptr()), mb.DT_BF16,
                                                   ctypes.c_void_p(st.cuda_stream)), reps, flush, st)
        rec("dequant", ms, raw.numel() + N * K * 2, [N, K])
    if mb.device_status() != 0:
        raise RuntimeError("a kernel reported a bounded-wait timeout")
    return out


def time_kernels(keep, device, peaks, reps=20):
    """Standalone CUDA-event timings of the dominant FLUX kernels on the launching stream."""
    raw, gtype, shape = keep["linear1"]
    return {"gemm_linear1": time_gemm(raw, gtype, shape, L_TXT + L_IMG, device, reps),
            "attention": time_attention(L_TXT + L_IMG, 24, device, reps)}


def profiled_traffic(name):
    """dram read + write bytes per launch from a committed ncu summary in profiles/ (None if absent)."""
    import re
    p = os.path.join(ROOT, "profiles", name)
    if not os.path.exists(p):
        return None
    m = re.search(r"traffic \(read \+ write\) \| ([0-9,]+) B per launch", open(p).read())
    return int(m.group(1).replace(",", "")) if m else None


def phys_gpu(local):
    """nvidia-smi -i argument for this rank's GPU (index or UUID from CUDA_VISIBLE_DEVICES)."""
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        items = [v.strip() for v in vis.split(",") if v.strip()]
        if local < len(items):
            return items[local]
    return str(local)


# ------------------------------------------------------------------ replica plumbing (one image per GPU)
def image_seed(rank):
    """Each rank denoises its own image: seed = rank, so 8 GPUs run seeds 0-7.
    The weights' generator streams are salted (WEIGHT_SALT) so no latent repeats a weight stream."""
    return rank


WEIGHT_SALT = 0x5EED0000


def max_over_ranks(value, world, device):
    """Max of a per-rank float over all ranks (the job time is the slowest rank's)."""
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(value)], device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def whole_job_rate(units_per_rank, world, ms_max):
    """Units of all ranks per second, timed by the slowest rank (weak scaling)."""
    return world * units_per_rank / (ms_max / 1e3)


# ------------------------------------------------------------------ config 2: GEMM sweep
SWEEP_M = (1536, 4608)
SWEEP_KN = (("qkv", 3072, 9216), ("mlp_in", 3072, 12288), ("mlp_out", 12288, 3072),
            ("single_proj_out", 15360, 3072), ("attn_out", 3072, 3072))


def sweep(args, local, peaks, reps=10):
    """Q4_K dequant-GEMM over M x (K->N) of BASELINE config 2 (weights quantized from N(0, 0.02),
    bf16 N(0, 1) activations, seed 0). Each launch is timed alone with CUDA events on the launching
    stream after 3 warm-ups; a 256 MB buffer is read between launches so that every launch reads
    its weight and activations from HBM (L2 flushed), and the median of `reps` launches is kept."""
    import torch
    import mold_b200 as mb
    dev = f"cuda:{local}"
    st = torch.cuda.current_stream()
    flush = torch.empty(64 << 20, dtype=torch.float32, device=dev)
    gtype, qfn, _ = quantizer(args.quant)
    g = torch.Generator(device=dev)
    only = tuple(args.sweep_only.split(":")) if args.sweep_only else None
    for name, K, N in SWEEP_KN:
        if only and only[0] != name:
            continue
        g.manual_seed(WEIGHT_SALT + K * 7 + N)
        raw = qfn(torch.randn((N, K), generator=g, device=dev) * 0.02)
        w = mb.QMatMul.from_device_bytes(raw, gtype, N, K, local)
        for M in SWEEP_M:
            if only and int(only[1]) != M:
                continue
            x = torch.randn((M, K), generator=g, device=dev).bfloat16()
            y = torch.empty((M, N), device=dev, dtype=torch.bfloat16)
            for _ in range(3):
                w.forward(x, out=y)
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
            for e0, e1 in ev:
                flush.sum()  # a 256 MB read: L2 holds none of the launch's inputs
                e0.record(st)
                w.forward(x, out=y)
                e1.record(st)
            torch.cuda.synchronize()
            ms = statistics.median(e0.elapsed_time(e1) for e0, e1 in ev)
            flops = 2.0 * M * N * K
            alg = raw.numel() + 2 * M * K + 2 * M * N
            print(json.dumps({"sweep": "config2_q4k_gemm", "linear": name, "quant": args.quant, "M": M, "K": K,
                              "N": N, "ms": ms, "tflops": flops / ms / 1e9,
                              "frac_of_burst": flops / ms / 1e9 / peaks["bf16_tflops"],
                              "peak": peaks["bf16_tflops"], "peak_source": peaks["source"],
                              "algorithmic_bytes": alg, "gbs": alg / ms / 1e6, "l2": "flushed (256 MB read) between launches"}),
                  flush=True)
        del w
    if mb.device_status() != 0:
        raise RuntimeError("a kernel reported a bounded-wait timeout")


# ------------------------------------------------------------------ main arm
def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return reference_arm(args, rank)

    import torch
    import torch.distributed as dist
    import mold_b200 as mb

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device(f"cuda:{local}"))
    mb.init(local)
    peaks = load_peaks()
    dev = f"cuda:{local}"

    if args.kernels_only:
        # the dominant kernels alone, on one linear1-shaped weight (small enough for an ncu capture)
        g = torch.Generator(device=dev).manual_seed(7)
        x = torch.randn((3 * 3072 + 12288, 3072), generator=g, device=dev) * 0.02
        gtype, qfn, _ = quantizer(args.quant)
        raw = qfn(x)
        del x
        want = set(args.kernel.split(","))
        k = {}
        if "gemm" in want:
            k["gemm_linear1"] = time_gemm(raw, gtype, (3 * 3072 + 12288, 3072), L_TXT + L_IMG, local, 5)
        if "attention" in want:
            k["attention"] = time_attention(L_TXT + L_IMG, 24, local, 5)
        if "gemm_qwen_mlp0" in want:  # Qwen-Image img_mlp.net.0.proj over the CFG batch's 2 x 4096 rows
            wq = qfn(torch.randn((12288, 3072), generator=g, device=dev) * 0.02)
            k["gemm_qwen_mlp0"] = time_gemm(wq, gtype, (12288, 3072), 2 * L_IMG, local, 5)
        k.update(time_hbm_kernels(want, raw, gtype, qfn, local, peaks))
        if rank == 0:
            print(json.dumps({"kernels": k}), flush=True)
        return

    if args.sweep:
        if rank == 0:
            sweep(args, local, peaks)
        return

    if args.model == "qwen":
        return main_qwen(args, world, rank, local, dev, peaks)

    model, cfg, keep = build_flux(args.quant, local, seed=0)

    gen = torch.Generator(device=dev).manual_seed(image_seed(rank))
    latent = torch.randn((16, LAT_H, LAT_W), generator=gen, device=dev)
    img0 = mb.sampling.patchify(latent).contiguous()
    img_ids = mb.sampling.img_ids(LAT_H // 2, LAT_W // 2, device=dev)
    txt = torch.randn((L_TXT, cfg.context_in_dim), generator=gen, device=dev)
    txt_ids = mb.sampling.txt_ids(L_TXT, device=dev)
    y = torch.randn((cfg.vec_in_dim,), generator=gen, device=dev)
    sched = mb.sampling.get_schedule(N_SCHEDULE, L_IMG)

    def steps_schedule(n):
        # n steps taken cyclically from the 28-step schedule
        ts = [sched[i % N_SCHEDULE] for i in range(n)]
        return ts + [sched[n % N_SCHEDULE] if n % N_SCHEDULE else 0.0]

    # the dominant kernels timed alone first, at burst clocks (their roofline peak is the burst figure)
    kern = None
    if rank == 0:
        kern = time_kernels(keep, local, peaks)
        gtype, qfn, _ = quantizer(args.quant)
        kern.update(time_hbm_kernels({"gemv", "ln_modulate", "qk_norm_rope"}, None, gtype, qfn, local, peaks))
    img = img0.clone()
    st = torch.cuda.current_stream()
    # warm-up: first call captures the step graph, then W replays
    model.denoise(img, img_ids, txt, txt_ids, y, steps_schedule(max(args.warmup, 1)), GUIDANCE)
    torch.cuda.synchronize()
    if mb.device_status() != 0:
        raise RuntimeError("a kernel reported a bounded-wait timeout during warm-up")
    img.copy_(img0)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    with ClockSampler(phys_gpu(local)) as clk:
        e0.record(st)
        model.denoise(img, img_ids, txt, txt_ids, y, steps_schedule(args.steps), GUIDANCE)
        e1.record(st)
        barrier()
    ms_max = max_over_ranks(e0.elapsed_time(e1), world, dev)
    finite = bool(torch.isfinite(img).all().item())
    steps_per_s = whole_job_rate(args.steps, world, ms_max)
    ms_per_step = ms_max / args.steps

    # ---- end to end through the public denoise call: pinned host buffers, copies inside the timed region
    e2e = None
    if not args.no_e2e:
        h_img = img0.cpu().pin_memory()
        h_txt = txt.cpu().pin_memory()
        h_y = y.cpu().pin_memory()
        h_out = torch.empty_like(h_img).pin_memory()
        n_e2e = N_SCHEDULE
        barrier()
        e0.record(st)
        img.copy_(h_img, non_blocking=True)
        txt.copy_(h_txt, non_blocking=True)
        y.copy_(h_y, non_blocking=True)
        model.denoise(img, img_ids, txt, txt_ids, y, sched, GUIDANCE)
        h_out.copy_(img, non_blocking=True)
        e1.record(st)
        barrier()
        ems = max_over_ranks(e0.elapsed_time(e1), world, dev)
        h2d = (h_img.numel() + h_txt.numel() + h_y.numel()) * 4
        e2e = {"value": whole_job_rate(n_e2e, world, ems), "unit": "steps/s",
               "h2d_bytes_per_step": h2d / n_e2e, "d2h_bytes_per_step": h_out.numel() * 4 / n_e2e,
               "images_per_s": world / (ems / 1e3),
               "note": "one mb_flux_denoise call per image (28 steps) from pinned host inputs to the host latent"}

    if world > 1:
        dist.barrier()
    if rank != 0:
        dist.destroy_process_group()
        return

    cpu = None  # the CPU sample is taken at N=1 only (rank 0 is the only rank there)
    if not args.no_cpu and world == 1:
        try:
            with all_host_threads():
                s = CpuSample(args.quant)
                s.run()
                tt = [s.run() for _ in range(2)]
            cpu = {"value": 1.0 / (statistics.mean(tt) * s.ratio), "unit": "steps/s", "cores": s.cores(),
                   "kind": "port",
                   "sample": "numpy/OpenBLAS oracle: %s (%s), mean of 2 timed runs, extrapolated x%.1f "
                             "by FLOPs to one full step" % (s.desc, args.quant.upper(), s.ratio)}
        except Exception as ex:  # the baseline must not hide the GPU number
            cpu = {"value": None, "unit": "steps/s", "cores": None, "kind": "port", "sample": f"failed: {ex}"}

    g = kern["gemm_linear1"]
    roof = {"bound": "tensor", "achieved": g["tflops"], "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
            "frac": g["tflops"] / peaks["bf16_tflops"],
            "traffic": profiled_traffic("k_qgemm_q4k_linear1_4608x21504x3072.md") if args.quant == "q4_k" else None,
            "algorithmic_bytes": g["weight_bytes"] + g["act_bytes"],
            "kernel": "k_qgemm<%s> single_blocks.linear1 M=4608 N=21504 K=3072" % args.quant.upper(),
            "peak_source": peaks["source"] + " bf16_tflops (burst; kernel timed alone)",
            "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, one launch of the same shape "
                              "(profiles/k_qgemm_q4k_linear1_4608x21504x3072.md)"}
    step_flops = mb.flux.step_flops(cfg, L_TXT, L_IMG)
    # launches per replayed step: timestep embeddings (2), batched GEMVs (3 x stage + run), casts (2),
    # stems (2), final LN + linear (2), Euler (1), prologue (1); 8 per double block, 5 per single block
    n_launch = 16 + cfg.depth * 8 + cfg.depth_single_blocks * 5
    line = {
        "metric": "flux_dev_1024_denoise_steps_per_s", "value": steps_per_s, "unit": "steps/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,0.02) weights quantized to GGUF on device, N(0,1) latents/text)",
        "config": {"workload": f"FLUX.1-dev {args.quant.upper()} 1024x1024 (4096 img + 512 txt tokens), "
                               f"28-step schedule, guidance 3.5, batch 1 per GPU",
                   "parallelism": f"replicas x{world} (one image per GPU, no collective)",
                   "l2": "inputs larger than L2 (6.7 GB of weights streamed per step)"},
        "images_per_s": steps_per_s / N_SCHEDULE,
        "step_tflops": step_flops / 1e12,
        "step_frac_of_sustained": step_flops * (steps_per_s / world) / 1e12 / peaks["bf16_tflops_sustained"],
        "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": n_launch * args.steps,
        "clocks": clk.summary(), "kernels": kern, "finite": finite,
    }
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def main_qwen(args, world, rank, local, dev, peaks):
    """Config 5: Qwen-Image 1024x1024, one image per GPU, each step a CFG batch of 2 sequences
    (conditional + unconditional prompt, 256 text tokens each) through mb_qwen_denoise."""
    import torch
    import torch.distributed as dist
    import mold_b200 as mb
    model, cfg, keep = build_qwen(args.quant, local, seed=0)
    gen = torch.Generator(device=dev).manual_seed(image_seed(rank))
    latent = torch.randn((16, LAT_H, LAT_W), generator=gen, device=dev)
    img0 = mb.sampling.patchify(latent).contiguous()
    txt = torch.randn((2, Q_TXT, cfg.joint_attention_dim), generator=gen, device=dev)
    mask = torch.ones((2, Q_TXT), dtype=torch.uint8, device=dev)
    hh, ww = LAT_H // 2, LAT_W // 2
    sig = mb.sampling.qwen_sigmas(Q_STEPS, L_IMG)

    def sigmas(n):
        s = [sig[i % Q_STEPS] for i in range(n)]
        return s + [sig[n % Q_STEPS] if n % Q_STEPS else 0.0]

    kern = None  # the dominant kernels timed alone first, at burst clocks
    if rank == 0:
        raw, gtype, shape = keep["mlp0"]
        kern = {"gemm_mlp0": time_gemm(raw, gtype, shape, 2 * L_IMG, local),
                "attention": time_attention(Q_TXT + L_IMG, 24, local)}
    st = torch.cuda.current_stream()
    img = img0.clone()
    model.denoise(img, txt, mask, hh, ww, sigmas(max(args.warmup, 1)), Q_GUIDANCE)
    torch.cuda.synchronize()
    if mb.device_status() != 0:
        raise RuntimeError("a kernel reported a bounded-wait timeout during warm-up")
    img.copy_(img0)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    with ClockSampler(phys_gpu(local)) as clk:
        e0.record(st)
        model.denoise(img, txt, mask, hh, ww, sigmas(args.steps), Q_GUIDANCE)
        e1.record(st)
        barrier()
    ms_max = max_over_ranks(e0.elapsed_time(e1), world, dev)
    finite = bool(torch.isfinite(img).all().item())
    steps_per_s = whole_job_rate(args.steps, world, ms_max)

    e2e = None
    if not args.no_e2e:
        h_img = img0.cpu().pin_memory()
        h_txt = txt.cpu().pin_memory()
        h_mask = mask.cpu().pin_memory()
        h_out = torch.empty_like(h_img).pin_memory()
        barrier()
        e0.record(st)
        img.copy_(h_img, non_blocking=True)
        txt.copy_(h_txt, non_blocking=True)
        mask.copy_(h_mask, non_blocking=True)
        model.denoise(img, txt, mask, hh, ww, sig, Q_GUIDANCE)
        h_out.copy_(img, non_blocking=True)
        e1.record(st)
        barrier()
        ems = max_over_ranks(e0.elapsed_time(e1), world, dev)
        h2d = h_img.numel() * 4 + h_txt.numel() * 4 + h_mask.numel()
        e2e = {"value": whole_job_rate(Q_STEPS, world, ems), "unit": "steps/s",
               "h2d_bytes_per_step": h2d / Q_STEPS, "d2h_bytes_per_step": h_out.numel() * 4 / Q_STEPS,
               "images_per_s": world / (ems / 1e3),
               "note": "one mb_qwen_denoise call per image (30 CFG steps) from pinned host inputs to the host latent"}

    if world > 1:
        dist.barrier()
    if rank != 0:
        dist.destroy_process_group()
        return
    cpu = None
    if not args.no_cpu and world == 1:
        try:
            with all_host_threads():
                s = QwenCpuSample(args.quant)
                s.run()
                tt = [s.run() for _ in range(2)]
            cpu = {"value": 1.0 / (statistics.mean(tt) * s.ratio), "unit": "steps/s", "cores": s.cores(),
                   "kind": "port",
                   "sample": "numpy/OpenBLAS oracle: %s (%s), mean of 2 timed runs, extrapolated x%.1f "
                             "by FLOPs to one full CFG step" % (s.desc, args.quant.upper(), s.ratio)}
        except Exception as ex:
            cpu = {"value": None, "unit": "steps/s", "cores": None, "kind": "port", "sample": f"failed: {ex}"}
    g = kern["gemm_mlp0"]
    roof = {"bound": "tensor", "achieved": g["tflops"], "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
            "frac": g["tflops"] / peaks["bf16_tflops"],
            "traffic": profiled_traffic("k_qgemm_q4k_qwen_mlp0_8192x12288x3072.md") if args.quant == "q4_k" else None,
            "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum, one launch of the same shape "
                              "(profiles/k_qgemm_q4k_qwen_mlp0_8192x12288x3072.md)",
            "algorithmic_bytes": g["weight_bytes"] + g["act_bytes"],
            "kernel": "k_qgemm<%s> img_mlp.net.0.proj M=8192 N=12288 K=3072" % args.quant.upper(),
            "peak_source": peaks["source"] + " bf16_tflops (burst; kernel timed alone)"}
    step_flops = mb.qwen.step_flops(cfg, Q_TXT, L_IMG, batch=2)
    # per replayed step: temb, 3 GEMVs (stage + run each), RMSNorm, txt_in, 2 casts, img_in, final
    # LN + linear, CFG-Euler, prologue (16); per block 2 LN, 4 grouped GEMMs, 1 QK-norm, 2 attention
    n_launch = 16 + cfg.num_layers * 9
    line = {
        "metric": METRIC["qwen"], "value": steps_per_s, "unit": "steps/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,0.02) weights quantized to GGUF on device, N(0,1) latents/text, "
                "all text tokens kept)",
        "config": {"workload": WORKLOAD["qwen"].format(q=args.quant.upper()),
                   "parallelism": f"replicas x{world} (one image per GPU, no collective)",
                   "l2": "inputs larger than L2 (11.5 GB of weights streamed per step)"},
        "images_per_s": world / (ms_max / args.steps * Q_STEPS / 1e3),
        "step_tflops": step_flops / 1e12,
        "step_frac_of_sustained": step_flops * steps_per_s / world / 1e12 / peaks["bf16_tflops_sustained"],
        "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": n_launch * args.steps,
        "clocks": clk.summary(), "kernels": kern, "finite": finite,
    }
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
