#!/usr/bin/env python
"""Benchmark of the B200-native LTX DiT denoise step.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N ...

Workload ("config 3"): full-size video DiT, 28 blocks, hidden 2048, 32x64 heads, FFN 8192,
latent 128 ch x 16x16x24 = 6144 tokens, CFG batch 2 (cond, uncond), text context
128 x 4096 ~ N(0,1), sigma 0.5, BF16, synthetic N(0, 0.02) weights. One step = the B=2
transformer forward + X0 + CFG + Euler update of one latent (cfg_denoise_step).
Prints one JSON line on rank 0.

  value     whole-job latent tokens/s = video tokens x CFG batch x steps/s, inputs
            resident in HBM, device-timed (CUDA events) over K steps, max over ranks.
  e2e       the same metric through the public API call (cfg_denoise_step) with the
            step's latent copied host->device from pinned memory and the next latent
            copied back every step.
  roofline  the dominant kernel (by time share) of an instrumented step, CUDA events
            on the launching stream, against MEASURED_PEAKS.json.
  cpu_baseline  the CPU oracle (the reference's PyTorch math restated) on this box's
            host cores for a bounded sample (one of the 28 blocks), scaled to a step.
N > 1: the same single step split over the N GPUs (strong scaling): CFG cond/uncond on
two GPU groups x Ulysses sequence parallelism over the video tokens inside each group
(ltx_parallel.ParallelDenoiser, NCCL all-to-all / all-gather over NVLink).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (str(ROOT), str(ROOT / "ltx-nv_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

METRIC = "DiT denoise steps/s & latent tokens/s at 1/2/4/8 B200; % BF16 TC peak"
UNIT = "latent tokens/s"
CFG3 = dict(num_layers=28, heads=32, head_dim=64, cross_dim=4096, f=16, h=16, w=24, text=128, sigma=0.5,
            sigma_next=0.25, cfg_scale=3.0)


def step_flops(c=CFG3, batch=2) -> float:
    """Algorithmic FLOPs of one CFG step (adaLN counted once per sample)."""
    t = c["f"] * c["h"] * c["w"]
    d = c["heads"] * c["head_dim"]
    f, s, cc, h = 4 * d, c["text"], c["cross_dim"], c["heads"]
    per_block = 8 * t * d * d + 4 * t * t * d + 4 * t * d * d + 4 * s * cc * d + 4 * t * s * d + 4 * t * d * f \
        + 4 * t * d * h
    return float((per_block * c["num_layers"] + 4 * t * d * 128) * batch)


def load_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        d["source"] = "measured"
        return d
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.rows = []
        if self.proc is None:
            return
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        for line in out.splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.rows.append(parts)

    def summary(self) -> dict:
        rows = getattr(self, "rows", [])
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ---------------------------------------------------------------------------------------
# our implementation
# ---------------------------------------------------------------------------------------


def build_model(dev: torch.device, seed: int = 1):
    """Config-3 model with N(0, 0.02) weights drawn on the device by the Philox kernel
    (q/k RMSNorm gains offset by +1, as in the oracle's synthetic weights)."""
    import ltx_dit

    c = CFG3
    cfg = ltx_dit.DiTConfig.video_only(num_layers=c["num_layers"], heads=c["heads"], head_dim=c["head_dim"],
                                       cross_dim=c["cross_dim"])
    with torch.device("meta"):
        model = ltx_dit.LTXModel(cfg)
    gen = ltx_dit.PhiloxGenerator(seed, dev)
    sd = {}
    for name, p in model.named_parameters():
        w = gen.randn(*p.shape, dtype=torch.bfloat16).mul_(0.02)
        if name.endswith(("q_norm.weight", "k_norm.weight")):
            w.add_(1.0)
        sd[name] = w
    model.load_state_dict(sd, assign=True)
    return model.eval(), cfg


def make_inputs(dev: torch.device, seed: int = 7):
    import ltx_dit

    c = CFG3
    t = c["f"] * c["h"] * c["w"]
    gen = ltx_dit.PhiloxGenerator(seed, dev)
    latent = gen.randn(1, t, 128, dtype=torch.bfloat16)
    ctx = gen.randn(2, c["text"], c["cross_dim"], dtype=torch.bfloat16)
    pos = ltx_dit.video_positions(1, c["f"], c["h"], c["w"], 24.0, dev)
    kf = torch.zeros(1, t, 1, device=dev)
    kf[:, : c["h"] * c["w"]] = 1.0
    sigmas = torch.tensor([c["sigma"], c["sigma_next"]], dtype=torch.float32)
    return latent, ctx, pos, kf, sigmas


def run_ours(args, rank: int, world: int, dev: torch.device) -> dict | None:
    import _native as nat
    import ltx_dit

    c = CFG3
    t = c["f"] * c["h"] * c["w"]
    model, cfg = build_model(dev)
    latent, ctx, pos, kf, sigmas = make_inputs(dev, seed=7)
    cpos, cneg = ctx[:1], ctx[1:]
    if world > 1:
        import ltx_parallel

        pdn = ltx_parallel.ParallelDenoiser(model)
        layout = pdn.layout

        def step(lat):
            return pdn.step(lat, pos, cpos, cneg, sigmas, 0, c["cfg_scale"], keyframes_mask=kf)
    else:
        layout = None

        def step(lat):
            return ltx_dit.cfg_denoise_step(model, lat, pos, cpos, cneg, sigmas, 0, c["cfg_scale"],
                                            keyframes_mask=kf)[2]

    stream = torch.cuda.current_stream(dev)
    # warm-up (eager), then capture one step in a CUDA graph (single GPU)
    for _ in range(max(args.warmup, 1)):
        step(latent)
    torch.cuda.synchronize(dev)
    graph = None
    if not args.no_graph:
        # one step captured in a CUDA graph (N > 1: the NCCL collectives of the step are
        # captured too; every rank captures the same sequence after the eager warm-up
        # has initialised the communicators)
        graph = torch.cuda.CUDAGraph()
        static_in = latent.clone()
        with torch.cuda.graph(graph):
            static_out = step(static_in)
        for _ in range(max(args.warmup, 1)):
            graph.replay()
        torch.cuda.synchronize(dev)

    launches_per_step = None
    n0 = nat.launch_count()
    step(latent)
    torch.cuda.synchronize(dev)
    launches_per_step = nat.launch_count() - n0

    # ---------------------------------------------------------------- timed region
    dist = torch.distributed if world > 1 else None
    if dist:
        dist.barrier()
    torch.cuda.synchronize(dev)
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index if dev.index is not None else 0) as clocks:
        ev0.record(stream)
        for _ in range(args.steps):
            if graph is not None:
                graph.replay()
            else:
                step(latent)
        ev1.record(stream)
        torch.cuda.synchronize(dev)
    ms = ev0.elapsed_time(ev1)
    if dist:
        tt = torch.tensor([ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    ms_per_step = ms / args.steps
    # one CFG step of one latent = 2 * T latent tokens for the whole job (all ranks
    # together: CFG split x sequence parallel = strong scaling)
    tokens_per_step = 2 * t
    value = tokens_per_step / (ms_per_step / 1e3)

    # ---------------------------------------------------------------- e2e (public API, host buffers)
    host_in = torch.empty(1, t, 128, dtype=torch.bfloat16, pin_memory=True)
    host_in.copy_(latent.cpu())
    host_out = torch.empty_like(host_in, pin_memory=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize(dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e2e_steps = max(1, min(args.steps, 10))
    e0.record(stream)
    for _ in range(e2e_steps):
        lat_dev = host_in.to(dev, non_blocking=True)
        out = step(lat_dev)
        host_out.copy_(out, non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = e0.elapsed_time(e1)
    if dist:
        tt = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_ms = float(tt.item())
    e2e_value = tokens_per_step / (e2e_ms / e2e_steps / 1e3)

    # ---------------------------------------------------------------- per-kernel breakdown
    with nat.profile() as prof:
        step(latent)
    kern = prof.summary()
    step_ms_instr = sum(v["total_ms"] for v in kern.values())
    # a graph that holds NCCL calls is released before the process group goes away
    used_graph = graph is not None
    del graph
    torch.cuda.synchronize(dev)

    if rank != 0:
        return None
    peaks = load_peaks()
    flops = step_flops()
    tflops = flops / (ms_per_step / 1e3) / 1e12
    # dominant kernel by total time
    dom_label, dom = max(kern.items(), key=lambda kv: kv[1]["total_ms"])
    dom_flops = kernel_flops(dom_label)
    achieved = dom_flops / (dom["avg_ms"] / 1e3) / 1e12 if dom_flops else None
    peak = peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])
    traffic = profile_traffic(dom_label)
    roofline = {"kernel": dom_label, "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                "frac": (achieved / peak) if achieved else None, "traffic": traffic,
                "peak_source": f"{peaks['source']} bf16_tflops_sustained",
                "flops_per_launch": dom_flops, "avg_launch_ms": dom["avg_ms"],
                "share_of_step": dom["total_ms"] / step_ms_instr}
    breakdown = {k: {"launches": v["launches"], "total_ms": round(v["total_ms"], 4),
                     "share": round(v["total_ms"] / step_ms_instr, 4)}
                 for k, v in sorted(kern.items(), key=lambda kv: -kv[1]["total_ms"])}
    return {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {"workload": "BASELINE config 3: full-size video DiT CFG denoise step", "model": "LTX-2.5 video DiT "
                   "28 blocks, hidden 2048, 32x64 heads, FFN 8192 (random-init N(0,0.02))", "global_batch": 2,
                   "latent_tokens": t, "seq_len": t, "text_tokens": CFG3["text"],
                   "parallelism": "single GPU" if world == 1 else f"cfg{layout.cfg} x sp{layout.sp} (Ulysses, NCCL)",
                   "l2": "inputs larger than L2 (4.2 GB weights, ~1 GB activations per step)",
                   "cuda_graph": used_graph},
        "steps_per_s": 1e3 / ms_per_step, "step_tflops_per_gpu": tflops / world,
        "pct_bf16_peak": tflops / world / peaks["bf16_tflops"], "pct_bf16_peak_sustained": tflops / world / peak,
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": host_in.numel() * 2,
                "d2h_bytes_per_step": host_out.numel() * 2, "steps": e2e_steps,
                "api": "ltx_dit.cfg_denoise_step" if world == 1 else "ltx_parallel.ParallelDenoiser.step"},
        "roofline": roofline,
        "gpu_launches": launches_per_step * args.steps,
        "gpu_launches_per_step": launches_per_step,
        "kernels": breakdown,
        "clocks": clocks.summary(),
    }


def kernel_flops(label: str) -> float | None:
    """Algorithmic FLOPs of one launch from a profile label."""
    kv = dict(p.split("=") for p in label.split()[1:] if "=" in p)
    if label.startswith("linear"):
        return 2.0 * int(kv["M"]) * int(kv["N"]) * int(kv["K"])
    if label.startswith("attention"):
        return 4.0 * int(kv["B"]) * int(kv["H"]) * int(kv["Tq"]) * int(kv["Tk"]) * int(kv["d"])
    return None


def profile_traffic(label: str) -> float | None:
    """DRAM bytes per launch of this kernel from the committed ncu summary, if any
    (lines 'traffic_bytes_per_launch: <label> = <bytes>' in profiles/*.md)."""
    for p in sorted((ROOT / "profiles").glob("*.md")):
        for line in p.read_text().splitlines():
            if line.startswith("traffic_bytes_per_launch:") and label in line:
                try:
                    return float(line.rsplit("=", 1)[1].strip())
                except ValueError:
                    return None
    return None


# ---------------------------------------------------------------------------------------
# CPU baseline / reference arm: the CPU oracle (reference math) on the host cores
# ---------------------------------------------------------------------------------------


def cpu_block_sample(threads: int) -> dict:
    """Time one of config 3's 28 blocks (B=2, T=6144, bf16) of the CPU oracle and scale
    it to a full step (x28; patchify/adaLN/head are <1% of the FLOPs and are left out)."""
    from types import SimpleNamespace

    from oracle import ltx_oracle

    torch.set_num_threads(threads)
    c = CFG3
    t = c["f"] * c["h"] * c["w"]
    d = c["heads"] * c["head_dim"]
    cfg = SimpleNamespace(num_layers=1, video_heads=c["heads"], video_head_dim=c["head_dim"], video_cross_dim=4096,
                          norm_eps=1e-6, gated_attention=True, cross_attention_adaln=False, audio_heads=2,
                          audio_head_dim=32)
    shapes = []
    for blk in ("attn1", "attn2"):
        cin = d if blk == "attn1" else c["cross_dim"]
        shapes += [(f"blocks.0.{blk}.q_norm.weight", (d,)), (f"blocks.0.{blk}.k_norm.weight", (d,)),
                   (f"blocks.0.{blk}.to_q.weight", (d, d)), (f"blocks.0.{blk}.to_q.bias", (d,)),
                   (f"blocks.0.{blk}.to_k.weight", (d, cin)), (f"blocks.0.{blk}.to_k.bias", (d,)),
                   (f"blocks.0.{blk}.to_v.weight", (d, cin)), (f"blocks.0.{blk}.to_v.bias", (d,)),
                   (f"blocks.0.{blk}.to_gate_logits.weight", (c["heads"], d)),
                   (f"blocks.0.{blk}.to_gate_logits.bias", (c["heads"],)),
                   (f"blocks.0.{blk}.to_out.weight", (d, d)), (f"blocks.0.{blk}.to_out.bias", (d,))]
    shapes += [("blocks.0.ff.proj_in.weight", (4 * d, d)), ("blocks.0.ff.proj_out.weight", (d, 4 * d)),
               ("blocks.0.scale_shift_table", (6, d))]
    w = ltx_oracle.synthetic_state_dict(shapes, 1, dtype=torch.bfloat16)
    g = torch.Generator().manual_seed(3)
    x = torch.randn(2, t, d, generator=g).to(torch.bfloat16)
    ctx = torch.randn(2, c["text"], c["cross_dim"], generator=g).to(torch.bfloat16)
    mod = (torch.randn(2, 1, 6 * d, generator=g) * 0.1).to(torch.bfloat16)
    pos = ltx_oracle.video_positions(2, c["f"], c["h"], c["w"], 24.0)
    pe = ltx_oracle.rope_tables(pos, d, torch.bfloat16, 10000.0, [20, 2048, 2048], c["heads"])
    va = ltx_oracle.StreamArgs(x=x, context=ctx, mod=mod, embedded=None, pe=pe, cross_pe=None, cross_ss=None,
                               cross_gate=None, prompt_mod=None, enabled=True)
    t0 = time.perf_counter()
    with torch.inference_mode():
        ltx_oracle.block(w, cfg, 0, va, None)
    sec = time.perf_counter() - t0
    step_sec = sec * c["num_layers"]
    return {"value": 2 * t / step_sec, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"1 of 28 blocks of one config-3 CFG step (B=2, T={t}, bf16) on the CPU oracle, "
                      f"{sec:.2f} s, scaled x28 (steps/s {1 / step_sec:.5f})",
            "block_sec": sec}


def run_reference(args, rank: int, world: int) -> dict | None:
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    vals = []
    if args.warmup > 0:
        cpu_block_sample(threads)  # one untimed sample warms the thread pool and caches
    samples = []
    for _ in range(max(1, args.steps)):
        s = cpu_block_sample(threads)
        samples.append(s)
        vals.append(s["value"])
    v = statistics.median(vals)
    cpu = dict(samples[0])
    cpu["value"] = v
    cpu.pop("block_sec", None)
    return {"impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 2 * CFG3["f"] * CFG3["h"] * CFG3["w"] / v * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "BASELINE config 3: full-size video DiT CFG denoise step", "latent_tokens":
                       CFG3["f"] * CFG3["h"] * CFG3["w"], "global_batch": 2, "parallelism": "CPU, host cores"},
            "cpu_baseline": cpu, "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


PROBES = {
    # name: (description, builder) -- one kernel at its config-3 shape
    "attention": "self-attention FMHA, B=2, H=32, T=6144, d=64 (q/k/v/gate read from the packed QKV buffer)",
    "ffn_in": "FFN-in tcgen05 GEMM + GELU epilogue, M=12288, N=8192, K=2048",
    "qkv": "packed QKV(+gate) tcgen05 GEMM, M=12288, N=6176, K=2048",
    "ffn_out": "FFN-out tcgen05 GEMM + gate*out+residual epilogue, M=12288, N=2048, K=8192",
    "attn_out": "attention out-projection tcgen05 GEMM + gate*out+residual epilogue, M=12288, N=2048, K=2048",
    "norm": "RMSNorm + adaLN modulate, [2*6144, 2048] bf16",
    "qknorm": "q RMSNorm (with weight) + split RoPE in place on the packed QKV buffer, [2*6144, 2048] bf16",
    "connector": "text connector (Embeddings1DConnector): 8 blocks, 32x128 heads, 128 registers, B=2 prompts x "
                 "1024 tokens, bf16",
    "vae": "video VAE decoder (ConvVideoDecoder), latent (1, 128, 9, 16, 24) -> 65 frames of 512x768, assumed "
           "block layout base 128, [res_x 5, compress_all 2] x 3 + res_x 5 (random weights), bf16",
    "conv3d": "one 3x3x3 decoder convolution at the last stage: 128 -> 128 channels over 65x128x192 voxels",
}

# Assumed production layout of the video decoder (the real one is read from the
# checkpoint's metadata, absent here): 8x temporal and 8x spatial upsampling by three
# compress_all stages, patch 4, so a (9, 16, 24) latent decodes to 65 frames of 512x768.
VAE_PROBE_CFG = {"decoder_blocks": [["res_x", {"num_layers": 5}], ["compress_all", {"multiplier": 2}],
                                    ["res_x", {"num_layers": 5}], ["compress_all", {"multiplier": 2}],
                                    ["res_x", {"num_layers": 5}], ["compress_all", {"multiplier": 2}],
                                    ["res_x", {"num_layers": 5}]],
                 "decoder_base_channels": 128, "patch_size": 4, "spatial_padding_mode": "zeros",
                 "latent_channels": 128, "out_channels": 3}


def vae_conv_flops(dec, latent_shape) -> float:
    """2 * voxels * taps * cin * cout summed over the decoder's convolutions."""
    import ltx_vae

    _, _, f, h, w = latent_shape
    total = 0.0

    def conv(c, vox):
        k = c.kernel_size[0] * c.kernel_size[1] * c.kernel_size[2]
        return 2.0 * vox * k * c.in_channels * c.out_channels

    vox = f * h * w
    total += conv(dec.conv_in.conv, vox)
    for blk in dec.up_blocks:
        res = blk.res_blocks if isinstance(blk, ltx_vae.UNetMidBlock3D) else (
            [blk] if isinstance(blk, ltx_vae.ResnetBlock3D) else [])
        for rb in res:
            total += conv(rb.conv1.conv, vox) + conv(rb.conv2.conv, vox)
            if isinstance(rb.conv_shortcut, torch.nn.Conv3d):
                total += conv(rb.conv_shortcut, vox)
        if isinstance(blk, ltx_vae.DepthToSpaceUpsample):
            total += conv(blk.conv.conv, vox)
            p1, p2, p3 = blk.stride
            f, h, w = f * p1 - (1 if p1 == 2 else 0), h * p2, w * p3
            vox = f * h * w
    return total + conv(dec.conv_out.conv, vox)


def vae_cpu_sample(decode_flops: float) -> dict:
    """The decoder's CPU restatement (oracle/vae_oracle.py, the reference's PyTorch ops) on
    the host cores: one output frame of the last-stage 3x3x3 convolution (128 -> 128
    channels, 128x192 voxels, bf16), the decode time extrapolated by FLOPs."""
    from oracle import vae_oracle

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    x = torch.randn(1, 128, 1, 128, 192, generator=g).to(torch.bfloat16)
    w = (torch.randn(128, 128, 3, 3, 3, generator=g) * (27 * 128) ** -0.5).to(torch.bfloat16)
    b = torch.zeros(128, dtype=torch.bfloat16)
    vae_oracle.conv3d_same(x, w, b)  # warm-up
    times = []
    for _ in range(5):
        t0 = time.perf_counter()
        vae_oracle.conv3d_same(x, w, b)
        times.append(time.perf_counter() - t0)
    sec = statistics.median(times)
    fl = 2.0 * 128 * 192 * 27 * 128 * 128
    return {"value": decode_flops / (fl / sec) * 1e3, "unit": "ms per decode (extrapolated)", "cores": threads,
            "kind": "port", "sample": f"one output frame of the last-stage 128->128 3x3x3 convolution "
                                      f"({fl / 1e9:.1f} GFLOP) on the CPU oracle, median of 5: {sec:.3f} s, "
                                      f"{fl / sec / 1e12:.3f} TFLOP/s, scaled to the decode's convolution FLOPs"}


def run_probe(args, dev: torch.device) -> dict:
    """Launch one kernel of the step at its config-3 shape W + K times and time the K
    launches with CUDA events (the small, single-kernel case for ncu captures)."""
    import _native as nat

    c = CFG3
    t = c["f"] * c["h"] * c["w"]
    d = c["heads"] * c["head_dim"]
    m = 2 * t
    g = torch.Generator(device=dev).manual_seed(0)

    def rnd(*shape, scale=1.0):
        return (torch.randn(*shape, generator=g, device=dev) * scale).to(torch.bfloat16)

    if args.probe == "attention":
        qkv = rnd(m, 3 * d + c["heads"])
        o = torch.empty(m, d, device=dev, dtype=torch.bfloat16)
        fn = lambda: nat.attention(qkv[:, :d], qkv[:, d:2 * d], qkv[:, 2 * d:3 * d], o, 2, t, t, c["heads"],  # noqa
                                   c["head_dim"], c["head_dim"] ** -0.5, qkv[:, 3 * d:])
        flops = 4.0 * 2 * c["heads"] * t * t * c["head_dim"]
        nbytes = 2 * (qkv.numel() + o.numel())
    elif args.probe in ("ffn_in", "qkv", "ffn_out", "attn_out"):
        n, k = {"ffn_in": (4 * d, d), "qkv": (3 * d + c["heads"], d), "ffn_out": (d, 4 * d),
                "attn_out": (d, d)}[args.probe]
        a, w, bias = rnd(m, k), rnd(n, k, scale=k ** -0.5), rnd(n)
        out = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
        if args.probe == "ffn_in":
            epi = nat.epilogue(nat.EPI_GELU_TANH, bias=bias)
        elif args.probe == "qkv":
            epi = nat.epilogue(bias=bias)
        else:
            table, mod = rnd(6, d, scale=0.1), rnd(2, 6 * d, scale=0.1)
            epi = nat.epilogue(nat.EPI_GATE_RESIDUAL, bias=bias, residual=out,
                               gate=nat.modulation(table, mod, shift=None, scale=(5 * d, 5 * d), mod_ld_batch=6 * d),
                               rows_per_batch=t)
        fn = lambda: nat.linear(a, w, out, epi)  # noqa: E731
        flops = 2.0 * m * n * k
        nbytes = 2 * (a.numel() + w.numel() + out.numel() * (2 if args.probe in ("ffn_out", "attn_out") else 1))
    elif args.probe == "norm":
        x, y = rnd(m, d), torch.empty(m, d, device=dev, dtype=torch.bfloat16)
        table, mod = rnd(6, d, scale=0.1), rnd(2, 6 * d, scale=0.1)
        mm = nat.modulation(table, mod, shift=(0, 0), scale=(d, d), mod_ld_batch=6 * d)
        fn = lambda: nat.norm_modulate(x, y, t, nat.LTX_NORM_RMS, 1e-6, mm)  # noqa: E731
        flops, nbytes = None, 2 * (x.numel() + y.numel())
    elif args.probe == "connector":
        import ltx_te

        conn = ltx_te.Embeddings1DConnector(heads=32, dim_head=128, num_layers=8, max_pos=[4096], registers=128,
                                            gated=False, ff_bias=True)
        for prm in conn.parameters():
            prm.data = rnd(*prm.shape, scale=0.02)
        conn = conn.to(dev).eval()
        s_len, dd = 1024, 4096
        hid = rnd(2, s_len, dd)
        amask = torch.zeros(2, 1, 1, s_len, device=dev, dtype=torch.bfloat16)
        amask[:, :, :, 300:] = -10000.0  # padded prompt tail -> registers
        fn = lambda: conn(hid, amask)  # noqa: E731
        m_rows = 2 * s_len
        flops = 8 * (2.0 * m_rows * dd * 3 * dd + 4.0 * 2 * s_len * s_len * dd + 2.0 * m_rows * dd * dd
                     + 2.0 * m_rows * dd * 4 * dd * 2)
        nbytes = 8 * 2 * (4 * dd * dd + 8 * dd * dd)  # weights streamed once per call
    elif args.probe == "vae":
        import ltx_vae

        with torch.device("meta"):
            dec = ltx_vae.ConvVideoDecoder(VAE_PROBE_CFG)
        sd = {}
        for name, prm in list(dec.named_parameters()) + list(dec.named_buffers()):
            if name.endswith("std-of-means"):
                sd[name] = torch.ones(prm.shape, device=dev)
            elif name.endswith("mean-of-means"):
                sd[name] = torch.zeros(prm.shape, device=dev)
            else:
                fan = prm[0].numel() if prm.dim() > 1 else 1
                sd[name] = torch.randn(prm.shape, generator=g, device=dev) * (fan ** -0.5 if prm.dim() > 1 else 0.02)
        dec.load_state_dict(sd, assign=True)
        dec = dec.eval()
        latent = rnd(1, 128, 9, 16, 24)
        fn = lambda: dec(latent)  # noqa: E731
        flops = vae_conv_flops(dec, latent.shape)
        nbytes = 2 * 3 * 65 * 512 * 768
    elif args.probe == "conv3d":
        f_, h_, w_, cc = 65, 128, 192, 128
        x = rnd(1, f_, h_, w_, cc)
        wt, bias = rnd(cc, 27, cc, scale=(27 * cc) ** -0.5), rnd(cc)
        out = torch.empty_like(x)
        fn = lambda: nat.conv3d(x, wt, bias, out, 3)  # noqa: E731
        flops = 2.0 * f_ * h_ * w_ * 27 * cc * cc
        nbytes = 2 * (x.numel() + out.numel() + wt.numel())
    elif args.probe == "qknorm":
        qkv = rnd(m, 3 * d + c["heads"])
        wq = (1 + rnd(d, scale=0.02).float()).to(torch.bfloat16)
        cos, sin = rnd(t, d // 2), rnd(t, d // 2)
        fn = lambda: nat.qk_norm_rope(qkv[:, :d], t, c["heads"], c["head_dim"], wq, 1e-6, cos, sin, 0)  # noqa
        flops, nbytes = None, 2 * (2 * m * d + cos.numel() + sin.numel())
    else:
        raise SystemExit(f"unknown probe {args.probe}")
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        fn()
    e1.record()
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1) / args.steps
    peaks = load_peaks()
    res = {"probe": args.probe, "what": PROBES[args.probe], "avg_launch_ms": ms, "launches": args.steps,
           "algorithmic_bytes": nbytes, "achieved_GBps": nbytes / (ms / 1e3) / 1e9}
    if args.probe == "vae":
        res["cpu_baseline"] = vae_cpu_sample(flops)
    if flops:
        res.update({"flops": flops, "achieved_TFLOPs": flops / (ms / 1e3) / 1e12,
                    "frac_of_measured_burst": flops / (ms / 1e3) / 1e12 / peaks["bf16_tflops"]})
    else:
        res["frac_of_measured_hbm"] = nbytes / (ms / 1e3) / 1e9 / peaks["hbm_gbs"]
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--probe", choices=sorted(PROBES), default=None,
                    help="time one kernel of the step at its config-3 shape instead of the step")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if world > 1 and rank != 0:
            return
        line = run_reference(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if args.probe:
        print(json.dumps(run_probe(args, dev)), flush=True)
        return
    # Libraries (NCCL's banner among them) write to file descriptor 1; keep stdout for the
    # one JSON line by pointing fd 1 at stderr until it is printed.
    sys.stdout.flush()
    json_out = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    if world > 1:
        from datetime import timedelta

        torch.distributed.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    try:
        line = run_ours(args, rank, world, dev)
        if line is not None and not args.no_cpu_baseline:
            cb = cpu_block_sample(os.cpu_count() or 1)
            cb.pop("block_sec", None)
            line["cpu_baseline"] = cb
        if line is not None:
            json_out.write(json.dumps(line) + "\n")
            json_out.flush()
    finally:
        if world > 1:
            torch.distributed.barrier()
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
