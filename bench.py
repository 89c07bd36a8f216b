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
            host cores: one whole 28-block CFG step (the --impl reference arm times as
            many whole steps as fit in 90 s).
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
CONFIGS = {
    # BASELINE.json configs; 1 (FP32 CPU loop) and 2 (microbench) are parity-test cases
    3: dict(kind="video", num_layers=28, heads=32, head_dim=64, cross_dim=4096, f=16, h=16, w=24, text=128,
            sigma=0.5, sigma_next=0.25, cfg_scale=3.0, loop=None,
            workload="BASELINE config 3: full-size video DiT CFG denoise step"),
    4: dict(kind="av", num_layers=48, heads=32, head_dim=128, cross_dim=3840, f=16, h=16, w=24, text=1024,
            audio_tokens=126, audio_text=1024, audio_cross=2048, sigma=0.5, sigma_next=0.25, cfg_scale=3.0, loop=None,
            workload="BASELINE config 4: dual-stream audio-video DiT CFG denoise step (video 4096 wide, 6144 "
                     "tokens; audio 2048 wide, 126 tokens; A<->V attention in every block; text 1024x3840 and "
                     "1024x2048)"),
    5: dict(kind="video", num_layers=28, heads=32, head_dim=64, cross_dim=4096, f=33, h=22, w=38, text=128,
            cfg_scale=3.0, loop=30,
            workload="BASELINE config 5: long high-res video, 27588 tokens, steps of the 30-step Euler loop "
                     "(ltx2_scheduler_sigmas(30))"),
}
CFG3 = CONFIGS[3]


def step_flops(c=CFG3, batch=2, text_kv_cached=True) -> float:
    """Algorithmic FLOPs of one CFG step (adaLN counted once per sample). The text-context
    K/V projection (4*S*C*D per block and sample) depends only on the constant context
    and weights; the step caches it across denoise steps, so with text_kv_cached it is not
    counted (0.4 % of the step at config 3)."""
    t = c["f"] * c["h"] * c["w"]
    d = c["heads"] * c["head_dim"]
    f, s, cc, h = 4 * d, c["text"], c["cross_dim"], c["heads"]
    per_block = 8 * t * d * d + 4 * t * t * d + 4 * t * d * d + 4 * t * s * d + 4 * t * d * f + 4 * t * d * h
    if not text_kv_cached:
        per_block += 4 * s * cc * d
    return float((per_block * c["num_layers"] + 4 * t * d * 128) * batch)


def workload_config(c=CFG3) -> dict:
    """The `config` object of both arms' JSON lines (the workload only, so the two arms'
    objects are equal; how it ran goes in `execution`)."""
    t = c["f"] * c["h"] * c["w"]
    d = c["heads"] * c["head_dim"]
    kind = "audio-video DiT" if c["kind"] == "av" else "video DiT"
    out = {"workload": c["workload"],
           "model": f"LTX-2.5 {kind} {c['num_layers']} blocks, hidden {d}, {c['heads']}x{c['head_dim']} heads, "
                    f"FFN {4 * d} (random-init N(0,0.02))",
           "global_batch": 2, "latent_tokens": t, "seq_len": t, "text_tokens": c["text"],
           "cfg_scale": c["cfg_scale"],
           "l2": "inputs larger than L2 (weights of several GB, activations of ~1 GB or more per step)"}
    if c.get("loop"):
        out["schedule"] = f"ltx2_scheduler_sigmas({c['loop']}), step k uses sigmas[k % {c['loop']}]"
    else:
        out["sigma"], out["sigma_next"] = c["sigma"], c["sigma_next"]
    if c["kind"] == "av":
        out.update(audio_tokens=c["audio_tokens"], audio_text_tokens=c["audio_text"], audio_hidden=2048)
    return out


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


def dit_config(c):
    import ltx_dit

    if c["kind"] == "av":
        return ltx_dit.DiTConfig(num_layers=c["num_layers"], video_heads=c["heads"], video_head_dim=c["head_dim"],
                                 video_cross_dim=c["cross_dim"], audio_cross_dim=c["audio_cross"],
                                 cross_attention_adaln=False)
    return ltx_dit.DiTConfig.video_only(num_layers=c["num_layers"], heads=c["heads"], head_dim=c["head_dim"],
                                        cross_dim=c["cross_dim"])


def build_model(dev: torch.device, seed: int = 1, c=CFG3):
    """The config's model with N(0, 0.02) weights drawn on the device by the Philox kernel
    (q/k RMSNorm gains offset by +1, as in the oracle's synthetic weights)."""
    import ltx_dit

    cfg = dit_config(c)
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


def make_inputs(dev: torch.device, seed: int = 7, c=CFG3):
    """Latent(s), text contexts, positions, keyframe mask and sigma schedule of the config."""
    import ltx_dit

    t = c["f"] * c["h"] * c["w"]
    gen = ltx_dit.PhiloxGenerator(seed, dev)
    inp = dict(latent=gen.randn(1, t, 128, dtype=torch.bfloat16),
               ctx=gen.randn(2, c["text"], c["cross_dim"], dtype=torch.bfloat16),
               pos=ltx_dit.video_positions(1, c["f"], c["h"], c["w"], 24.0, dev))
    kf = torch.zeros(1, t, 1, device=dev)
    kf[:, : c["h"] * c["w"]] = 1.0
    inp["kf"] = kf
    if c.get("loop"):
        inp["sigmas"] = ltx_dit.ltx2_scheduler_sigmas(c["loop"])
    else:
        inp["sigmas"] = torch.tensor([c["sigma"], c["sigma_next"]], dtype=torch.float32)
    if c["kind"] == "av":
        ta = c["audio_tokens"]
        inp["a_latent"] = gen.randn(1, ta, 128, dtype=torch.bfloat16)
        inp["a_ctx"] = gen.randn(2, c["audio_text"], c["audio_cross"], dtype=torch.bfloat16)
        inp["a_pos"] = ltx_dit.audio_positions(1, ta, dev)
    return inp


def run_ours(args, rank: int, world: int, dev: torch.device) -> dict | None:
    import _native as nat
    import ltx_dit

    c = CONFIGS[args.config]
    t = c["f"] * c["h"] * c["w"]
    model, cfg = build_model(dev, c=c)
    inp = make_inputs(dev, seed=7, c=c)
    latent, pos, kf, sigmas = inp["latent"], inp["pos"], inp["kf"], inp["sigmas"]
    cpos, cneg = inp["ctx"][:1], inp["ctx"][1:]
    n_sig = len(sigmas) - 1
    if c["kind"] == "av":
        a_lat, a_pos, a_ctx = inp["a_latent"], inp["a_pos"], inp["a_ctx"]
        if world > 1:
            import ltx_parallel

            pdn = ltx_parallel.ParallelDenoiser(model, cfg_split=args.cfg_split, exchange=args.exchange)
            layout = pdn.layout

            def step(lat, idx=0):
                return pdn.step_av(lat, a_lat, pos, a_pos, cpos, cneg, a_ctx[:1], a_ctx[1:], sigmas, idx % n_sig,
                                   c["cfg_scale"], v_keyframes_mask=kf)[0]
        else:
            layout = None

            def step(lat, idx=0):
                return ltx_dit.av_cfg_denoise_step(model, lat, a_lat, pos, a_pos, cpos, cneg, a_ctx[:1], a_ctx[1:],
                                                   sigmas, idx % n_sig, c["cfg_scale"], v_keyframes_mask=kf)[0]
    elif world > 1:
        import ltx_parallel

        pdn = ltx_parallel.ParallelDenoiser(model, cfg_split=args.cfg_split, exchange=args.exchange)
        layout = pdn.layout

        def step(lat, idx=0):
            return pdn.step(lat, pos, cpos, cneg, sigmas, idx % n_sig, c["cfg_scale"], keyframes_mask=kf)
    else:
        layout = None

        def step(lat, idx=0):
            return ltx_dit.cfg_denoise_step(model, lat, pos, cpos, cneg, sigmas, idx % n_sig, c["cfg_scale"],
                                            keyframes_mask=kf)[2]

    stream = torch.cuda.current_stream(dev)
    # warm-up (eager), then capture one step in a CUDA graph (single GPU)
    for _ in range(max(args.warmup, 1)):
        step(latent)
    torch.cuda.synchronize(dev)
    graph = None
    # a denoise loop (config 5) walks the schedule: every step has its own sigmas, so it
    # runs eagerly (a captured graph would replay one step's sigmas)
    if not args.no_graph and not c.get("loop"):
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
        lat = latent
        for k in range(args.steps):
            if graph is not None:
                graph.replay()
            elif c.get("loop"):
                lat = step(lat, k)
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
    for k in range(e2e_steps):
        lat_dev = host_in.to(dev, non_blocking=True)
        out = step(lat_dev, k)
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
    if world > 1:
        pdn.close()  # the peer-memory exchange buffers, on every rank
    torch.cuda.synchronize(dev)

    if rank != 0:
        return None
    peaks = load_peaks()
    # algorithmic FLOPs of the step as executed: 2MNK per GEMM and 4*B*H*Tq*Tk*d per
    # attention launch of the profiled step (config 3: equals step_flops())
    flops = sum((kernel_flops(k) or 0.0) * v["launches"] for k, v in kern.items())
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
        "config": workload_config(c),
        "execution": {"parallelism": "single GPU" if world == 1 else
                      f"cfg{layout.cfg} x sp{layout.sp} (Ulysses, exchange: "
                      f"{'NVLink peer memory in the q/k and attention kernels' if pdn.exchange_kind == 'peer' else 'NCCL all-to-all'})",
                      "cuda_graph": used_graph,
                      "step_flops": flops, "text_kv": "projected once, cached across denoise steps (the context "
                      "is constant); not counted in step_flops"},
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


def cpu_reference_setup(threads: int, num_layers: int | None = None):
    """Config-3 weights (bf16, N(0, 0.02), q/k RMSNorm gains +1, in the reference's
    parameter order) and inputs on the host for the CPU oracle."""
    import ltx_dit

    from oracle import ltx_oracle

    torch.set_num_threads(threads)
    c = CFG3
    cfg = ltx_dit.DiTConfig.video_only(num_layers=num_layers or c["num_layers"], heads=c["heads"],
                                       head_dim=c["head_dim"], cross_dim=c["cross_dim"])
    with torch.device("meta"):
        shapes = [(n, tuple(p.shape)) for n, p in ltx_dit.LTXModel(cfg).named_parameters()]
    g = torch.Generator().manual_seed(1)
    w = {}
    for name, shape in shapes:
        t = torch.randn(shape, generator=g, dtype=torch.bfloat16).mul_(0.02)
        if name.endswith(("q_norm.weight", "k_norm.weight")):
            t.add_(1.0)
        w[name] = t
    t = c["f"] * c["h"] * c["w"]
    latent = torch.randn(1, t, 128, generator=g).to(torch.bfloat16)
    ctx = torch.randn(2, c["text"], c["cross_dim"], generator=g).to(torch.bfloat16)
    pos = ltx_oracle.video_positions(1, c["f"], c["h"], c["w"], 24.0)
    kf = torch.zeros(1, t, 1)
    kf[:, : c["h"] * c["w"]] = 1.0
    sigmas = torch.tensor([c["sigma"], c["sigma_next"]])
    return cfg, w, (latent, pos, ctx[:1], ctx[1:], sigmas, kf)


def cpu_oracle_step(cfg, w, inputs) -> float:
    """One CFG denoise step (patchify, adaLN, every block, head, X0, CFG, Euler) of the
    CPU oracle; returns its wall time in seconds."""
    from oracle import ltx_oracle

    latent, pos, cpos, cneg, sigmas, kf = inputs
    t0 = time.perf_counter()
    with torch.inference_mode():
        ltx_oracle.cfg_denoise_step(w, cfg, latent, pos, cpos, cneg, sigmas, 0, CFG3["cfg_scale"], keyframes_mask=kf)
    return time.perf_counter() - t0


def cpu_full_steps(threads: int, warmup: int, steps: int, budget_s: float) -> dict:
    """The CPU oracle (the reference's PyTorch math, restated op for op) running whole
    config-3 CFG steps on `threads` host cores. Warm-up: `warmup` one-block samples
    (untimed; they start the thread pool and the allocator). Timed: whole 28-block steps,
    as many of the `steps` requested as fit in `budget_s` seconds by the warm-up's
    estimate (at least one)."""
    from dataclasses import replace

    cfg, w, inputs = cpu_reference_setup(threads)
    one_block = replace(cfg, num_layers=1)
    est = None
    for _ in range(max(1, warmup)):
        est = cpu_oracle_step(one_block, w, inputs) * cfg.num_layers
    n = int(max(1, min(steps, budget_s // max(est, 1e-3))))
    times = [cpu_oracle_step(cfg, w, inputs) for _ in range(n)]
    sec = sum(times) / n
    t = CFG3["f"] * CFG3["h"] * CFG3["w"]
    return {"value": 2 * t / sec, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{n} whole config-3 CFG step(s) ({cfg.num_layers} blocks, B=2, T={t}, bf16) of the CPU oracle, "
                      f"{sec:.2f} s each (steps/s {1 / sec:.5f}); warm-up {max(1, warmup)} one-block sample(s)",
            "steps_timed": n, "step_s": sec, "timed_s": sum(times)}


def cpu_one_block_sample(c, threads: int) -> dict:
    """Configs 4 and 5 are too slow for a whole step on the CPU: the CPU oracle runs the
    config's model with ONE block (patchify, adaLN, one block, head, and for config 5
    X0 + CFG + Euler), timed once after a small warm-up, and the time is multiplied by
    the number of blocks. Labelled extrapolated."""
    import ltx_dit

    from oracle import ltx_oracle

    torch.set_num_threads(threads)
    cfg = dit_config({**c, "num_layers": 1})
    with torch.device("meta"):
        shapes = [(n, tuple(p.shape)) for n, p in ltx_dit.LTXModel(cfg).named_parameters()]
    g = torch.Generator().manual_seed(1)
    w = {}
    for name, shape in shapes:
        x = torch.randn(shape, generator=g, dtype=torch.bfloat16).mul_(0.02)
        if name.endswith(("q_norm.weight", "k_norm.weight")):
            x.add_(1.0)
        w[name] = x
    t = c["f"] * c["h"] * c["w"]
    lat = torch.randn(1, t, 128, generator=g).to(torch.bfloat16)
    ctx = torch.randn(2, c["text"], c["cross_dim"], generator=g).to(torch.bfloat16)
    pos = ltx_oracle.video_positions(1, c["f"], c["h"], c["w"], 24.0)
    sig = torch.tensor([0.5, 0.25])

    def run(tv_pos, tv_lat, tv_ctx):
        with torch.inference_mode():
            if c["kind"] == "av":
                ta = c["audio_tokens"]
                s2 = torch.full((2,), 0.5)
                vid = ltx_oracle.Modality(latent=tv_lat.repeat(2, 1, 1), sigma=s2,
                                          timesteps=torch.full((2, tv_lat.shape[1], 1), 0.5),
                                          positions=tv_pos.repeat(2, 1, 1, 1), context=tv_ctx)
                aud = ltx_oracle.Modality(latent=torch.randn(2, ta, 128, generator=g).to(torch.bfloat16), sigma=s2,
                                          timesteps=torch.full((2, ta, 1), 0.5),
                                          positions=ltx_oracle.audio_positions(2, ta),
                                          context=torch.randn(2, c["audio_text"], c["audio_cross"],
                                                              generator=g).to(torch.bfloat16))
                ltx_oracle.forward(w, cfg, vid, aud)
            else:
                ltx_oracle.cfg_denoise_step(w, cfg, tv_lat, tv_pos, tv_ctx[:1], tv_ctx[1:], sig, 0, c["cfg_scale"])

    run(pos[:, :, :256], lat[:, :256], ctx)  # warm-up on 256 tokens
    t0 = time.perf_counter()
    run(pos, lat, ctx)
    sec = time.perf_counter() - t0
    step_sec = sec * c["num_layers"]
    return {"value": 2 * t / step_sec, "unit": UNIT, "cores": threads, "kind": "port", "extrapolated": True,
            "sample": f"one-block model of this config (B=2, T={t}, bf16) on the CPU oracle: {sec:.2f} s, "
                      f"multiplied by {c['num_layers']} blocks (extrapolated; patchify, adaLN and head counted "
                      f"{c['num_layers']} times)"}


def run_reference(args, rank: int, world: int) -> dict | None:
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    c = CONFIGS[args.config]
    if args.config == 3:
        cpu = cpu_full_steps(threads, args.warmup, args.steps, budget_s=90.0)
        n, sec = cpu.pop("steps_timed"), cpu.pop("step_s")
        cpu.pop("timed_s")
    else:
        cpu = cpu_one_block_sample(c, threads)
        n, sec = 1, 2 * c["f"] * c["h"] * c["w"] / cpu["value"]
    v = cpu["value"]
    return {"impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": world, "steps": n,
            "steps_requested": args.steps, "warmup": args.warmup, "ms_per_step": sec * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": workload_config(c),
            "execution": {"parallelism": f"CPU, {threads} host threads (rank 0 only)", "cuda_graph": False,
                          "step_flops": step_flops(text_kv_cached=False),
                          "text_kv": "recomputed every step, as the reference does",
                          "note": "steps = whole steps timed (as many of the requested ones as fit in 90 s); "
                                  "warm-up = one-block samples"},
            "cpu_baseline": cpu, "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


PROBES = {
    # name: (description, builder) -- one kernel at its config-3 shape
    "attention": "self-attention FMHA, B=2, H=32, T=6144, d=64 (q/k/v/gate read from the packed QKV buffer)",
    "attention128": "self-attention FMHA at config 4's video width: B=2, H=32, T=6144, d=128 (packed QKV buffer)",
    "attention_rank8": "self-attention of one rank at 8 GPUs (CFG2 x SP4): B=1, H=8, T=6144, d=64, units of the "
                       "partly filled last wave split over key ranges (packed QKV buffer)",
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
    "gpu_bar": "the reference's GPU libraries at the step's shapes on the same B200: torch SDPA (cuDNN and "
               "flash backends, the reference's cuDNN-first sdpa) against our attention at config 3 (d=64) and "
               "config 4 (d=128), and cuBLAS (F.linear) against our GEMMs at the five config-3 GEMM shapes",
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


def _time_ms(fn, warmup: int, steps: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def run_gpu_bar(args, dev: torch.device) -> dict:
    """Per-op comparison with the libraries the reference calls on a GPU (its sdpa tries
    cuDNN first, ltx_nn.py:15,22-26; its projections are nn.Linear, ltx_nn.py:188-192,
    244-245), same shapes, same process, CUDA events. Our GEMM rows use the plain bias
    epilogue (the step fuses more into some of them)."""
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel

    import _native as nat

    g = torch.Generator(device=dev).manual_seed(0)

    def rnd(*shape, scale=1.0):
        return (torch.randn(*shape, generator=g, device=dev) * scale).to(torch.bfloat16)

    w_, k_ = max(args.warmup, 3), max(args.steps, 10)
    peaks = load_peaks()
    rows = {}
    t = CFG3["f"] * CFG3["h"] * CFG3["w"]
    for name, heads, hd in (("attention cfg3 B=2 H=32 T=6144 d=64", 32, 64),
                            ("attention cfg4 B=2 H=32 T=6144 d=128", 32, 128)):
        d = heads * hd
        qkv = rnd(2 * t, 3 * d + heads)
        o = torch.empty(2 * t, d, device=dev, dtype=torch.bfloat16)
        flops = 4.0 * 2 * heads * t * t * hd
        ours = _time_ms(lambda: nat.attention(qkv[:, :d], qkv[:, d:2 * d], qkv[:, 2 * d:3 * d], o, 2, t, t, heads,
                                              hd, hd ** -0.5, qkv[:, 3 * d:]), w_, k_)
        ours_ng = _time_ms(lambda: nat.attention(qkv[:, :d], qkv[:, d:2 * d], qkv[:, 2 * d:3 * d], o, 2, t, t,
                                                 heads, hd, hd ** -0.5, None), w_, k_)
        # the reference's layout: (B, T, H, d) views transposed to (B, H, T, d)
        q4 = qkv[:, :d].reshape(2, t, heads, hd).transpose(1, 2)
        k4 = qkv[:, d:2 * d].reshape(2, t, heads, hd).transpose(1, 2)
        v4 = qkv[:, 2 * d:3 * d].reshape(2, t, heads, hd).transpose(1, 2)
        row = {"flops": flops, "ours_ms": ours, "ours_no_gate_ms": ours_ng}
        for bname, be in (("cudnn", SDPBackend.CUDNN_ATTENTION), ("flash", SDPBackend.FLASH_ATTENTION)):
            try:
                with sdpa_kernel([be]):
                    row[f"torch_{bname}_ms"] = _time_ms(lambda: F.scaled_dot_product_attention(q4, k4, v4), w_, k_)
            except RuntimeError as e:  # backend not available for this shape / build
                row[f"torch_{bname}_ms"] = None
                row[f"torch_{bname}_error"] = str(e).splitlines()[0][:160]
        rows[name] = row
    d = CFG3["heads"] * CFG3["head_dim"]
    m = 2 * t
    for name, n, k in (("qkv+gate", 3 * d + CFG3["heads"], d), ("attn out / text out", d, d),
                       ("text q+gate", d + CFG3["heads"], d), ("ffn in", 4 * d, d), ("ffn out", d, 4 * d)):
        a, wt, bias = rnd(m, k), rnd(n, k, scale=k ** -0.5), rnd(n)
        out = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
        epi = nat.epilogue(bias=bias)
        npad = (n + 7) // 8 * 8
        wp = torch.zeros(npad, k, device=dev, dtype=torch.bfloat16)
        wp[:n] = wt
        bp = torch.zeros(npad, device=dev, dtype=torch.bfloat16)
        bp[:n] = bias
        outp = torch.empty(m, npad, device=dev, dtype=torch.bfloat16)
        ours = _time_ms(lambda: nat.linear(a, wp, outp, nat.epilogue(bias=bp)), w_, k_) if npad != n else \
            _time_ms(lambda: nat.linear(a, wt, out, epi), w_, k_)
        cub = _time_ms(lambda: F.linear(a, wt, bias), w_, k_)
        rows[f"gemm {name} M={m} N={n} K={k}"] = {"flops": 2.0 * m * n * k, "ours_ms": ours, "torch_cublas_ms": cub}
    for r in rows.values():
        for key in list(r):
            if key.endswith("_ms") and r[key]:
                r[key.replace("_ms", "_TFLOPs")] = r["flops"] / (r[key] / 1e3) / 1e12
        lib = [v for kk, v in r.items() if kk.startswith("torch_") and kk.endswith("_ms") and v]
        r["best_library_over_ours"] = min(lib) / r["ours_ms"] if lib else None
    return {"probe": "gpu_bar", "what": PROBES["gpu_bar"], "peak_bf16_tflops": peaks["bf16_tflops"],
            "torch": torch.__version__, "cudnn": torch.backends.cudnn.version(), "ops": rows}


# Guidance of the reference's production run (run_all.py:43-44): video cfg 3, STG 1,
# rescale 0.7, modality 3; audio cfg 7, STG 1, rescale 0.7, modality 3. STG perturbs the
# self-attention of one block (block 29 of the 48-block model; block 14 of config 3's 28).
GUIDED_V = (3.0, 1.0, 0.7, 3.0)
GUIDED_A = (7.0, 1.0, 0.7, 3.0)


def run_guided(args, dev: torch.device) -> dict:
    """The production sampling step on one GPU: guided_denoise_step (one transformer call
    on the B = 4 guidance batch [cond, uncond, STG-perturbed, A<->V-isolated], X0 per pass,
    guidance with std rescale) and the Euler update per modality, as run_dit runs it. The
    step has host synchronisations (keep masks, per-sample timesteps), so it runs eagerly."""
    import _native as nat
    import ltx_dit

    c = CONFIGS[args.config]
    if c.get("loop"):
        raise SystemExit("--guided takes config 3 or 4")
    t = c["f"] * c["h"] * c["w"]
    model, cfg = build_model(dev, c=c)
    inp = make_inputs(dev, seed=7, c=c)
    stg_block = (29 if c["num_layers"] > 29 else c["num_layers"] // 2,)
    vp = ltx_dit.GuiderParams(*GUIDED_V, stg_blocks=stg_block)
    video = ltx_dit.LatentState(latent=inp["latent"], denoise_mask=torch.ones(1, t, 1, device=dev),
                                positions=inp["pos"], clean_latent=inp["latent"], keyframes_mask=inp["kf"])
    contexts = {"v_pos": inp["ctx"][:1], "v_neg": inp["ctx"][1:]}
    audio, ap = None, None
    if c["kind"] == "av":
        ta = c["audio_tokens"]
        audio = ltx_dit.LatentState(latent=inp["a_latent"], denoise_mask=torch.ones(1, ta, 1, device=dev),
                                    positions=inp["a_pos"], clean_latent=inp["a_latent"])
        contexts.update(a_pos=inp["a_ctx"][:1], a_neg=inp["a_ctx"][1:])
        ap = ltx_dit.GuiderParams(*GUIDED_A, stg_blocks=stg_block)
    sigmas = inp["sigmas"]

    def step():
        dv, da, _ = ltx_dit.guided_denoise_step(model, video, audio, contexts, sigmas[0], 0, vp, ap, cfg)
        nv = ltx_dit.euler_step(video.latent, dv, sigmas, 0)
        na = ltx_dit.euler_step(audio.latent, da, sigmas, 0) if audio is not None else None
        return nv, na

    stream = torch.cuda.current_stream(dev)
    for _ in range(max(args.warmup, 1)):
        step()
    torch.cuda.synchronize(dev)
    n0 = nat.launch_count()
    step()
    torch.cuda.synchronize(dev)
    launches_per_step = nat.launch_count() - n0
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(dev.index if dev.index is not None else 0) as clocks:
        ev0.record(stream)
        for _ in range(args.steps):
            step()
        ev1.record(stream)
        torch.cuda.synchronize(dev)
    ms_per_step = ev0.elapsed_time(ev1) / args.steps
    with nat.profile() as prof:
        step()
    kern = prof.summary()
    flops = sum((kernel_flops(k) or 0.0) * v["launches"] for k, v in kern.items())
    step_ms_instr = sum(v["total_ms"] for v in kern.values())
    peaks = load_peaks()
    peak = peaks.get("bf16_tflops_sustained", peaks["bf16_tflops"])
    dom_label, dom = max(kern.items(), key=lambda kv: kv[1]["total_ms"])
    dom_flops = kernel_flops(dom_label)
    achieved = dom_flops / (dom["avg_ms"] / 1e3) / 1e12 if dom_flops else None
    tokens = 4 * t  # the four guidance passes of one latent
    tflops = flops / (ms_per_step / 1e3) / 1e12
    workload = dict(workload_config(c))
    workload["workload"] = (f"production sampling step of {c['workload'].split(':')[0]}: run_dit's guided_denoise_step "
                            "(B = 4 guidance batch [cond, uncond, STG, A<->V-isolated], X0, guidance with std "
                            "rescale) + Euler per modality")
    workload["global_batch"] = 4
    workload["guidance"] = {"video": list(GUIDED_V) + [list(stg_block)],
                            "audio": (list(GUIDED_A) + [list(stg_block)]) if ap is not None else None}
    return {
        "metric": METRIC, "value": tokens / (ms_per_step / 1e3), "unit": "latent tokens/s (4 passes x T)",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": workload,
        "execution": {"parallelism": "single GPU", "cuda_graph": False, "step_flops": flops,
                      "note": "eager: the guided step synchronises with the host (keep masks, timesteps)"},
        "steps_per_s": 1e3 / ms_per_step, "step_tflops_per_gpu": tflops,
        "pct_bf16_peak": tflops / peaks["bf16_tflops"], "pct_bf16_peak_sustained": tflops / peak,
        "roofline": {"kernel": dom_label, "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": (achieved / peak) if achieved else None, "traffic": None,
                     "peak_source": f"{peaks['source']} bf16_tflops_sustained",
                     "avg_launch_ms": dom["avg_ms"], "share_of_step": dom["total_ms"] / step_ms_instr},
        "gpu_launches": launches_per_step * args.steps, "gpu_launches_per_step": launches_per_step,
        "kernels": {k: {"launches": v["launches"], "total_ms": round(v["total_ms"], 4),
                        "share": round(v["total_ms"] / step_ms_instr, 4)}
                    for k, v in sorted(kern.items(), key=lambda kv: -kv[1]["total_ms"])[:12]},
        "clocks": clocks.summary(),
        "cpu_baseline": None,
    }


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

    if args.probe in ("attention", "attention128", "attention_rank8"):
        hd = 128 if args.probe == "attention128" else 64
        # attention_rank8: what one rank of 8 attends over (CFG2 x SP4: 1 sample, 8 heads)
        nb, heads = (1, c["heads"] // 4) if args.probe == "attention_rank8" else (2, c["heads"])
        d = heads * hd
        qkv = rnd(nb * t, 3 * d + ((heads + 7) // 8) * 8)
        o = torch.empty(nb * t, d, device=dev, dtype=torch.bfloat16)
        fn = lambda: nat.attention(qkv[:, :d], qkv[:, d:2 * d], qkv[:, 2 * d:3 * d], o, nb, t, t, heads,  # noqa
                                   hd, hd ** -0.5, qkv[:, 3 * d:3 * d + heads])
        flops = 4.0 * nb * heads * t * t * hd
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
    ap.add_argument("--config", type=int, choices=sorted(CONFIGS), default=3,
                    help="BASELINE.json workload: 3 (default, the headline), 4 (audio-video, one GPU) or 5 "
                         "(27588-token denoise loop)")
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--guided", action="store_true",
                    help="one GPU: the production sampling step (B = 4 guidance batch, run_dit) instead of the CFG step")
    ap.add_argument("--cfg-split", type=int, choices=[1, 2], default=None,
                    help="N > 1: CFG groups (default 2: cond and uncond on separate ranks)")
    ap.add_argument("--exchange", choices=["auto", "peer", "nccl"], default="auto",
                    help="N > 1: the Ulysses exchange fused into the kernels over peer memory, or NCCL all-to-all")
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
    if args.probe == "gpu_bar":
        print(json.dumps(run_gpu_bar(args, dev)), flush=True)
        return
    if args.probe:
        print(json.dumps(run_probe(args, dev)), flush=True)
        return
    if args.guided:
        if world > 1:
            raise SystemExit("--guided runs on one GPU")
        print(json.dumps(run_guided(args, dev)), flush=True)
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
            if args.config == 3:
                cb = cpu_full_steps(os.cpu_count() or 1, warmup=1, steps=1, budget_s=0.0)
                for k in ("steps_timed", "step_s", "timed_s"):
                    cb.pop(k)
            else:
                cb = cpu_one_block_sample(CONFIGS[args.config], os.cpu_count() or 1)
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
