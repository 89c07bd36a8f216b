"""Parity at the benchmark configurations' full size: the native step against the CPU
oracle on the same seeded inputs, at the depth and token counts BASELINE configs 3-5 run.

  config 3  all 28 blocks, T = 6144 (16x16x24), B = 2 (CFG), text 128 x 4096, BF16:
            velocity and next latent of one CFG denoise step (cfg_denoise_step, the
            benchmarked call with the fused X0 + CFG + Euler head).
  config 4  the audio-video model at full width and real token counts: video 4096 wide
            (32x128 heads, FFN 16384), 6144 tokens, text 1024 x 3840; audio 2048 wide
            (32x64), 126 tokens, text 1024 x 2048; A<->V attention in every block; B = 2.
            8 of the 48 blocks (the 48-block weights are 37 GB, which the oracle would
            have to hold in host memory and run for minutes); velocities of both streams
            and the next latents after X0 + CFG + Euler.
  config 5  the config-3 model at T = 27588 (33x22x38) with 2 of its 28 blocks: one CFG step.

Weights are N(0, 0.02) drawn on the device by the Philox kernel (q/k RMSNorm gains
1 + N(0, 0.02)) and copied to the host for the oracle; latents and contexts come from a
seeded CPU generator.

The bar. Two BF16 implementations of the same arithmetic round at different points inside
the attention softmax and the GEMM reductions, and through 28 residual blocks those 1-ulp
differences accumulate to more than 1e-2 in rel-L2: the reference's own code run on the
GPU (cuBLAS + cuDNN SDPA) differs from the same code on the CPU by about as much as the
native step does. So each checked tensor must satisfy, against the CPU oracle:
  rel-L2(native, oracle CPU bf16) <= 1e-2, or <= 1.25 x rel-L2(oracle GPU bf16, oracle CPU
  bf16) -- no further from the reference than the reference is from itself on a B200;
and against exact arithmetic (the oracle in fp32 on the GPU, TF32 off, same bf16-valued
weights and inputs):
  rel-L2(native, fp32) <= 1.25 x max(rel-L2(oracle CPU bf16, fp32), rel-L2(oracle GPU bf16,
  fp32)) -- at least as accurate as the reference's BF16 path, up to 25 %.
Each test prints every measured distance."""

import pytest
import torch

import _native as nat
import ltx_dit
from model_fixtures import philox_model
from oracle import ltx_oracle

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
TOL = 1e-2


def rel_l2(a, b):
    a, b = a.detach().float().cpu(), b.detach().float().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def _dev_weights(host, dtype):
    return {k: v.to(DEV, dtype) for k, v in host.items()}


def _check(label, names, ours, ref_cpu, ref_gpu, truth):
    """Print and assert the two criteria of the module docstring for each tensor."""
    rows, bad = [], []
    for n, o, c, g, t in zip(names, ours, ref_cpu, ref_gpu, truth):
        e_ours, e_ref = rel_l2(o, c), rel_l2(g, c)
        a_ours, a_cpu, a_gpu = rel_l2(o, t), rel_l2(c, t), rel_l2(g, t)
        rows.append(f"  {n:18s} native-vs-oracle {e_ours:.3e}  oracleGPU-vs-oracle {e_ref:.3e}  "
                    f"native-vs-fp32 {a_ours:.3e}  oracle-vs-fp32 {a_cpu:.3e}  oracleGPU-vs-fp32 {a_gpu:.3e}")
        if not (e_ours <= TOL or e_ours <= 1.25 * e_ref):
            bad.append((n, "distance to the CPU oracle", e_ours, e_ref))
        if not a_ours <= 1.25 * max(a_cpu, a_gpu):
            bad.append((n, "accuracy vs fp32", a_ours, a_cpu, a_gpu))
    print(f"\n{label}\n" + "\n".join(rows))
    assert not bad, bad


def _oracle_runs(host, run):
    """run(weights, device, dtype) on: the CPU in bf16 (the reference's CPU path), the GPU
    in bf16 (the same code on cuBLAS / cuDNN) and the GPU in fp32 (TF32 off)."""
    torch.set_num_threads(max(1, torch.get_num_threads()))
    ref_cpu = run(host, torch.device("cpu"), torch.bfloat16)
    w = _dev_weights(host, torch.bfloat16)
    ref_gpu = run(w, DEV, torch.bfloat16)
    del w
    mm, cd = torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = torch.backends.cudnn.allow_tf32 = False
    try:
        w = _dev_weights(host, torch.float32)
        truth = run(w, DEV, torch.float32)
        del w
    finally:
        torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = mm, cd
    torch.cuda.empty_cache()
    return ref_cpu, ref_gpu, truth


def _time_ms(fn, reps=3):
    fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / reps


def _cfg_step_vs_oracle(cfg, f, h, w, text, cross_dim, seed, label, time_both=False):
    model, host = philox_model(cfg, seed)
    t = f * h * w
    g = torch.Generator().manual_seed(seed + 100)
    latent = torch.randn(1, t, 128, generator=g).to(torch.bfloat16)
    ctx = torch.randn(2, text, cross_dim, generator=g).to(torch.bfloat16)
    pos = ltx_oracle.video_positions(1, f, h, w, 24.0)
    kf = torch.zeros(1, t, 1)
    kf[:, : h * w] = 1.0
    sigmas = torch.tensor([0.5, 0.25])
    args = (latent.to(DEV), pos.to(DEV), ctx[:1].to(DEV), ctx[1:].to(DEV), sigmas, 0, 3.0)
    ours = ltx_dit.cfg_denoise_step(model, *args, keyframes_mask=kf.to(DEV))
    torch.cuda.synchronize()
    assert nat.device_error_flags() == 0
    ours = [o.cpu() for o in ours]
    t_native = _time_ms(lambda: ltx_dit.cfg_denoise_step(model, *args, keyframes_mask=kf.to(DEV))) \
        if time_both else None
    del model
    torch.cuda.empty_cache()

    def run(wt, dev, dt):
        out = ltx_oracle.cfg_denoise_step(wt, cfg, latent.to(dev, dt), pos.to(dev), ctx[:1].to(dev, dt),
                                          ctx[1:].to(dev, dt), sigmas, 0, 3.0, keyframes_mask=kf.to(dev))
        return [o.cpu() for o in out]

    ref_cpu, ref_gpu, truth = _oracle_runs(host, run)
    _check(label, ["velocity", "denoised", "next latent"], ours, ref_cpu, ref_gpu, truth)
    if time_both:
        # the GPU bar: the reference's module (restated op for op) on cuBLAS + cuDNN SDPA,
        # eager, against the native step, eager (no CUDA graph on either side)
        wdev = _dev_weights(host, torch.bfloat16)
        t_ref = _time_ms(lambda: run(wdev, DEV, torch.bfloat16))
        print(f"  step time on this B200 (eager): native {t_native:.1f} ms, reference module on cuBLAS/cuDNN "
              f"{t_ref:.1f} ms ({t_ref / t_native:.2f}x)")
        assert t_native < t_ref


def test_config3_all_28_blocks_cfg_step_matches_oracle():
    """BASELINE config 3 exactly as benchmarked: 28 blocks, D=2048, 32x64, FFN 8192,
    T=6144, text 128x4096, sigma 0.5 -> 0.25, CFG 3, keyframe mask on the first frame."""
    cfg = ltx_dit.DiTConfig.video_only(num_layers=28, heads=32, head_dim=64, cross_dim=4096)
    _cfg_step_vs_oracle(cfg, 16, 16, 24, 128, 4096, seed=11, label="config 3, 28 blocks, T=6144", time_both=True)


def test_config5_tokens_two_blocks_cfg_step_matches_oracle():
    """BASELINE config 5's latent, 1216x704x257 -> 33x22x38 = 27588 tokens, through 2 of
    the config-3 model's 28 blocks (self-attention over all 27588 tokens)."""
    cfg = ltx_dit.DiTConfig.video_only(num_layers=2, heads=32, head_dim=64, cross_dim=4096)
    _cfg_step_vs_oracle(cfg, 33, 22, 38, 128, 4096, seed=12, label="config 5 tokens, 2 blocks, T=27588")


def test_config4_full_width_av_eight_blocks_matches_oracle():
    """BASELINE config 4's audio-video model at full width and token counts with 8 of
    its 48 blocks: forward of the CFG batch [cond, uncond] for both streams, then X0 +
    CFG (scale 3) + Euler (sigma 0.5 -> 0.25) per stream on the native kernels."""
    cfg = ltx_dit.DiTConfig(num_layers=8, video_cross_dim=3840, cross_attention_adaln=False)
    model, host = philox_model(cfg, seed=13)
    g = torch.Generator().manual_seed(113)
    f, h, w = 16, 16, 24
    tv, ta, s = f * h * w, 126, 1024
    sig = torch.full((2,), 0.5)
    v_lat = torch.randn(1, tv, 128, generator=g).to(torch.bfloat16)
    a_lat = torch.randn(1, ta, 128, generator=g).to(torch.bfloat16)
    vid = dict(latent=v_lat.repeat(2, 1, 1), sigma=sig, timesteps=torch.full((2, tv, 1), 0.5),
               positions=ltx_oracle.video_positions(2, f, h, w, 24.0),
               context=torch.randn(2, s, 3840, generator=g).to(torch.bfloat16))
    aud = dict(latent=a_lat.repeat(2, 1, 1), sigma=sig, timesteps=torch.full((2, ta, 1), 0.5),
               positions=ltx_oracle.audio_positions(2, ta),
               context=torch.randn(2, s, 2048, generator=g).to(torch.bfloat16))
    sigmas = torch.tensor([0.5, 0.25])
    p = ltx_dit.GuiderParams(cfg_scale=3.0, stg_scale=0.0, rescale_scale=0.0, modality_scale=1.0, stg_blocks=())

    def native_next(lat, vel, ts):
        x0 = torch.empty_like(vel)
        nat.x0(lat.to(DEV).contiguous(), vel.contiguous(), ts.to(DEV).reshape(-1).contiguous(), x0)
        c, u = x0.chunk(2)
        den = ltx_dit.guide(c, u, c, c, p)
        return ltx_dit.euler_step(lat[:1].to(DEV), den, sigmas, 0)

    vx, ax = model(ltx_dit.Modality(**{k: v.to(DEV) for k, v in vid.items()}),
                   ltx_dit.Modality(**{k: v.to(DEV) for k, v in aud.items()}), None)
    v_next = native_next(vid["latent"], vx, vid["timesteps"])
    a_next = native_next(aud["latent"], ax, aud["timesteps"])
    # the fused audio-video step (X0 + CFG + Euler in both heads' proj_out epilogues) is
    # the same arithmetic: identical next latents
    fv, fa = ltx_dit.av_cfg_denoise_step(model, v_lat.to(DEV), a_lat.to(DEV), vid["positions"][:1].to(DEV),
                                         aud["positions"][:1].to(DEV), vid["context"][:1].to(DEV),
                                         vid["context"][1:].to(DEV), aud["context"][:1].to(DEV),
                                         aud["context"][1:].to(DEV), sigmas, 0, 3.0)
    torch.cuda.synchronize()
    assert nat.device_error_flags() == 0
    assert torch.equal(fv, v_next) and torch.equal(fa, a_next)
    ours = [vx.cpu(), ax.cpu(), v_next.cpu(), a_next.cpu()]
    del model
    torch.cuda.empty_cache()

    def run(wt, dev, dt):
        def mv(d):
            return ltx_oracle.Modality(**{k: (v.to(dev, dt) if k in ("latent", "context") else v.to(dev))
                                         for k, v in d.items()})

        def nxt(lat, vel, ts):
            x0 = (lat.float() - vel.float() * ts.float()).to(vel.dtype)
            den = ltx_oracle.guide_cfg(x0[0:1], x0[1:2], 3.0)
            return ltx_oracle.euler_step(lat[:1], den, sigmas, 0)

        mvid, maud = mv(vid), mv(aud)
        rvx, rax = ltx_oracle.forward(wt, cfg, mvid, maud)
        return [rvx.cpu(), rax.cpu(), nxt(mvid.latent, rvx, mvid.timesteps).cpu(),
                nxt(maud.latent, rax, maud.timesteps).cpu()]

    ref_cpu, ref_gpu, truth = _oracle_runs(host, run)
    _check("config 4 width and tokens, 8 blocks", ["video velocity", "audio velocity", "video next latent",
                                                   "audio next latent"], ours, ref_cpu, ref_gpu, truth)
