"""Model-level parity on the B200: the drop-in LTXModel / cfg_denoise_step (all native
kernels) against the reference's golden outputs and the CPU oracle on the same seeded
inputs. Tolerances (relative L2): 1e-4 in FP32 mode, 1e-2 in BF16."""

import dataclasses

import pytest
import torch

import _native as nat
import golden_cases as gc
import ltx_dit
from oracle import ltx_oracle

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda")
TOL = {"float32": 1e-4, "bfloat16": 1e-2}


def rel_l2(a, b):
    a, b = a.detach().float().cpu(), b.detach().float().cpu()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def _cfg(rec):
    return ltx_dit.DiTConfig(**{k: (tuple(v) if isinstance(v, list) else v) for k, v in rec["config"].items()})


def _model(rec, dtype):
    cfg = _cfg(rec)
    model = ltx_dit.LTXModel(cfg)
    sd = ltx_oracle.synthetic_state_dict(rec["param_shapes"], rec["weight_seed"], dtype=torch.float32)
    model.load_state_dict(sd)
    return model.to(DEV, dtype).eval(), cfg


def _mod(d, dtype):
    if d is None:
        return None
    t = {k: (v.to(DEV) if torch.is_tensor(v) else v) for k, v in d.items()}
    t["latent"] = t["latent"].to(dtype)
    t["context"] = t["context"].to(dtype)
    return ltx_dit.Modality(**t)


@pytest.mark.parametrize("case", gc.CASES)
def test_forward_matches_reference_golden(case):
    rec = gc.load(case)
    dtype = getattr(torch, rec["dtype"])
    model, _ = _model(rec, dtype)
    video = _mod(rec["video"], dtype)
    audio = _mod(rec["audio"], dtype)
    vx, ax = model(video, audio, None)
    torch.cuda.synchronize()
    assert nat.device_error_flags() == 0
    assert rel_l2(vx, rec["vx"]) < TOL[rec["dtype"]], rel_l2(vx, rec["vx"])
    if rec["ax"] is not None:
        assert rel_l2(ax, rec["ax"]) < TOL[rec["dtype"]], rel_l2(ax, rec["ax"])


@pytest.mark.parametrize("case", ["tiny_video_float32", "tiny_video_bfloat16"])
@pytest.mark.parametrize("fused", [True, False])
def test_cfg_steps_match_reference_golden(case, fused):
    rec = gc.load(case)
    dtype = getattr(torch, rec["dtype"])
    if fused is False and dtype == torch.float32:
        pytest.skip("fp32 always runs the projection then the element-wise update")
    model, _ = _model(rec, dtype)
    st = rec["steps"]
    for idx, r in enumerate(st["records"]):
        vel, den, nxt = ltx_dit.cfg_denoise_step(
            model, r["latent_in"].to(DEV, dtype), st["positions"].to(DEV), st["context_pos"].to(DEV, dtype),
            st["context_neg"].to(DEV, dtype), st["sigmas"], idx, st["cfg_scale"],
            keyframes_mask=st["keyframes_mask"].to(DEV), fused_head=fused)
        tol = TOL[rec["dtype"]]
        assert rel_l2(vel, r["velocity"]) < tol
        assert rel_l2(den, r["denoised"]) < tol
        assert rel_l2(nxt, r["latent_out"]) < tol


def _state(d, dtype):
    t = {k: (v.to(DEV) if torch.is_tensor(v) else v) for k, v in d.items()}
    t["latent"] = t["latent"].to(dtype)
    return ltx_dit.LatentState(**t)


@pytest.mark.parametrize("case", gc.GUIDED_CASES)
def test_guided_steps_match_reference_golden(case):
    """Full guidance (cond / uncond / STG-perturbed / modality-isolated passes in one B=4
    forward, std rescale) on the tiny AV model with a conditioned first frame: every
    pass's x0, the blended x0 and the Euler-updated latents of two steps against the
    reference; then run_dit over the same schedule."""
    rec = gc.load_guided(case)
    dtype = getattr(torch, rec["dtype"])
    tol = TOL[rec["dtype"]]
    model, cfg = _model(rec, dtype)
    vp, ap = ltx_dit.GuiderParams(*rec["v_params"]), ltx_dit.GuiderParams(*rec["a_params"])
    ctx = {k: v.to(DEV, dtype) for k, v in rec["contexts"].items()}
    sig = rec["sigmas"].to(DEV)
    vs0, as0 = _state(rec["video_state"], dtype), _state(rec["audio_state"], dtype)
    vs, aus = vs0, as0
    for idx, ref in enumerate(rec["steps"]):
        dv, da, passes = ltx_dit.guided_denoise_step(model, vs, aus, ctx, sig[idx], idx, vp, ap, cfg)
        torch.cuda.synchronize()
        assert nat.device_error_flags() == 0
        for name in ("cond", "uncond", "ptb", "mod"):
            assert rel_l2(passes[name][0], ref["passes"][name][0]) < tol, (idx, name, "video")
            assert rel_l2(passes[name][1], ref["passes"][name][1]) < tol, (idx, name, "audio")
        # the blend weights pass differences by up to 1 + (cfg-1) + stg + (mod-1) (= 10 for
        # the audio parameters), so the blended x0 gets that factor on top of the per-pass
        # tolerance in BF16; the guidance arithmetic itself is checked exactly below
        blend_tol = tol if rec["dtype"] == "float32" else 3 * tol
        assert rel_l2(dv, ref["denoised_video"]) < blend_tol
        assert rel_l2(da, ref["denoised_audio"]) < blend_tol
        for got, par, k in ((dv, vp, 0), (da, ap, 1)):
            mine = ltx_oracle.guide(*[passes[p][k].cpu() for p in ("cond", "uncond", "ptb", "mod")],
                                    par.cfg_scale, par.stg_scale, par.rescale_scale, par.modality_scale)
            assert rel_l2(got, mine) < (1e-6 if rec["dtype"] == "float32" else 4e-3)
        vs = dataclasses.replace(vs, latent=ltx_dit.euler_step(vs.latent, dv, sig, idx))
        aus = dataclasses.replace(aus, latent=ltx_dit.euler_step(aus.latent, da, sig, idx))
        assert rel_l2(vs.latent, ref["video_latent"]) < tol
        assert rel_l2(aus.latent, ref["audio_latent"]) < tol
    lv, la = ltx_dit.run_dit(model, cfg, ctx, vs0, as0, sig, vp, ap)
    assert torch.equal(lv, vs.latent) and torch.equal(la, aus.latent)


def _config1(num_layers=8):
    return ltx_dit.DiTConfig.video_only(num_layers=num_layers, heads=32, head_dim=64, cross_dim=4096)


def _synthetic(cfg, dtype, seed=1):
    with torch.device("meta"):
        shapes = [(n, tuple(p.shape)) for n, p in ltx_dit.LTXModel(cfg).named_parameters()]
    sd = ltx_oracle.synthetic_state_dict(shapes, seed, dtype=torch.float32)
    model = ltx_dit.LTXModel(cfg)
    model.load_state_dict(sd)
    return model.to(DEV, dtype).eval(), sd


def test_config1_fp32_full_loop_matches_oracle_every_step():
    """8 blocks, D=2048, 32x64 heads, FFN 8192, text 128x4096, latent
    128 x 5x8x12 = 480 tokens, CFG 3, 8 Euler steps sigma linspace(1, 0, 9), weights
    N(0, 0.02) seed 1, Philox noise seed 0, FP32. Each step is checked against the oracle
    started from the same latent (rel-L2 <= 1e-4 for velocity and latent)."""
    cfg = _config1()
    model, sd = _synthetic(cfg, torch.float32)
    f, h, w = 5, 8, 12
    t = f * h * w
    gen = ltx_dit.PhiloxGenerator(0, DEV)
    latent = gen.randn(1, t, 128, dtype=torch.float32)
    g = torch.Generator().manual_seed(1234)
    ctx = torch.randn(2, 128, 4096, generator=g)
    pos = ltx_oracle.video_positions(1, f, h, w, 24.0)
    sigmas = torch.linspace(1.0, 0.0, 9)
    torch.set_num_threads(max(1, torch.get_num_threads()))
    for idx in range(8):
        vel, den, nxt = ltx_dit.cfg_denoise_step(model, latent, pos.to(DEV), ctx[:1].to(DEV), ctx[1:].to(DEV),
                                                 sigmas, idx, 3.0)
        rvel, rden, rnxt = ltx_oracle.cfg_denoise_step(sd, cfg, latent.cpu(), pos, ctx[:1], ctx[1:], sigmas, idx, 3.0)
        assert rel_l2(vel, rvel) < 1e-4, (idx, rel_l2(vel, rvel))
        assert rel_l2(nxt, rnxt) < 1e-4, (idx, rel_l2(nxt, rnxt))
        latent = nxt


@pytest.mark.parametrize("t_shape", [(4, 16, 24), (24, 16, 16)])
def test_bf16_two_blocks_at_benchmark_width_matches_oracle(t_shape):
    """BASELINE config 3 geometry (D=2048, 32x64, FFN 8192, text 128x4096, sigma 0.5, CFG
    batch 2) with 2 blocks so the CPU oracle stays fast; the second shape is the full
    6144-token latent."""
    cfg = _config1(num_layers=2)
    model, sd = _synthetic(cfg, torch.bfloat16, seed=3)
    f, h, w = t_shape
    t = f * h * w
    g = torch.Generator().manual_seed(5)
    latent = torch.randn(1, t, 128, generator=g).to(torch.bfloat16)
    ctx = torch.randn(2, 128, 4096, generator=g).to(torch.bfloat16)
    pos = ltx_oracle.video_positions(1, f, h, w, 24.0)
    sigmas = torch.tensor([0.5, 0.25])
    vel, den, nxt = ltx_dit.cfg_denoise_step(model, latent.to(DEV), pos.to(DEV), ctx[:1].to(DEV), ctx[1:].to(DEV),
                                             sigmas, 0, 3.0)
    wb = {k: v.to(torch.bfloat16) for k, v in sd.items()}
    rvel, rden, rnxt = ltx_oracle.cfg_denoise_step(wb, cfg, latent, pos, ctx[:1], ctx[1:], sigmas, 0, 3.0)
    assert rel_l2(vel, rvel) < 1e-2, rel_l2(vel, rvel)
    assert rel_l2(nxt, rnxt) < 1e-2, rel_l2(nxt, rnxt)


def test_bf16_config4_width_av_two_blocks_matches_oracle():
    """BASELINE config 4 geometry with 2 of its 48 blocks: video D=4096 (32x128 heads, FFN
    16384, head_dim 128 attention), audio D=2048 (32x64), A<->V attention every block,
    text contexts 3840 (video) and 2048 (audio) wide, cross-adaLN off, BF16, CFG batch 2.
    Token counts are cut (192 video, 25 audio, 64 text) so the CPU oracle stays fast."""
    cfg = ltx_dit.DiTConfig(num_layers=2, video_cross_dim=3840, cross_attention_adaln=False)
    model, sd = _synthetic(cfg, torch.bfloat16, seed=4)
    wb = {k: v.to(torch.bfloat16) for k, v in sd.items()}
    g = torch.Generator().manual_seed(9)
    f, h, w = 2, 8, 12
    tv, ta, s = f * h * w, 25, 64
    sig = torch.full((2,), 0.5)
    vid = dict(latent=torch.randn(2, tv, 128, generator=g).to(torch.bfloat16), sigma=sig,
               timesteps=torch.full((2, tv, 1), 0.5), positions=ltx_oracle.video_positions(2, f, h, w, 24.0),
               context=torch.randn(2, s, 3840, generator=g).to(torch.bfloat16))
    aud = dict(latent=torch.randn(2, ta, 128, generator=g).to(torch.bfloat16), sigma=sig,
               timesteps=torch.full((2, ta, 1), 0.5), positions=ltx_oracle.audio_positions(2, ta),
               context=torch.randn(2, s, 2048, generator=g).to(torch.bfloat16))
    vx, ax = model(ltx_dit.Modality(**{k: v.to(DEV) for k, v in vid.items()}),
                   ltx_dit.Modality(**{k: v.to(DEV) for k, v in aud.items()}), None)
    torch.cuda.synchronize()
    assert nat.device_error_flags() == 0
    rvx, rax = ltx_oracle.forward(wb, cfg, ltx_oracle.Modality(**vid), ltx_oracle.Modality(**aud))
    assert rel_l2(vx, rvx) < 1e-2, rel_l2(vx, rvx)
    assert rel_l2(ax, rax) < 1e-2, rel_l2(ax, rax)


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_text_connector_matches_reference_golden(dtype):
    """The text connector on the native kernels against the reference's
    Embeddings1DConnector outputs (padded tokens replaced by learnable registers)."""
    import ltx_te

    rec = torch.load(gc.GOLDEN / f"connector_{dtype}.pt", weights_only=False)
    dt = getattr(torch, dtype)
    conn = ltx_te.Embeddings1DConnector(**rec["config"])
    conn.load_state_dict(ltx_oracle.synthetic_state_dict(rec["param_shapes"], rec["weight_seed"], dtype=torch.float32))
    conn = conn.to(DEV, dt).eval()
    out, mask = conn(rec["hidden"].to(DEV), rec["mask"].to(DEV))
    torch.cuda.synchronize()
    assert nat.device_error_flags() == 0
    assert rel_l2(out, rec["out"]) < TOL[dtype], rel_l2(out, rec["out"])
    assert torch.equal(mask.cpu(), rec["out_mask"])


def test_create_noised_states_bit_exact_vs_torch():
    vs, as_ = ltx_dit.create_noised_states(1, 65, 512, 768, 24.0, 10, DEV, torch.bfloat16)
    g = torch.Generator(device=DEV).manual_seed(10)
    rv = torch.randn(1, vs.latent.shape[1], 128, device=DEV, dtype=torch.bfloat16, generator=g)
    ra = torch.randn(1, as_.latent.shape[1], 128, device=DEV, dtype=torch.bfloat16, generator=g)
    assert torch.equal(vs.latent, rv) and torch.equal(as_.latent, ra)


def test_guide_and_euler_kernels_match_oracle():
    g = torch.Generator().manual_seed(6)
    c, u = torch.randn(1, 50, 128, generator=g), torch.randn(1, 50, 128, generator=g)
    p = ltx_dit.GuiderParams(cfg_scale=3.0, stg_scale=0.0, rescale_scale=0.0, modality_scale=1.0, stg_blocks=())
    out = ltx_dit.guide(c.to(DEV), u.to(DEV), c.to(DEV), c.to(DEV), p)
    assert torch.equal(out.cpu(), ltx_oracle.guide_cfg(c, u, 3.0))
    sig = torch.linspace(1.0, 0.0, 9)
    e = ltx_dit.euler_step(u.to(DEV), out, sig, 3)
    assert torch.equal(e.cpu(), ltx_oracle.euler_step(u, out.cpu(), sig, 3))
