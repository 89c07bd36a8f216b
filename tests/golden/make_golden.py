"""Generate the golden fixtures in tests/golden/ from the reference implementation.

The reference (lipaul/ltx-nv, standalone/ltx_dit.py + ltx_nn.py) is pure PyTorch and is
importable in the build container, so this script runs it on CPU for small
configurations and records inputs and outputs. The fixtures pin the CPU oracle
(oracle/ltx_oracle.py, oracle/philox_oracle.c); the GPU parity tests then compare the
sm_100a kernels with that oracle. The reference is not needed at test time.

    python tests/golden/make_golden.py --reference /path/to/lipaul/ltx-nv [--only KIND]

Fixtures written:
  philox_m1.npz       the reference's own golden noise (cuda_c_standalone/artifacts/
                      m1_philox: torch.randn seed 10, bf16, video [1,3456,128] then audio
                      [1,68,128], RTX 6000 Ada launch grid): the audio tensor and the
                      first 65536 video values as uint16 bits, and a SHA-256 of all
                      video bits.
  dit_<case>.pt       config, parameter (name, shape) list, weight seed, inputs and the
                      reference's outputs for LTXModel.forward and for two CFG denoise
                      steps (X0 + guide + Euler).
  sched.pt            ltx2_scheduler_sigmas(30), video/audio positions.
  guide.pt            guide() with and without the std rescale on seeded x0 predictions.
  connector_<dtype>.pt  the text connector (Embeddings1DConnector) on seeded inputs.
  ckpt_keys.json      dev-checkpoint key -> parameter name as the reference's
                      load_transformer maps it (tiny AV model), with parameter shapes.
  guided_tiny_av_<dtype>.pt  two steps of guided_denoise_step (cond / uncond / STG /
                      modality passes, rescale) + Euler on the tiny AV model.
  vae_tiny_<dtype>.pt the video VAE decoder (ConvVideoDecoder) with every block kind on
                      a seeded (2, 128, 3, 4, 6) latent (oracle/vae_oracle.py weights).

Weights are N(0, 0.02) from numpy's PCG64 (platform independent) in the reference's
named_parameters() order, q/k RMSNorm gains offset by +1 (oracle.synthetic_state_dict).
"""

from __future__ import annotations

import argparse
import dataclasses
import hashlib
import os
import sys
from pathlib import Path

import numpy as np
import torch

ROOT = Path(__file__).resolve().parents[2]
OUT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from oracle import ltx_oracle, vae_oracle  # noqa: E402


def _import_reference(ref_root: Path):
    sys.path.insert(0, str(ref_root / "standalone"))
    import ltx_dit  # noqa: F401

    return sys.modules["ltx_dit"]


def rng_normal(shape, seed, scale=1.0, dtype=torch.float32):
    g = np.random.default_rng(seed)
    return torch.from_numpy(g.standard_normal(shape, dtype=np.float32) * np.float32(scale)).to(dtype)


CASES = {
    # video-only benchmark geometry in miniature: context width != hidden, no cross-adaLN
    # (the audio dims are those of DiTConfig.video_only: a stream that never runs)
    "tiny_video": dict(num_layers=2, video_heads=4, video_head_dim=64, video_cross_dim=384, audio_heads=2,
                       audio_head_dim=32, audio_cross_dim=64, cross_attention_adaln=False),
    # the real LTX-2.5 AV structure (cross-adaLN, A<->V attention) in miniature
    "tiny_av": dict(num_layers=2, video_heads=4, video_head_dim=64, video_cross_dim=256, audio_heads=2,
                    audio_head_dim=64, audio_cross_dim=128, cross_attention_adaln=True),
}
FRAMES = (2, 3, 4)  # latent f, h, w -> 24 video tokens
AUDIO_T = 5
TEXT_S = 8
WEIGHT_SEED = 1


def build_reference_model(ld, cfg, dtype):
    torch.manual_seed(0)
    model = ld.LTXModel(cfg)
    shapes = [(n, tuple(p.shape)) for n, p in model.named_parameters()]
    sd = ltx_oracle.synthetic_state_dict(shapes, WEIGHT_SEED, dtype=torch.float32)
    model.load_state_dict(sd)
    return model.to(dtype).eval(), shapes


def patch_context_view(ld):
    """The survey's adapter for context width != hidden: undo the view at ltx_dit.py:157."""
    orig = ld.ArgsPreprocessor.prepare

    def prepare(self, modality, cross):
        ctx = modality.context
        b = ctx.shape[0]
        hidden = self.m.cfg.audio_dim if self.stream == "audio" else self.m.cfg.video_dim
        if ctx.numel() % (b * hidden) != 0:
            raise ValueError("context size not viewable; pick another fixture size")
        args = orig(self, modality, cross)
        return dataclasses.replace(args, context=ctx)

    ld.ArgsPreprocessor.prepare = prepare
    return orig


def video_inputs(ld, cfg, dtype, batch, sigma, seed):
    f, h, w = FRAMES
    t = f * h * w
    latent = rng_normal((batch, t, cfg.video_in), seed).to(dtype)
    positions = ld.video_positions(batch, f, h, w, 24.0, "cpu")
    kf = torch.zeros(batch, t, 1)
    kf[:, : h * w] = 1.0
    ctx = rng_normal((batch, TEXT_S, cfg.video_cross_dim), seed + 1).to(dtype)
    sig = torch.full((batch,), float(sigma), dtype=torch.float32)
    ts = torch.ones(batch, t, 1) * sig.view(batch, 1, 1)
    return ld.Modality(latent=latent, sigma=sig, timesteps=ts, positions=positions, context=ctx, keyframes_mask=kf)


def audio_inputs(ld, cfg, dtype, batch, sigma, seed, enabled=True, t=AUDIO_T):
    latent = rng_normal((batch, t, cfg.audio_in), seed + 2).to(dtype)
    positions = ld.audio_positions(batch, t, "cpu")
    ctx = rng_normal((batch, TEXT_S, cfg.audio_cross_dim), seed + 3).to(dtype)
    sig = torch.full((batch,), float(sigma), dtype=torch.float32)
    ts = torch.ones(batch, t, 1) * sig.view(batch, 1, 1)
    return ld.Modality(latent=latent, sigma=sig, timesteps=ts, positions=positions, context=ctx, enabled=enabled)


def modality_dict(m):
    return {k: v for k, v in dataclasses.asdict(m).items()}


@torch.inference_mode()
def make_case(ld, name, overrides, dtype):
    cfg = ld.DiTConfig(**overrides)
    model, shapes = build_reference_model(ld, cfg, dtype)
    video_only = name == "tiny_video"
    batch = 2
    video = video_inputs(ld, cfg, dtype, batch, 0.7, seed=100)
    if video_only:
        # Disabled 1-token audio stream + zero A2V row (ltx_dit.py:253-257, 286).
        audio = audio_inputs(ld, cfg, dtype, batch, 0.7, seed=100, enabled=False, t=1)
        pert = torch.ones(4, cfg.num_layers, batch, dtype=dtype)
        pert[2] = 0
    else:
        audio = audio_inputs(ld, cfg, dtype, batch, 0.7, seed=100)
        pert = None
    vx, ax = model(video, audio, pert)
    rec = {
        "case": name,
        "dtype": str(dtype).replace("torch.", ""),
        "config": dataclasses.asdict(cfg),
        "param_shapes": shapes,
        "weight_seed": WEIGHT_SEED,
        "video": modality_dict(video),
        "audio": None if video_only else modality_dict(audio),
        "vx": vx.clone(),
        "ax": None if video_only else ax.clone(),
    }
    # Two CFG denoise steps of the video stream (B=2 forward, X0, guide, Euler) on a
    # (1, T, C) latent with sigmas linspace(1, 0, 9) (BASELINE config 1's schedule).
    if video_only:
        sigmas = torch.linspace(1.0, 0.0, 9)
        latent = video.latent[:1].clone()
        ctx_pos, ctx_neg = video.context[:1].clone(), video.context[1:].clone()
        params = ld.GuiderParams(cfg_scale=3.0, stg_scale=0.0, rescale_scale=0.0, modality_scale=1.0, stg_blocks=())
        steps = []
        for idx in range(2):
            sig = sigmas[idx]
            sig2 = sig.expand(2)
            lat2 = latent.repeat(2, 1, 1)
            ts = torch.ones(2, latent.shape[1], 1) * sig2.view(2, 1, 1)
            vm = ld.Modality(latent=lat2, sigma=sig2, timesteps=ts, positions=video.positions,
                             context=torch.cat([ctx_pos, ctx_neg]), keyframes_mask=video.keyframes_mask)
            am = audio_inputs(ld, cfg, dtype, 2, float(sig), seed=100, enabled=False, t=1)
            vel, _ = model(vm, am, pert)
            x0 = (lat2.float() - vel.float() * ts.float()).to(vel.dtype)
            den = ld.guide(x0[0:1], x0[1:2], x0[0:1], x0[0:1], params)
            nxt = ld.euler_step(latent, den, sigmas, idx)
            steps.append({"latent_in": latent.clone(), "velocity": vel.clone(), "denoised": den.clone(),
                          "latent_out": nxt.clone()})
            latent = nxt
        rec["steps"] = {"sigmas": sigmas, "cfg_scale": 3.0, "context_pos": ctx_pos, "context_neg": ctx_neg,
                        "positions": video.positions[:1].clone(), "keyframes_mask": video.keyframes_mask[:1].clone(),
                        "records": steps}
    return rec


def make_philox(ref_root: Path):
    art = ref_root / "cuda_c_standalone" / "artifacts" / "m1_philox"
    v = np.fromfile(art / "video_noise.bin", dtype=np.uint16)
    a = np.fromfile(art / "audio_noise.bin", dtype=np.uint16)
    assert v.size == 3456 * 128 and a.size == 68 * 128
    np.savez(OUT / "philox_m1.npz", video_prefix=v[:65536], audio=a, video_numel=np.int64(v.size),
             video_sha256=np.frombuffer(hashlib.sha256(v.tobytes()).digest(), dtype=np.uint8), seed=np.int64(10),
             ada_grid_video=np.int64(852), ada_grid_audio=np.int64(34))


def make_sched(ld):
    torch.save({"sigmas30": ld.ltx2_scheduler_sigmas(30), "sigmas8_tokens480": ld.ltx2_scheduler_sigmas(8, 480),
                "video_positions": ld.video_positions(1, 3, 4, 5, 24.0, "cpu"),
                "audio_positions": ld.audio_positions(1, 7, "cpu")}, OUT / "sched.pt")


GUIDE_PARAMS = [  # (cfg, stg, rescale, modality)
    (3.0, 1.0, 0.7, 3.0),
    (4.5, 0.0, 1.0, 1.0),
    (3.0, 1.0, 0.0, 3.0),
]


def make_guide(ld):
    """The reference's guide() (ltx_dit.py:551-562), std rescale included, on seeded
    (1, 384, 128) x0 predictions in fp32 and bf16."""
    rec = {"params": GUIDE_PARAMS, "cases": {}}
    for dtype in (torch.float32, torch.bfloat16):
        xs = [rng_normal((1, 384, 128), 500 + i, scale=1.0 + 0.1 * i, dtype=dtype) for i in range(4)]
        outs = [ld.guide(*xs, ld.GuiderParams(cfg, stg, rs, mod, ())) for cfg, stg, rs, mod in GUIDE_PARAMS]
        rec["cases"][str(dtype).replace("torch.", "")] = {"inputs": xs, "outputs": outs}
    torch.save(rec, OUT / "guide.pt")


GUIDED_V = (3.0, 1.0, 0.7, 3.0, (1,))  # cfg, stg, rescale, modality, stg_blocks (run_all.py:43-44 values)
GUIDED_A = (7.0, 1.0, 0.7, 3.0, (1,))
GUIDED_SIGMAS = [1.0, 0.7, 0.4]


@torch.inference_mode()
def make_guided(ld, dtype):
    """Two steps of the reference's full guidance (guided_denoise_step: cond / uncond / STG /
    modality-isolated passes in one B=4 call, std rescale, Euler) on the tiny AV model,
    with a conditioned first frame (denoise mask 0, keyframes mask 1)."""
    cfg = ld.DiTConfig(**CASES["tiny_av"])
    model, shapes = build_reference_model(ld, cfg, dtype)
    f, h, w = FRAMES
    t = f * h * w
    dmask = torch.ones(1, t, 1)
    dmask[:, : h * w] = 0.0
    kf = 1.0 - dmask
    vs = ld.LatentState(latent=rng_normal((1, t, cfg.video_in), 300).to(dtype), denoise_mask=dmask,
                        positions=ld.video_positions(1, f, h, w, 24.0, "cpu"),
                        clean_latent=torch.zeros(1, t, cfg.video_in, dtype=dtype), keyframes_mask=kf)
    aus = ld.LatentState(latent=rng_normal((1, AUDIO_T, cfg.audio_in), 301).to(dtype),
                         denoise_mask=torch.ones(1, AUDIO_T, 1), positions=ld.audio_positions(1, AUDIO_T, "cpu"),
                         clean_latent=torch.zeros(1, AUDIO_T, cfg.audio_in, dtype=dtype))
    contexts = {"v_pos": rng_normal((1, TEXT_S, cfg.video_cross_dim), 302).to(dtype),
                "v_neg": rng_normal((1, TEXT_S, cfg.video_cross_dim), 303).to(dtype),
                "a_pos": rng_normal((1, TEXT_S, cfg.audio_cross_dim), 304).to(dtype),
                "a_neg": rng_normal((1, TEXT_S, cfg.audio_cross_dim), 305).to(dtype)}
    sigmas = torch.tensor(GUIDED_SIGMAS, dtype=torch.float32)
    vp, ap = ld.GuiderParams(*GUIDED_V), ld.GuiderParams(*GUIDED_A)
    rec = {"config": dataclasses.asdict(cfg), "param_shapes": shapes, "weight_seed": WEIGHT_SEED,
           "dtype": str(dtype).replace("torch.", ""), "v_params": GUIDED_V, "a_params": GUIDED_A,
           "sigmas": sigmas, "contexts": contexts,
           "video_state": dataclasses.asdict(vs), "audio_state": dataclasses.asdict(aus), "steps": []}
    for idx in range(len(GUIDED_SIGMAS) - 1):
        dv, da, passes = ld.guided_denoise_step(model, vs, aus, contexts, sigmas[idx], idx, vp, ap, cfg)
        vs = dataclasses.replace(vs, latent=ld.euler_step(vs.latent, dv, sigmas, idx))
        aus = dataclasses.replace(aus, latent=ld.euler_step(aus.latent, da, sigmas, idx))
        rec["steps"].append({"denoised_video": dv, "denoised_audio": da, "passes": passes,
                             "video_latent": vs.latent, "audio_latent": aus.latent})
    return rec


def make_ckpt_keys(ld):
    """The reference's load_transformer (ltx_dit.py:414-432) on a tiny checkpoint written
    in the dev-checkpoint key format: records, per checkpoint key, the parameter name the
    reference loads it into (None = dropped) and the parameter shapes."""
    import json
    import tempfile

    import common as ref_common
    from safetensors.torch import save_file

    cfg = ld.DiTConfig(**CASES["tiny_av"])
    _, shapes = build_reference_model(ld, cfg, torch.float32)

    def to_ckpt(n):
        k = n.replace("blocks.", "transformer_blocks.", 1) if n.startswith("blocks.") else n
        k = k.replace("to_out.", "to_out.0.")
        k = k.replace("audio_ff.proj_in.", "audio_ff.net.0.proj.").replace("audio_ff.proj_out.", "audio_ff.net.2.")
        k = k.replace(".ff.proj_in.", ".ff.net.0.proj.").replace(".ff.proj_out.", ".ff.net.2.")
        return "model.diffusion_model." + k

    keys = [to_ckpt(n) for n, _ in shapes] + ["vae.decoder.conv_in.weight", "text_embedding_projection.weight"]
    tensors = {k: torch.zeros(2, 2) for k in keys}
    for (n, shp), k in zip(shapes, keys):
        tensors[k] = torch.zeros(shp)
    captured = {}

    def cpu_load(path, rename=None, **kw):
        captured["rename"] = rename
        return ref_common.load_state_dict(path, device="cpu", dtype=torch.float32, rename=rename)

    saved = ld.load_state_dict, ld.DEVICE
    ld.load_state_dict, ld.DEVICE = cpu_load, "cpu"
    try:
        with tempfile.TemporaryDirectory() as d:
            path = f"{d}/tiny.safetensors"
            save_file(tensors, path)
            ld.load_transformer(path, cfg)  # raises on any missing parameter
    finally:
        ld.load_state_dict, ld.DEVICE = saved
    rec = {"config": "tiny_av", "shapes": [[n, list(shp)] for n, shp in shapes],
           "keys": {k: captured["rename"](k) for k in keys}}
    (OUT / "ckpt_keys.json").write_text(json.dumps(rec, indent=0))


CONNECTOR = dict(heads=4, dim_head=64, num_layers=2, max_pos=[4096], registers=8, gated=True, ff_bias=True)


@torch.inference_mode()
def make_connector(ref_root: Path, dtype):
    """The reference's Embeddings1DConnector (ltx_te.py:187-229) on seeded inputs: sample 0
    has its last 12 of 32 tokens padded (negative additive mask), sample 1 none."""
    sys.path.insert(0, str(ref_root / "standalone"))
    import ltx_te

    conn = ltx_te.Embeddings1DConnector(**CONNECTOR)
    shapes = [(n, tuple(p.shape)) for n, p in conn.named_parameters()]
    conn.load_state_dict(ltx_oracle.synthetic_state_dict(shapes, WEIGHT_SEED + 5, dtype=torch.float32))
    conn = conn.to(dtype).eval()
    inner = CONNECTOR["heads"] * CONNECTOR["dim_head"]
    hidden = rng_normal((2, 32, inner), 400).to(dtype)
    mask = torch.zeros(2, 1, 1, 32, dtype=dtype)
    mask[0, :, :, 20:] = -10000.0
    out, out_mask = conn(hidden, mask)
    return {"config": CONNECTOR, "param_shapes": shapes, "weight_seed": WEIGHT_SEED + 5,
            "dtype": str(dtype).replace("torch.", ""), "hidden": hidden, "mask": mask, "out": out,
            "out_mask": out_mask}


# Every decoder block kind (res_x, res_x_y with the GroupNorm + 1x1 shortcut,
# compress_time / compress_space / compress_all) at channel counts the tcgen05
# convolution takes (input channels a multiple of 64).
VAE_CFG = {"decoder_blocks": [["res_x", {"num_layers": 1}], ["compress_all", {"multiplier": 2}],
                              ["res_x_y", {"multiplier": 2}], ["compress_time", {"multiplier": 1}],
                              ["compress_space", {"multiplier": 1}], ["res_x", {"num_layers": 1}]],
           "decoder_base_channels": 64, "patch_size": 4, "spatial_padding_mode": "zeros", "latent_channels": 128,
           "out_channels": 3}


@torch.inference_mode()
def make_vae(ref_root: Path, dtype):
    """The reference's ConvVideoDecoder (ltx_vae.py:161-216) on a seeded (2, 128, 3, 4, 6)
    latent -> (2, 3, 9, 64, 96)."""
    sys.path.insert(0, str(ref_root / "standalone"))
    import ltx_vae

    dec = ltx_vae.ConvVideoDecoder(VAE_CFG)
    shapes = [(n, tuple(p.shape)) for n, p in dec.named_parameters()]
    sd = vae_oracle.synthetic_decoder_state_dict(shapes, WEIGHT_SEED + 7, VAE_CFG["latent_channels"])
    dec.load_state_dict(sd)
    dec = dec.to(dtype).eval()
    latent = rng_normal((2, 128, 3, 4, 6), 500).to(dtype)
    out = dec(latent)
    return {"config": VAE_CFG, "param_shapes": shapes, "weight_seed": WEIGHT_SEED + 7,
            "dtype": str(dtype).replace("torch.", ""), "latent": latent, "out": out}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("LTX_NV_REFERENCE"), required="LTX_NV_REFERENCE" not in os.environ,
                    help="checkout of lipaul/ltx-nv (default: $LTX_NV_REFERENCE)")
    ap.add_argument("--only", choices=["guide", "guided", "ckpt", "connector", "vae"], default=None,
                    help="regenerate one fixture only")
    args = ap.parse_args()
    ref_root = Path(args.reference)
    ld = _import_reference(ref_root)
    patch_context_view(ld)
    if args.only in (None, "guide"):
        make_guide(ld)
    if args.only in (None, "guided"):
        for dtype in (torch.float32, torch.bfloat16):
            rec = make_guided(ld, dtype)
            torch.save(rec, OUT / f"guided_tiny_av_{rec['dtype']}.pt")
    if args.only in (None, "ckpt"):
        make_ckpt_keys(ld)
    if args.only in (None, "connector"):
        for dtype in (torch.float32, torch.bfloat16):
            rec = make_connector(ref_root, dtype)
            torch.save(rec, OUT / f"connector_{rec['dtype']}.pt")
    if args.only in (None, "vae"):
        for dtype in (torch.float32, torch.bfloat16):
            rec = make_vae(ref_root, dtype)
            torch.save(rec, OUT / f"vae_tiny_{rec['dtype']}.pt")
    if args.only is not None:
        return
    make_philox(ref_root)
    make_sched(ld)
    for name, ov in CASES.items():
        for dtype in (torch.float32, torch.bfloat16):
            rec = make_case(ld, name, ov, dtype)
            torch.save(rec, OUT / f"dit_{name}_{rec['dtype']}.pt")
            print("wrote", name, rec["dtype"], tuple(rec["vx"].shape))


if __name__ == "__main__":
    main()
