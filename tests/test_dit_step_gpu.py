"""The whole-step C entry point (ltx_ctx_create / ltx_dit_reserve / ltx_dit_step, called
through ctypes) against the Python drop-in's cfg_denoise_step: same kernels, same
arguments, so velocity, denoised and next latent must be bit-identical, including a
second step that reuses the step-invariant RoPE tables and text K/V."""

import pytest
import torch

import _native as nat
import ltx_dit
from model_fixtures import DEV, philox_model
from oracle import ltx_oracle

pytestmark = pytest.mark.gpu


def _inputs(f, h, w, text, cross_dim, dtype, seed):
    t = f * h * w
    g = torch.Generator().manual_seed(seed)
    latent = torch.randn(1, t, 128, generator=g).to(dtype).to(DEV)
    ctx = torch.randn(2, text, cross_dim, generator=g).to(dtype).to(DEV)
    pos = ltx_oracle.video_positions(1, f, h, w, 24.0).to(DEV)
    kf = torch.zeros(1, t, 1, device=DEV)
    kf[:, : h * w] = 1.0
    return latent, ctx, pos, kf


def _two_steps_equal(model, f, h, w, text, cross_dim, dtype, seed):
    latent, ctx, pos, kf = _inputs(f, h, w, text, cross_dim, dtype, seed)
    sigmas = torch.tensor([1.0, 0.5, 0.25])
    step = ltx_dit.NativeStep(model, f * h * w, text)
    lat_a = lat_b = latent
    for idx in range(2):
        ref = ltx_dit.cfg_denoise_step(model, lat_a, pos, ctx[:1], ctx[1:], sigmas, idx, 3.0, keyframes_mask=kf)
        got = step(lat_b, pos, ctx[:1], ctx[1:], sigmas, idx, 3.0, keyframes_mask=kf, reuse=idx > 0)
        torch.cuda.synchronize()
        assert nat.device_error_flags() == 0
        for name, r, g in zip(("velocity", "denoised", "next latent"), ref, got):
            assert torch.equal(r, g), (idx, name, float((r.float() - g.float()).abs().max()))
        lat_a, lat_b = ref[2], got[2]
    step.close()


def test_dit_step_config3_bit_identical_to_cfg_denoise_step():
    """BASELINE config 3 at full size: 28 blocks, T = 6144, text 128 x 4096, BF16."""
    cfg = ltx_dit.DiTConfig.video_only(num_layers=28, heads=32, head_dim=64, cross_dim=4096)
    model, _ = philox_model(cfg, seed=21, host_copy=False)
    _two_steps_equal(model, 16, 16, 24, 128, 4096, torch.bfloat16, seed=22)


def test_dit_step_fp32_config1_geometry_bit_identical():
    """The FP32 accuracy mode (BASELINE config 1 geometry, 2 of its 8 blocks, T = 480)."""
    cfg = ltx_dit.DiTConfig.video_only(num_layers=2, heads=32, head_dim=64, cross_dim=4096)
    model, _ = philox_model(cfg, seed=23, host_copy=False, dtype=torch.float32)
    _two_steps_equal(model, 5, 8, 12, 128, 4096, torch.float32, seed=24)


def test_dit_step_rejects_unreserved_sizes():
    cfg = ltx_dit.DiTConfig.video_only(num_layers=1, heads=32, head_dim=64, cross_dim=4096)
    model, _ = philox_model(cfg, seed=25, host_copy=False)
    step = ltx_dit.NativeStep(model, 96, 16)
    latent, ctx, pos, kf = _inputs(4, 4, 12, 32, 4096, torch.bfloat16, seed=26)  # T = 192 > 96
    with pytest.raises(nat.LtxError, match="workspace too small"):
        step(latent, pos, ctx[:1], ctx[1:], torch.tensor([0.5, 0.25]), 0, 3.0)
    step.close()
