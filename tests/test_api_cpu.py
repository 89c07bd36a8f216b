"""Host-side checks that need no GPU: the C ABI exports what include/ltxb200.h declares,
the drop-in module's parameter layout equals the reference's, and the host helpers
(schedule, positions, perturbation masks, Philox bookkeeping) agree with the oracle."""

import ctypes
import re
from pathlib import Path

import pytest
import torch

import _native as nat
import golden_cases as gc
import ltx_dit
from oracle import ltx_oracle, philox_oracle

ROOT = Path(__file__).resolve().parents[1]


def header_functions() -> list[str]:
    """Every function declared in include/*.h (the public ABI and the test hooks)."""
    names = set()
    for h in sorted((ROOT / "include").glob("*.h")):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(ltx_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(nat.LIB_PATH))
    names = header_functions()
    assert len(names) >= 20
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # and the Python binding covers the whole header
    assert set(names) <= set(nat._SIGNATURES), set(names) - set(nat._SIGNATURES)


def test_library_status_codes_without_a_gpu():
    lib = nat.load_library()
    assert lib.ltx_abi_version() == 1
    # argument validation happens before any CUDA call
    st = lib.ltx_philox_randn(None, 16, 0, 1, 0, 1, None)
    assert st == 1 and b"out is NULL" in lib.ltx_last_error()
    st = lib.ltx_linear(None, 8, None, 8, None, 8, 8, 8, 8, None, 1, None)
    assert st == 1
    assert lib.ltx_philox_offset_increment(442368, 852) == 4
    assert lib.ltx_philox_offset_increment(1572864, 1184) == 8
    assert lib.ltx_philox_offset_increment(1572864, 1184) == philox_oracle.offset_increment(1572864, 1184)


def test_whole_step_entry_points_without_a_gpu():
    """ltx_dit_workspace_bytes is host arithmetic; the context / step entry points
    validate their arguments and report errors as status codes, never by crashing."""
    lib = nat.load_library()
    c = nat.DitConfig()
    c.num_layers, c.heads, c.head_dim = 28, 32, 64
    c.in_channels = c.out_channels = 128
    c.cross_dim, c.ffn_dim, c.gated_attention = 4096, 8192, 1
    c.norm_eps, c.theta, c.timestep_scale_multiplier, c.dtype = 1e-6, 10000.0, 1000.0, nat.LTX_BF16
    c.max_pos[:] = [20.0, 2048.0, 2048.0]
    t, s, d = 6144, 128, 2048
    nbytes = nat.dit_workspace_bytes(c, t, s)
    # x, h, o (2T x D), the shared QKV / text-q / FFN buffer (2T x F), text K/V of every block
    assert nbytes >= 2 * (3 * 2 * t * d + 2 * t * 8192 + 28 * 2 * s * 2 * d)
    assert nbytes < 2 * (3 * 2 * t * d + 2 * t * 8192 + 28 * 2 * s * 2 * d) + 64 << 20
    assert lib.ltx_dit_workspace_bytes(None, t, s) == 0
    assert lib.ltx_ctx_destroy(None) == 0
    st = lib.ltx_dit_step(None, ctypes.byref(c), None, None, None, None, None, None)
    assert st == 1 and b"NULL" in lib.ltx_last_error()
    st = lib.ltx_dit_reserve(None, ctypes.byref(c), t, s)
    assert st == 1
    h = ctypes.c_void_p()
    assert lib.ltx_ctx_create(0, ctypes.byref(h)) != 0  # no CUDA device here
    assert h.value is None


def test_vae_decoder_parameter_layout_matches_reference():
    """ConvVideoDecoder has the reference's parameter names, shapes and order (and its
    per-channel statistics buffers), so reference state dicts load unchanged."""
    import ltx_vae

    rec = torch.load(gc.GOLDEN / "vae_tiny_bfloat16.pt", weights_only=False)
    with torch.device("meta"):
        dec = ltx_vae.ConvVideoDecoder(rec["config"])
    assert [(n, tuple(p.shape)) for n, p in dec.named_parameters()] == [(n, tuple(s)) for n, s in rec["param_shapes"]]
    assert {n for n, _ in dec.named_buffers()} == {"per_channel_statistics.std-of-means",
                                                    "per_channel_statistics.mean-of-means"}


def test_load_video_decoder_maps_checkpoint_keys(tmp_path):
    """load_video_decoder reads the config from the checkpoint's metadata and takes
    `decoder.*` (prefix removed) and `per_channel_statistics.*` keys, ignoring the rest,
    as the reference's load_video_decoder (ltx_vae.py:225-235)."""
    import json

    from safetensors.torch import save_file

    import ltx_vae
    from oracle import vae_oracle

    rec = torch.load(gc.GOLDEN / "vae_tiny_bfloat16.pt", weights_only=False)
    sd = vae_oracle.synthetic_decoder_state_dict(rec["param_shapes"], rec["weight_seed"],
                                                 rec["config"]["latent_channels"])
    tensors = {(k if k.startswith("per_channel_statistics.") else "decoder." + k): v.contiguous()
               for k, v in sd.items()}
    tensors["encoder.conv_in.conv.weight"] = torch.zeros(4)  # other parts of the VAE file
    path = tmp_path / "vae.safetensors"
    save_file(tensors, str(path), metadata={"config": json.dumps({"vae": rec["config"]})})
    dec = ltx_vae.load_video_decoder(str(path), device="cpu")
    got = dict(dec.named_parameters()) | dict(dec.named_buffers())
    assert set(got) == set(sd)
    for name, t in sd.items():
        assert torch.equal(got[name], t), name


def test_native_wrappers_refuse_cpu_tensors():
    with pytest.raises(ValueError):
        nat.gelu_tanh(torch.zeros(8), torch.zeros(8))


@pytest.mark.parametrize("case", ["tiny_video_float32", "tiny_av_float32"])
def test_parameter_layout_matches_reference(case):
    rec = gc.load(case)
    cfg = ltx_dit.DiTConfig(**{k: (tuple(v) if isinstance(v, list) else v) for k, v in rec["config"].items()})
    with torch.device("meta"):
        model = ltx_dit.LTXModel(cfg)
    mine = [(n, tuple(p.shape)) for n, p in model.named_parameters()]
    ref = [(n, tuple(s)) for n, s in rec["param_shapes"]]
    assert mine == ref


def test_video_only_config_matches_golden_geometry():
    rec = gc.load("tiny_video_float32")
    cfg = ltx_dit.DiTConfig.video_only(num_layers=2, heads=4, head_dim=64, cross_dim=384)
    for k, v in rec["config"].items():
        mine = getattr(cfg, k)
        assert (tuple(mine) if isinstance(mine, tuple) else mine) == (tuple(v) if isinstance(v, list) else v), k


def test_schedule_positions_and_perturbations_match_oracle():
    assert torch.equal(ltx_dit.ltx2_scheduler_sigmas(30), ltx_oracle.scheduler_sigmas(30))
    assert torch.equal(ltx_dit.video_positions(2, 3, 4, 5, 24.0, "cpu"), ltx_oracle.video_positions(2, 3, 4, 5, 24.0))
    assert torch.equal(ltx_dit.audio_positions(2, 9, "cpu"), ltx_oracle.audio_positions(2, 9))
    keep = ltx_dit.build_perturbation_config(4, ["cond", "uncond", "ptb", "mod"], [2], [1], "cpu", torch.float32)
    assert keep.shape == (4, 4, 4)
    assert keep[0, 2, 2] == 0 and keep[1, 1, 2] == 0 and keep[2:, :, 3].eq(0).all() and keep[:, :, :2].eq(1).all()


def test_perturbation_config_and_mask_checks():
    """The guidance batch's keep-mask matches the oracle's restatement of
    build_perturbation_config, and masks other than 0 / 1 are rejected loudly."""
    from oracle import ltx_oracle

    passes = ["cond", "uncond", "ptb", "mod"]
    keep = ltx_dit.build_perturbation_config(6, passes, [5], [2, 5], torch.device("cpu"), torch.bfloat16)
    assert torch.equal(keep, ltx_oracle.build_perturbation_config(6, passes, [5], [2, 5], torch.bfloat16))
    with torch.device("meta"):
        model = ltx_dit.LTXModel(ltx_dit.DiTConfig.video_only(num_layers=6, heads=2, head_dim=64, cross_dim=128))
    assert model._keep_masks(keep, 4)[0][5] == [1.0, 1.0, 0.0, 1.0]
    with pytest.raises(NotImplementedError):
        model._keep_masks(keep * 0.5, 4)
    with pytest.raises(ValueError):
        model._keep_masks(keep, 2)


def test_load_transformer_maps_checkpoint_keys_like_the_reference(tmp_path):
    """A dev-format checkpoint of the tiny AV model (keys recorded from the reference's
    load_transformer, tests/golden/ckpt_keys.json) loads into the same parameters."""
    import json

    from safetensors.torch import save_file

    from oracle import ltx_oracle

    rec = json.loads((gc.GOLDEN / "ckpt_keys.json").read_text())
    shapes = [(n, tuple(s)) for n, s in rec["shapes"]]
    sd = ltx_oracle.synthetic_state_dict(shapes, 7, dtype=torch.float32)
    tensors = {}
    for key, name in rec["keys"].items():
        tensors[key] = sd[name].contiguous() if name is not None else torch.ones(3)
    path = tmp_path / "tiny.safetensors"
    save_file(tensors, str(path))
    case = gc.load("tiny_av_float32")
    cfg = ltx_dit.DiTConfig(**{k: (tuple(v) if isinstance(v, list) else v) for k, v in case["config"].items()})
    model = ltx_dit.load_transformer(str(path), cfg, device=torch.device("cpu"), dtype=torch.float32)
    got = dict(model.named_parameters())
    assert set(got) == set(sd)
    for name, t in sd.items():
        assert torch.equal(got[name], t), name


def test_attention_split_plan():
    """The attention launch's split plan (host arithmetic, ltx_test_attention_plan): the
    per-rank self-attention shapes of config 3 at 1, 2, 4 and 8 GPUs, config 5 (keys not a
    multiple of the 128-key tile: never split) and the 126 audio queries over 6144 video
    keys (64 units, fewer than the SMs: all split). Every plan keeps whole units to full
    waves, splits into a divisor of the key tiles with at least 3 tiles per part, and has
    the least cost of the measured model (whole unit 11 + n key-tile times, part 16 + n/k)."""
    sms = 148
    cases = {(2, 32, 6144, 6144): (1480, 2), (1, 32, 6144, 6144): (740, 4), (1, 16, 6144, 6144): (384, 1),
             (1, 8, 6144, 6144): (148, 3), (2, 32, 27588, 27588): (6912, 1), (2, 32, 126, 6144): (0, 2)}
    for (b, h, tq, tk), want in cases.items():
        units = b * h * ((tq + 255) // 256)
        assert nat.attention_plan(units, tk, sms) == want, (b, h, tq, tk)
    for units in range(1, 1200, 7):
        for tk in (384, 1024, 1536, 6144, 6000):
            n_full, k = nat.attention_plan(units, tk, sms)
            r = units % sms
            if k == 1:
                assert n_full == units
                continue
            n = tk // 128
            assert tk % 128 == 0 and n % k == 0 and n // k >= 3
            assert n_full == units - r and n_full % sms == 0 and r * k <= 4 * sms
            cost = -(-(r * k) // sms) * (16 + n / k)
            assert cost < 11 + n
            for k2 in range(2, 9):
                if n % k2 == 0 and n // k2 >= 3 and r * k2 <= 4 * sms:
                    assert cost <= -(-(r * k2) // sms) * (16 + n / k2) + 1e-9


def test_exchange_entry_points_validate_without_a_gpu():
    """The peer-memory exchange entry points reject bad arguments with a status code
    before any CUDA call."""
    lib = nat.load_library()
    fake = (ctypes.c_void_p * 9)(*([16] * 9))
    cnt = ctypes.c_void_p(16)
    assert lib.ltx_sp_barrier(fake, cnt, 9, 0, 1000, None) == 1  # more than 8 ranks
    assert lib.ltx_sp_barrier(fake, cnt, 2, 2, 1000, None) == 1  # rank out of range
    assert lib.ltx_sp_barrier(None, cnt, 2, 0, 1000, None) == 1
    x = ctypes.c_void_p(256)
    # 30 heads do not split over 4 ranks
    assert lib.ltx_qk_norm_rope_scatter(x, 6200, 64, 64, 30, 64, x, x, ctypes.c_float(1e-6), None, None, 0, 0, 1,
                                        4, 0, fake, 1600, None) == 1
    # attention_scatter needs more than 128 keys and parts dividing T
    assert lib.ltx_attention_scatter(x, 1544, x, 1544, x, 1544, 1, 128, 8, 64, ctypes.c_float(0.125), None, 0, None,
                                     0, 4, fake, 2048, 0, None) == 1
    assert lib.ltx_attention_scatter(x, 1544, x, 1544, x, 1544, 1, 1000, 8, 64, ctypes.c_float(0.125), None, 0,
                                     None, 0, 3, fake, 2048, 0, None) == 1
    assert lib.ltx_peer_alloc(0, None, None) == 1
    assert lib.ltx_peer_close(None) == 0 and lib.ltx_peer_free(None) == 0
