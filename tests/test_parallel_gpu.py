"""Multi-GPU step (ltx_parallel) against the single-GPU step on the same inputs.

With attention running every (sample, head, 256-query) unit whole, each rank runs the
same kernels on the same rows as the single GPU, so the next latent must be identical.
With the automatic attention plan the units that would only partly fill the last wave
of SMs are split over key ranges, and ranks with fewer heads split other units than the
single GPU does: there the next latent must agree to bf16 rounding (rel-L2 <= 1e-2).
Needs >= 2 (or 4) visible GPUs; skipped otherwise."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, cfg_split, exchange, q):
    import sys
    from datetime import timedelta
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    for p in (str(root), str(root / "ltx-nv_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    import torch.distributed as dist

    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    try:
        import ltx_dit
        import ltx_parallel

        cfg = ltx_dit.DiTConfig.video_only(num_layers=2, heads=32, head_dim=64, cross_dim=4096)
        with torch.device("meta"):
            model = ltx_dit.LTXModel(cfg)
        gen = ltx_dit.PhiloxGenerator(11, dev)
        sd = {}
        for name, p in model.named_parameters():
            w = gen.randn(*p.shape, dtype=torch.bfloat16).mul_(0.02)
            if name.endswith(("q_norm.weight", "k_norm.weight")):
                w.add_(1.0)
            sd[name] = w
        model.load_state_dict(sd, assign=True)
        f, h, w_ = 8, 16, 16
        t = f * h * w_
        latent = gen.randn(1, t, 128, dtype=torch.bfloat16)
        ctx = gen.randn(2, 128, 4096, dtype=torch.bfloat16)
        pos = ltx_dit.video_positions(1, f, h, w_, 24.0, dev)
        kf = torch.zeros(1, t, 1, device=dev)
        kf[:, : h * w_] = 1
        sigmas = torch.tensor([0.5, 0.25])
        import _native as nat

        def single():
            return ltx_dit.cfg_denoise_step(model, latent, pos, ctx[:1], ctx[1:], sigmas, 0, 3.0, keyframes_mask=kf,
                                            fused_head=False)[2]

        nat.attention_force_split(-1)  # whole units everywhere: the exact comparison
        ref = single()
        pdn = ltx_parallel.ParallelDenoiser(model, cfg_split=cfg_split, exchange=exchange)
        sp = model._sp
        out = pdn.step(latent, pos, ctx[:1], ctx[1:], sigmas, 0, 3.0, keyframes_mask=kf)
        nat.attention_force_split(0)  # the automatic plan
        model._sp = None
        ref_auto = single()
        model._sp = sp
        out_auto = pdn.step(latent, pos, ctx[:1], ctx[1:], sigmas, 0, 3.0, keyframes_mask=kf)
        torch.cuda.synchronize()
        model._sp = None
        diff = (out.float() - ref.float()).abs().max().item()
        rel = float((out_auto.float() - ref_auto.float()).norm() / ref_auto.float().norm())
        q.put((rank, diff, rel, pdn.layout.cfg, pdn.layout.sp))
        pdn.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,cfg_split,exchange", [(2, 2, "nccl"), (2, 1, "nccl"), (2, 1, "peer"), (4, 2, "nccl"),
                                                     (4, 2, "peer")])
def test_parallel_step_equals_single_gpu(world, cfg_split, exchange):
    """exchange "nccl": pack + all_to_all + unpack; "peer": the exchange fused into the q/k
    and attention kernels over NVLink peer memory."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, cfg_split, exchange, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    print("\nper rank (max |diff| whole units, rel-L2 automatic plan):", [(r, d, e) for r, d, e, _, _ in res])
    assert all(d == 0.0 for _, d, _, _, _ in res), res
    assert all(e < 1e-2 for _, _, e, _, _ in res), res


def _av_worker(rank, world, port, cfg_split, exchange, q):
    import sys
    from datetime import timedelta
    from pathlib import Path

    root = Path(__file__).resolve().parents[1]
    for p in (str(root), str(root / "ltx-nv_b200")):
        if p not in sys.path:
            sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    import torch.distributed as dist

    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    try:
        import ltx_dit
        import ltx_parallel

        # config-4 widths (video 32x128, audio 32x64, A<->V attention), 2 blocks, small tokens
        cfg = ltx_dit.DiTConfig(num_layers=2, video_cross_dim=3840, cross_attention_adaln=False)
        with torch.device("meta"):
            model = ltx_dit.LTXModel(cfg)
        gen = ltx_dit.PhiloxGenerator(13, dev)
        sd = {}
        for name, p in model.named_parameters():
            w = gen.randn(*p.shape, dtype=torch.bfloat16).mul_(0.02)
            if name.endswith(("q_norm.weight", "k_norm.weight")):
                w.add_(1.0)
            sd[name] = w
        model.load_state_dict(sd, assign=True)
        f, h, w_ = 4, 8, 16
        tv, ta = f * h * w_, 126
        v_lat = gen.randn(1, tv, 128, dtype=torch.bfloat16)
        a_lat = gen.randn(1, ta, 128, dtype=torch.bfloat16)
        v_ctx = gen.randn(2, 256, 3840, dtype=torch.bfloat16)
        a_ctx = gen.randn(2, 256, 2048, dtype=torch.bfloat16)
        v_pos = ltx_dit.video_positions(1, f, h, w_, 24.0, dev)
        a_pos = ltx_dit.audio_positions(1, ta, dev)
        kf = torch.zeros(1, tv, 1, device=dev)
        kf[:, : h * w_] = 1
        sigmas = torch.tensor([0.5, 0.25])
        args = (v_lat, a_lat, v_pos, a_pos, v_ctx[:1], v_ctx[1:], a_ctx[:1], a_ctx[1:], sigmas, 0, 3.0)
        ref_v, ref_a = ltx_dit.av_cfg_denoise_step(model, *args, v_keyframes_mask=kf)
        pdn = ltx_parallel.ParallelDenoiser(model, cfg_split=cfg_split, exchange=exchange)
        out_v, out_a = pdn.step_av(*args, v_keyframes_mask=kf)
        torch.cuda.synchronize()
        model._sp = None

        def rel(a, b):
            return float((a.float() - b.float()).norm() / b.float().norm())

        q.put((rank, rel(out_v, ref_v), rel(out_a, ref_a), pdn.layout.cfg, pdn.layout.sp))
        pdn.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,cfg_split,exchange", [(2, 1, "nccl"), (2, 1, "peer"), (4, 2, "peer")])
def test_parallel_av_step_matches_single_gpu(world, cfg_split, exchange):
    """Audio-video step under sequence parallelism (audio replicated, video-to-audio
    attention merged from split-KV partials) against the single-GPU av_cfg_denoise_step.
    The split softmax rounds differently from the single pass, so the check is relative
    L2 <= 1e-2 (a few 1e-3 expected); video is token-local except self-attention, whose
    Ulysses exchange is exact."""
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_av_worker, args=(r, world, port, cfg_split, exchange, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    print("\nAV SP rel-L2 per rank (video, audio):", [(r, v, a) for r, v, a, _, _ in res])
    assert all(v < 1e-2 and a < 1e-2 for _, v, a, _, _ in res), res
