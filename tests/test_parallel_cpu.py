"""Host-side logic of the multi-GPU step, on CPU with gloo ranks (world size 2 and 4):
rank layouts, token shards, and the Ulysses all-to-all exchange pattern. The pack /
unpack semantics of ltx_sp_pack / ltx_sp_unpack (include/ltxb200.h) are restated here
in torch so the exchange can run without a GPU; attention over the exchanged buffers
must equal attention over the full sequence."""

import math
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn.functional as F

from ltx_parallel import Layout, qkv_segments


def test_layouts():
    lay = [Layout.make(8, r) for r in range(8)]
    assert all(x.cfg == 2 and x.sp == 4 for x in lay)
    assert [x.sample for x in lay] == [0, 0, 0, 0, 1, 1, 1, 1]
    assert lay[5].sp_rank == 1 and lay[5].tokens(6144) == (1536, 3072)
    assert lay[0].sp_groups() == [[0, 1, 2, 3], [4, 5, 6, 7]]
    assert lay[0].cfg_groups() == [[0, 4], [1, 5], [2, 6], [3, 7]]
    two = Layout.make(2, 1)
    assert two.cfg == 2 and two.sp == 1 and two.sample == 1 and two.tokens(6144) == (0, 6144)
    sp_only = Layout.make(2, 1, cfg=1)
    assert sp_only.sample == -1 and sp_only.tokens(480) == (240, 480)
    assert Layout.make(1, 0).sp == 1
    with pytest.raises(ValueError):
        Layout.make(8, 0).tokens(27588 * 2 + 2)
    assert Layout.make(8, 3).tokens(27588) == (3 * 6897, 4 * 6897)


def test_qkv_segments():
    assert qkv_segments(2048, 32, 4, True) == [(0, 512), (2048, 512), (4096, 512), (6144, 8)]
    assert qkv_segments(2048, 32, 2, False) == [(0, 1024), (2048, 1024), (4096, 1024)]


def pack_ref(src, parts, segs):
    return torch.stack([torch.cat([src[:, o + j * w:o + (j + 1) * w] for o, w in segs], dim=1) for j in range(parts)])


def unpack_ref(src):
    p, rows, w = src.shape
    return src.permute(1, 0, 2).reshape(rows, p * w)


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.manual_seed(0)
        heads, d, t = 8, 16, 24 * world
        dim = heads * d
        qkv_full = torch.randn(t, 3 * dim + heads)
        lay = Layout.make(world, rank, cfg=1)
        t0, t1 = lay.tokens(t)
        local = qkv_full[t0:t1]
        segs = qkv_segments(dim, heads, world, True)
        w = sum(s[1] for s in segs)
        send = pack_ref(local, world, segs)
        recv = torch.empty(t, w)
        dist.all_to_all_single(recv, send.reshape(world * (t1 - t0), w))
        hp, dp = heads // world, dim // world
        qh = recv[:, :dp].view(t, hp, d).transpose(0, 1)
        kh = recv[:, dp:2 * dp].view(t, hp, d).transpose(0, 1)
        vh = recv[:, 2 * dp:3 * dp].view(t, hp, d).transpose(0, 1)
        gate = 2 * torch.sigmoid(recv[:, 3 * dp:3 * dp + hp])
        out = (F.scaled_dot_product_attention(qh, kh, vh).transpose(0, 1) * gate[..., None]).reshape(t, dp)
        back = torch.empty(t, dp)
        dist.all_to_all_single(back, out.contiguous())
        mine = unpack_ref(back.view(world, t1 - t0, dp))
        # full-sequence reference on this rank's tokens
        qf = qkv_full[:, :dim].view(t, heads, d).transpose(0, 1)
        kf = qkv_full[:, dim:2 * dim].view(t, heads, d).transpose(0, 1)
        vf = qkv_full[:, 2 * dim:3 * dim].view(t, heads, d).transpose(0, 1)
        gf = 2 * torch.sigmoid(qkv_full[:, 3 * dim:])
        ref = (F.scaled_dot_product_attention(qf, kf, vf).transpose(0, 1) * gf[..., None]).reshape(t, dim)[t0:t1]
        q.put((rank, float((mine - ref).abs().max())))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
def test_ulysses_exchange_equals_full_attention_gloo(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(err < 1e-5 for _, err in res), res


def merge_ref(o_all, lse_all):
    """The merge of ltx_attention_merge (without the gate): weights 2^(lse_r - max)."""
    m = lse_all.max(dim=0, keepdim=True).values
    w = torch.exp2(lse_all - m)  # (R, rows, H)
    num = (o_all.view(*lse_all.shape, -1) * w[..., None]).sum(0)
    return num / w.sum(0)[..., None]


def _split_kv_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.manual_seed(1)
        heads, d, tq, tk = 4, 16, 10, 12 * world
        scale = d ** -0.5
        qh = torch.randn(heads, tq, d)  # replicated audio queries
        kf, vf = torch.randn(heads, tk, d), torch.randn(heads, tk, d)  # all video keys
        lay = Layout.make(world, rank, cfg=1)
        t0, t1 = lay.tokens(tk)
        k, v = kf[:, t0:t1], vf[:, t0:t1]  # this rank's shard
        s = torch.einsum("hqd,hkd->hqk", qh, k) * scale
        o_part = torch.softmax(s, dim=-1) @ v  # O / l over the local keys
        lse = torch.logsumexp(s, dim=-1) / math.log(2.0)  # log2-sum-exp
        o_all = torch.empty(world * heads, tq, d)
        lse_all = torch.empty(world * heads, tq)
        dist.all_gather_into_tensor(o_all, o_part.contiguous())
        dist.all_gather_into_tensor(lse_all, lse.contiguous())
        o_all, lse_all = o_all.view(world, heads, tq, d), lse_all.view(world, heads, tq)
        merged = merge_ref(o_all.permute(0, 2, 1, 3).reshape(world, tq, heads * d), lse_all.permute(0, 2, 1))
        ref = F.scaled_dot_product_attention(qh, kf, vf).transpose(0, 1)
        q.put((rank, float((merged - ref).abs().max())))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4])
def test_split_kv_merge_equals_full_attention_gloo(world):
    """Video-to-audio attention under sequence parallelism: each rank attends the
    replicated audio queries to its shard of the video keys, the (O / l, log2-sum-exp)
    partials are all-gathered and merged; every rank must get the attention over all keys."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_split_kv_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert all(err < 1e-5 for _, err in res), res


def _transport_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import ltx_dit
        import ltx_parallel

        cfg = ltx_dit.DiTConfig.video_only(num_layers=1, heads=8, head_dim=16, cross_dim=32)
        with torch.device("meta"):
            model = ltx_dit.LTXModel(cfg)
        got = []
        for cfg_split, exchange in ((2, "auto"), (1, "auto"), (1, "nccl")):
            pdn = ltx_parallel.ParallelDenoiser(model, cfg_split=cfg_split, exchange=exchange)
            got.append((pdn.layout.sp, pdn.exchange_kind, pdn.exchange is None,
                        model._sp is not None and model._sp.exchange is None))
            pdn.close()
        try:
            ltx_parallel.ParallelDenoiser(model, exchange="shared-memory")
            got.append("no error")
        except ValueError:
            got.append("ValueError")
        q.put((rank, got))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_exchange_transport_choice_gloo():
    """ParallelDenoiser's exchange transport: with CFG2 at 2 ranks there is no sequence
    parallelism (no exchange); with SP2 "auto" picks the NCCL formulation when the process
    group is not NCCL on CUDA (here gloo on CPU), and an unknown transport is refused."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_transport_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(2)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for _, got in res:
        assert got == [(1, "none", True, False), (2, "nccl", True, True), (2, "nccl", True, True), "ValueError"]
