"""Multi-GPU denoise step: CFG split x Ulysses sequence parallelism over NCCL.

One process per GPU. The world of W ranks is split into `cfg` CFG groups (2 when W >= 2:
cond on the first W/2 ranks, uncond on the rest) of `sp = W / cfg` ranks each. Inside a
CFG group the latent's T tokens are sharded contiguously over the sp ranks; everything
except self-attention is token-local (GEMMs, norms, FFN, text cross-attention against
the replicated 128-token context). Self-attention runs Ulysses-style:

    QKV(+gate) GEMM on local tokens -> q/k RMSNorm + RoPE (needs all heads of a token)
    -> ltx_sp_pack -> NCCL all_to_all (tokens -> heads) -> tcgen05 attention over all T
    tokens for the rank's H/sp heads -> NCCL all_to_all back -> ltx_sp_unpack -> out GEMM

The step ends with one all_gather of the (T/sp, 128) velocity inside each CFG pair (the
X0 + CFG + Euler update needs cond and uncond of the same tokens) and one all_gather of
the next latent's shards inside each SP group, so every rank holds the full next latent.
Each rank runs the same kernels on the same rows as the single-GPU step, so the result
equals the single-GPU result.

No remote memory is read by any kernel: NCCL moves every byte into local HBM first.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist

import _native as nat
import ltx_dit


@dataclass(frozen=True)
class Layout:
    """Rank -> (CFG sample, SP rank) map and the token shard of each rank."""

    world: int
    rank: int
    cfg: int  # CFG groups: 1 (both samples on every rank) or 2 (one sample per rank)

    @staticmethod
    def make(world: int, rank: int, cfg: int | None = None) -> "Layout":
        if cfg is None:
            cfg = 2 if world >= 2 and world % 2 == 0 else 1
        if world % cfg:
            raise ValueError(f"world {world} is not divisible by the CFG split {cfg}")
        return Layout(world, rank, cfg)

    @property
    def sp(self) -> int:
        return self.world // self.cfg

    @property
    def sample(self) -> int:
        """CFG sample of this rank (0 = cond, 1 = uncond); -1 when every rank runs both."""
        return self.rank // self.sp if self.cfg == 2 else -1

    @property
    def sp_rank(self) -> int:
        return self.rank % self.sp

    def sp_groups(self) -> list[list[int]]:
        return [[c * self.sp + i for i in range(self.sp)] for c in range(self.cfg)]

    def cfg_groups(self) -> list[list[int]]:
        return [[c * self.sp + i for c in range(self.cfg)] for i in range(self.sp)]

    def tokens(self, t: int) -> tuple[int, int]:
        if t % self.sp:
            raise ValueError(f"{t} tokens do not split evenly over {self.sp} sequence-parallel ranks")
        n = t // self.sp
        return self.sp_rank * n, (self.sp_rank + 1) * n


def qkv_segments(dim: int, heads: int, sp: int, gated: bool) -> list[tuple[int, int]]:
    """(offset, width-per-destination) of q, k, v (and gate logits) in the packed
    (T, 3D + H) projection: destination j gets heads [j*H/sp, (j+1)*H/sp)."""
    segs = [(0, dim // sp), (dim, dim // sp), (2 * dim, dim // sp)]
    if gated:
        segs.append((3 * dim, heads // sp))
    return segs


class SequenceParallel:
    """Self-attention replacement installed as `model._sp` (see LTXModel._self_and_text)."""

    def __init__(self, group, size: int):
        self.group = group
        self.size = size

    def self_attention(self, attn, qkv: torch.Tensor, st) -> torch.Tensor:
        p = self.size
        heads, d = attn.heads, attn.dim_head
        dim = heads * d
        if heads % p:
            raise ValueError(f"{heads} heads do not split over {p} ranks")
        gated = attn.to_gate_logits is not None
        segs = qkv_segments(dim, heads, p, gated)
        w = sum(s[1] for s in segs)
        if w % 8:
            raise ValueError("the per-rank q/k/v/gate row must be a multiple of 8 elements")
        dp, hp = dim // p, heads // p
        rows = st.T
        t_full = rows * p
        o = torch.empty(st.B * rows, dim, device=qkv.device, dtype=qkv.dtype)
        for b in range(st.B):
            src = qkv[b * rows:(b + 1) * rows]
            send = torch.empty(p, rows, w, device=qkv.device, dtype=qkv.dtype)
            nat.sp_pack(src, p, segs, send)
            recv = torch.empty(t_full, w, device=qkv.device, dtype=qkv.dtype)
            dist.all_to_all_single(recv, send.view(t_full, w), group=self.group)
            out = torch.empty(t_full, dp, device=qkv.device, dtype=qkv.dtype)
            nat.attention(recv[:, :dp], recv[:, dp:2 * dp], recv[:, 2 * dp:3 * dp], out, 1, t_full, t_full, hp, d,
                          d ** -0.5, recv[:, 3 * dp:3 * dp + hp] if gated else None)
            back = torch.empty(t_full, dp, device=qkv.device, dtype=qkv.dtype)
            dist.all_to_all_single(back, out, group=self.group)
            nat.sp_unpack(back.view(p, rows, dp), p, o[b * rows:(b + 1) * rows])
        return o


class ParallelDenoiser:
    """CFG x SP execution of ltx_dit.cfg_denoise_step across the default process group."""

    def __init__(self, model: ltx_dit.LTXModel, cfg_split: int | None = None):
        self.model = model
        self.layout = Layout.make(dist.get_world_size(), dist.get_rank(), cfg_split)
        lay = self.layout
        self.sp_group = self.cfg_group = None
        for ranks in lay.sp_groups():  # every rank creates every group, in the same order
            g = dist.new_group(ranks)
            if lay.rank in ranks:
                self.sp_group = g
        for ranks in lay.cfg_groups():
            g = dist.new_group(ranks)
            if lay.rank in ranks:
                self.cfg_group = g
        model._sp = SequenceParallel(self.sp_group, lay.sp) if lay.sp > 1 else None

    @torch.inference_mode()
    def step(self, latent: torch.Tensor, positions: torch.Tensor, context_pos: torch.Tensor,
             context_neg: torch.Tensor, sigmas: torch.Tensor, idx: int, cfg_scale: float,
             keyframes_mask: torch.Tensor | None = None) -> torch.Tensor:
        """latent (1, T, C) (identical on every rank) -> next latent (1, T, C) on every rank."""
        lay, model = self.layout, self.model
        dtype = model.proj_out.weight.dtype
        dev = latent.device
        _, t, c = latent.shape
        t0, t1 = lay.tokens(t)
        tl = t1 - t0
        sigma, sigma_next = ltx_dit._sigma_pair(sigmas, idx)
        nb = 1 if lay.cfg == 2 else 2
        lat_l = latent[:, t0:t1].to(dtype)
        if lay.cfg == 2:
            ctx = context_pos if lay.sample == 0 else context_neg
        else:
            ctx = model.cached_cat(context_pos, context_neg, dtype)
        video = ltx_dit.Modality(
            latent=lat_l.expand(nb, -1, -1), sigma=torch.full((nb,), sigma, device=dev),
            timesteps=torch.full((nb, tl, 1), sigma, device=dev), positions=positions[:, :, t0:t1].expand(nb, -1, -1, -1),
            context=ctx.to(dtype),
            keyframes_mask=keyframes_mask[:, t0:t1].expand(nb, -1, -1) if keyframes_mask is not None else None)
        va, _ = model.prepare(video, None, uniform_timesteps=True)
        model.run_blocks(va, None)
        h = model.head_hidden(va)
        vel_l = torch.empty(nb * tl, c, device=dev, dtype=dtype)
        nat.linear(h, model.proj_out.weight, vel_l, nat.epilogue(bias=model.proj_out.bias))
        if lay.cfg == 2:
            vel = torch.empty(2 * tl, c, device=dev, dtype=dtype)
            dist.all_gather_into_tensor(vel, vel_l, group=self.cfg_group)
        else:
            vel = vel_l
        ts = torch.full((2, tl), sigma, device=dev, dtype=torch.float32)
        nxt_l = torch.empty(tl, c, device=dev, dtype=dtype)
        nat.cfg_euler(vel, lat_l.reshape(tl, c).contiguous(), ts, cfg_scale, sigma, sigma_next, nxt_l)
        if lay.sp == 1:
            return nxt_l.view(1, t, c)
        nxt = torch.empty(t, c, device=dev, dtype=dtype)
        dist.all_gather_into_tensor(nxt, nxt_l, group=self.sp_group)
        return nxt.view(1, t, c)
