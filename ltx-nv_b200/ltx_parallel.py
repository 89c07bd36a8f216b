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

The audio-video model (step_av) keeps the audio stream (126 tokens) replicated on every
rank of a CFG group: audio-to-video attention reads the full audio keys locally, and
video-to-audio attention runs over the sharded video keys as split-KV partial attentions
(fp32 O / l and log2-sum-exp per row and head) merged after an all_gather.

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

    def split_kv_attention(self, attn, qg: torch.Tensor, kv: torch.Tensor, batch: int, tq: int, tk_local: int,
                           gated: bool) -> torch.Tensor:
        """Attention of replicated queries qg (B*Tq, >= H*d (+H gate logits)) over keys and
        values sharded over the SP group (kv (B*Tk_local, 2*H*d) on each rank): partial
        attention over the local keys (fp32 O / l and log2-sum-exp per row and head), an
        all_gather of the partials, and the exact softmax merge with the gate applied.
        Every rank ends with the same (B*Tq, H*d) output."""
        heads, d = attn.heads, attn.dim_head
        inner = heads * d
        rows = batch * tq
        dev = qg.device
        o_part = torch.empty(rows, inner, device=dev, dtype=torch.float32)
        lse = torch.empty(rows, heads, device=dev, dtype=torch.float32)
        nat.attention_partial(qg[:, :inner], kv[:, :inner], kv[:, inner:2 * inner], o_part, lse, batch, tq, tk_local,
                              heads, d, d ** -0.5)
        o_all = torch.empty(self.size * rows, inner, device=dev, dtype=torch.float32)
        lse_all = torch.empty(self.size * rows, heads, device=dev, dtype=torch.float32)
        dist.all_gather_into_tensor(o_all, o_part, group=self.group)
        dist.all_gather_into_tensor(lse_all, lse, group=self.group)
        o = torch.empty(rows, inner, device=dev, dtype=qg.dtype)
        nat.attention_merge(o_all.view(self.size, rows, inner), lse_all.view(self.size, rows, heads),
                            qg[:, inner:inner + heads] if gated else None, o, heads, d)
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

    @torch.inference_mode()
    def step_av(self, v_latent: torch.Tensor, a_latent: torch.Tensor, v_positions: torch.Tensor,
                a_positions: torch.Tensor, v_context_pos: torch.Tensor, v_context_neg: torch.Tensor,
                a_context_pos: torch.Tensor, a_context_neg: torch.Tensor, sigmas: torch.Tensor, idx: int,
                cfg_scale: float, v_keyframes_mask: torch.Tensor | None = None):
        """ltx_dit.av_cfg_denoise_step across the process group: the video tokens are
        sharded over the SP ranks as in step(); the audio stream (126 tokens) is
        replicated on every rank of a CFG group, audio-to-video attention reads the full
        audio keys locally, and video-to-audio attention merges partial attentions over the
        sharded video keys (SequenceParallel.split_kv_attention). Returns the next video
        latent (1, Tv, C) and the next audio latent (1, Ta, C) on every rank."""
        lay, model = self.layout, self.model
        dtype = model.proj_out.weight.dtype
        dev = v_latent.device
        _, tv, c = v_latent.shape
        ta = a_latent.shape[1]
        t0, t1 = lay.tokens(tv)
        tl = t1 - t0
        sigma, sigma_next = ltx_dit._sigma_pair(sigmas, idx)
        nb = 1 if lay.cfg == 2 else 2

        def ctx_of(cpos, cneg):
            if lay.cfg == 2:
                return (cpos if lay.sample == 0 else cneg).to(dtype)
            return torch.cat([cpos, cneg], dim=0).to(dtype)

        sig = torch.full((nb,), sigma, device=dev)
        vlat_l = v_latent[:, t0:t1].to(dtype)
        video = ltx_dit.Modality(
            latent=vlat_l.expand(nb, -1, -1), sigma=sig, timesteps=torch.full((nb, tl, 1), sigma, device=dev),
            positions=v_positions[:, :, t0:t1].expand(nb, -1, -1, -1), context=ctx_of(v_context_pos, v_context_neg),
            keyframes_mask=v_keyframes_mask[:, t0:t1].expand(nb, -1, -1) if v_keyframes_mask is not None else None)
        alat = a_latent.to(dtype)
        audio = ltx_dit.Modality(latent=alat.expand(nb, -1, -1), sigma=sig,
                                 timesteps=torch.full((nb, ta, 1), sigma, device=dev),
                                 positions=a_positions.expand(nb, -1, -1, -1),
                                 context=ctx_of(a_context_pos, a_context_neg))
        va, aa = model.prepare(video, audio, uniform_timesteps=True)
        model.run_blocks(va, aa)
        outs = []
        for st, lat2, proj, rows, group_gather in ((va, vlat_l.reshape(tl, c), model.proj_out, tl, True),
                                                   (aa, alat.reshape(ta, c), model.audio_proj_out, ta, False)):
            h = model.head_hidden(st)
            vel_l = torch.empty(nb * rows, c, device=dev, dtype=dtype)
            nat.linear(h, proj.weight, vel_l, nat.epilogue(bias=proj.bias))
            if lay.cfg == 2:
                vel = torch.empty(2 * rows, c, device=dev, dtype=dtype)
                dist.all_gather_into_tensor(vel, vel_l, group=self.cfg_group)
            else:
                vel = vel_l
            ts = torch.full((2, rows), sigma, device=dev, dtype=torch.float32)
            nxt_l = torch.empty(rows, c, device=dev, dtype=dtype)
            nat.cfg_euler(vel, lat2.contiguous(), ts, cfg_scale, sigma, sigma_next, nxt_l)
            if group_gather and lay.sp > 1:
                nxt = torch.empty(tv, c, device=dev, dtype=dtype)
                dist.all_gather_into_tensor(nxt, nxt_l, group=self.sp_group)
                outs.append(nxt.view(1, tv, c))
            else:
                outs.append(nxt_l.view(1, rows, c))
        return outs[0], outs[1]
