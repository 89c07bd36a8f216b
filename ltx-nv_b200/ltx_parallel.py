"""Multi-GPU denoise step: CFG split x Ulysses sequence parallelism.

One process per GPU. The world of W ranks is split into `cfg` CFG groups (2 when W >= 2:
cond on the first W/2 ranks, uncond on the rest) of `sp = W / cfg` ranks each. Inside a
CFG group the latent's T tokens are sharded contiguously over the sp ranks; everything
except self-attention is token-local (GEMMs, norms, FFN, text cross-attention against
the replicated text context). Self-attention runs Ulysses-style:

    QKV(+gate) GEMM on local tokens -> q/k RMSNorm + RoPE (needs all heads of a token)
    -> exchange (tokens -> heads) -> tcgen05 attention over all T tokens for the rank's
    H/sp heads -> exchange back (heads -> tokens) -> out GEMM

On one node the exchange runs inside the kernels over NVLink peer memory (PeerExchange):
the q/k kernel stores each row's head blocks into the receive buffer of the rank owning
those heads, the attention epilogue stores each output row into the buffer of the rank
owning the token, and a flag barrier separates writers from readers; kernels only store
to peer memory and read local memory. Otherwise (exchange="nccl") it is ltx_sp_pack ->
NCCL all_to_all -> attention -> all_to_all -> ltx_sp_unpack.

The step ends with one all_gather of the (T/sp, 128) velocity inside each CFG pair (the
X0 + CFG + Euler update needs cond and uncond of the same tokens) and one all_gather of
the next latent's shards inside each SP group, so every rank holds the full next latent.
Each rank runs the same kernels on the same rows as the single-GPU step: with attention
running every (sample, head, 256-query) unit whole the result equals the single-GPU
result bit for bit; the attention tail split makes other units split on a rank than on
one GPU, which changes the result by bf16 rounding only.

The audio-video model (step_av) keeps the audio stream (126 tokens) replicated on every
rank of a CFG group: audio-to-video attention reads the full audio keys locally, and
video-to-audio attention runs over the sharded video keys as split-KV partial attentions
(fp32 O / l and log2-sum-exp per row and head) merged after an all_gather.
"""

from __future__ import annotations

import os
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


class _CudaArray:
    """A device buffer of this process seen as a torch tensor (__cuda_array_interface__)."""

    def __init__(self, ptr: int, shape: tuple[int, ...], typestr: str):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False), "version": 2,
                                         "strides": None}


def _bf16_view(ptr: int, rows: int, cols: int, device: torch.device) -> torch.Tensor:
    return torch.as_tensor(_CudaArray(ptr, (rows, cols), "<i2"), device=device).view(torch.bfloat16)


class PeerExchange:
    """Buffers of the Ulysses exchange over NVLink peer memory for one SP group.

    Every rank allocates one buffer (nat.peer_alloc) laid out as
        [flags: one int per rank | counter | receive buffer (B*T, W) | output (B*T/P, D)]
    and maps the others' through CUDA IPC handles gathered over the group. The q/k pass
    stores each row's head blocks into the owners' receive buffers, the attention
    epilogue stores each output row into its token owner's output buffer, and
    nat.sp_barrier separates writers from readers. Buffers are made per shape on first
    use (outside any graph capture) and kept until close()."""

    def __init__(self, group, size: int, rank: int, device: torch.device):
        self.group, self.size, self.rank, self.device = group, size, rank, device
        self._bufs: dict[tuple, dict] = {}

    def get(self, batch: int, rows: int, width: int, dim: int) -> dict:
        key = (batch, rows, width, dim)
        if key in self._bufs:
            return self._bufs[key]
        t_full = rows * self.size
        head = 512  # flags and counter
        recv_bytes = batch * t_full * width * 2
        out_off = head + (recv_bytes + 255) // 256 * 256
        total = out_off + batch * rows * dim * 2
        ptr, handle = nat.peer_alloc(total)
        handles = [None] * self.size
        dist.all_gather_object(handles, handle, group=self.group)
        bases = [ptr if j == self.rank else nat.peer_open(handles[j]) for j in range(self.size)]
        buf = {"own": ptr, "bases": bases, "flags": list(bases), "counter": ptr + 256,
               "recv": [b + head for b in bases], "out": [b + out_off for b in bases],
               "recv_local": _bf16_view(ptr + head, batch * t_full, width, self.device),
               "out_local": _bf16_view(ptr + out_off, batch * rows, dim, self.device)}
        self._bufs[key] = buf
        return buf

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (call on every rank, after a
        barrier, with no exchange in flight)."""
        for buf in self._bufs.values():
            for j, b in enumerate(buf["bases"]):
                if j != self.rank:
                    nat.peer_close(b)
            nat.peer_free(buf["own"])
        self._bufs.clear()


class SequenceParallel:
    """Self-attention replacement installed as `model._sp` (see LTXModel._self_and_text)."""

    def __init__(self, group, size: int, exchange: PeerExchange | None = None):
        self.group = group
        self.size = size
        self.exchange = exchange

    def fused_for(self, attn, st) -> bool:
        """Whether this self-attention runs the fused peer-memory exchange."""
        if self.exchange is None or st.x.dtype != torch.bfloat16 or attn.dim_head not in (64, 128):
            return False
        heads = attn.heads
        if heads % self.size or (heads // self.size) % 8 or (heads * attn.dim_head // 16) % 32 \
                or heads * attn.dim_head // 16 > 128 or st.T * self.size <= 128:
            return False
        return st.pe is None or st.pe.heads == heads

    def self_attention_fused(self, attn, qkv: torch.Tensor, st) -> torch.Tensor:
        """q/k RMSNorm + RoPE with the rows sent to their heads' owners, a barrier, attention
        over all tokens of this rank's heads with each output row sent to its token's
        owner, a barrier: returns this rank's (B*T, D) attention output."""
        p, heads, d = self.size, attn.heads, attn.dim_head
        dim, hp = heads * d, heads // p
        dp = hp * d
        gated = attn.to_gate_logits is not None
        width = (3 * dp + (hp if gated else 0) + 7) // 8 * 8
        ex = self.exchange
        buf = ex.get(st.B, st.T, width, dim)
        pe = st.pe
        cos = sin = None
        ld_batch = 0
        if pe is not None:
            cos = pe.cos.view(-1, dim // 2) if pe.cos.dim() == 3 else pe.cos
            sin = pe.sin.view(-1, dim // 2) if pe.sin.dim() == 3 else pe.sin
            ld_batch = pe.ld_batch
        nat.qk_norm_rope_scatter(qkv, st.T, heads, d, attn.q_norm.weight, attn.k_norm.weight, attn.norm_eps, cos, sin,
                                 gated, ex.rank, buf["recv"], width, rope_ld_batch=ld_batch)
        nat.sp_barrier(buf["flags"], buf["counter"], ex.rank)
        recv = buf["recv_local"]
        t_full = st.T * p
        nat.attention_scatter(recv[:, :dp], recv[:, dp:2 * dp], recv[:, 2 * dp:3 * dp], st.B, t_full, hp, d,
                              d ** -0.5, recv[:, 3 * dp:3 * dp + hp] if gated else None, buf["out"], dim, ex.rank * dp)
        nat.sp_barrier(buf["flags"], buf["counter"], ex.rank)
        return buf["out_local"]

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

    def __init__(self, model: ltx_dit.LTXModel, cfg_split: int | None = None, exchange: str = "auto"):
        """exchange: "peer" runs the Ulysses exchange inside the q/k and attention kernels
        over NVLink peer memory (one node, NCCL process group), "nccl" as pack +
        all_to_all + unpack; "auto" picks "peer" when the whole group is on one node."""
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
        if exchange not in ("auto", "peer", "nccl"):
            raise ValueError(f"unknown exchange {exchange!r}")
        one_node = int(os.environ.get("LOCAL_WORLD_SIZE", lay.world)) == lay.world
        use_peer = lay.sp > 1 and (exchange == "peer" or (
            exchange == "auto" and one_node and dist.get_backend() == "nccl" and torch.cuda.is_available()))
        self.exchange = PeerExchange(self.sp_group, lay.sp, lay.sp_rank,
                                     torch.device("cuda", torch.cuda.current_device())) if use_peer else None
        self.exchange_kind = "peer" if use_peer else ("nccl" if lay.sp > 1 else "none")
        model._sp = SequenceParallel(self.sp_group, lay.sp, self.exchange) if lay.sp > 1 else None

    def close(self) -> None:
        """Release the peer-memory exchange (every rank; no step in flight)."""
        if self.exchange is not None:
            torch.cuda.synchronize()
            dist.barrier()
            self.exchange.close()
            self.exchange = None
            if self.model._sp is not None:
                self.model._sp.exchange = None

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
