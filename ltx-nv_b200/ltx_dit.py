"""B200-native LTX-2.5 DiT denoising step (drop-in for lipaul/ltx-nv standalone/ltx_dit.py).

Same public names and signatures as the reference module: DiTConfig, Modality,
LTXModel(cfg).forward(video, audio, perturbations) -> (vx, ax), load_transformer,
video_positions / audio_positions, (un)patchify_*, LatentState, create_noised_states,
ltx2_scheduler_sigmas, GuiderParams, guide, euler_step, guided_denoise_step, run_dit,
build_perturbation_config. The parameters of LTXModel have the reference's names,
shapes and registration order, so its state dicts and checkpoints load unchanged.

What runs underneath: every op of the forward is a libltxb200 sm_100a kernel called
through _native (no cuBLAS, no cuDNN, no torch element-wise math on the path):
  patchify  tcgen05 GEMM (+ keyframe add in the epilogue)
  adaLN     weight-streaming GEMMs on one row per sample (timesteps are uniform over
            tokens in every denoise step; a per-token path exists for general masks)
  block     norm+modulate -> packed QKV(+gate) GEMM -> q/k RMSNorm+RoPE -> tcgen05
            attention (gate fused) -> out GEMM with gate*out+residual epilogue;
            the same for text cross-attention and A<->V attention; norm+modulate ->
            FFN-in GEMM with GELU epilogue -> FFN-out GEMM with gated residual epilogue
  head      LayerNorm+modulate -> proj_out GEMM; in cfg_denoise_step the proj_out
            epilogue also applies X0 + CFG + Euler and writes the next latent.
Activations are (B*T, D) row-major buffers in HBM; the residual stream is updated in
place by the GEMM epilogues.

Guidance: cfg_denoise_step is the fused CFG-only step (B=2, X0 + CFG + Euler in the
proj_out epilogue). guided_denoise_step / run_dit run the reference's full guidance: one
B=4 forward over [cond, uncond, STG-perturbed, modality-isolated] (perturbed
self-attention outputs V, ltx_value_gate; isolated samples skip the A<->V residual
update), X0, and the blend with the two-pass std rescale (ltx_guide_rescale).
"""

from __future__ import annotations

import json
import math
import time
from dataclasses import dataclass, replace

import torch

import _native as nat
from ltx_nn import AdaLayerNormSingle, Attention, FeedForward, RopeTables, rope_tables

DEVICE = torch.device("cuda")


def _version(t: torch.Tensor) -> int:
    """In-place modification counter of a tensor; -1 for inference-mode tensors, which do
    not track one (the caches below then rely on the documented contract that positions
    and text contexts are not modified in place while a model reuses them)."""
    try:
        return t._version
    except RuntimeError:
        return -1

# ---------------------------------------------------------------------------------------
# Config (ltx_dit.py:28-82)
# ---------------------------------------------------------------------------------------


@dataclass(frozen=True)
class DiTConfig:
    num_layers: int = 48
    video_heads: int = 32
    video_head_dim: int = 128
    video_in: int = 128
    video_out: int = 128
    video_cross_dim: int = 4096
    audio_heads: int = 32
    audio_head_dim: int = 64
    audio_in: int = 128
    audio_out: int = 128
    audio_cross_dim: int = 2048
    norm_eps: float = 1e-6
    theta: float = 10000.0
    video_max_pos: tuple = (20, 2048, 2048)
    audio_max_pos: tuple = (20,)
    timestep_scale_multiplier: int = 1000
    av_ca_timestep_scale_multiplier: float = 1000.0
    double_rope: bool = True
    gated_attention: bool = True
    cross_attention_adaln: bool = True
    ff_bias: bool = False
    audio_ff_bias: bool = True
    use_keyframes: bool = True

    @staticmethod
    def from_checkpoint(transformer_path: str) -> "DiTConfig":
        """Read the transformer config from a safetensors file's metadata (ltx_dit.py:54-73)."""
        from safetensors import safe_open

        with safe_open(transformer_path, framework="pt") as f:
            meta = f.metadata() or {}
        c = json.loads(meta["config"])["transformer"]
        return DiTConfig(
            num_layers=c["num_layers"], video_heads=c["num_attention_heads"],
            video_head_dim=c["attention_head_dim"], video_in=c["in_channels"], video_out=c["out_channels"],
            video_cross_dim=c["cross_attention_dim"], audio_heads=c["audio_num_attention_heads"],
            audio_head_dim=c["audio_attention_head_dim"], audio_in=c.get("audio_in_channels", 128),
            audio_out=c["audio_out_channels"], audio_cross_dim=c["audio_cross_attention_dim"],
            norm_eps=c["norm_eps"], theta=c["positional_embedding_theta"],
            video_max_pos=tuple(c["positional_embedding_max_pos"]),
            audio_max_pos=tuple(c["audio_positional_embedding_max_pos"]),
            timestep_scale_multiplier=c["timestep_scale_multiplier"],
            av_ca_timestep_scale_multiplier=c["av_ca_timestep_scale_multiplier"],
            double_rope=c.get("frequencies_precision", False) == "float64",
            gated_attention=c.get("apply_gated_attention", False),
            cross_attention_adaln=c.get("cross_attention_adaln", False),
            ff_bias=c.get("ff_bias", True), audio_ff_bias=c.get("audio_ff_bias", True),
            use_keyframes=c.get("use_keyframes_abs_pos_embedding", False),
        )

    @staticmethod
    def video_only(num_layers: int, heads: int, head_dim: int, cross_dim: int) -> "DiTConfig":
        """Video-only DiT (3, 5): text cross-attention without
        cross-adaLN, and a minimal audio stream that is never run (its parameters exist
        only so the state dict matches the reference's AV model)."""
        return DiTConfig(num_layers=num_layers, video_heads=heads, video_head_dim=head_dim, video_cross_dim=cross_dim,
                         audio_heads=2, audio_head_dim=32, audio_cross_dim=max(2 * heads, 64),
                         cross_attention_adaln=False)

    @property
    def video_dim(self) -> int:
        return self.video_heads * self.video_head_dim

    @property
    def audio_dim(self) -> int:
        return self.audio_heads * self.audio_head_dim


# ---------------------------------------------------------------------------------------
# Per-modality inputs (ltx_dit.py:89-117)
# ---------------------------------------------------------------------------------------


@dataclass
class Modality:
    latent: torch.Tensor  # (B, T, 128) patchified
    sigma: torch.Tensor  # (B,)
    timesteps: torch.Tensor  # (B, T, 1) = denoise_mask * sigma
    positions: torch.Tensor  # video (B,3,T,2) pixel-space bounds; audio (B,1,T,2) seconds
    context: torch.Tensor  # (B, S, cross_dim) text encoding
    keyframes_mask: torch.Tensor | None = None  # (B, T, 1)
    enabled: bool = True


@dataclass
class _Stream:
    """Prepared state of one stream for the block loop (the reference's TransformerArgs)."""

    name: str
    B: int
    T: int
    D: int
    heads: int
    head_dim: int
    x: torch.Tensor  # (B*T, D) residual stream
    tmod: torch.Tensor  # (N, n*D) timestep modulation, N = B (per sample) or B*T
    tmod_ld_tok: int
    emb: torch.Tensor  # (N, D) embedded timestep
    prompt_mod: torch.Tensor | None  # (B, 2D)
    context: torch.Tensor  # (B*S, C)
    S: int
    pe: RopeTables
    cross_pe: RopeTables | None
    cross_ss: torch.Tensor | None  # (N, 4D)
    cross_gate: torch.Tensor | None  # (B, D)
    enabled: bool
    context_src: torch.Tensor | None = None  # the caller's context tensor (cache identity)

    def mod(self, table: torch.Tensor, tmod: torch.Tensor, shift: int | None, scale: int | None,
            n_total: int | None = None, ld_tok: int | None = None) -> nat.Modulation:
        """Modulation from rows `shift` / `scale` of an adaLN table (n, D) and the
        matching slices of a (N, n*D) timestep modulation."""
        d = table.shape[-1]
        ld_row = tmod.shape[-1]
        per_tok = self.tmod_ld_tok if ld_tok is None else ld_tok
        return nat.modulation(table, tmod,
                              shift=(shift * d, shift * d) if shift is not None else None,
                              scale=(scale * d, scale * d) if scale is not None else None,
                              mod_ld_batch=ld_row * (self.T if per_tok else 1), mod_ld_tok=ld_row if per_tok else 0)


# ---------------------------------------------------------------------------------------
# Model (ltx_dit.py:209-378)
# ---------------------------------------------------------------------------------------


class Block(torch.nn.Module):
    """BasicAVTransformerBlock parameters (ltx_dit.py:209-235)."""

    def __init__(self, cfg: DiTConfig):
        super().__init__()
        v, a = cfg.video_dim, cfg.audio_dim
        n_ca = 9 if cfg.cross_attention_adaln else 6
        self.attn1 = Attention(v, None, cfg.video_heads, cfg.video_head_dim, cfg.norm_eps, cfg.gated_attention)
        self.attn2 = Attention(v, cfg.video_cross_dim, cfg.video_heads, cfg.video_head_dim, cfg.norm_eps,
                               cfg.gated_attention)
        self.ff = FeedForward(v, v, bias=cfg.ff_bias)
        self.scale_shift_table = torch.nn.Parameter(torch.empty(n_ca, v))
        self.audio_attn1 = Attention(a, None, cfg.audio_heads, cfg.audio_head_dim, cfg.norm_eps, cfg.gated_attention)
        self.audio_attn2 = Attention(a, cfg.audio_cross_dim, cfg.audio_heads, cfg.audio_head_dim, cfg.norm_eps,
                                     cfg.gated_attention)
        self.audio_ff = FeedForward(a, a, bias=cfg.audio_ff_bias)
        self.audio_scale_shift_table = torch.nn.Parameter(torch.empty(n_ca, a))
        self.audio_to_video_attn = Attention(v, a, cfg.audio_heads, cfg.audio_head_dim, cfg.norm_eps,
                                             cfg.gated_attention)
        self.video_to_audio_attn = Attention(a, v, cfg.audio_heads, cfg.audio_head_dim, cfg.norm_eps,
                                             cfg.gated_attention)
        self.scale_shift_table_a2v_ca_audio = torch.nn.Parameter(torch.empty(5, a))
        self.scale_shift_table_a2v_ca_video = torch.nn.Parameter(torch.empty(5, v))
        if cfg.cross_attention_adaln:
            self.prompt_scale_shift_table = torch.nn.Parameter(torch.empty(2, v))
            self.audio_prompt_scale_shift_table = torch.nn.Parameter(torch.empty(2, a))


class LTXModel(torch.nn.Module):
    """LTX-2.5 AV transformer (ltx_dit.py:325-378) executed by libltxb200 kernels."""

    def __init__(self, cfg: DiTConfig):
        super().__init__()
        self.cfg = cfg
        v, a = cfg.video_dim, cfg.audio_dim
        n_adaln = 9 if cfg.cross_attention_adaln else 6
        self.patchify_proj = torch.nn.Linear(cfg.video_in, v, bias=True)
        self.keyframes_abs_pos_embedding = torch.nn.Parameter(torch.zeros(1, v)) if cfg.use_keyframes else None
        self.adaln_single = AdaLayerNormSingle(v, n_adaln)
        self.prompt_adaln_single = AdaLayerNormSingle(v, 2) if cfg.cross_attention_adaln else None
        self.scale_shift_table = torch.nn.Parameter(torch.empty(2, v))
        self.norm_out = torch.nn.LayerNorm(v, elementwise_affine=False, eps=cfg.norm_eps)
        self.proj_out = torch.nn.Linear(v, cfg.video_out)
        self.audio_patchify_proj = torch.nn.Linear(cfg.audio_in, a, bias=True)
        self.audio_adaln_single = AdaLayerNormSingle(a, n_adaln)
        self.audio_prompt_adaln_single = AdaLayerNormSingle(a, 2) if cfg.cross_attention_adaln else None
        self.audio_scale_shift_table = torch.nn.Parameter(torch.empty(2, a))
        self.audio_norm_out = torch.nn.LayerNorm(a, elementwise_affine=False, eps=cfg.norm_eps)
        self.audio_proj_out = torch.nn.Linear(a, cfg.audio_out)
        self.av_ca_video_scale_shift_adaln_single = AdaLayerNormSingle(v, 4)
        self.av_ca_audio_scale_shift_adaln_single = AdaLayerNormSingle(a, 4)
        self.av_ca_a2v_gate_adaln_single = AdaLayerNormSingle(v, 1)
        self.av_ca_v2a_gate_adaln_single = AdaLayerNormSingle(a, 1)
        self.blocks = torch.nn.ModuleList([Block(cfg) for _ in range(cfg.num_layers)])
        self._rope_cache: dict = {}
        self._kv_cache: dict = {}
        self._cat_cache = None
        self._sp = None  # ltx_parallel.SequenceParallel when the video tokens are sharded

    # ------------------------------------------------------------------ preparation
    def _rope(self, positions: torch.Tensor, dim: int, dtype: torch.dtype, max_pos: list, heads: int) -> RopeTables:
        """RoPE tables, cached per positions tensor (positions are constant across the
        denoise steps). The entry keeps a reference to the positions storage, so a new
        tensor cannot reuse its address while the entry lives."""
        key = (positions.data_ptr(), _version(positions), tuple(positions.shape), tuple(positions.stride()), dim,
               dtype, tuple(max_pos), heads)
        hit = self._rope_cache.get(key)
        if hit is None:
            if len(self._rope_cache) > 16:
                self._rope_cache.clear()
            tabs = rope_tables(positions, dim, dtype, self.cfg.theta, max_pos, heads, self.cfg.double_rope)
            hit = (positions, tabs)
            self._rope_cache[key] = hit
        return hit[1]

    def _text_kv(self, attn: Attention, ctx: torch.Tensor, rows: int, src: torch.Tensor) -> torch.Tensor:
        """K/V projection of the text context with the k RMSNorm applied. Without
        cross-adaLN it depends only on the context and the weights, both constant across
        the denoise steps, so it is cached per (module, caller's context tensor `src`,
        weights); the entry keeps `src` alive so its address cannot be reused."""
        inner = attn.heads * attn.dim_head
        wkv, bkv = attn.packed_kv()
        key = id(attn)
        hit = self._kv_cache.get(key)
        if hit is not None:
            c_ref, c_ver, shape, w_ptr, kv = hit
            if c_ref is src and c_ver == _version(src) and shape == tuple(ctx.shape) and w_ptr == wkv.data_ptr():
                return kv
        kv = torch.empty(ctx.shape[0], wkv.shape[0], device=ctx.device, dtype=ctx.dtype)
        nat.linear(ctx, wkv, kv, nat.epilogue(bias=bkv))
        attn._norm_rope(kv[:, :inner], rows, attn.k_norm.weight, None)
        self._kv_cache[key] = (src, _version(src), tuple(ctx.shape), wkv.data_ptr(), kv)
        return kv

    def cached_cat(self, a: torch.Tensor, b: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
        """torch.cat([a, b]).to(dtype), reused while a and b are unchanged (the CFG
        context pair is constant across the denoise loop)."""
        c = self._cat_cache
        if c is not None and c[0] is a and c[1] is b and c[2] == (_version(a), _version(b), dtype):
            return c[3]
        out = torch.cat([a, b], dim=0).to(dtype).contiguous()
        self._cat_cache = (a, b, (_version(a), _version(b), dtype), out)
        return out

    @staticmethod
    def _per_sample_timesteps(ts: torch.Tensor) -> torch.Tensor | None:
        """(B,) timesteps when every token of a sample shares its timestep, else None."""
        first = ts[:, :1]
        if bool((ts == first).all()):
            return first.reshape(ts.shape[0]).to(torch.float32).contiguous()
        return None

    def _prepare(self, stream: str, m: Modality, cross: Modality | None, uniform_timesteps: bool = False) -> _Stream:
        """ArgsPreprocessor.prepare (ltx_dit.py:131-184). `uniform_timesteps` asserts that
        every token of a sample has the same timestep (a full denoise mask), which skips
        the device-to-host check."""
        cfg = self.cfg
        a = stream == "audio"
        patch = self.audio_patchify_proj if a else self.patchify_proj
        adaln = self.audio_adaln_single if a else self.adaln_single
        prompt_adaln = self.audio_prompt_adaln_single if a else self.prompt_adaln_single
        dim = cfg.audio_dim if a else cfg.video_dim
        heads = cfg.audio_heads if a else cfg.video_heads
        hd = cfg.audio_head_dim if a else cfg.video_head_dim
        dtype = patch.weight.dtype
        b, t, cin = m.latent.shape
        lat = m.latent.to(dtype).reshape(b * t, cin).contiguous()
        x = torch.empty(b * t, dim, device=lat.device, dtype=dtype)
        kf = self.keyframes_abs_pos_embedding
        if not a and m.keyframes_mask is not None and kf is not None:
            mask = m.keyframes_mask.reshape(b * t).to(torch.float32).contiguous()
            nat.linear(lat, patch.weight, x, nat.epilogue(nat.EPI_ROW_MASK_ADD, bias=patch.bias, row_mask=mask,
                                                          row_vec=kf.reshape(-1)))
        else:
            nat.linear(lat, patch.weight, x, nat.epilogue(bias=patch.bias))
        scale = float(cfg.timestep_scale_multiplier)
        ts = m.timesteps.reshape(b, t).to(torch.float32)
        if uniform_timesteps:
            t_sample = ts[:, 0].contiguous()
        else:
            t_sample = self._per_sample_timesteps(ts)
        t_in = t_sample if t_sample is not None else ts.reshape(-1).contiguous()
        tmod, emb = adaln(t_in, dtype, scale)
        prompt = None
        if prompt_adaln is not None:
            prompt, _ = prompt_adaln(m.sigma.to(torch.float32).reshape(-1).contiguous(), dtype, scale)
        s_len = m.context.shape[1]
        context = m.context.to(dtype).reshape(b * s_len, -1).contiguous()
        max_pos = list(cfg.audio_max_pos if a else cfg.video_max_pos)
        pe = self._rope(m.positions, dim, dtype, max_pos, heads)
        cross_pe = cross_ss = cross_gate = None
        if cross is not None:
            cross_pe = self._rope(m.positions[:, 0:1], cfg.audio_cross_dim, dtype,
                                  [max(cfg.video_max_pos[0], cfg.audio_max_pos[0])], heads)
            ss_mod = self.av_ca_audio_scale_shift_adaln_single if a else self.av_ca_video_scale_shift_adaln_single
            g_mod = self.av_ca_v2a_gate_adaln_single if a else self.av_ca_a2v_gate_adaln_single
            cross_ss, _ = ss_mod(t_in, dtype, scale)
            factor = cfg.av_ca_timestep_scale_multiplier / cfg.timestep_scale_multiplier
            cross_gate, _ = g_mod(cross.sigma.to(torch.float32).reshape(-1).contiguous(), dtype, scale * factor)
        return _Stream(stream, b, t, dim, heads, hd, x, tmod, 0 if t_sample is not None else 1, emb, prompt,
                       context, s_len, pe, cross_pe, cross_ss, cross_gate, m.enabled, context_src=m.context)

    # ------------------------------------------------------------------ block pieces
    def _self_and_text(self, blk: Block, st: _Stream, h: torch.Tensor, keep_self: list | None = None):
        """Self-attention + text cross-attention of one stream (ltx_dit.py:259-282).
        keep_self: per-sample self-attention keep flags of this block (STG: 0 = the
        attention output is V, ltx_nn.py:209-210, 229-230)."""
        cfg = self.cfg
        a = st.name == "audio"
        attn1 = blk.audio_attn1 if a else blk.attn1
        attn2 = blk.audio_attn2 if a else blk.attn2
        table = blk.audio_scale_shift_table if a else blk.scale_shift_table
        d, eps, rows = st.D, cfg.norm_eps, st.B * st.T
        inner = attn1.heads * attn1.dim_head
        gated = cfg.gated_attention
        # self-attention
        nat.norm_modulate(st.x, h, st.T, nat.LTX_NORM_RMS, eps, st.mod(table, st.tmod, 0, 1))
        perturbed = [b for b, k in enumerate(keep_self) if k == 0] if keep_self is not None else []
        if self._sp is not None and not a and not perturbed and self._sp.fused_for(attn1, st):
            # sequence-parallel over peer memory: q/k normalisation fused into the exchange
            qkv = attn1.project_qkv(h, st.T, st.pe, normalize=False)
            o = self._sp.self_attention_fused(attn1, qkv, st)
            nat.linear(o, attn1.to_out.weight, st.x,
                       nat.epilogue(nat.EPI_GATE_RESIDUAL, bias=attn1.to_out.bias, residual=st.x,
                                    gate=st.mod(table, st.tmod, None, 2), rows_per_batch=st.T))
            return self._text_cross(blk, st, h, attn2, table, d, eps, rows, inner, gated)
        qkv = attn1.project_qkv(h, st.T, st.pe)
        v_cols = qkv[:, 2 * inner:3 * inner]
        g_cols = qkv[:, 3 * inner:3 * inner + attn1.heads] if gated else None
        if self._sp is not None and not a:
            # sequence-parallel: this rank holds st.T of the video tokens (ltx_parallel)
            if perturbed:
                raise NotImplementedError("STG perturbation under sequence parallelism")
            o = self._sp.self_attention(attn1, qkv, st)
        elif len(perturbed) == st.B:
            # every sample perturbed: no attention at all (ltx_nn.py:209-210)
            o = torch.empty(rows, inner, device=h.device, dtype=h.dtype)
            nat.value_gate(v_cols, g_cols, o, attn1.heads, attn1.dim_head)
        else:
            o = attn1.attend(qkv[:, :inner], qkv[:, inner:2 * inner], v_cols, g_cols, st.B, st.T, st.T)
            for b in perturbed:
                r0, r1 = b * st.T, (b + 1) * st.T
                nat.value_gate(v_cols[r0:r1], g_cols[r0:r1] if gated else None, o[r0:r1], attn1.heads,
                               attn1.dim_head)
        nat.linear(o, attn1.to_out.weight, st.x,
                   nat.epilogue(nat.EPI_GATE_RESIDUAL, bias=attn1.to_out.bias, residual=st.x,
                                gate=st.mod(table, st.tmod, None, 2), rows_per_batch=st.T))
        self._text_cross(blk, st, h, attn2, table, d, eps, rows, inner, gated)

    def _text_cross(self, blk: Block, st: _Stream, h: torch.Tensor, attn2, table, d: int, eps: float, rows: int,
                    inner: int, gated: bool):
        """Text cross-attention of one stream (ltx_dit.py:267-282)."""
        cfg = self.cfg
        a = st.name == "audio"
        # text cross-attention
        if cfg.cross_attention_adaln:
            nat.norm_modulate(st.x, h, st.T, nat.LTX_NORM_RMS, eps, st.mod(table, st.tmod, 6, 7))
        else:
            nat.norm_modulate(st.x, h, st.T, nat.LTX_NORM_RMS, eps, None)
        wq, bq = attn2.packed_q()
        qg = torch.empty(rows, wq.shape[0], device=h.device, dtype=h.dtype)
        nat.linear(h, wq, qg, nat.epilogue(bias=bq))
        attn2._norm_rope(qg[:, :inner], st.T, attn2.q_norm.weight, None)
        ctx = st.context
        if cfg.cross_attention_adaln:
            psst = blk.audio_prompt_scale_shift_table if a else blk.prompt_scale_shift_table
            if ctx.shape[1] != d:
                raise ValueError("cross-adaLN needs the text context width to equal the hidden size")
            enc = torch.empty_like(ctx)
            nat.norm_modulate(ctx, enc, st.S, nat.LTX_NORM_NONE, eps,
                              nat.modulation(psst, st.prompt_mod, shift=(0, 0), scale=(d, d),
                                             mod_ld_batch=st.prompt_mod.shape[-1]))
            wkv, bkv = attn2.packed_kv()
            kv = torch.empty(enc.shape[0], wkv.shape[0], device=h.device, dtype=h.dtype)
            nat.linear(enc, wkv, kv, nat.epilogue(bias=bkv))
            attn2._norm_rope(kv[:, :inner], st.S, attn2.k_norm.weight, None)
        else:
            kv = self._text_kv(attn2, ctx, st.S, st.context_src if st.context_src is not None else ctx)
        o = attn2.attend(qg[:, :inner], kv[:, :inner], kv[:, inner:2 * inner], qg[:, inner:] if gated else None,
                         st.B, st.T, st.S)
        gate = st.mod(table, st.tmod, None, 8) if cfg.cross_attention_adaln else None
        nat.linear(o, attn2.to_out.weight, st.x,
                   nat.epilogue(nat.EPI_GATE_RESIDUAL, bias=attn2.to_out.bias, residual=st.x, gate=gate,
                                rows_per_batch=st.T))

    def _ffn(self, blk: Block, st: _Stream, h: torch.Tensor):
        """Feed-forward with adaLN (ltx_dit.py:309-314)."""
        a = st.name == "audio"
        ff = blk.audio_ff if a else blk.ff
        table = blk.audio_scale_shift_table if a else blk.scale_shift_table
        nat.norm_modulate(st.x, h, st.T, nat.LTX_NORM_RMS, self.cfg.norm_eps, st.mod(table, st.tmod, 3, 4))
        f = torch.empty(st.B * st.T, ff.proj_in.out_features, device=h.device, dtype=h.dtype)
        nat.linear(h, ff.proj_in.weight, f, nat.epilogue(nat.EPI_GELU_TANH, bias=ff.proj_in.bias))
        nat.linear(f, ff.proj_out.weight, st.x,
                   nat.epilogue(nat.EPI_GATE_RESIDUAL, bias=ff.proj_out.bias, residual=st.x,
                                gate=st.mod(table, st.tmod, None, 5), rows_per_batch=st.T))

    def _av_cross(self, blk: Block, vs: _Stream, as_: _Stream, run_a2v: bool, run_v2a: bool,
                  keep_a2v: list | None = None, keep_v2a: list | None = None):
        """Audio<->video cross-attention (ltx_dit.py:284-307); both read the pre-AV states.
        keep_*: per-sample keep flags (modality isolation: 0 = the sample's update is
        skipped, which is what the reference's multiply by a 0 mask leaves)."""
        cfg = self.cfg
        eps = cfg.norm_eps
        tv, ta = blk.scale_shift_table_a2v_ca_video, blk.scale_shift_table_a2v_ca_audio

        def normed(st, table, rows_sl):
            out = torch.empty_like(st.x)
            # get_av_ca_ada_values returns (scale, shift) = table rows (r0, r0 + 1)
            r0 = rows_sl
            nat.norm_modulate(st.x, out, st.T, nat.LTX_NORM_RMS, eps, st.mod(table, st.cross_ss, r0 + 1, r0))
            return out

        def gate_of(st, table):
            d = table.shape[-1]
            return lambda b0: nat.modulation(table, st.cross_gate[b0:], shift=None, scale=(4 * d, 0), mod_ld_batch=d)

        a2v_v = normed(vs, tv, 0) if run_a2v else None
        a2v_a = normed(as_, ta, 0) if run_a2v else None
        v2a_a = normed(as_, ta, 2) if run_v2a else None
        v2a_v = normed(vs, tv, 2) if run_v2a else None
        if run_a2v:
            self._cross_attend(blk.audio_to_video_attn, a2v_v, vs, a2v_a, as_, vs.cross_pe, as_.cross_pe,
                               gate_of(vs, tv), vs, keep_a2v)
        if run_v2a:
            self._cross_attend(blk.video_to_audio_attn, v2a_a, as_, v2a_v, vs, as_.cross_pe, vs.cross_pe,
                               gate_of(as_, ta), as_, keep_v2a)

    def _cross_attend(self, attn: Attention, q_in, q_st: _Stream, kv_in, kv_st: _Stream, q_pe, k_pe, gate_at,
                      out_st: _Stream, keep: list | None = None):
        """gate_at(b0): the gate modulation seen from sample b0 on. The residual update
        runs over the runs of kept samples only."""
        inner = attn.heads * attn.dim_head
        gated = self.cfg.gated_attention
        wq, bq = attn.packed_q()
        qg = torch.empty(q_in.shape[0], wq.shape[0], device=q_in.device, dtype=q_in.dtype)
        nat.linear(q_in, wq, qg, nat.epilogue(bias=bq))
        attn._norm_rope(qg[:, :inner], q_st.T, attn.q_norm.weight, q_pe)
        wkv, bkv = attn.packed_kv()
        kv = torch.empty(kv_in.shape[0], wkv.shape[0], device=q_in.device, dtype=q_in.dtype)
        nat.linear(kv_in, wkv, kv, nat.epilogue(bias=bkv))
        attn._norm_rope(kv[:, :inner], kv_st.T, attn.k_norm.weight, k_pe)
        if self._sp is not None and kv_st.name == "video":
            # video-to-audio under sequence parallelism: the video keys are sharded over
            # the ranks, the audio queries are replicated -> split-KV attention merged
            # across the ranks (ltx_parallel)
            o = self._sp.split_kv_attention(attn, qg, kv, q_st.B, q_st.T, kv_st.T, gated)
        else:
            o = attn.attend(qg[:, :inner], kv[:, :inner], kv[:, inner:2 * inner], qg[:, inner:] if gated else None,
                            q_st.B, q_st.T, kv_st.T)
        runs, b = [], 0
        kept = keep if keep is not None else [1.0] * out_st.B
        while b < out_st.B:
            if kept[b] == 0:
                b += 1
                continue
            b0 = b
            while b < out_st.B and kept[b] != 0:
                b += 1
            runs.append((b0, b))
        t = out_st.T
        for b0, b1 in runs:
            x = out_st.x[b0 * t:b1 * t]
            nat.linear(o[b0 * t:b1 * t], attn.to_out.weight, x,
                       nat.epilogue(nat.EPI_GATE_RESIDUAL, bias=attn.to_out.bias, residual=x, gate=gate_at(b0),
                                    rows_per_batch=t))

    # ------------------------------------------------------------------ forward
    def _keep_masks(self, perturbations, batch: int):
        """Host copy of the (4, L, B) keep-mask (ltx_dit.py:381-411) as nested lists; None =
        all ones. Entries are 0 (perturbed / skipped) or 1, as build_perturbation_config
        makes them."""
        if perturbations is None:
            return None
        keep = perturbations.detach().to("cpu", torch.float32)
        if bool(((keep != 0) & (keep != 1)).any()):
            raise NotImplementedError("perturbation keep-masks other than 0 / 1")
        if keep.shape[-1] != batch:
            raise ValueError(f"perturbation batch {keep.shape[-1]} != model batch {batch}")
        return keep.tolist()

    def run_blocks(self, va: _Stream | None, aa: _Stream | None, perturbations=None):
        keep = self._keep_masks(perturbations, (va or aa).B)
        hv = torch.empty_like(va.x) if va is not None else None
        ha = torch.empty_like(aa.x) if aa is not None else None
        for i, blk in enumerate(self.blocks):
            run_v = va is not None and va.enabled and va.x.numel() > 0
            run_a = aa is not None and aa.enabled and aa.x.numel() > 0
            run_a2v = run_v and aa is not None and aa.x.numel() > 0
            run_v2a = run_a and va is not None and va.x.numel() > 0
            k_a2v = k_v2a = None
            if keep is not None:
                k_a2v, k_v2a = keep[2][i], keep[3][i]
                run_a2v = run_a2v and any(k != 0 for k in k_a2v)
                run_v2a = run_v2a and any(k != 0 for k in k_v2a)
            if run_v:
                self._self_and_text(blk, va, hv, keep[0][i] if keep is not None else None)
            if run_a:
                self._self_and_text(blk, aa, ha, keep[1][i] if keep is not None else None)
            if run_a2v or run_v2a:
                self._av_cross(blk, va, aa, run_a2v, run_v2a, k_a2v, k_v2a)
            if run_v:
                self._ffn(blk, va, hv)
            if run_a:
                self._ffn(blk, aa, ha)

    def head_hidden(self, st: _Stream) -> torch.Tensor:
        """LayerNorm + (1 + scale) / shift of the output head (ltx_dit.py:371-377)."""
        a = st.name == "audio"
        sst = self.audio_scale_shift_table if a else self.scale_shift_table
        h = torch.empty_like(st.x)
        d = st.D
        per_tok = st.tmod_ld_tok
        m = nat.modulation(sst, st.emb, shift=(0, 0), scale=(d, 0), mod_ld_batch=d * (st.T if per_tok else 1),
                           mod_ld_tok=d if per_tok else 0)
        nat.norm_modulate(st.x, h, st.T, nat.LTX_NORM_LAYER, self.cfg.norm_eps, m)
        return h

    def _output(self, st: _Stream) -> torch.Tensor:
        proj = self.audio_proj_out if st.name == "audio" else self.proj_out
        h = self.head_hidden(st)
        out = torch.empty(st.B * st.T, proj.out_features, device=h.device, dtype=h.dtype)
        nat.linear(h, proj.weight, out, nat.epilogue(bias=proj.bias))
        return out.view(st.B, st.T, -1)

    def prepare(self, video: Modality | None, audio: Modality | None, uniform_timesteps: bool = False):
        va = self._prepare("video", video, audio, uniform_timesteps) if video is not None else None
        aa = self._prepare("audio", audio, video, uniform_timesteps) if audio is not None else None
        return va, aa

    @torch.inference_mode()
    def forward(self, video: Modality | None, audio: Modality | None, perturbations=None) -> tuple:
        """(vx, ax) velocities (ltx_dit.py:354-369)."""
        va, aa = self.prepare(video, audio)
        self.run_blocks(va, aa, perturbations)
        vx = self._output(va) if va is not None else None
        ax = self._output(aa) if aa is not None else None
        return vx, ax


# ---------------------------------------------------------------------------------------
# Perturbations / loading (ltx_dit.py:381-432)
# ---------------------------------------------------------------------------------------


def build_perturbation_config(num_blocks: int, passes: list[str], v_stg_blocks: list[int], a_stg_blocks: list[int],
                              device: torch.device, dtype: torch.dtype) -> torch.Tensor:
    """(4, num_blocks, B) keep-mask: 0 skip-video-self, 1 skip-audio-self, 2 skip-A2V, 3 skip-V2A."""
    keep = torch.ones(4, num_blocks, len(passes), dtype=dtype)
    for i, name in enumerate(passes):
        if name == "ptb":
            for blk in v_stg_blocks:
                keep[0, blk, i] = 0
            for blk in a_stg_blocks:
                keep[1, blk, i] = 0
        elif name == "mod":
            keep[2, :, i] = 0
            keep[3, :, i] = 0
    return keep.to(device)


def _rename(key: str) -> str | None:
    if not key.startswith("model.diffusion_model."):
        return None
    k = key.removeprefix("model.diffusion_model.")
    k = k.replace("transformer_blocks.", "blocks.")
    k = k.replace("to_out.0.", "to_out.").replace("ff.net.0.proj.", "ff.proj_in.").replace("ff.net.2.", "ff.proj_out.")
    k = k.replace("audio_ff.net.0.proj.", "audio_ff.proj_in.").replace("audio_ff.net.2.", "audio_ff.proj_out.")
    return k


def load_transformer(path: str, cfg: DiTConfig, device: torch.device = DEVICE,
                     dtype: torch.dtype = torch.bfloat16) -> LTXModel:
    """Build the model and load a dev-transformer safetensors checkpoint (ltx_dit.py:414-432)."""
    from safetensors import safe_open

    with torch.device("meta"):
        model = LTXModel(cfg)
    sd = {}
    with safe_open(path, framework="pt", device=str(device)) as f:
        for name in f.keys():  # noqa: SIM118
            new = _rename(name)
            if new is None:
                continue
            t = f.get_tensor(name)
            sd[new] = t.to(dtype) if t.is_floating_point() else t
    res = model.load_state_dict(sd, strict=False, assign=True)
    missing = [k for k in res.missing_keys if k != "keyframes_abs_pos_embedding"]
    if missing:
        raise RuntimeError(f"transformer missing keys: {missing[:10]} ({len(missing)} total)")
    if model.keyframes_abs_pos_embedding is not None and model.keyframes_abs_pos_embedding.is_meta:
        model.keyframes_abs_pos_embedding = torch.nn.Parameter(torch.zeros(1, cfg.video_dim, device=device,
                                                                           dtype=dtype))
    return model.to(device).eval()


# ---------------------------------------------------------------------------------------
# Latent state (ltx_dit.py:439-520)
# ---------------------------------------------------------------------------------------

SCALE_T, SCALE_H, SCALE_W = 8, 32, 32


def video_positions(batch: int, f: int, h: int, w: int, fps: float, device) -> torch.Tensor:
    """(B, 3, T, 2) pixel-space [start, end) per token; time / fps with the causal fix."""
    coords = torch.meshgrid(torch.arange(f, device=device), torch.arange(h, device=device),
                            torch.arange(w, device=device), indexing="ij")
    starts = torch.stack(coords, dim=0)
    bounds = torch.stack([starts, starts + 1], dim=-1).reshape(3, -1, 2)
    bounds = bounds.unsqueeze(0).expand(batch, -1, -1, -1).clone().float()
    bounds = bounds * torch.tensor([SCALE_T, SCALE_H, SCALE_W], device=device).view(1, 3, 1, 1)
    bounds[:, 0] = (bounds[:, 0] + 1 - SCALE_T).clamp(min=0)
    bounds[:, 0] = bounds[:, 0] / fps
    return bounds


def audio_positions(batch: int, frames: int, device) -> torch.Tensor:
    """(B, 1, T, 2) latent-frame [start, end) bounds in seconds."""
    idx = torch.arange(frames, dtype=torch.float32, device=device)
    start = ((idx * 4 + 1 - 4).clamp(min=0)) * 160 / 16000
    end = (((idx + 1) * 4 + 1 - 4).clamp(min=0)) * 160 / 16000
    return torch.stack([start, end], dim=-1)[None, None].expand(batch, 1, -1, -1).contiguous()


def patchify_video(latent: torch.Tensor) -> torch.Tensor:
    return latent.permute(0, 2, 3, 4, 1).reshape(latent.shape[0], -1, latent.shape[1])


def unpatchify_video(tokens: torch.Tensor, f: int, h: int, w: int) -> torch.Tensor:
    b, _, c = tokens.shape
    return tokens.view(b, f, h, w, c).permute(0, 4, 1, 2, 3)


def patchify_audio(latent: torch.Tensor) -> torch.Tensor:
    return latent.permute(0, 2, 1, 3).reshape(latent.shape[0], latent.shape[2], -1)


def unpatchify_audio(tokens: torch.Tensor, channels: int, mel_bins: int) -> torch.Tensor:
    b, t, _ = tokens.shape
    return tokens.view(b, t, channels, mel_bins).permute(0, 2, 1, 3)


@dataclass
class LatentState:
    latent: torch.Tensor
    denoise_mask: torch.Tensor
    positions: torch.Tensor
    clean_latent: torch.Tensor
    keyframes_mask: torch.Tensor | None = None


class PhiloxGenerator:
    """torch.Generator(device='cuda').manual_seed(seed) equivalent for randn: the same
    Philox stream, launch policy and offset bookkeeping, filled by libltxb200."""

    def __init__(self, seed: int, device: torch.device | str = DEVICE):
        self.seed = int(seed)
        self.offset = 0
        self.device = torch.device(device)

    def randn(self, *shape: int, dtype: torch.dtype = torch.float32) -> torch.Tensor:
        out = torch.empty(*shape, device=self.device, dtype=dtype)
        n = out.numel()
        if n == 0:
            return out
        grid = nat.philox_grid(n, self.device.index if self.device.index is not None else torch.cuda.current_device())
        nat.philox_randn(out, self.seed, self.offset, grid)
        self.offset += nat.philox_offset_increment(n, grid)
        return out


def create_noised_states(batch: int, num_video_frames: int, height: int, width: int, fps: float, seed: int,
                         device: torch.device, dtype: torch.dtype) -> tuple[LatentState, LatentState]:
    """Unconditioned t2v initial state (ltx_dit.py:495-520), noise from the Philox kernel."""
    gen = PhiloxGenerator(seed, device)
    f = (num_video_frames - 1) // SCALE_T + 1
    h, w = height // SCALE_H, width // SCALE_W
    v_tokens = f * h * w
    video_noise = gen.randn(batch, v_tokens, 128, dtype=dtype)
    keyframes_mask = torch.zeros(batch, v_tokens, 1, device=device, dtype=torch.float32)
    keyframes_mask[:, : h * w] = 1.0
    video_state = LatentState(latent=video_noise,
                              denoise_mask=torch.ones(batch, v_tokens, 1, device=device, dtype=torch.float32),
                              positions=video_positions(batch, f, h, w, fps, device),
                              clean_latent=torch.zeros_like(video_noise), keyframes_mask=keyframes_mask)
    audio_frames = round(num_video_frames / fps * 25.0)
    audio_noise = gen.randn(batch, audio_frames, 128, dtype=dtype)
    audio_state = LatentState(latent=audio_noise,
                              denoise_mask=torch.ones(batch, audio_frames, 1, device=device, dtype=torch.float32),
                              positions=audio_positions(batch, audio_frames, device),
                              clean_latent=torch.zeros_like(audio_noise))
    return video_state, audio_state


# ---------------------------------------------------------------------------------------
# Scheduler + guidance + sampling (ltx_dit.py:528-621)
# ---------------------------------------------------------------------------------------


def ltx2_scheduler_sigmas(steps: int, tokens: int = 4096, max_shift: float = 2.05, base_shift: float = 0.95,
                          terminal: float = 0.1) -> torch.Tensor:
    """Shifted flow-matching sigmas (host-side, 31 values)."""
    sigmas = torch.linspace(1.0, 0.0, steps + 1)
    mm = (max_shift - base_shift) / (4096 - 1024)
    shift = tokens * mm + (base_shift - mm * 1024)
    e = math.exp(shift)
    sigmas = torch.where(sigmas != 0, e / (e + (1 / sigmas - 1)), sigmas)
    nz = sigmas != 0
    one_minus = 1.0 - sigmas[nz]
    scale = one_minus[-1] / (1.0 - terminal)
    sigmas[nz] = 1.0 - one_minus / scale
    return sigmas.to(torch.float32)


@dataclass(frozen=True)
class GuiderParams:
    cfg_scale: float
    stg_scale: float
    rescale_scale: float
    modality_scale: float
    stg_blocks: tuple[int, ...]

    @property
    def cfg_only(self) -> bool:
        return self.stg_scale == 0 and self.modality_scale == 1 and self.rescale_scale == 0


def _sigma_pair(sigmas: torch.Tensor, idx: int) -> tuple[float, float]:
    s = sigmas.detach().to("cpu", torch.float32)
    return float(s[idx]), float(s[idx + 1])


@torch.inference_mode()
def cfg_denoise_step(model: LTXModel, latent: torch.Tensor, positions: torch.Tensor, context_pos: torch.Tensor,
                     context_neg: torch.Tensor, sigmas: torch.Tensor, idx: int, cfg_scale: float,
                     keyframes_mask: torch.Tensor | None = None, fused_head: bool = True):
    """One CFG denoise step of the video stream (B = 2 [cond, uncond] forward, X0,
    guide, Euler; ltx_dit.py:565-606 with CFG-only guidance).

    latent (1, T, C), positions (1, 3, T, 2), contexts (1, S, Cctx). Returns
    (velocity (2, T, C), denoised (1, T, C), next latent (1, T, C)). The X0 + CFG + Euler
    update runs in the proj_out GEMM epilogue (bf16) or right after it (fp32)."""
    dtype = model.proj_out.weight.dtype
    dev = latent.device
    _, t, c = latent.shape
    sigma, sigma_next = _sigma_pair(sigmas, idx)
    sig = torch.full((2,), sigma, device=dev, dtype=torch.float32)
    ts = torch.full((2, t, 1), sigma, device=dev, dtype=torch.float32)
    lat = latent.to(dtype)
    video = Modality(latent=lat.expand(2, -1, -1), sigma=sig, timesteps=ts, positions=positions.expand(2, -1, -1, -1),
                     context=model.cached_cat(context_pos, context_neg, dtype),
                     keyframes_mask=keyframes_mask.expand(2, -1, -1) if keyframes_mask is not None else None)
    va, _ = model.prepare(video, None, uniform_timesteps=True)
    model.run_blocks(va, None)
    h = model.head_hidden(va)
    lat2 = lat.reshape(t, c).contiguous()
    vel = torch.empty(2 * t, c, device=dev, dtype=dtype)
    den = torch.empty(t, c, device=dev, dtype=dtype)
    nxt = torch.empty(t, c, device=dev, dtype=dtype)
    ts2 = ts.reshape(2, t)
    if fused_head:
        nat.proj_out_cfg_euler(h, model.proj_out.weight, model.proj_out.bias, lat2, ts2, cfg_scale, sigma, sigma_next,
                               nxt, den, vel)
    else:
        nat.linear(h, model.proj_out.weight, vel, nat.epilogue(bias=model.proj_out.bias))
        nat.cfg_euler(vel, lat2, ts2, cfg_scale, sigma, sigma_next, nxt, den)
    return vel.view(2, t, c), den.view(1, t, c), nxt.view(1, t, c)


@torch.inference_mode()
def av_cfg_denoise_step(model: LTXModel, v_latent: torch.Tensor, a_latent: torch.Tensor, v_positions: torch.Tensor,
                        a_positions: torch.Tensor, v_context_pos: torch.Tensor, v_context_neg: torch.Tensor,
                        a_context_pos: torch.Tensor, a_context_neg: torch.Tensor, sigmas: torch.Tensor, idx: int,
                        cfg_scale: float, v_keyframes_mask: torch.Tensor | None = None):
    """One CFG denoise step of the audio-video model: the B = 2 [cond, uncond] forward of
    both streams with A<->V attention in every block, then X0 + CFG + Euler per stream in
    the proj_out epilogues (ltx_dit.py:565-606 with CFG-only guidance).

    v_latent (1, Tv, C), a_latent (1, Ta, C), positions (1, 3, Tv, 2) / (1, 1, Ta, 2),
    contexts (1, S, C_v) / (1, S_a, C_a). Returns (next video latent (1, Tv, C), next audio
    latent (1, Ta, C))."""
    dtype = model.proj_out.weight.dtype
    dev = v_latent.device
    sigma, sigma_next = _sigma_pair(sigmas, idx)
    sig = torch.full((2,), sigma, device=dev, dtype=torch.float32)

    def modality(lat, pos, cpos, cneg, kf):
        t = lat.shape[1]
        return Modality(latent=lat.to(dtype).expand(2, -1, -1), sigma=sig,
                        timesteps=torch.full((2, t, 1), sigma, device=dev, dtype=torch.float32),
                        positions=pos.expand(2, -1, -1, -1), context=torch.cat([cpos, cneg], dim=0).to(dtype),
                        keyframes_mask=kf.expand(2, -1, -1) if kf is not None else None)

    video = modality(v_latent, v_positions, v_context_pos, v_context_neg, v_keyframes_mask)
    audio = modality(a_latent, a_positions, a_context_pos, a_context_neg, None)
    va, aa = model.prepare(video, audio, uniform_timesteps=True)
    model.run_blocks(va, aa)
    outs = []
    for st, lat, proj in ((va, v_latent, model.proj_out), (aa, a_latent, model.audio_proj_out)):
        h = model.head_hidden(st)
        t, c = lat.shape[1], lat.shape[2]
        lat2 = lat.to(dtype).reshape(t, c).contiguous()
        ts2 = torch.full((2, t), sigma, device=dev, dtype=torch.float32)
        nxt = torch.empty(t, c, device=dev, dtype=dtype)
        if dtype == torch.bfloat16:
            nat.proj_out_cfg_euler(h, proj.weight, proj.bias, lat2, ts2, cfg_scale, sigma, sigma_next, nxt)
        else:
            vel = torch.empty(2 * t, c, device=dev, dtype=dtype)
            nat.linear(h, proj.weight, vel, nat.epilogue(bias=proj.bias))
            nat.cfg_euler(vel, lat2, ts2, cfg_scale, sigma, sigma_next, nxt)
        outs.append(nxt.view(1, t, c))
    return outs[0], outs[1]


class NativeStep:
    """cfg_denoise_step through the library's whole-step C entry point (ltx_dit_step):
    the path a C or C++ caller takes without Python. It owns an ltx_ctx (TMA descriptor
    cache, step workspace sized for T latent and S text tokens) and the weight table of
    `model` (the packed attention weights of ltx_nn). Video-only models without
    cross-adaLN (3, 5). Results equal cfg_denoise_step bit for bit."""

    def __init__(self, model: LTXModel, tokens: int, text_tokens: int):
        cfg = model.cfg
        if cfg.cross_attention_adaln:
            raise NotImplementedError("ltx_dit_step runs the video DiT without cross-adaLN")
        dev = model.proj_out.weight.device
        self.device = dev
        dtype = model.proj_out.weight.dtype
        c = nat.DitConfig()
        c.num_layers, c.heads, c.head_dim = cfg.num_layers, cfg.video_heads, cfg.video_head_dim
        c.in_channels, c.out_channels, c.cross_dim = cfg.video_in, cfg.video_out, cfg.video_cross_dim
        c.ffn_dim = model.blocks[0].ff.proj_in.out_features
        c.gated_attention = int(cfg.gated_attention)
        c.norm_eps, c.theta = cfg.norm_eps, cfg.theta
        c.max_pos[:] = [float(v) for v in cfg.video_max_pos]
        c.timestep_scale_multiplier = float(cfg.timestep_scale_multiplier)
        c.dtype = nat.LTX_BF16 if dtype == torch.bfloat16 else nat.LTX_F32
        self.cfg_c = c
        keep = []

        def p(t):
            if t is None:
                return None
            t = t.detach()
            if not t.is_contiguous():
                raise ValueError("weights must be contiguous")
            keep.append(t)
            return t.data_ptr()

        blocks = (nat.DitBlockWeights * cfg.num_layers)()
        for i, blk in enumerate(model.blocks):
            wqkv, bqkv = blk.attn1.packed_self()
            wq, bq = blk.attn2.packed_q()
            wkv, bkv = blk.attn2.packed_kv()
            vals = [blk.scale_shift_table, wqkv, bqkv, blk.attn1.q_norm.weight, blk.attn1.k_norm.weight,
                    blk.attn1.to_out.weight, blk.attn1.to_out.bias, wq, bq, wkv, bkv, blk.attn2.q_norm.weight,
                    blk.attn2.k_norm.weight, blk.attn2.to_out.weight, blk.attn2.to_out.bias, blk.ff.proj_in.weight,
                    blk.ff.proj_in.bias, blk.ff.proj_out.weight, blk.ff.proj_out.bias]
            for name, v in zip(nat.DIT_BLOCK_FIELDS, vals):
                setattr(blocks[i], name, p(v))
        te = model.adaln_single.emb.timestep_embedder
        w = nat.DitWeights()
        w.patchify_w, w.patchify_b = p(model.patchify_proj.weight), p(model.patchify_proj.bias)
        kf = model.keyframes_abs_pos_embedding
        w.keyframes_emb = p(kf.reshape(-1)) if kf is not None else None
        w.t_linear_1_w, w.t_linear_1_b = p(te.linear_1.weight), p(te.linear_1.bias)
        w.t_linear_2_w, w.t_linear_2_b = p(te.linear_2.weight), p(te.linear_2.bias)
        w.adaln_w, w.adaln_b = p(model.adaln_single.linear.weight), p(model.adaln_single.linear.bias)
        w.scale_shift_table = p(model.scale_shift_table)
        w.proj_out_w, w.proj_out_b = p(model.proj_out.weight), p(model.proj_out.bias)
        w.blocks = blocks
        self.weights, self._blocks, self._keep = w, blocks, keep
        self.dtype, self.T, self.S = dtype, tokens, text_tokens
        self.ctx = nat.ctx_create(dev.index if dev.index is not None else torch.cuda.current_device())
        nat.dit_reserve(self.ctx, c, tokens, text_tokens)

    def close(self) -> None:
        if getattr(self, "ctx", None):
            nat.ctx_destroy(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:  # noqa: BLE001 - interpreter shutdown
            pass

    def __call__(self, latent: torch.Tensor, positions: torch.Tensor, context_pos: torch.Tensor,
                 context_neg: torch.Tensor, sigmas: torch.Tensor, idx: int, cfg_scale: float,
                 keyframes_mask: torch.Tensor | None = None, reuse: bool = False, out: tuple | None = None):
        """Same arguments and results as cfg_denoise_step. reuse=True keeps the RoPE tables
        and text K/V of the previous call (same positions and contexts). `out` optionally
        gives (velocity (2, T, C), denoised (1, T, C), next latent (1, T, C)) buffers."""
        sigma, sigma_next = _sigma_pair(sigmas, idx)
        _, t, c = latent.shape
        dt = self.dtype
        lat = latent.to(dt).reshape(t, c).contiguous()
        pos = positions.reshape(-1, 3, t, 2)[0].to(torch.float32).contiguous()
        cp = context_pos.to(dt).reshape(-1, context_pos.shape[-1]).contiguous()
        cn = context_neg.to(dt).reshape(-1, context_neg.shape[-1]).contiguous()
        kf = keyframes_mask.reshape(-1, t)[0].to(torch.float32).contiguous() if keyframes_mask is not None else None
        a = nat.DitStepArgs()
        a.latent, a.positions, a.context_pos, a.context_neg = lat.data_ptr(), pos.data_ptr(), cp.data_ptr(), cn.data_ptr()
        a.keyframes_mask = kf.data_ptr() if kf is not None else None
        a.T, a.S = t, cp.shape[0]
        a.sigma, a.sigma_next, a.cfg_scale = sigma, sigma_next, float(cfg_scale)
        a.flags = (nat.STEP_REUSE_TEXT_KV | nat.STEP_REUSE_ROPE) if reuse else 0
        if out is None:
            vel = torch.empty(2, t, c, device=lat.device, dtype=dt)
            den = torch.empty(1, t, c, device=lat.device, dtype=dt)
            nxt = torch.empty(1, t, c, device=lat.device, dtype=dt)
        else:
            vel, den, nxt = out
        self._args = (lat, pos, cp, cn, kf)  # alive until the stream has consumed them
        nat.dit_step(self.ctx, self.cfg_c, self.weights, a, vel, den, nxt)
        return vel, den, nxt


_guide_ws: dict = {}


def guide(cond, uncond, ptb, mod, p: GuiderParams) -> torch.Tensor:
    """Guidance blend cond + (cfg-1)(cond-uncond) + stg(cond-ptb) + (mod-1)(cond-mod)
    (ltx_dit.py:551-562): one device kernel, or with rescale_scale != 0 the two-pass
    std rescale (factor = r*std(cond)/std(pred) + 1 - r) through a cached workspace."""
    out = torch.empty_like(cond)
    args = (cond.contiguous(), uncond.contiguous(), ptb.contiguous(), mod.contiguous())
    if p.rescale_scale == 0:
        nat.guide(*args, p.cfg_scale, p.stg_scale, p.modality_scale, out)
        return out
    key = (cond.device, cond.numel())
    ws = _guide_ws.get(key)
    if ws is None:
        ws = _guide_ws[key] = nat.guide_rescale_workspace(cond.numel(), cond.device)
    nat.guide_rescale(*args, p.cfg_scale, p.stg_scale, p.modality_scale, p.rescale_scale, out, ws)
    return out


def euler_step(sample: torch.Tensor, denoised: torch.Tensor, sigmas: torch.Tensor, idx: int) -> torch.Tensor:
    """Flow-matching Euler update (ltx_dit.py:602-606) as one device kernel."""
    sigma, sigma_next = _sigma_pair(sigmas, idx)
    out = torch.empty_like(sample)
    nat.euler(sample.contiguous(), denoised.contiguous(), sigma, sigma_next, out)
    return out


@torch.inference_mode()
def guided_denoise_step(model: LTXModel, video_state: LatentState, audio_state: LatentState | None, contexts: dict,
                        sigma: torch.Tensor, step_idx: int, v_params: GuiderParams, a_params: GuiderParams | None,
                        cfg: DiTConfig):
    """One transformer call with the B=4 guidance passes [cond, uncond, ptb (STG), mod
    (A<->V isolated)] -> blended x0 per modality (ltx_dit.py:565-599): the perturbation
    keep-mask of build_perturbation_config, X0 per pass, guide() with rescale."""
    passes = ["cond", "uncond", "ptb", "mod"]
    n = len(passes)
    sigma = sigma.reshape(()).to(torch.float32)
    dev = video_state.latent.device
    sigma_b = sigma.to(dev).expand(n)
    dtype = model.proj_out.weight.dtype
    v_ctx = torch.cat([contexts["v_pos"], contexts["v_neg"], contexts["v_pos"], contexts["v_pos"]], dim=0)
    v_lat = video_state.latent.repeat(n, 1, 1)
    video = Modality(latent=v_lat, sigma=sigma_b,
                     timesteps=video_state.denoise_mask.repeat(n, 1, 1) * sigma_b.view(n, 1, 1),
                     positions=video_state.positions.repeat(n, 1, 1, 1), context=v_ctx,
                     keyframes_mask=video_state.keyframes_mask.repeat(n, 1, 1)
                     if video_state.keyframes_mask is not None else None)
    audio = None
    if audio_state is not None:
        a_ctx = torch.cat([contexts["a_pos"], contexts["a_neg"], contexts["a_pos"], contexts["a_pos"]], dim=0)
        a_lat = audio_state.latent.repeat(n, 1, 1)
        audio = Modality(latent=a_lat, sigma=sigma_b,
                         timesteps=audio_state.denoise_mask.repeat(n, 1, 1) * sigma_b.view(n, 1, 1),
                         positions=audio_state.positions.repeat(n, 1, 1, 1), context=a_ctx)
    a_blocks = list(a_params.stg_blocks) if a_params is not None else []
    keep = build_perturbation_config(cfg.num_layers, passes, list(v_params.stg_blocks), a_blocks, dev, dtype)
    vx, ax = model(video, audio, keep)
    def x0(lat, vel, ts):
        out = torch.empty_like(vel)
        nat.x0(lat.to(vel.dtype).contiguous(), vel.contiguous(), ts.to(torch.float32).reshape(-1).contiguous(), out)
        return out

    vs_ = x0(v_lat, vx, video.timesteps).chunk(n)
    if audio is not None:
        as_ = x0(audio.latent, ax, audio.timesteps).chunk(n)
    else:
        as_ = (None,) * n
    r = dict(zip(passes, zip(vs_, as_)))
    denoised_video = guide(*[r[p][0] for p in passes], v_params)
    denoised_audio = guide(*[r[p][1] for p in passes], a_params) if audio is not None else None
    return denoised_video, denoised_audio, r


@torch.inference_mode()
def run_dit(model: LTXModel, cfg: DiTConfig, contexts: dict, video_state: LatentState,
            audio_state: LatentState | None, sigmas: torch.Tensor, v_params: GuiderParams,
            a_params: GuiderParams | None, on_step=None) -> tuple[torch.Tensor, torch.Tensor | None]:
    """Denoising loop (ltx_dit.py:609-621): guided_denoise_step (the 4-pass guidance
    batch) and an Euler update per modality at every step. Without an audio state the
    audio stream is left out of the batch."""
    for idx in range(len(sigmas) - 1):
        t0 = time.perf_counter()
        dv, da, passes = guided_denoise_step(model, video_state, audio_state, contexts, sigmas[idx], idx, v_params,
                                             a_params, cfg)
        video_state = replace(video_state, latent=euler_step(video_state.latent, dv, sigmas, idx))
        if audio_state is not None:
            audio_state = replace(audio_state, latent=euler_step(audio_state.latent, da, sigmas, idx))
        if on_step:
            on_step(idx, time.perf_counter() - t0, dv, da, passes, video_state, audio_state)
    return video_state.latent, audio_state.latent if audio_state is not None else None
