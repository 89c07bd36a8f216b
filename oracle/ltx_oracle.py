"""CPU restatement of the LTX-2.5 DiT denoising step -- TEST INFRASTRUCTURE ONLY.

This module is the checker for the product path (ltx-nv_b200/): only tests/,
__graft_entry__.smoke() and bench.py's cpu_baseline / reference legs may import it. It
restates, op for op and in the same torch dtype, the reference implementation in
lipaul/ltx-nv standalone/ltx_dit.py and standalone/ltx_nn.py, as plain functions over
a state dict that uses the reference's parameter names, and runs on CPU tensors.

Differences from the reference, all of them its documented adapters for the
benchmark configurations (the reference itself cannot run those configurations):
  * `audio=None` runs the video stream alone (the reference evaluates None.numel() at
    ltx_dit.py:253-256); A2V/V2A are skipped, which is what a disabled 1-token audio
    stream plus a zero A2V perturbation row produces in the reference.
  * the text context keeps its own width (B, S, C): the reference's
    `context.view(b, -1, hidden)` (ltx_dit.py:157) only works for C == hidden; attn2's
    to_k/to_v already map C -> hidden (ltx_nn.py:189-190).
  * CFG-only guidance: the model runs with B=2 [cond, uncond] and the guide is
    guide(c, u, c, c) (ltx_dit.py:551-562), i.e. cond + (cfg-1)(cond-uncond).
The tests pin every function here against fixtures produced by the reference itself
(tests/golden/make_golden.py).
"""

from __future__ import annotations

import functools
import math
from dataclasses import dataclass

import numpy as np
import torch
import torch.nn.functional as F

# ----------------------------------------------------------------------------------------
# primitives (ltx_nn.py)
# ----------------------------------------------------------------------------------------


def rms_norm(x, eps=1e-6, weight=None):
    """ltx_nn.py:18-19."""
    return F.rms_norm(x, (x.shape[-1],), weight=weight, eps=eps)


def sdpa(q, k, v, mask=None):
    """ltx_nn.py:22-26. (B, H, T, d); mask an additive (B, 1, 1, T) mask or None."""
    return F.scaled_dot_product_attention(q, k, v, attn_mask=mask, dropout_p=0.0, is_causal=False)


@functools.lru_cache(maxsize=16)
def freq_grid(theta: float, n_axes: int, inner_dim: int, double: bool = True) -> torch.Tensor:
    """ltx_nn.py:34-60: theta ** linspace(0, 1, inner_dim // (2 n_axes)) * pi/2."""
    n = inner_dim // (2 * n_axes)
    if double:
        g = np.power(theta, np.linspace(np.log(1.0) / np.log(theta), np.log(theta) / np.log(theta), n,
                                        dtype=np.float64))
        return torch.as_tensor(g * math.pi / 2, dtype=torch.float32)
    g = theta ** torch.linspace(math.log(1.0, theta), math.log(theta, theta), n, dtype=torch.float32)
    return g.to(torch.float32) * math.pi / 2


def rope_tables(positions, dim, out_dtype, theta, max_pos, heads, double=True):
    """ltx_nn.py:63-96: positions (B, n_axes, T, 2) -> (cos, sin) each (B, H, T, dim/2/H)."""
    n_axes = positions.shape[1]
    freqs = freq_grid(float(theta), n_axes, dim, double).to(positions.device)
    grid = (positions[..., 0] + positions[..., 1]) / 2.0
    frac = torch.stack([grid[:, i] / max_pos[i] for i in range(n_axes)], dim=-1)
    ang = (freqs * (frac.unsqueeze(-1) * 2 - 1)).transpose(-1, -2).flatten(2)
    pad = dim // 2 - ang.shape[-1]
    cos, sin = ang.cos(), ang.sin()
    if pad:
        cos = torch.cat([torch.ones_like(cos[:, :, :pad]), cos], dim=-1)
        sin = torch.cat([torch.zeros_like(sin[:, :, :pad]), sin], dim=-1)
    b, t = cos.shape[0], cos.shape[1]
    cos = cos.reshape(b, t, heads, -1).swapaxes(1, 2)
    sin = sin.reshape(b, t, heads, -1).swapaxes(1, 2)
    return cos.to(out_dtype), sin.to(out_dtype)


def apply_rope(x, tables):
    """ltx_nn.py:99-115 on (B, T, H*d) activations."""
    cos, sin = tables
    h = cos.shape[1]
    xh = x.unflatten(-1, (h, -1)).transpose(1, 2)
    pair = xh.reshape(*xh.shape[:-1], 2, xh.shape[-1] // 2)
    a, b = pair[..., :1, :], pair[..., 1:, :]
    c, s = cos.unsqueeze(-2), sin.unsqueeze(-2)
    out = torch.cat([a * c - b * s, b * c + a * s], dim=-2).reshape(*xh.shape)
    return out.transpose(1, 2).flatten(-2)


def timestep_sinusoid(t, dim=256, max_period=10000):
    """standalone/common.py:138-148 ([cos, sin], flip_sin_to_cos)."""
    half = dim // 2
    freqs = torch.exp(-math.log(max_period) * torch.arange(0, half, dtype=torch.float32, device=t.device) / half)
    args = t[:, None].float() * freqs[None, :]
    emb = torch.cat([torch.cos(args), torch.sin(args)], dim=-1)
    if dim % 2:
        emb = F.pad(emb, (0, 1))
    return emb


def linear(w, name, x):
    return F.linear(x, w[name + ".weight"], w.get(name + ".bias"))


def adaln_single(w, name, t, dtype):
    """ltx_nn.py:123-158 -> (modulation, embedded_timestep)."""
    proj = timestep_sinusoid(t, 256).to(dtype)
    h = linear(w, name + ".emb.timestep_embedder.linear_1", proj)
    emb = linear(w, name + ".emb.timestep_embedder.linear_2", F.silu(h))
    return linear(w, name + ".linear", F.silu(emb)), emb


def attention(w, name, x, heads, dim_head, eps, context=None, pe=None, k_pe=None, gated=True,
              perturbation_mask=None, all_perturbed=False, mask=None):
    """ltx_nn.py:194-236. STG: all_perturbed -> out = V (:209-210); a per-sample
    perturbation_mask (B, 1, 1) blends out * mask + V * (1 - mask) (:229-230)."""
    context = x if context is None else context
    b = x.shape[0]
    v = linear(w, name + ".to_v", context)
    if all_perturbed:
        out = v
    else:
        q = rms_norm(linear(w, name + ".to_q", x), eps, w[name + ".q_norm.weight"])
        k = rms_norm(linear(w, name + ".to_k", context), eps, w[name + ".k_norm.weight"])
        if pe is not None:
            q = apply_rope(q, pe)
            k = apply_rope(k, pe if k_pe is None else k_pe)
        q = q.view(b, -1, heads, dim_head).transpose(1, 2)
        k = k.view(b, -1, heads, dim_head).transpose(1, 2)
        v4 = v.view(b, -1, heads, dim_head).transpose(1, 2)
        out = sdpa(q, k, v4, mask).transpose(1, 2).reshape(b, -1, heads * dim_head)
        if perturbation_mask is not None:
            out = out * perturbation_mask + v * (1 - perturbation_mask)
    if gated and (name + ".to_gate_logits.weight") in w:
        g = linear(w, name + ".to_gate_logits", x)
        t = out.shape[1]
        out = (out.view(b, t, heads, dim_head) * (2.0 * torch.sigmoid(g)).unsqueeze(-1)).view(b, t, heads * dim_head)
    return linear(w, name + ".to_out", out)


def feed_forward(w, name, x):
    """ltx_nn.py:239-248."""
    return linear(w, name + ".proj_out", F.gelu(linear(w, name + ".proj_in", x), approximate="tanh"))


# ----------------------------------------------------------------------------------------
# model (ltx_dit.py)
# ----------------------------------------------------------------------------------------


@dataclass
class Modality:
    """ltx_dit.py:89-97."""

    latent: torch.Tensor
    sigma: torch.Tensor
    timesteps: torch.Tensor
    positions: torch.Tensor
    context: torch.Tensor
    keyframes_mask: torch.Tensor | None = None
    enabled: bool = True


@dataclass
class StreamArgs:
    x: torch.Tensor
    context: torch.Tensor
    mod: torch.Tensor
    embedded: torch.Tensor
    pe: tuple
    cross_pe: tuple | None
    cross_ss: torch.Tensor | None
    cross_gate: torch.Tensor | None
    prompt_mod: torch.Tensor | None
    enabled: bool


def _dims(cfg, stream):
    if stream == "audio":
        return cfg.audio_heads * cfg.audio_head_dim, cfg.audio_heads, cfg.audio_head_dim
    return cfg.video_heads * cfg.video_head_dim, cfg.video_heads, cfg.video_head_dim


def prepare(w, cfg, stream, mod: Modality, cross: Modality | None) -> StreamArgs:
    """ltx_dit.py:131-184 (context kept at its own width, see module docstring)."""
    a = stream == "audio"
    pre = "audio_" if a else ""
    dim, heads, _ = _dims(cfg, stream)
    x = linear(w, pre + "patchify_proj", mod.latent)
    kf = w.get("keyframes_abs_pos_embedding")
    if not a and mod.keyframes_mask is not None and kf is not None:
        x = x + (mod.keyframes_mask > 0).to(x.dtype) * kf.to(x.dtype)
    ts = mod.timesteps * cfg.timestep_scale_multiplier
    t_mod, emb = adaln_single(w, pre + "adaln_single", ts.flatten(), mod.latent.dtype)
    b = x.shape[0]
    t_mod = t_mod.view(b, -1, t_mod.shape[-1])
    emb = emb.view(b, -1, emb.shape[-1])
    prompt = None
    if cfg.cross_attention_adaln:
        pt, _ = adaln_single(w, pre + "prompt_adaln_single", (mod.sigma * cfg.timestep_scale_multiplier).flatten(),
                             mod.latent.dtype)
        prompt = pt.view(b, -1, pt.shape[-1])
    max_pos = list(cfg.audio_max_pos if a else cfg.video_max_pos)
    pe = rope_tables(mod.positions, dim, x.dtype, cfg.theta, max_pos, heads, cfg.double_rope)
    cross_pe = cross_ss = cross_gate = None
    if cross is not None:
        cross_pe = rope_tables(mod.positions[:, 0:1, :], cfg.audio_cross_dim, x.dtype, cfg.theta,
                               [max(cfg.video_max_pos[0], cfg.audio_max_pos[0])], heads, cfg.double_rope)
        ss_name = "av_ca_audio_scale_shift_adaln_single" if a else "av_ca_video_scale_shift_adaln_single"
        g_name = "av_ca_v2a_gate_adaln_single" if a else "av_ca_a2v_gate_adaln_single"
        cst, _ = adaln_single(w, ss_name, ts.flatten(), x.dtype)
        cross_ss = cst.view(b, -1, cst.shape[-1])
        factor = cfg.av_ca_timestep_scale_multiplier / cfg.timestep_scale_multiplier
        cgt, _ = adaln_single(w, g_name, (cross.sigma * cfg.timestep_scale_multiplier * factor).flatten(), x.dtype)
        cross_gate = cgt.view(b, -1, cgt.shape[-1])
    return StreamArgs(x, mod.context, t_mod, emb, pe, cross_pe, cross_ss, cross_gate, prompt, mod.enabled)


def ada(table, batch, t_mod, sl):
    """ltx_dit.py:192-198: table[sl] + t_mod viewed (B, T, n, D)."""
    n = table.shape[0]
    vals = table[sl].unsqueeze(0).unsqueeze(0).to(t_mod.dtype) + t_mod.reshape(batch, t_mod.shape[1], n, -1)[:, :, sl]
    return vals.unbind(dim=2)


def av_ada(table, batch, ss_ts, gate_ts, sl):
    """ltx_dit.py:201-206."""
    scale, shift = (t.squeeze(2) for t in ada(table[:4], batch, ss_ts, sl))
    (gate,) = (t.squeeze(2) for t in ada(table[4:], batch, gate_ts, slice(None)))
    return scale, shift, gate


def text_cross(w, cfg, name, sst_name, psst_name, x_normed, args: StreamArgs, heads, d):
    """ltx_dit.py:237-248."""
    if cfg.cross_attention_adaln:
        shift_q, scale_q, gate = ada(w[sst_name], x_normed.shape[0], args.mod, slice(6, 9))
        kv = w[psst_name][None, None].to(x_normed.dtype)
        if args.prompt_mod is not None:
            kv = kv + args.prompt_mod.reshape(x_normed.shape[0], args.prompt_mod.shape[1], 2, -1)
        shift_kv, scale_kv = kv.unbind(dim=2)
        q_in = x_normed * (1 + scale_q) + shift_q
        enc = args.context * (1 + scale_kv) + shift_kv
        return attention(w, name, q_in, heads, d, cfg.norm_eps, context=enc, gated=cfg.gated_attention) * gate
    return attention(w, name, x_normed, heads, d, cfg.norm_eps, context=args.context, gated=cfg.gated_attention)


def _self_ptb(keep_row):
    """apply_block_perturbations (ltx_dit.py:381-394) for one self-attention row:
    (perturbation_mask or None, all_perturbed)."""
    if keep_row is None:
        return None, False
    all_p = bool((keep_row == 0).all())
    any_p = bool((keep_row == 0).any())
    return (keep_row.reshape(-1, 1, 1) if any_p and not all_p else None), all_p


def block(w, cfg, i, va: StreamArgs | None, aa: StreamArgs | None, keep=None):
    """ltx_dit.py:250-317. keep: (4, B) keep-mask rows of this block, or None (all ones)."""
    p = f"blocks.{i}."
    eps = cfg.norm_eps
    vdim, vh, vd = _dims(cfg, "video")
    adim, ah, ad = _dims(cfg, "audio")
    vx = va.x if va is not None else None
    ax = aa.x if aa is not None else None
    run_v = va is not None and va.enabled and vx.numel() > 0
    run_a = aa is not None and aa.enabled and ax.numel() > 0
    run_a2v = run_v and ax is not None and ax.numel() > 0
    run_v2a = run_a and vx is not None and vx.numel() > 0
    if run_v:
        sh, sc, g = ada(w[p + "scale_shift_table"], vx.shape[0], va.mod, slice(0, 3))
        pm, allp = _self_ptb(keep[0] if keep is not None else None)
        out = attention(w, p + "attn1", rms_norm(vx, eps) * (1 + sc) + sh, vh, vd, eps, pe=va.pe,
                        gated=cfg.gated_attention, perturbation_mask=pm, all_perturbed=allp)
        vx = vx + out * g
        vx = vx + text_cross(w, cfg, p + "attn2", p + "scale_shift_table", p + "prompt_scale_shift_table",
                             rms_norm(vx, eps), va, vh, vd)
    if run_a:
        sh, sc, g = ada(w[p + "audio_scale_shift_table"], ax.shape[0], aa.mod, slice(0, 3))
        pm, allp = _self_ptb(keep[1] if keep is not None else None)
        out = attention(w, p + "audio_attn1", rms_norm(ax, eps) * (1 + sc) + sh, ah, ad, eps, pe=aa.pe,
                        gated=cfg.gated_attention, perturbation_mask=pm, all_perturbed=allp)
        ax = ax + out * g
        ax = ax + text_cross(w, cfg, p + "audio_attn2", p + "audio_scale_shift_table",
                             p + "audio_prompt_scale_shift_table", rms_norm(ax, eps), aa, ah, ad)
    if run_a2v or run_v2a:
        vx_pre, ax_pre = vx, ax
        kv_mask = keep if keep is not None else torch.ones(4, vx.shape[0], dtype=vx.dtype, device=vx.device)
        if run_a2v and bool((kv_mask[2] != 0).any()):
            s, shv, g = av_ada(w[p + "scale_shift_table_a2v_ca_video"], vx.shape[0], va.cross_ss, va.cross_gate,
                               slice(0, 2))
            q_in = rms_norm(vx_pre, eps) * (1 + s) + shv
            s, sha, _ = av_ada(w[p + "scale_shift_table_a2v_ca_audio"], ax.shape[0], aa.cross_ss, aa.cross_gate,
                               slice(0, 2))
            kv_in = rms_norm(ax_pre, eps) * (1 + s) + sha
            vx = vx + attention(w, p + "audio_to_video_attn", q_in, ah, ad, eps, context=kv_in, pe=va.cross_pe,
                                k_pe=aa.cross_pe, gated=cfg.gated_attention) * g * kv_mask[2].reshape(-1, 1, 1)
        if run_v2a and bool((kv_mask[3] != 0).any()):
            s, sha, g = av_ada(w[p + "scale_shift_table_a2v_ca_audio"], ax.shape[0], aa.cross_ss, aa.cross_gate,
                               slice(2, 4))
            q_in = rms_norm(ax_pre, eps) * (1 + s) + sha
            s, shv, _ = av_ada(w[p + "scale_shift_table_a2v_ca_video"], vx.shape[0], va.cross_ss, va.cross_gate,
                               slice(2, 4))
            kv_in = rms_norm(vx_pre, eps) * (1 + s) + shv
            ax = ax + attention(w, p + "video_to_audio_attn", q_in, ah, ad, eps, context=kv_in, pe=aa.cross_pe,
                                k_pe=va.cross_pe, gated=cfg.gated_attention) * g * kv_mask[3].reshape(-1, 1, 1)
    if run_v:
        sh, sc, g = ada(w[p + "scale_shift_table"], vx.shape[0], va.mod, slice(3, 6))
        vx = vx + feed_forward(w, p + "ff", rms_norm(vx, eps) * (1 + sc) + sh) * g
    if run_a:
        sh, sc, g = ada(w[p + "audio_scale_shift_table"], ax.shape[0], aa.mod, slice(3, 6))
        ax = ax + feed_forward(w, p + "audio_ff", rms_norm(ax, eps) * (1 + sc) + sh) * g
    if va is not None:
        va = StreamArgs(**{**va.__dict__, "x": vx})
    if aa is not None:
        aa = StreamArgs(**{**aa.__dict__, "x": ax})
    return va, aa


def output_head(w, pre, eps, args: StreamArgs):
    """ltx_dit.py:371-378."""
    x = args.x
    ss = w[pre + "scale_shift_table"][None, None].to(x.dtype) + args.embedded[:, :, None]
    shift, scale = ss[:, :, 0], ss[:, :, 1]
    x = F.layer_norm(x, (x.shape[-1],), eps=eps)
    x = x * (1 + scale) + shift
    return linear(w, pre + "proj_out", x)


@torch.inference_mode()
def forward(w, cfg, video: Modality | None, audio: Modality | None = None, keep=None):
    """LTXModel.forward (ltx_dit.py:354-369). keep: (4, L, B) perturbation keep-mask."""
    va = prepare(w, cfg, "video", video, audio) if video is not None else None
    aa = prepare(w, cfg, "audio", audio, video) if audio is not None else None
    for i in range(cfg.num_layers):
        va, aa = block(w, cfg, i, va, aa, keep[:, i] if keep is not None else None)
    vx = output_head(w, "", cfg.norm_eps, va) if va is not None else None
    ax = output_head(w, "audio_", cfg.norm_eps, aa) if aa is not None else None
    return vx, ax


# ----------------------------------------------------------------------------------------
# latent state + sampling (ltx_dit.py:442-621)
# ----------------------------------------------------------------------------------------


def video_positions(batch, f, h, w, fps):
    """ltx_dit.py:442-456 (B, 3, T, 2)."""
    coords = torch.meshgrid(torch.arange(f), torch.arange(h), torch.arange(w), indexing="ij")
    starts = torch.stack(coords, dim=0)
    bounds = torch.stack([starts, starts + 1], dim=-1).reshape(3, -1, 2)
    bounds = bounds.unsqueeze(0).expand(batch, -1, -1, -1).clone().float()
    bounds = bounds * torch.tensor([8, 32, 32]).view(1, 3, 1, 1)
    bounds[:, 0] = (bounds[:, 0] + 1 - 8).clamp(min=0) / fps
    return bounds


def audio_positions(batch, frames):
    """ltx_dit.py:459-465 (B, 1, T, 2) seconds."""
    idx = torch.arange(frames, dtype=torch.float32)
    start = ((idx * 4 + 1 - 4).clamp(min=0)) * 160 / 16000
    end = (((idx + 1) * 4 + 1 - 4).clamp(min=0)) * 160 / 16000
    return torch.stack([start, end], dim=-1)[None, None].expand(batch, 1, -1, -1).contiguous()


def scheduler_sigmas(steps, tokens=4096, max_shift=2.05, base_shift=0.95, terminal=0.1):
    """ltx_dit.py:528-539."""
    s = torch.linspace(1.0, 0.0, steps + 1)
    mm = (max_shift - base_shift) / (4096 - 1024)
    shift = tokens * mm + (base_shift - mm * 1024)
    e = math.exp(shift)
    s = torch.where(s != 0, e / (e + (1 / s - 1)), s)
    nz = s != 0
    one_minus = 1.0 - s[nz]
    scale = one_minus[-1] / (1.0 - terminal)
    s[nz] = 1.0 - one_minus / scale
    return s.to(torch.float32)


def guide(cond, uncond, ptb, mod, cfg_scale, stg_scale, rescale_scale, modality_scale):
    """ltx_dit.py:551-562: the four-way blend in fp32, optional std rescale, cast back."""
    c = cond.float()
    pred = c + (cfg_scale - 1) * (c - uncond.float()) + stg_scale * (c - ptb.float()) \
        + (modality_scale - 1) * (c - mod.float())
    if rescale_scale != 0:
        factor = c.std() / pred.std()
        factor = rescale_scale * factor + (1 - rescale_scale)
        pred = pred * factor
    return pred.to(cond.dtype)


def guide_cfg(cond, uncond, cfg_scale):
    """ltx_dit.py:551-562 with ptb = mod = cond, stg = 0, rescale = 0."""
    c = cond.float()
    pred = c + (cfg_scale - 1) * (c - uncond.float()) + 0.0 * (c - c) + (1.0 - 1) * (c - c)
    return pred.to(cond.dtype)


def euler_step(sample, denoised, sigmas, idx):
    """ltx_dit.py:602-606."""
    sigma = sigmas[idx].float()
    dt = (sigmas[idx + 1] - sigmas[idx]).float()
    velocity = ((sample.float() - denoised.float()) / sigma).to(sample.dtype)
    return (sample.float() + velocity.float() * dt).to(sample.dtype)


@torch.inference_mode()
def cfg_denoise_step(w, cfg, latent, positions, context_pos, context_neg, sigmas, idx, cfg_scale,
                     keyframes_mask=None, denoise_mask=None):
    """One CFG step of the video stream: B=2 [cond, uncond] forward, X0
    (ltx_dit.py:591-593), CFG guide, Euler. latent (1, T, C). Returns
    (velocity (2, T, C), denoised (1, T, C), next latent (1, T, C))."""
    t = latent.shape[1]
    sigma = sigmas[idx].to(latent.device)
    dm = torch.ones(1, t, 1, device=latent.device) if denoise_mask is None else denoise_mask
    sigma_b = sigma.expand(2)
    lat2 = latent.repeat(2, 1, 1)
    ts = dm.repeat(2, 1, 1) * sigma_b.view(2, 1, 1)
    mod = Modality(latent=lat2, sigma=sigma_b, timesteps=ts, positions=positions.repeat(2, 1, 1, 1),
                   context=torch.cat([context_pos, context_neg], dim=0),
                   keyframes_mask=keyframes_mask.repeat(2, 1, 1) if keyframes_mask is not None else None)
    vx, _ = forward(w, cfg, mod, None)
    x0 = (lat2.float() - vx.float() * ts.float()).to(vx.dtype)
    den = guide_cfg(x0[0:1], x0[1:2], cfg_scale)
    nxt = euler_step(latent, den, sigmas, idx)
    return vx, den, nxt


def build_perturbation_config(num_blocks, passes, v_stg_blocks, a_stg_blocks, dtype):
    """ltx_dit.py:397-411: (4, L, B) keep-mask; 0 skip-video-self, 1 skip-audio-self,
    2 skip-A2V, 3 skip-V2A."""
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
    return keep


@torch.inference_mode()
def guided_denoise_step(w, cfg, video_state, audio_state, contexts, sigma, v_params, a_params):
    """ltx_dit.py:565-599: one B=4 forward over [cond, uncond, ptb, mod], X0 per modality
    and the guidance blend (with rescale). State objects carry latent, denoise_mask,
    positions and (video) keyframes_mask; params are (cfg, stg, rescale, modality,
    stg_blocks). Returns (denoised video, denoised audio, {pass: (x0_v, x0_a)})."""
    passes = ["cond", "uncond", "ptb", "mod"]
    n = len(passes)
    v_ctx = torch.cat([contexts["v_pos"], contexts["v_neg"], contexts["v_pos"], contexts["v_pos"]], dim=0)
    a_ctx = torch.cat([contexts["a_pos"], contexts["a_neg"], contexts["a_pos"], contexts["a_pos"]], dim=0)
    sigma_b = sigma.expand(n)
    v_lat = video_state["latent"].repeat(n, 1, 1)
    a_lat = audio_state["latent"].repeat(n, 1, 1)
    kf = video_state.get("keyframes_mask")
    video = Modality(latent=v_lat, sigma=sigma_b,
                     timesteps=video_state["denoise_mask"].repeat(n, 1, 1) * sigma_b.view(n, 1, 1),
                     positions=video_state["positions"].repeat(n, 1, 1, 1), context=v_ctx,
                     keyframes_mask=kf.repeat(n, 1, 1) if kf is not None else None)
    audio = Modality(latent=a_lat, sigma=sigma_b,
                     timesteps=audio_state["denoise_mask"].repeat(n, 1, 1) * sigma_b.view(n, 1, 1),
                     positions=audio_state["positions"].repeat(n, 1, 1, 1), context=a_ctx)
    keep = build_perturbation_config(cfg.num_layers, passes, list(v_params[4]), list(a_params[4]),
                                     video_state["latent"].dtype)
    vx, ax = forward(w, cfg, video, audio, keep)
    x0_v = (v_lat.float() - vx.float() * video.timesteps.float()).to(vx.dtype)
    x0_a = (a_lat.float() - ax.float() * audio.timesteps.float()).to(ax.dtype)
    r = dict(zip(passes, zip(x0_v.chunk(n), x0_a.chunk(n))))
    gv = guide(*[r[p][0] for p in passes], *v_params[:4])
    ga = guide(*[r[p][1] for p in passes], *a_params[:4])
    return gv, ga, r


# ----------------------------------------------------------------------------------------
# text connector (ltx_te.py:187-229)
# ----------------------------------------------------------------------------------------


@torch.inference_mode()
def connector_forward(w, prefix, heads, dim_head, num_layers, max_pos, registers, gated, hidden, additive_mask):
    """Embeddings1DConnector.forward (ltx_te.py:212-229): learnable-register fill of
    padded tokens, 1D RoPE over token indices (no mid-point grid), `num_layers` blocks of
    x + attn1(rms(x)) and x + ff(rms(x)), final RMS norm. Returns (out, mask)."""
    b, s, _ = hidden.shape
    inner = heads * dim_head
    if registers:
        regs = w[prefix + "learnable_registers"].repeat(s // registers, 1).to(hidden.dtype)
        regs = regs.unsqueeze(0).expand(b, -1, -1)
        binary = (additive_mask[:, 0, 0, :] >= 0).to(hidden.dtype).unsqueeze(-1)
        hidden = binary * hidden + (1 - binary) * regs
        additive_mask = torch.zeros_like(additive_mask)
    grid = torch.arange(s, dtype=torch.float32)[None, None, :].expand(b, -1, -1)
    pe = rope_tables(torch.stack([grid, grid], dim=-1), inner, hidden.dtype, 10000.0, list(max_pos), heads, True)
    x = hidden
    for i in range(num_layers):
        p = f"{prefix}blocks.{i}."
        x = x + attention(w, p + "attn1", rms_norm(x), heads, dim_head, 1e-6, pe=pe, gated=gated,
                          mask=additive_mask)
        x = x + feed_forward(w, p + "ff", rms_norm(x))
    return rms_norm(x), additive_mask


# ----------------------------------------------------------------------------------------
# synthetic weights (every parameter ~ N(0, 0.02), fixed seed)
# ----------------------------------------------------------------------------------------


def synthetic_state_dict(param_shapes, seed, dtype=torch.float32, norm_gain_offset=1.0):
    """N(0, 0.02) for every parameter in the given (name, shape) order, drawn from
    numpy's PCG64 generator seeded with `seed` (identical on every platform); q_norm /
    k_norm gains then get +norm_gain_offset so attention is not uniform (the gains
    would otherwise be ~0.02)."""
    g = np.random.default_rng(seed)
    sd = {}
    for name, shape in param_shapes:
        t = torch.from_numpy(g.standard_normal(tuple(shape), dtype=np.float32) * np.float32(0.02))
        if name.endswith(("q_norm.weight", "k_norm.weight")):
            t = t + norm_gain_offset
        sd[name] = t.to(dtype)
    return sd
