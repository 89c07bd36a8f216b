"""CPU restatement of the LTX-2.5 video VAE decoder -- TEST INFRASTRUCTURE ONLY.

The checker for ltx-nv_b200/ltx_vae.py: only tests/ may import it. It restates, op for op
in the input's torch dtype, ConvVideoDecoder.forward of lipaul/ltx-nv
standalone/ltx_vae.py:161-216 (timestep_conditioning=False, 'zeros' spatial padding,
non-causal temporal padding as the decoder calls it) as plain functions over a state
dict with the reference's parameter names, on (B, C, F, H, W) CPU tensors. The tests pin
it against fixtures produced by the reference itself (tests/golden/make_golden.py,
vae_tiny_*.pt).
"""

from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F


def pixel_norm(x: torch.Tensor, eps: float = 1e-8) -> torch.Tensor:
    """ltx_vae.py:20-28: RMS over the channel dim."""
    return x / torch.sqrt(torch.mean(x ** 2, dim=1, keepdim=True) + eps)


def conv3d_same(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, causal: bool = False) -> torch.Tensor:
    """CausalConv3d.forward (ltx_vae.py:47-57), kernel 3: edge frames repeated in time
    (both ends, or twice in front when causal), zero padding 1 in H and W."""
    if causal:
        xp = torch.cat([x[:, :, :1]] * 2 + [x], dim=2)
    else:
        xp = torch.cat([x[:, :, :1], x, x[:, :, -1:]], dim=2)
    return F.conv3d(xp, w, b, padding=(0, 1, 1))


def resnet_block(sd: dict, p: str, x: torch.Tensor, cin: int, cout: int) -> torch.Tensor:
    """ResnetBlock3D.forward (ltx_vae.py:107-112)."""
    h = F.silu(pixel_norm(x))
    h = conv3d_same(h, sd[p + "conv1.conv.weight"], sd[p + "conv1.conv.bias"])
    h = F.silu(pixel_norm(h))
    h = conv3d_same(h, sd[p + "conv2.conv.weight"], sd[p + "conv2.conv.bias"])
    if cin != cout:
        s = F.group_norm(x, 1, sd[p + "norm3.weight"], sd[p + "norm3.bias"], 1e-6)
        s = F.conv3d(s, sd[p + "conv_shortcut.weight"], sd[p + "conv_shortcut.bias"])
    else:
        s = x
    return s + h


def depth_to_space(x: torch.Tensor, stride) -> torch.Tensor:
    """DepthToSpaceUpsample's rearrange (ltx_vae.py:138-143)."""
    p1, p2, p3 = stride
    b, c, d, h, w = x.shape
    c2 = c // (p1 * p2 * p3)
    y = x.reshape(b, c2, p1, p2, p3, d, h, w).permute(0, 1, 5, 2, 6, 3, 7, 4)
    y = y.reshape(b, c2, d * p1, h * p2, w * p3)
    return y[:, :, 1:] if p1 == 2 else y


def decoder_plan(cfg: dict):
    """The decoder's block list in execution order (ltx_vae.py:150-200): (kind, prefix,
    cin, cout, extra), plus the patch size and final channel count."""
    blocks = cfg["decoder_blocks"]
    base = cfg.get("decoder_base_channels", 128)
    mult = 1
    for name, params in blocks:
        c = {"multiplier": params} if isinstance(params, int) else params
        if name in ("compress_time", "compress_space", "compress_all"):
            mult *= c.get("multiplier", 1)
        elif name == "res_x_y":
            mult *= c.get("multiplier", 2)
    ch = base * mult
    plan = []
    for i, (name, params) in enumerate(reversed(blocks)):
        c = {"num_layers": params} if isinstance(params, int) else params
        p = f"up_blocks.{i}."
        if name == "res_x":
            for j in range(c["num_layers"]):
                plan.append(("res", f"{p}res_blocks.{j}.", ch, ch, None))
        elif name == "res_x_y":
            m = c.get("multiplier", 2)
            plan.append(("res", p, ch, ch // m, None))
            ch //= m
        else:
            stride = {"compress_time": (2, 1, 1), "compress_space": (1, 2, 2), "compress_all": (2, 2, 2)}[name]
            red = c.get("multiplier", 1)
            plan.append(("d2s", p, ch, math.prod(stride) * ch // red, stride))
            ch //= red
    return plan, cfg.get("patch_size", 4), ch


def decode(sd: dict, cfg: dict, latent: torch.Tensor) -> torch.Tensor:
    """ConvVideoDecoder.forward (ltx_vae.py:201-216): (B, C, F, H, W) latent ->
    (B, 3, F', H'*p, W'*p) in the latent's dtype."""
    dt = latent.dtype
    std = sd["per_channel_statistics.std-of-means"].to(dt).view(1, -1, 1, 1, 1)
    mean = sd["per_channel_statistics.mean-of-means"].to(dt).view(1, -1, 1, 1, 1)
    x = latent * std + mean
    x = conv3d_same(x, sd["conv_in.conv.weight"], sd["conv_in.conv.bias"])
    plan, p, _ = decoder_plan(cfg)
    for kind, pre, cin, cout, stride in plan:
        if kind == "res":
            x = resnet_block(sd, pre, x, cin, cout)
        else:
            x = depth_to_space(conv3d_same(x, sd[pre + "conv.conv.weight"], sd[pre + "conv.conv.bias"]), stride)
    x = F.silu(pixel_norm(x))
    x = conv3d_same(x, sd["conv_out.conv.weight"], sd["conv_out.conv.bias"])
    b, c, f, h, w = x.shape
    # channel = ((c * 1 + pt) * p + r) * p + q; r -> width offset, q -> height offset
    x = x.reshape(b, c // (p * p), 1, p, p, f, h, w).permute(0, 1, 5, 2, 6, 4, 7, 3)
    return x.reshape(b, c // (p * p), f, h * p, w * p)


def decode_video_frames(out: torch.Tensor) -> torch.Tensor:
    """decode_video's post-processing (ltx_vae.py:218-222) of a forward output."""
    return out[0].permute(1, 2, 3, 0).float().add(1.0).mul(0.5).clamp(0.0, 1.0)


def synthetic_decoder_state_dict(param_shapes, seed: int, latent_channels: int) -> dict:
    """Seeded synthetic decoder weights (numpy PCG64, platform-independent): N(0, 0.02)
    for every parameter in order, GroupNorm gains 1 + N(0, 0.02), and the per-channel
    statistics std = 1 + 0.1 N, mean = 0.1 N (seeds seed + 1, seed + 2)."""
    g = np.random.default_rng(seed)
    sd = {}
    for name, shape in param_shapes:
        t = torch.from_numpy(g.standard_normal(tuple(shape), dtype=np.float32) * np.float32(0.02))
        sd[name] = t + 1.0 if name.endswith("norm3.weight") else t
    for key, sd_seed, off, scale in (("std-of-means", seed + 1, 1.0, 0.1), ("mean-of-means", seed + 2, 0.0, 0.1)):
        v = np.random.default_rng(sd_seed).standard_normal((latent_channels,), dtype=np.float32) * np.float32(scale)
        sd["per_channel_statistics." + key] = torch.from_numpy(v) + off
    return sd
