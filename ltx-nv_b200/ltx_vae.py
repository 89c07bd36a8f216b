"""Video VAE decoder of LTX-2.5 on the sm_100a kernels (drop-in for ConvVideoDecoder in
lipaul/ltx-nv standalone/ltx_vae.py:167-222).

Same class names, constructor arguments, parameter and buffer names as the reference,
so its state dicts (and `load_video_decoder`'s key mapping) load unchanged. The modules
keep torch Conv3d / GroupNorm objects only as parameter holders: every op of the forward
is a libltxb200 kernel on channels-last (B, F, H, W, C) bf16 activations:

  un_normalize + NCDHW -> channels-last   ltx_vae_latent_in
  CausalConv3d / 1x1x1 shortcut           ltx_conv3d (tcgen05 implicit GEMM, bias and
                                          residual add in the epilogue)
  PixelNorm + SiLU                        ltx_pixel_norm
  GroupNorm(1, C)                         ltx_group_norm1 (two passes)
  depth-to-space                          ltx_depth_to_space
  unpatchify / decode_video frames        ltx_vae_unpatchify

Only the decoder's configuration (timestep_conditioning=False, 'zeros' spatial
padding) is supported, as in the reference; other padding modes raise.
"""

from __future__ import annotations

import math

import torch

import _native as nat

PIXEL_NORM_EPS = 1e-8


def _cl_empty(like: torch.Tensor, shape) -> torch.Tensor:
    return torch.empty(tuple(shape), device=like.device, dtype=torch.bfloat16)


class PixelNorm(torch.nn.Module):
    """ltx_vae.py:20-28 (per-voxel RMS norm over channels)."""

    def __init__(self, dim: int = 1, eps: float = PIXEL_NORM_EPS):
        super().__init__()
        self.dim, self.eps = dim, eps

    def run(self, x: torch.Tensor, out: torch.Tensor, silu: bool) -> None:
        nat.pixel_norm(x, out, self.eps, silu)


class CausalConv3d(torch.nn.Module):
    """ltx_vae.py:31-57: 3x3x3 convolution, zero padding in H/W, edge-frame padding in time."""

    def __init__(self, in_channels, out_channels, kernel_size=3, spatial_padding_mode="zeros", **kw):
        super().__init__()
        if spatial_padding_mode != "zeros":
            raise NotImplementedError(f"spatial_padding_mode {spatial_padding_mode!r}")
        if kernel_size != 3:
            raise NotImplementedError("kernel_size 3 only (the decoder's convolutions)")
        self.time_kernel = kernel_size
        k = (kernel_size, kernel_size, kernel_size)
        self.conv = torch.nn.Conv3d(in_channels, out_channels, k, padding=(0, 1, 1), padding_mode=spatial_padding_mode,
                                    **kw)
        self._packed = None

    def packed(self) -> tuple[torch.Tensor, torch.Tensor]:
        return _pack_conv(self, self.conv, 27)

    def run(self, x: torch.Tensor, causal: bool = False, residual: torch.Tensor | None = None,
            out: torch.Tensor | None = None, norm_silu_eps: float | None = None) -> torch.Tensor:
        w, b = self.packed()
        if out is None:
            out = _cl_empty(x, x.shape[:-1] + (w.shape[0],))
        nat.conv3d(x, w, b, out, 3, causal, residual, norm_silu_eps)
        return out


def _pack_conv(owner: torch.nn.Module, conv: torch.nn.Conv3d, taps: int):
    """(cout, cin, kt, kh, kw) -> (cout, taps, cin) bf16, tap = (dt*3 + dh)*3 + dw; cached
    until the weight tensor changes."""
    wt = conv.weight
    key = (wt.data_ptr(), wt._version, conv.bias.data_ptr(), conv.bias._version)
    if owner._packed is None or owner._packed[0] != key:
        w = wt.detach().to(torch.bfloat16).permute(0, 2, 3, 4, 1).reshape(wt.shape[0], taps, wt.shape[1]).contiguous()
        b = conv.bias.detach().to(torch.bfloat16).contiguous()
        owner._packed = (key, w, b)
    return owner._packed[1], owner._packed[2]


class PerChannelStatistics(torch.nn.Module):
    """ltx_vae.py:76-87."""

    def __init__(self, channels: int):
        super().__init__()
        self.register_buffer("std-of-means", torch.ones(channels))
        self.register_buffer("mean-of-means", torch.zeros(channels))


class ResnetBlock3D(torch.nn.Module):
    """ltx_vae.py:94-115: x -> conv2(silu(norm(conv1(silu(norm(x)))))) + shortcut(x)."""

    def __init__(self, in_channels: int, out_channels: int, spatial_padding_mode: str):
        super().__init__()
        self.norm1 = PixelNorm()
        self.conv1 = CausalConv3d(in_channels, out_channels, 3, spatial_padding_mode)
        self.norm2 = PixelNorm()
        self.conv2 = CausalConv3d(out_channels, out_channels, 3, spatial_padding_mode)
        if in_channels != out_channels:
            self.norm3 = torch.nn.GroupNorm(1, in_channels, eps=1e-6)
            self.conv_shortcut = torch.nn.Conv3d(in_channels, out_channels, 1)
        else:
            self.norm3 = torch.nn.Identity()
            self.conv_shortcut = torch.nn.Identity()
        self._packed = None
        self._gn_ws = None
        self._gn = None

    def _norm3_params(self) -> tuple[torch.Tensor, torch.Tensor]:
        """GroupNorm weight and bias as bf16, cached until the parameters change."""
        w, b = self.norm3.weight, self.norm3.bias
        key = (w.data_ptr(), w._version, b.data_ptr(), b._version)
        if self._gn is None or self._gn[0] != key:
            self._gn = (key, w.detach().to(torch.bfloat16).contiguous(), b.detach().to(torch.bfloat16).contiguous())
        return self._gn[1], self._gn[2]

    def run(self, x: torch.Tensor, causal: bool = False) -> torch.Tensor:
        cout = self.conv1.conv.out_channels
        h = torch.empty_like(x)
        self.norm1.run(x, h, silu=True)
        if cout <= 256:
            # norm2 + SiLU in conv1's epilogue (the tile holds all cout channels of a voxel)
            h2 = self.conv1.run(h, causal, norm_silu_eps=self.norm2.eps)
        else:
            h2 = self.conv1.run(h, causal)
            self.norm2.run(h2, h2, silu=True)
        if isinstance(self.conv_shortcut, torch.nn.Conv3d):
            g = torch.empty_like(x)
            if self._gn_ws is None or self._gn_ws.device != x.device or self._gn_ws.numel() < x.shape[0] * 256:
                self._gn_ws = nat.group_norm1_workspace(x.shape[0], x.device)
            gw, gb = self._norm3_params()
            nat.group_norm1(x, gw, gb, self.norm3.eps, g, self._gn_ws)
            w, b = _pack_conv(self, self.conv_shortcut, 1)
            sc = _cl_empty(x, x.shape[:-1] + (cout,))
            nat.conv3d(g, w, b, sc, 1)
        else:
            sc = x
        return self.conv2.run(h2, causal, residual=sc)


class UNetMidBlock3D(torch.nn.Module):
    """ltx_vae.py:118-128."""

    def __init__(self, in_channels: int, num_layers: int, spatial_padding_mode: str):
        super().__init__()
        self.res_blocks = torch.nn.ModuleList(
            [ResnetBlock3D(in_channels, in_channels, spatial_padding_mode) for _ in range(num_layers)])

    def run(self, x: torch.Tensor, causal: bool = False) -> torch.Tensor:
        for blk in self.res_blocks:
            x = blk.run(x, causal)
        return x


class DepthToSpaceUpsample(torch.nn.Module):
    """ltx_vae.py:131-147: conv, then channels (c p1 p2 p3) -> (d p1)(h p2)(w p3); the first
    frame is dropped when the time stride is 2."""

    def __init__(self, in_channels: int, stride: tuple, out_channels_reduction: int, spatial_padding_mode: str):
        super().__init__()
        self.stride = stride
        self.out_channels = math.prod(stride) * in_channels // out_channels_reduction
        self.final_channels = in_channels // out_channels_reduction
        self.conv = CausalConv3d(in_channels, self.out_channels, 3, spatial_padding_mode)

    def run(self, x: torch.Tensor, causal: bool = False) -> torch.Tensor:
        p1, p2, p3 = self.stride
        y = self.conv.run(x, causal)
        b, f, h, w, _ = y.shape
        out = _cl_empty(x, (b, f * p1 - int(p1 == 2), h * p2, w * p3, self.final_channels))
        nat.depth_to_space(y, self.stride, p1 == 2, out)
        return out


def _bottleneck_channels(base: int, decoder_blocks: list) -> int:
    """ltx_vae.py:150-158."""
    mult = 1
    for name, params in decoder_blocks:
        cfg = {"multiplier": params} if isinstance(params, int) else params
        if name in ("compress_time", "compress_space", "compress_all"):
            mult *= cfg.get("multiplier", 1)
        elif name == "res_x_y":
            mult *= cfg.get("multiplier", 2)
    return base * mult


class ConvVideoDecoder(torch.nn.Module):
    """ltx_vae.py:161-222 (timestep_conditioning=False variant)."""

    def __init__(self, vae_cfg: dict):
        super().__init__()
        blocks = vae_cfg["decoder_blocks"]
        base = vae_cfg.get("decoder_base_channels", 128)
        patch = vae_cfg.get("patch_size", 4)
        pad_mode = vae_cfg.get("spatial_padding_mode", "zeros")
        in_ch = vae_cfg.get("latent_channels", 128)
        out_ch = vae_cfg.get("out_channels", 3) * patch ** 2
        ch = _bottleneck_channels(base, blocks)
        self.patch_size = patch
        self.per_channel_statistics = PerChannelStatistics(in_ch)
        self.conv_in = CausalConv3d(in_ch, ch, 3, pad_mode)
        self.up_blocks = torch.nn.ModuleList()
        for name, params in reversed(blocks):
            cfg = {"num_layers": params} if isinstance(params, int) else params
            if name == "res_x":
                blk: torch.nn.Module = UNetMidBlock3D(ch, cfg["num_layers"], pad_mode)
            elif name == "res_x_y":
                ch //= cfg.get("multiplier", 2)
                blk = ResnetBlock3D(ch * cfg.get("multiplier", 2), ch, pad_mode)
            elif name == "compress_time":
                blk = DepthToSpaceUpsample(ch, (2, 1, 1), cfg.get("multiplier", 1), pad_mode)
                ch = blk.final_channels
            elif name == "compress_space":
                blk = DepthToSpaceUpsample(ch, (1, 2, 2), cfg.get("multiplier", 1), pad_mode)
                ch = blk.final_channels
            elif name == "compress_all":
                blk = DepthToSpaceUpsample(ch, (2, 2, 2), cfg.get("multiplier", 1), pad_mode)
                ch = blk.final_channels
            else:
                raise ValueError(name)
            self.up_blocks.append(blk)
        self.conv_norm_out = PixelNorm()
        self.conv_out = CausalConv3d(ch, out_ch, 3, pad_mode)

    def _decode_cl(self, sample: torch.Tensor) -> torch.Tensor:
        """(B, C, F, H, W) latent -> channels-last (B, F, H, W, 3*p*p) output of conv_out."""
        if not sample.is_cuda:
            raise ValueError("ConvVideoDecoder runs on CUDA tensors only")
        b, c, f, h, w = sample.shape
        x = torch.empty(b, f, h, w, c, device=sample.device, dtype=torch.bfloat16)
        stats = self.per_channel_statistics
        nat.vae_latent_in(sample.to(torch.bfloat16), stats.get_buffer("std-of-means"),
                          stats.get_buffer("mean-of-means"), x)
        x = self.conv_in.run(x, causal=False)
        for blk in self.up_blocks:
            x = blk.run(x, causal=False)
        h_ = torch.empty_like(x)
        self.conv_norm_out.run(x, h_, silu=True)
        return self.conv_out.run(h_, causal=False)

    @torch.inference_mode()
    def forward(self, sample: torch.Tensor) -> torch.Tensor:
        """(B, latent C, F, H, W) -> (B, 3, F', H'*p, W'*p) bf16, as the reference."""
        y = self._decode_cl(sample)
        b, f, h, w, cc = y.shape
        p = self.patch_size
        out = torch.empty(b, cc // (p * p), f, h * p, w * p, device=y.device, dtype=torch.bfloat16)
        nat.vae_unpatchify(y, p, out)
        return out

    @torch.inference_mode()
    def decode_video(self, latent: torch.Tensor) -> torch.Tensor:
        """latent (B, 128, F', H', W') -> RGB frames (f, h, w, c) float in [0, 1] of sample 0
        (ltx_vae.py:218-222)."""
        y = self._decode_cl(latent)
        b, f, h, w, cc = y.shape
        p = self.patch_size
        frames = torch.empty(f, h * p, w * p, cc // (p * p), device=y.device, dtype=torch.float32)
        nat.vae_unpatchify(y, p, frames, frames=True)
        return frames


def load_video_decoder(path: str, device: torch.device | str = "cuda") -> ConvVideoDecoder:
    """ltx_vae.py:225-235: the decoder's config from the checkpoint metadata and its
    weights (keys `decoder.*` without the prefix, `per_channel_statistics.*` as is)."""
    import json

    from safetensors import safe_open

    with safe_open(path, framework="pt") as fh:
        meta = fh.metadata() or {}
        cfg = json.loads(meta["config"])["vae"]
        with torch.device("meta"):
            model = ConvVideoDecoder(cfg)
        sd = {}
        for k in fh.keys():
            if k.startswith("decoder."):
                sd[k.removeprefix("decoder.")] = fh.get_tensor(k)
            elif k.startswith("per_channel_statistics."):
                sd[k] = fh.get_tensor(k)
    res = model.load_state_dict(sd, strict=False, assign=True)
    if res.missing_keys:
        raise RuntimeError(f"video decoder missing: {res.missing_keys[:8]}")
    return model.to(device).eval()
