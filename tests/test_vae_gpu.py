"""Video VAE decoder on the B200: each kernel against a float32 PyTorch restatement of
its op (convolution, GroupNorm) or the CPU oracle (PixelNorm, rearranges, bit-exact
where the op is a permutation), and the whole drop-in ConvVideoDecoder against the
reference's own output (tests/golden/vae_tiny_*.pt)."""

import pytest
import torch
import torch.nn.functional as F

import _native as nat
import golden_cases as gc
from oracle import vae_oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rel_l2(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def to_cl(x):  # (B, C, F, H, W) -> (B, F, H, W, C)
    return x.permute(0, 2, 3, 4, 1).contiguous()


def from_cl(x):
    return x.permute(0, 4, 1, 2, 3).contiguous()


def conv_ref(x_cl, w, b, ksize, causal):
    """float32 restatement of CausalConv3d / the 1x1x1 Conv3d on the device."""
    x = from_cl(x_cl).float()
    if ksize == 1:
        return to_cl(F.conv3d(x, w.float(), b.float()))
    return to_cl(vae_oracle.conv3d_same(x, w.float(), b.float(), causal))


@pytest.mark.parametrize("b,f,h,w,cin,cout,k,causal,res", [
    (2, 3, 5, 7, 64, 48, 3, False, False),     # cout < 64: one 64-wide tile, masked
    (1, 4, 8, 20, 128, 256, 3, False, True),   # residual add in the epilogue
    (1, 2, 3, 45, 64, 320, 3, True, False),    # causal padding, ragged N (320 = 256 + 64), ragged M
    (2, 2, 4, 6, 256, 128, 1, False, True),    # 1x1x1 shortcut with residual
    (1, 9, 16, 24, 64, 64, 3, False, False),   # the fixture's last-stage shape
])
def test_conv3d_matches_float32(b, f, h, w, cin, cout, k, causal, res):
    torch.manual_seed(21)
    x = torch.randn(b, f, h, w, cin, device=DEV).to(torch.bfloat16)
    wt = (torch.randn(cout, cin, k, k, k, device=DEV) * (cin * k ** 3) ** -0.5).to(torch.bfloat16)
    bias = torch.randn(cout, device=DEV).to(torch.bfloat16)
    packed = wt.permute(0, 2, 3, 4, 1).reshape(cout, k ** 3, cin).contiguous()
    r = torch.randn(b, f, h, w, cout, device=DEV).to(torch.bfloat16) if res else None
    out = torch.empty(b, f, h, w, cout, device=DEV, dtype=torch.bfloat16)
    nat.conv3d(x, packed, bias, out, k, causal, r)
    torch.cuda.synchronize()
    assert nat.device_error_flags() == 0
    ref = conv_ref(x, wt, bias, k, causal) + (r.float() if res else 0)
    assert rel_l2(out, ref) < 4e-3


@pytest.mark.parametrize("cout", [64, 128, 256])
def test_conv3d_fused_pixel_norm_matches_unfused(cout):
    """conv + bias, then PixelNorm + SiLU in the epilogue == the conv followed by
    ltx_pixel_norm (up to the channel-sum order of the mean)."""
    torch.manual_seed(27)
    x = torch.randn(1, 3, 6, 20, 128, device=DEV).to(torch.bfloat16)
    wt = (torch.randn(cout, 27, 128, device=DEV) * (27 * 128) ** -0.5).to(torch.bfloat16)
    bias = (0.1 * torch.randn(cout, device=DEV)).to(torch.bfloat16)
    fused = torch.empty(1, 3, 6, 20, cout, device=DEV, dtype=torch.bfloat16)
    nat.conv3d(x, wt, bias, fused, 3, norm_silu_eps=1e-8)
    plain = torch.empty_like(fused)
    nat.conv3d(x, wt, bias, plain, 3)
    nat.pixel_norm(plain, plain, 1e-8, True)
    torch.cuda.synchronize()
    assert nat.device_error_flags() == 0
    assert rel_l2(fused, plain) < 2e-3
    assert (fused.float() - plain.float()).abs().max() <= 2 ** -6 * plain.float().abs().max()
    with pytest.raises(nat.LtxError):
        nat.conv3d(x, wt, bias, fused, 3, residual=fused, norm_silu_eps=1e-8)


def test_conv3d_residual_in_place_and_errors():
    torch.manual_seed(22)
    x = torch.randn(1, 2, 4, 4, 64, device=DEV).to(torch.bfloat16)
    wt = (torch.randn(64, 27, 64, device=DEV) * 0.02).to(torch.bfloat16)
    bias = torch.zeros(64, device=DEV, dtype=torch.bfloat16)
    acc = torch.randn(1, 2, 4, 4, 64, device=DEV).to(torch.bfloat16)
    expect = torch.empty_like(acc)
    nat.conv3d(x, wt, bias, expect, 3, False, acc.clone())
    nat.conv3d(x, wt, bias, acc, 3, False, acc)  # out is its own residual
    torch.cuda.synchronize()
    assert torch.equal(acc, expect)
    with pytest.raises(nat.LtxError):
        nat.conv3d(x, wt, bias, x, 3)  # in place over the input
    with pytest.raises(ValueError):
        nat.conv3d(x, wt[:, :1], bias, acc, 3)


@pytest.mark.parametrize("c", [64, 128, 256, 512, 1024, 96])
def test_pixel_norm_silu_matches_oracle(c):
    """Every channel count the decoder uses (and a generic one), with a voxel count that is
    not a multiple of the voxels a warp takes."""
    torch.manual_seed(23)
    x = (torch.randn(2, 3, 5, 7, c, device=DEV) * 3).to(torch.bfloat16)
    for silu in (False, True):
        y = torch.empty_like(x)
        nat.pixel_norm(x, y, 1e-8, silu)
        ref = vae_oracle.pixel_norm(from_cl(x).cpu())
        ref = to_cl(F.silu(ref) if silu else ref)
        assert rel_l2(y.cpu(), ref) < 4e-3
        assert (y.cpu().float() - ref.float()).abs().max() <= 2 ** -6 * ref.float().abs().max()


def test_group_norm1_matches_float32():
    torch.manual_seed(24)
    x = (torch.randn(2, 3, 4, 5, 128, device=DEV) * 2 + 0.5).to(torch.bfloat16)
    wt = (1 + 0.1 * torch.randn(128, device=DEV)).to(torch.bfloat16)
    bs = (0.1 * torch.randn(128, device=DEV)).to(torch.bfloat16)
    y = torch.empty_like(x)
    nat.group_norm1(x, wt, bs, 1e-6, y, nat.group_norm1_workspace(2, x.device))
    ref = to_cl(F.group_norm(from_cl(x).float(), 1, wt.float(), bs.float(), 1e-6))
    assert rel_l2(y, ref) < 4e-3


@pytest.mark.parametrize("stride", [(2, 2, 2), (2, 1, 1), (1, 2, 2)])
def test_depth_to_space_is_the_reference_rearrange(stride):
    p1, p2, p3 = stride
    torch.manual_seed(25)
    x = torch.randn(2, 3, 4, 5, 16 * p1 * p2 * p3, device=DEV).to(torch.bfloat16)
    y = torch.empty(2, 3 * p1 - int(p1 == 2), 4 * p2, 5 * p3, 16, device=DEV, dtype=torch.bfloat16)
    nat.depth_to_space(x, stride, p1 == 2, y)
    ref = to_cl(vae_oracle.depth_to_space(from_cl(x).cpu(), stride))
    assert torch.equal(y.cpu(), ref)


def test_latent_in_and_unpatchify_are_exact():
    torch.manual_seed(26)
    lat = torch.randn(2, 128, 3, 4, 6).to(torch.bfloat16)
    std, mean = 1 + 0.1 * torch.randn(128), 0.1 * torch.randn(128)
    y = torch.empty(2, 3, 4, 6, 128, device=DEV, dtype=torch.bfloat16)
    nat.vae_latent_in(lat.to(DEV), std.to(DEV), mean.to(DEV), y)
    ref = to_cl(lat * std.to(lat).view(1, -1, 1, 1, 1) + mean.to(lat).view(1, -1, 1, 1, 1))
    assert torch.equal(y.cpu(), ref)
    for w_ in (5, 6):  # 16-byte stores when W * p is a multiple of 8, scalar stores otherwise
        z = torch.randn(2, 5, 4, w_, 48).to(torch.bfloat16)
        out = torch.empty(2, 3, 5, 16, w_ * 4, device=DEV, dtype=torch.bfloat16)
        nat.vae_unpatchify(z.to(DEV), 4, out)
        b, f, h, w, c = z.shape
        zr = from_cl(z).reshape(b, 3, 1, 4, 4, f, h, w).permute(0, 1, 5, 2, 6, 4, 7, 3).reshape(b, 3, f, h * 4, w * 4)
        assert torch.equal(out.cpu(), zr)
    frames = torch.empty(5, 16, 24, 3, device=DEV)
    nat.vae_unpatchify(z.to(DEV), 4, frames, frames=True)
    assert torch.equal(frames.cpu(), vae_oracle.decode_video_frames(zr))


def _decoder(rec):
    import ltx_vae

    dec = ltx_vae.ConvVideoDecoder(rec["config"])
    sd = vae_oracle.synthetic_decoder_state_dict(rec["param_shapes"], rec["weight_seed"],
                                                 rec["config"]["latent_channels"])
    dec.load_state_dict(sd)
    return dec.to(DEV).eval()


def test_vae_decoder_matches_reference_golden():
    """The drop-in ConvVideoDecoder (bf16, as the reference runs it) against the
    reference's output: the bf16 run at the 1e-2 bar, the float32 run at 2e-2 (our
    decoder computes in bf16 only)."""
    rec = torch.load(gc.GOLDEN / "vae_tiny_bfloat16.pt", weights_only=False)
    rec32 = torch.load(gc.GOLDEN / "vae_tiny_float32.pt", weights_only=False)
    dec = _decoder(rec)
    out = dec(rec["latent"].to(DEV))
    torch.cuda.synchronize()
    assert nat.device_error_flags() == 0
    assert out.shape == rec["out"].shape and out.dtype == torch.bfloat16
    assert rel_l2(out.cpu(), rec["out"]) < 1e-2
    assert rel_l2(out.cpu(), rec32["out"]) < 2e-2
    frames = dec.decode_video(rec["latent"].to(DEV))
    assert frames.shape == (9, 64, 96, 3) and frames.dtype == torch.float32
    assert rel_l2(frames.cpu(), vae_oracle.decode_video_frames(rec["out"])) < 1e-2
