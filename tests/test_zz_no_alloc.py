"""ltx_guide_rescale_noalloc (static-scratch variant) against ltx_guide_rescale with a
caller workspace. Collected last; it also passes on its own."""

import pytest
import torch

import _native as nat

DEV = "cuda"


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("n", [2, 4096, 4097, 6144 * 128, 256 * 4096])
def test_noalloc_matches_workspace_variant_two_calls(dtype, n):
    """n covers the smallest input, one block (4096 elements per block), two blocks, one
    benchmark video latent (192 blocks) and the limit, where 256 blocks fill the static
    scratch exactly."""
    torch.manual_seed(21)
    xs = [(torch.randn(n, device=DEV) * (1.0 + 0.1 * i)).to(dtype) for i in range(4)]
    ws = nat.guide_rescale_workspace(n, xs[0].device)
    for cfg, stg, mod, rs in ((3.0, 1.0, 3.0, 0.7), (4.5, 0.0, 1.0, 1.0)):
        ref = torch.empty_like(xs[0])
        nat.guide_rescale(*xs, cfg, stg, mod, rs, ref, ws)
        # two calls in a row: the second one starts from the counter the first left
        for _ in range(2):
            out = torch.full_like(xs[0], float("nan"))
            nat.guide_rescale_noalloc(*xs, cfg, stg, mod, rs, out)
            torch.cuda.synchronize()
            assert nat.device_error_flags() == 0
            assert torch.equal(out, ref)


@pytest.mark.gpu
def test_noalloc_rejects_oversize_n():
    n = 256 * 4096 + 1
    xs = [torch.zeros(n, device=DEV) for _ in range(4)]
    out = torch.empty_like(xs[0])
    with pytest.raises(nat.LtxError, match="static scratch"):
        nat.guide_rescale_noalloc(*xs, 3.0, 1.0, 3.0, 0.7, out)
