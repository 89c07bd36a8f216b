"""Kernel-level parity on the B200: every libltxb200 entry point against the CPU oracle
(Philox) or a float32 PyTorch restatement of the same op (floating-point kernels)."""

import hashlib
import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F

import _native as nat
import golden_cases as gc
from oracle import ltx_oracle, philox_oracle

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rel_l2(a, b):
    a, b = a.float(), b.float()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


def bits16(t):
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)


# ------------------------------------------------------------------------------ Philox


def test_philox_matches_reference_golden_noise_bit_exact():
    g = np.load(gc.GOLDEN / "philox_m1.npz")
    n_v = int(g["video_numel"])
    grid_v, grid_a = int(g["ada_grid_video"]), int(g["ada_grid_audio"])
    v = torch.empty(n_v, dtype=torch.bfloat16, device=DEV)
    nat.philox_randn(v, int(g["seed"]), 0, grid_v)
    off = nat.philox_offset_increment(n_v, grid_v)
    a = torch.empty(g["audio"].size, dtype=torch.bfloat16, device=DEV)
    nat.philox_randn(a, int(g["seed"]), off, grid_a)
    vb = bits16(v)
    assert hashlib.sha256(vb.tobytes()).digest() == g["video_sha256"].tobytes()
    assert (vb[: g["video_prefix"].size] == g["video_prefix"]).all()
    assert (bits16(a) == g["audio"]).all()


@pytest.mark.parametrize("shape,seed,dtype", [((2, 128, 16, 16, 24), 42, torch.float32),
                                               ((1, 480, 128), 0, torch.float32),
                                               ((1, 3456, 128), 10, torch.bfloat16),
                                               ((3, 1001), 7, torch.float32),
                                               ((5,), 3, torch.bfloat16)])
def test_philox_bit_exact_vs_torch_randn_on_this_device(shape, seed, dtype):
    gen = torch.Generator(device=DEV).manual_seed(seed)
    ref1 = torch.randn(shape, dtype=dtype, device=DEV, generator=gen)
    ref2 = torch.randn(shape, dtype=dtype, device=DEV, generator=gen)
    n = ref1.numel()
    grid = nat.philox_grid(n)
    out = torch.empty(shape, dtype=dtype, device=DEV)
    nat.philox_randn(out, seed, 0, grid)
    assert torch.equal(out, ref1)
    nat.philox_randn(out, seed, nat.philox_offset_increment(n, grid), grid)
    assert torch.equal(out, ref2)


def test_philox_raw_words_match_c_restatement():
    threads, rounds, seed, offset = 700, 3, 0x1234_5678_9ABC, 8
    out = torch.empty(threads * rounds * 4, dtype=torch.int32, device=DEV)
    nat.philox_raw(out, threads, rounds, seed, offset)
    got = out.cpu().numpy().view(np.uint32)
    ref = philox_oracle.philox_raw(threads, rounds, seed, offset)
    assert (got == ref).all()


def test_philox_fp32_within_ulp_of_oracle_at_b200_grid():
    n = 2 * 128 * 16 * 16 * 24
    grid = nat.philox_grid(n)
    out = torch.empty(n, dtype=torch.float32, device=DEV)
    nat.philox_randn(out, 42, 0, grid)
    ref = philox_oracle.randn(n, 42, 0, grid)
    got = out.cpu().numpy().astype(np.float64)
    assert np.abs(got - ref).max() < 1e-4


# ------------------------------------------------------------------------- element-wise


def _mod_ref(table, mod, b, idx, d):
    return (table[idx].float() + mod.view(mod.shape[0], -1)[b, idx * d:(idx + 1) * d].float())


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("d", [64, 2048, 4096])
@pytest.mark.parametrize("kind", [nat.LTX_NORM_RMS, nat.LTX_NORM_LAYER])
def test_norm_modulate(dtype, d, kind):
    torch.manual_seed(0)
    b, t = 2, 37
    x = torch.randn(b * t, d, device=DEV).to(dtype)
    table = (torch.randn(6, d, device=DEV) * 0.1).to(dtype)
    mod = (torch.randn(b, 6 * d, device=DEV) * 0.1).to(dtype)
    y = torch.empty_like(x)
    m = nat.modulation(table, mod, shift=(0, 0), scale=(d, d), mod_ld_batch=6 * d)
    nat.norm_modulate(x, y, t, kind, 1e-6, m)
    xf = x.float().view(b, t, d)
    n = F.rms_norm(xf, (d,), eps=1e-6) if kind == nat.LTX_NORM_RMS else F.layer_norm(xf, (d,), eps=1e-6)
    sh = torch.stack([_mod_ref(table, mod, i, 0, d) for i in range(b)])[:, None]
    sc = torch.stack([_mod_ref(table, mod, i, 1, d) for i in range(b)])[:, None]
    ref = (n * (1 + sc) + sh).view(b * t, d)
    assert rel_l2(y, ref) < (1e-6 if dtype == torch.float32 else 8e-3)


@pytest.mark.parametrize("kind", [nat.LTX_NORM_RMS, nat.LTX_NORM_LAYER])
def test_norm_modulate_rows_path_matches_generic(kind):
    """bf16, D = 2048 with per-sample modulation takes the warp-per-row kernel; the same
    values given as a per-token modulation take the generic kernel. Apart from the order
    of the row reduction the two compute the same rounding sequence."""
    torch.manual_seed(3)
    b, t, d = 2, 300, 2048
    x = torch.randn(b * t, d, device=DEV, dtype=torch.bfloat16)
    table = (torch.randn(6, d, device=DEV) * 0.1).to(torch.bfloat16)
    mod = (torch.randn(b, 6 * d, device=DEV) * 0.1).to(torch.bfloat16)
    y_rows = torch.empty_like(x)
    nat.norm_modulate(x, y_rows, t, kind, 1e-6, nat.modulation(table, mod, shift=(0, 0), scale=(d, d),
                                                                   mod_ld_batch=6 * d))
    mod_tok = mod[:, None, :].expand(b, t, 6 * d).contiguous()
    y_gen = torch.empty_like(x)
    nat.norm_modulate(x, y_gen, t, kind, 1e-6, nat.modulation(table, mod_tok, shift=(0, 0), scale=(d, d),
                                                                  mod_ld_batch=t * 6 * d, mod_ld_tok=6 * d))
    torch.cuda.synchronize()
    assert rel_l2(y_rows, y_gen) < 1e-3
    assert (y_rows != y_gen).float().mean().item() < 0.01


def test_norm_modulate_per_token_and_plain():
    torch.manual_seed(1)
    b, t, d = 2, 16, 256
    x = torch.randn(b * t, d, device=DEV, dtype=torch.bfloat16)
    mod = (torch.randn(b, t, 2 * d, device=DEV) * 0.1).to(torch.bfloat16)
    y = torch.empty_like(x)
    m = nat.modulation(None, mod, shift=(0, 0), scale=(0, d), mod_ld_batch=t * 2 * d, mod_ld_tok=2 * d)
    nat.norm_modulate(x, y, t, nat.LTX_NORM_RMS, 1e-6, m)
    n = F.rms_norm(x.float().view(b, t, d), (d,), eps=1e-6)
    ref = n * (1 + mod[..., d:].float()) + mod[..., :d].float()
    assert rel_l2(y.view(b, t, d), ref) < 8e-3
    nat.norm_modulate(x, y, t, nat.LTX_NORM_RMS, 1e-6, None)
    assert rel_l2(y.view(b, t, d), n) < 5e-3


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("heads,hd", [(32, 64), (4, 16)])
def test_qk_norm_rope_pair_equals_two_passes(dtype, heads, hd):
    torch.manual_seed(16)
    rows, t = 2 * 300, 300
    d = heads * hd
    x = torch.randn(rows, 3 * d + 8, device=DEV).to(dtype)
    wq = (1 + 0.02 * torch.randn(d, device=DEV)).to(dtype)
    wk = (1 + 0.02 * torch.randn(d, device=DEV)).to(dtype)
    cos = torch.randn(t, d // 2, device=DEV).to(dtype)
    sin = torch.randn(t, d // 2, device=DEV).to(dtype)
    a, b = x.clone(), x.clone()
    nat.qk_norm_rope_pair(a, d, t, heads, hd, wq, wk, 1e-6, cos, sin, 0)
    nat.qk_norm_rope(b[:, :d], t, heads, hd, wq, 1e-6, cos, sin, 0)
    nat.qk_norm_rope(b[:, d:2 * d], t, heads, hd, wk, 1e-6, cos, sin, 0)
    torch.cuda.synchronize()
    assert torch.equal(a, b)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("heads,hd", [(32, 64), (32, 128), (4, 16), (2, 32)])
def test_qk_norm_rope_vs_oracle(dtype, heads, hd):
    torch.manual_seed(2)
    b, f, h, w = 2, 2, 3, 5
    t = f * h * w
    d = heads * hd
    pos = ltx_oracle.video_positions(b, f, h, w, 24.0)
    cos_r, sin_r = ltx_oracle.rope_tables(pos, d, dtype, 10000.0, [20, 2048, 2048], heads)
    x = torch.randn(b, t, d).to(dtype)
    wgt = (1 + 0.02 * torch.randn(d)).to(dtype)
    ref = ltx_oracle.apply_rope(ltx_oracle.rms_norm(x, 1e-6, wgt), (cos_r, sin_r))
    # tables on the GPU from the same positions
    freqs = ltx_oracle.freq_grid(10000.0, 3, d).to(DEV)
    cos = torch.empty(t, d // 2, device=DEV, dtype=dtype)
    sin = torch.empty_like(cos)
    nat.rope_tables(pos[0].contiguous().to(DEV), freqs, torch.tensor([20.0, 2048.0, 2048.0], device=DEV), d, cos,
                    sin)
    ref_cos = cos_r[0].transpose(0, 1).reshape(t, d // 2)
    assert rel_l2(cos.cpu(), ref_cos) < (1e-6 if dtype == torch.float32 else 4e-3)
    xd = x.view(b * t, d).to(DEV).clone()
    nat.qk_norm_rope(xd, t, heads, hd, wgt.to(DEV), 1e-6, cos, sin, rope_ld_batch=0)
    assert rel_l2(xd.cpu().view(b, t, d), ref) < (2e-6 if dtype == torch.float32 else 1e-2)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_gelu_gate_residual_timestep(dtype):
    torch.manual_seed(3)
    x = torch.randn(1000, 64, device=DEV).to(dtype)
    y = torch.empty_like(x)
    nat.gelu_tanh(x, y)
    assert rel_l2(y, F.gelu(x.float(), approximate="tanh")) < (1e-6 if dtype == torch.float32 else 5e-3)
    odd = torch.randn(1003, device=DEV).to(dtype)
    oy = torch.empty_like(odd)
    nat.gelu_tanh(odd, oy)
    assert rel_l2(oy, F.gelu(odd.float(), approximate="tanh")) < (1e-6 if dtype == torch.float32 else 5e-3)
    b, t, d = 2, 50, 64
    r = torch.randn(b * t, d, device=DEV).to(dtype)
    u = torch.randn(b * t, d, device=DEV).to(dtype)
    g = (torch.randn(b, 6 * d, device=DEV) * 0.5).to(dtype)
    table = torch.randn(6, d, device=DEV).to(dtype) * 0.1
    out = torch.empty_like(r)
    gm = nat.modulation(table, g, shift=None, scale=(2 * d, 2 * d), mod_ld_batch=6 * d)
    nat.gate_residual(r, u, out, t, gm)
    gate = torch.stack([_mod_ref(table, g, i, 2, d) for i in range(b)])[:, None]
    ref = (r.float().view(b, t, d) + u.float().view(b, t, d) * gate).view(b * t, d)
    assert rel_l2(out, ref) < (1e-6 if dtype == torch.float32 else 5e-3)
    ts = torch.tensor([0.5, 1.0, 0.03], device=DEV)
    emb = torch.empty(3, 256, device=DEV, dtype=dtype)
    nat.timestep_embedding(ts, 1000.0, 256, 10000.0, emb)
    ref = ltx_oracle.timestep_sinusoid(ts.cpu() * 1000, 256)
    assert (emb.float().cpu() - ref).abs().max() < (2e-3 if dtype == torch.float32 else 1e-2)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_cfg_euler_vs_oracle(dtype):
    torch.manual_seed(4)
    t, c = 300, 128
    lat = torch.randn(1, t, c).to(dtype)
    vel = torch.randn(2, t, c).to(dtype)
    sigmas = torch.linspace(1.0, 0.0, 9)
    idx = 2
    ts = torch.full((2, t), float(sigmas[idx]))
    x0 = (lat.repeat(2, 1, 1).float() - vel.float() * ts[..., None]).to(dtype)
    den_ref = ltx_oracle.guide_cfg(x0[0:1], x0[1:2], 3.0)
    nxt_ref = ltx_oracle.euler_step(lat, den_ref, sigmas, idx)
    den = torch.empty(1, t, c, device=DEV, dtype=dtype)
    nxt = torch.empty_like(den)
    nat.cfg_euler(vel.to(DEV), lat.to(DEV), ts.to(DEV), 3.0, float(sigmas[idx]), float(sigmas[idx + 1]), nxt, den)
    assert torch.equal(den.cpu(), den_ref)
    assert torch.equal(nxt.cpu(), nxt_ref)


# ------------------------------------------------------------------------------- GEMM


def _lin_ref(a, w, bias):
    return a.float() @ w.float().t() + (bias.float() if bias is not None else 0)


@pytest.mark.parametrize("m,n,k,bn", [(128, 256, 64, 0), (256, 256, 128, 0), (300, 384, 192, 128),
                                      (1000, 6176, 256, 0), (777, 2048, 2048, 128), (4096, 2048, 2048, 256),
                                      (40, 136, 72, 0), (12288, 512, 128, 0)])
def test_linear_bf16_tcgen05(m, n, k, bn):
    torch.manual_seed(5)
    a = torch.randn(m, k, device=DEV, dtype=torch.bfloat16)
    w = (torch.randn(n, k, device=DEV) * k ** -0.5).to(torch.bfloat16)
    bias = torch.randn(n, device=DEV, dtype=torch.bfloat16)
    c = torch.empty(m, n, device=DEV, dtype=torch.bfloat16)
    nat.gemm_set_tile_n(bn)
    try:
        nat.linear(a, w, c, nat.epilogue(bias=bias))
    finally:
        nat.gemm_set_tile_n(0)
    torch.cuda.synchronize()
    assert nat.device_error_flags() == 0
    assert rel_l2(c, _lin_ref(a, w, bias)) < 4e-3


@pytest.mark.parametrize("m,n,k", [(1000, 2080, 512), (12288, 2048, 2048), (300, 512, 128)])
def test_linear_bf16_cta_pair_matches_single(m, n, k):
    """The automatic choice runs N >= 512, M >= 256 on CTA pairs (cta_group::2, 256-row
    tiles); forcing 256-column single-CTA tiles runs the same K order per output, so the
    two must agree bit for bit for every epilogue kind, ragged M and N included."""
    torch.manual_seed(12)
    b = 2
    t = m // b
    a = torch.randn(m, k, device=DEV, dtype=torch.bfloat16)
    w = (torch.randn(n, k, device=DEV) * k ** -0.5).to(torch.bfloat16)
    bias = torch.randn(n, device=DEV, dtype=torch.bfloat16)
    table = torch.randn(6, n, device=DEV, dtype=torch.bfloat16) * 0.1
    mod = torch.randn(b, 6 * n, device=DEV, dtype=torch.bfloat16) * 0.1
    mask = (torch.arange(m, device=DEV) % 5 == 0).float()
    vec = torch.randn(n, device=DEV, dtype=torch.bfloat16)
    res = torch.randn(m, n, device=DEV, dtype=torch.bfloat16)
    epis = {
        "none": lambda c: nat.epilogue(bias=bias),
        "gelu": lambda c: nat.epilogue(nat.EPI_GELU_TANH, bias=bias),
        "gate_residual": lambda c: nat.epilogue(
            nat.EPI_GATE_RESIDUAL, bias=bias, residual=c,
            gate=nat.modulation(table, mod, shift=None, scale=(5 * n, 5 * n), mod_ld_batch=6 * n), rows_per_batch=t),
        "row_mask_add": lambda c: nat.epilogue(nat.EPI_ROW_MASK_ADD, bias=bias, row_mask=mask, row_vec=vec),
    }
    for name, mk in epis.items():
        outs = []
        for bn in (0, 256):
            c = res.clone()
            nat.gemm_set_tile_n(bn)
            try:
                nat.linear(a, w, c, mk(c))
            finally:
                nat.gemm_set_tile_n(0)
            outs.append(c)
        torch.cuda.synchronize()
        assert nat.device_error_flags() == 0
        assert torch.equal(outs[0], outs[1]), name
    assert rel_l2(outs[0], res.float() * 0 + _lin_ref(a, w, bias) + mask[:, None] * vec.float()) < 4e-3


def test_linear_bf16_strided_operands_and_epilogues():
    torch.manual_seed(6)
    b, t, d, k = 2, 200, 256, 512
    m = b * t
    big = torch.randn(m, 3 * k, device=DEV, dtype=torch.bfloat16)
    a = big[:, k:2 * k]  # strided view (ld = 3k)
    w = (torch.randn(d, k, device=DEV) * k ** -0.5).to(torch.bfloat16)
    bias = torch.randn(d, device=DEV, dtype=torch.bfloat16)
    base = _lin_ref(a, w, bias)
    # GELU
    c = torch.empty(m, d, device=DEV, dtype=torch.bfloat16)
    nat.linear(a, w, c, nat.epilogue(nat.EPI_GELU_TANH, bias=bias))
    assert rel_l2(c, F.gelu(base.to(torch.bfloat16).float(), approximate="tanh")) < 6e-3
    # gate * residual, in place
    res = torch.randn(m, d, device=DEV, dtype=torch.bfloat16)
    res0 = res.clone()
    table = torch.randn(6, d, device=DEV, dtype=torch.bfloat16) * 0.1
    mod = torch.randn(b, 6 * d, device=DEV, dtype=torch.bfloat16) * 0.1
    gm = nat.modulation(table, mod, shift=None, scale=(5 * d, 5 * d), mod_ld_batch=6 * d)
    nat.linear(a, w, res, nat.epilogue(nat.EPI_GATE_RESIDUAL, bias=bias, residual=res, gate=gm, rows_per_batch=t))
    gate = torch.stack([_mod_ref(table, mod, i, 5, d) for i in range(b)])[:, None]
    ref = (res0.float().view(b, t, d) + base.view(b, t, d) * gate).view(m, d)
    assert rel_l2(res, ref) < 5e-3
    # keyframe row add
    mask = (torch.arange(m, device=DEV) % 7 == 0).float()
    vec = torch.randn(d, device=DEV, dtype=torch.bfloat16)
    nat.linear(a, w, c, nat.epilogue(nat.EPI_ROW_MASK_ADD, bias=bias, row_mask=mask, row_vec=vec))
    assert rel_l2(c, base + mask[:, None] * vec.float()) < 4e-3


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("m,n,k", [(2, 12288, 2048), (3, 64, 256), (31, 300, 8192), (2, 2048, 256)])
def test_linear_skinny(dtype, m, n, k):
    torch.manual_seed(7)
    a = torch.randn(m, k, device=DEV).to(dtype)
    w = (torch.randn(n, k, device=DEV) * k ** -0.5).to(dtype)
    bias = torch.randn(n, device=DEV).to(dtype)
    c = torch.empty(m, n, device=DEV, dtype=dtype)
    nat.linear(a, w, c, nat.epilogue(bias=bias))
    assert rel_l2(c, _lin_ref(a, w, bias)) < (1e-5 if dtype == torch.float32 else 4e-3)
    nat.linear(a, w, c, nat.epilogue(nat.EPI_SILU, bias=bias, silu_input=True))
    ref = F.silu(_lin_ref(F.silu(a.float()).to(dtype), w, bias).to(dtype).float())
    assert rel_l2(c, ref) < (1e-5 if dtype == torch.float32 else 6e-3)


@pytest.mark.parametrize("m,n,k", [(480, 2048, 2048), (960, 8192, 512), (100, 100, 200)])
def test_linear_fp32_cuda_cores(m, n, k):
    torch.manual_seed(8)
    a = torch.randn(m, k, device=DEV)
    w = torch.randn(n, k, device=DEV) * k ** -0.5
    bias = torch.randn(n, device=DEV)
    c = torch.empty(m, n, device=DEV)
    nat.linear(a, w, c, nat.epilogue(bias=bias))
    ref = (a.double() @ w.double().t() + bias.double()).float()
    assert rel_l2(c, ref) < 1e-6


# -------------------------------------------------------------------------- attention


def _attn_ref(q, k, v, b, tq, tk, h, d, gate=None):
    qh = q.float().view(b, tq, h, d).transpose(1, 2)
    kh = k.float().view(b, tk, h, d).transpose(1, 2)
    vh = v.float().view(b, tk, h, d).transpose(1, 2)
    o = F.scaled_dot_product_attention(qh, kh, vh).transpose(1, 2)
    if gate is not None:
        o = o * (2 * torch.sigmoid(gate.float().view(b, tq, h, 1)))
    return o.reshape(b * tq, h * d)


# Tk <= 128 takes the persistent short-context kernel: ragged Tk and Tq, one key, runs of
# tasks that change (sample, head) inside a CTA, and the full text cross-attention shape.
@pytest.mark.parametrize("b,tq,tk,h,d", [(1, 128, 128, 2, 64), (2, 200, 300, 4, 64), (2, 6144, 128, 2, 64),
                                         (2, 126, 1000, 3, 64), (1, 256, 640, 2, 128), (2, 100, 126, 2, 128),
                                         (2, 1536, 1536, 32, 64), (3, 300, 77, 5, 64), (3, 1000, 1, 3, 128),
                                         (4, 40, 128, 7, 64), (2, 5000, 100, 37, 64), (2, 6144, 128, 32, 64)])
def test_attention_bf16_tcgen05(b, tq, tk, h, d):
    torch.manual_seed(9)
    # a fused QKV-like buffer: q, k, v and gate logits side by side (strided operands);
    # the gate block is padded so the row stride stays a multiple of 8 elements
    qkv = torch.randn(b * max(tq, tk), 3 * h * d + ((h + 7) // 8) * 8, device=DEV, dtype=torch.bfloat16)
    q = qkv[: b * tq, : h * d]
    k = qkv[: b * tk, h * d:2 * h * d]
    v = qkv[: b * tk, 2 * h * d:3 * h * d]
    gate = qkv[: b * tq, 3 * h * d:3 * h * d + h]
    o = torch.empty(b * tq, h * d, device=DEV, dtype=torch.bfloat16)
    nat.attention(q, k, v, o, b, tq, tk, h, d, d ** -0.5, gate)
    torch.cuda.synchronize()
    assert nat.device_error_flags() == 0
    assert rel_l2(o, _attn_ref(q, k, v, b, tq, tk, h, d, gate)) < 1e-2
    nat.attention(q, k, v, o, b, tq, tk, h, d, d ** -0.5, None)
    assert rel_l2(o, _attn_ref(q, k, v, b, tq, tk, h, d)) < 1e-2


# ltx_attention_ws splits the (sample, head, 256-query) units that would only partly fill
# a last wave of SMs into key-range parts merged by the last one. parts = 0: the
# automatic plan at the per-rank self-attention shapes of 1, 2 and 8 GPUs (it must
# split them); parts > 0: every unit forced through the part kernel, on a ragged query
# count, one key tile per part, parts = 1 (the merge of a single part), and head_dim 128.
@pytest.mark.parametrize("b,tq,tk,h,d,parts", [(2, 6144, 6144, 32, 64, 0), (1, 6144, 6144, 32, 64, 0),
                                               (1, 6144, 6144, 8, 64, 0), (1, 6144, 6144, 8, 128, 0),
                                               (2, 2000, 2048, 4, 64, 4), (1, 1000, 1536, 3, 64, 3),
                                               (1, 300, 384, 2, 64, 3), (2, 700, 1024, 2, 64, 1),
                                               (1, 1536, 1536, 2, 128, 2), (2, 520, 1024, 3, 128, 8)])
def test_attention_split_tail_matches_single_pass(b, tq, tk, h, d, parts):
    torch.manual_seed(16)
    nat.attention_force_split(parts)
    try:
        assert nat.load_library().ltx_attention_workspace_bytes(b, tq, tk, h, d) > 0, "shape must exercise the split"
        qkv = torch.randn(b * max(tq, tk), 3 * h * d + ((h + 7) // 8) * 8, device=DEV, dtype=torch.bfloat16)
        q, k, v = qkv[:b * tq, :h * d], qkv[:b * tk, h * d:2 * h * d], qkv[:b * tk, 2 * h * d:3 * h * d]
        gate = qkv[:b * tq, 3 * h * d:3 * h * d + h]
        whole = torch.empty(b * tq, h * d, device=DEV, dtype=torch.bfloat16)
        nat.attention(q, k, v, whole, b, tq, tk, h, d, d ** -0.5, gate, split_tail=False)
        ref = _attn_ref(q, k, v, b, tq, tk, h, d, gate)
        e_whole = rel_l2(whole, ref)
        first = None
        for _ in range(2):  # the second call starts from the counters the first one left
            split = torch.full_like(whole, float("nan"))
            nat.attention(q, k, v, split, b, tq, tk, h, d, d ** -0.5, gate)
            torch.cuda.synchronize()
            assert nat.device_error_flags() == 0
            # Each part rounds P = 2^(s - m) to bf16 against its own running maximum, so
            # split rows differ from the single pass by bf16 rounding; they must be as
            # accurate against exact arithmetic.
            e_split = rel_l2(split, ref)
            assert e_split < 1e-2 and e_split <= max(1.25 * e_whole, 5e-3), (e_split, e_whole)
            if first is None:
                first = split
            else:
                assert torch.equal(split, first), "the merge order is fixed: repeated calls are bit-identical"
        ws = nat.attention_workspace(b, tq, tk, h, d, torch.device(DEV))
        assert int(ws[:4096].view(torch.int32).abs().sum()) == 0, "arrival counters must return to zero"
    finally:
        nat.attention_force_split(0)


def test_attention_bf16_config5_sequence():
    """BASELINE config 5 length (T = 33x22x38 = 27588, not a multiple of the 128-key tile)
    for two heads, against a float32 reference computed in query chunks."""
    torch.manual_seed(15)
    t, h, d = 27588, 2, 64
    qkv = torch.randn(t, 3 * h * d + 8, device=DEV, dtype=torch.bfloat16)
    q, k, v = qkv[:, :h * d], qkv[:, h * d:2 * h * d], qkv[:, 2 * h * d:3 * h * d]
    gate = qkv[:, 3 * h * d:3 * h * d + h]
    o = torch.empty(t, h * d, device=DEV, dtype=torch.bfloat16)
    nat.attention(q, k, v, o, 1, t, t, h, d, d ** -0.5, gate)
    torch.cuda.synchronize()
    assert nat.device_error_flags() == 0
    ref = torch.empty(t, h * d, device=DEV)
    kh = k.float().view(t, h, d).transpose(0, 1)
    vh = v.float().view(t, h, d).transpose(0, 1)
    for r0 in range(0, t, 4096):
        qh = q[r0:r0 + 4096].float().view(-1, h, d).transpose(0, 1)
        p = torch.softmax(qh @ kh.transpose(1, 2) * d ** -0.5, dim=-1)
        out = (p @ vh).transpose(0, 1) * (2 * torch.sigmoid(gate[r0:r0 + 4096].float()))[..., None]
        ref[r0:r0 + 4096] = out.reshape(-1, h * d)
    assert rel_l2(o, ref) < 1e-2


@pytest.mark.parametrize("b,tq,tk,h,d", [(2, 480, 480, 32, 64), (2, 100, 8, 4, 16 * 2), (1, 70, 90, 2, 128)])
def test_attention_fp32(b, tq, tk, h, d):
    torch.manual_seed(10)
    q = torch.randn(b * tq, h * d, device=DEV)
    k = torch.randn(b * tk, h * d, device=DEV)
    v = torch.randn(b * tk, h * d, device=DEV)
    gate = torch.randn(b * tq, h, device=DEV)
    o = torch.empty(b * tq, h * d, device=DEV)
    nat.attention(q, k, v, o, b, tq, tk, h, d, d ** -0.5, gate)
    ref = _attn_ref(q.double(), k.double(), v.double(), b, tq, tk, h, d, gate.double())
    assert rel_l2(o, ref) < 1e-5


# ------------------------------------------------------------------- STG value pass-through, X0


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_value_gate_and_x0(dtype):
    torch.manual_seed(14)
    rows, h, d = 300, 4, 64
    qkv = torch.randn(rows, 3 * h * d + 8, device=DEV).to(dtype)
    v, g = qkv[:, 2 * h * d:3 * h * d], qkv[:, 3 * h * d:3 * h * d + h]
    o = torch.empty(rows, h * d, device=DEV, dtype=dtype)
    nat.value_gate(v, g, o, h, d)
    # reference op order: 2.0 * sigmoid(logit) in the activation dtype, then v * gate
    gate = (2.0 * torch.sigmoid(g)).to(dtype)
    ref = (v.view(rows, h, d) * gate.unsqueeze(-1)).reshape(rows, h * d)
    if dtype == torch.bfloat16:
        assert torch.equal(o, ref)
    else:
        assert rel_l2(o, ref) < 1e-6
    nat.value_gate(v, None, o, h, d)
    assert torch.equal(o, v)
    lat = torch.randn(rows, 128, device=DEV).to(dtype)
    vel = torch.randn(rows, 128, device=DEV).to(dtype)
    ts = torch.rand(rows, device=DEV)
    x = torch.empty_like(lat)
    nat.x0(lat, vel, ts, x)
    assert torch.equal(x, (lat.float() - vel.float() * ts[:, None]).to(dtype))


# ------------------------------------------------------------------- guidance


def test_guide_rescale_vs_reference_golden():
    """The reference's guide() outputs (std rescale on and off) against the device
    kernels through ltx_dit.guide; the workspace is reused across calls (its completion
    counter is left at zero by every call)."""
    import ltx_dit

    rec = torch.load(gc.GOLDEN / "guide.pt", weights_only=False)
    for dt, case in rec["cases"].items():
        xs = [x.to(DEV) for x in case["inputs"]]
        for (cfg, stg, rs, mod), ref in zip(rec["params"], case["outputs"]):
            p = ltx_dit.GuiderParams(cfg, stg, rs, mod, ())
            out1 = ltx_dit.guide(*xs, p)
            out2 = ltx_dit.guide(*xs, p)
            torch.cuda.synchronize()
            assert nat.device_error_flags() == 0
            assert torch.equal(out1, out2)
            tol = 1e-6 if dt == "float32" else 4e-3
            assert rel_l2(out1, ref.to(DEV)) < tol, (dt, cfg, stg, rs, mod)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_guide_rescale_zero_equals_plain_guide(dtype):
    torch.manual_seed(13)
    n = 3 * 4096 + 77
    xs = [torch.randn(n, device=DEV).to(dtype) for _ in range(4)]
    plain = torch.empty_like(xs[0])
    nat.guide(*xs, 3.0, 1.0, 2.0, plain)
    ws = nat.guide_rescale_workspace(n, xs[0].device)
    res = torch.empty_like(xs[0])
    nat.guide_rescale(*xs, 3.0, 1.0, 2.0, 0.0, res, ws)
    assert torch.equal(plain, res)
    # a large input (more blocks than the partial-sum table holds: grid-stride)
    n = 9_000_000
    xs = [torch.randn(n, device=DEV) for _ in range(4)]
    ws = nat.guide_rescale_workspace(n, xs[0].device)
    res = torch.empty_like(xs[0])
    nat.guide_rescale(*xs, 3.0, 1.0, 2.0, 0.5, res, ws)
    ref = ltx_oracle.guide(*[x.double() for x in xs], 3.0, 1.0, 0.5, 2.0)
    assert rel_l2(res, ref) < 1e-6


# ------------------------------------------------------------------- fused head + Euler


@pytest.mark.parametrize("t,k", [(300, 256), (6144, 2048)])
def test_proj_out_cfg_euler_bf16(t, k):
    torch.manual_seed(11)
    x = torch.randn(2 * t, k, device=DEV, dtype=torch.bfloat16)
    w = (torch.randn(128, k, device=DEV) * k ** -0.5).to(torch.bfloat16)
    bias = torch.randn(128, device=DEV, dtype=torch.bfloat16) * 0.1
    lat = torch.randn(t, 128, device=DEV, dtype=torch.bfloat16)
    ts = torch.full((2, t), 0.75, device=DEV)
    vel = torch.empty(2 * t, 128, device=DEV, dtype=torch.bfloat16)
    den = torch.empty(t, 128, device=DEV, dtype=torch.bfloat16)
    nxt = torch.empty_like(den)
    nat.proj_out_cfg_euler(x, w, bias, lat, ts, 3.0, 0.75, 0.625, nxt, den, vel)
    torch.cuda.synchronize()
    assert rel_l2(vel, _lin_ref(x, w, bias)) < 4e-3
    # the epilogue's update applied to the kernel's own velocity must equal the
    # element-wise kernel exactly
    den2 = torch.empty_like(den)
    nxt2 = torch.empty_like(den)
    nat.cfg_euler(vel, lat, ts, 3.0, 0.75, 0.625, nxt2, den2)
    assert torch.equal(den, den2) and torch.equal(nxt, nxt2)


@pytest.mark.parametrize("hd,parts,tk", [(64, 2, 6144), (64, 4, 6144), (128, 4, 1536)])
def test_split_kv_attention_merge_matches_full_attention(hd, parts, tk):
    """Split-KV attention as the video-to-audio attention runs under sequence
    parallelism: the keys cut into `parts` contiguous shards (one per rank), a partial
    attention per shard (fp32 O / l and log2-sum-exp), then the merge with the gate.
    Against the single-pass attention over all keys and against fp32 SDPA."""
    torch.manual_seed(3)
    heads, tq = 32, 126
    d = heads * hd
    q = torch.randn(tq, d + heads, device=DEV).to(torch.bfloat16)
    kv = torch.randn(tk, 2 * d, device=DEV).to(torch.bfloat16)
    full = torch.empty(tq, d, device=DEV, dtype=torch.bfloat16)
    nat.attention(q[:, :d], kv[:, :d], kv[:, d:], full, 1, tq, tk, heads, hd, hd ** -0.5, q[:, d:])
    sl = tk // parts
    o_all = torch.empty(parts, tq, d, device=DEV)
    lse_all = torch.empty(parts, tq, heads, device=DEV)
    for r in range(parts):
        shard = kv[r * sl:(r + 1) * sl]
        nat.attention_partial(q[:, :d], shard[:, :d], shard[:, d:], o_all[r], lse_all[r], 1, tq, sl, heads, hd,
                              hd ** -0.5)
    merged = torch.empty(tq, d, device=DEV, dtype=torch.bfloat16)
    nat.attention_merge(o_all, lse_all, q[:, d:], merged, heads, hd)
    torch.cuda.synchronize()
    assert nat.device_error_flags() == 0
    q4 = q[:, :d].float().view(tq, heads, hd).transpose(0, 1)
    k4 = kv[:, :d].float().view(tk, heads, hd).transpose(0, 1)
    v4 = kv[:, d:].float().view(tk, heads, hd).transpose(0, 1)
    ref = torch.nn.functional.scaled_dot_product_attention(q4, k4, v4).transpose(0, 1)
    ref = (ref * (2 * torch.sigmoid(q[:, d:].float()))[..., None]).reshape(tq, d)
    e_full, e_merged = rel_l2(full, ref), rel_l2(merged, ref)
    assert e_merged < 1e-2 and e_merged < 1.5 * e_full + 1e-3, (e_merged, e_full)
    assert rel_l2(merged, full) < 1e-2
    # the partial log-sum-exp is the natural one over the scaled scores, in log2 units
    s = torch.einsum("hqd,hkd->hqk", q4, k4[:, :sl]) * hd ** -0.5
    lse_ref = torch.logsumexp(s, dim=-1).transpose(0, 1) / math.log(2.0)
    assert torch.allclose(lse_all[0], lse_ref, atol=2e-2, rtol=1e-3)


def test_peer_barrier_wait_expires_and_reports_on_the_host():
    """The sequence-parallel flag barrier with a peer that never arrives (rank 0 of 2, the
    peer's slot in this rank's flag array stays 0) gives up after its limit, sets bit 2
    of the device error word and returns; the context keeps working."""
    assert nat.device_error_flags(clear=True) == 0
    flags = torch.zeros(2, dtype=torch.int32, device=DEV)
    counter = torch.zeros(1, dtype=torch.int32, device=DEV)
    nat.sp_barrier([flags.data_ptr(), flags.data_ptr()], counter.data_ptr(), 0, limit_cycles=2_000_000)
    torch.cuda.synchronize()
    assert int(counter.item()) == 1
    # both "ranks'" flag arrays are this one: rank 0 published its count in slot 0 and
    # waited for slot 1, which nothing writes
    assert flags.tolist() == [1, 0]
    assert nat.device_error_flags(clear=True) == 2
    assert nat.device_error_flags() == 0
    x = torch.randn(4096, device=DEV).to(torch.bfloat16)
    y = torch.empty_like(x)
    nat.gelu_tanh(x, y)
    torch.cuda.synchronize()
    assert rel_l2(y, torch.nn.functional.gelu(x.float(), approximate="tanh")) < 1e-2


def test_bounded_wait_expires_and_reports_on_the_host():
    """Failure detection without a GPU fault: a bounded mbarrier wait on a barrier that
    nothing arrives on (the wait the tcgen05 kernels use, with a 2M-cycle limit instead
    of ~4 s) gives up, sets the device error word and returns; the host reads the flag,
    clears it, and the context keeps working."""
    assert nat.device_error_flags(clear=True) == 0
    ret = torch.zeros(1, dtype=torch.int32, device=DEV)
    nat.test_bounded_wait(2_000_000, ret)
    torch.cuda.synchronize()
    assert int(ret.item()) == 1  # returned after giving up (2 would mean the wait completed)
    assert nat.device_error_flags(clear=True) == 1  # LTX_DEVERR_MBAR_TIMEOUT
    assert nat.device_error_flags() == 0
    x = torch.randn(4096, device=DEV).to(torch.bfloat16)
    y = torch.empty_like(x)
    nat.gelu_tanh(x, y)
    torch.cuda.synchronize()
    ref = torch.nn.functional.gelu(x.float(), approximate="tanh")
    assert rel_l2(y, ref) < 1e-2


# ------------------------------------------------------- sequence-parallel exchange kernels


@pytest.mark.parametrize("p,b,heads,hd,gated", [(4, 1, 32, 64, True), (2, 2, 32, 64, True), (2, 1, 16, 128, False)])
def test_sp_scatter_kernels_emulating_ranks_on_one_gpu(p, b, heads, hd, gated):
    """The fused Ulysses exchange with every "rank" on this GPU (all destination buffers
    local): ltx_qk_norm_rope_scatter must fill the receive buffers exactly as q/k norm +
    RoPE in place followed by pack and all-to-all would, and ltx_attention_scatter must
    deliver exactly what attention followed by all-to-all and unpack would."""
    torch.manual_seed(30)
    n = 384  # tokens per rank and sample
    dim, hp = heads * hd, heads // p
    dp = hp * hd
    t_full = n * p
    width = (3 * dp + (hp if gated else 0) + 7) // 8 * 8
    ldx = 3 * dim + (((heads + 7) // 8) * 8 if gated else 0)
    wq = (1 + 0.02 * torch.randn(dim, device=DEV)).to(torch.bfloat16)
    wk = (1 + 0.02 * torch.randn(dim, device=DEV)).to(torch.bfloat16)
    xs = [torch.randn(b * n, ldx, device=DEV).to(torch.bfloat16) for _ in range(p)]
    cos = [torch.randn(n, dim // 2, device=DEV).to(torch.bfloat16) for _ in range(p)]
    sin = [torch.randn(n, dim // 2, device=DEV).to(torch.bfloat16) for _ in range(p)]
    # reference: normalise in place, then the receive buffers all-to-all would deliver
    want = [torch.zeros(b * t_full, width, device=DEV, dtype=torch.bfloat16) for _ in range(p)]
    for r in range(p):
        y = xs[r].clone()
        nat.qk_norm_rope_pair(y, dim, n, heads, hd, wq, wk, 1e-6, cos[r], sin[r], 0)
        for j in range(p):
            rows = [bb * t_full + r * n + t for bb in range(b) for t in range(n)]
            blk = [y[:, j * dp:(j + 1) * dp], y[:, dim + j * dp:dim + (j + 1) * dp],
                   y[:, 2 * dim + j * dp:2 * dim + (j + 1) * dp]]
            if gated:
                blk.append(y[:, 3 * dim + j * hp:3 * dim + (j + 1) * hp])
            want[j][rows, :sum(t.shape[1] for t in blk)] = torch.cat(blk, 1)
    recv = [torch.zeros(b * t_full, width, device=DEV, dtype=torch.bfloat16) for _ in range(p)]
    for r in range(p):
        nat.qk_norm_rope_scatter(xs[r], n, heads, hd, wq, wk, 1e-6, cos[r], sin[r], gated, r,
                                 [t.data_ptr() for t in recv], width)
    torch.cuda.synchronize()
    for j in range(p):
        assert torch.equal(recv[j], want[j]), j
    # attention over each rank's heads, output rows to their token owners
    outs = [torch.zeros(b * n, dim, device=DEV, dtype=torch.bfloat16) for _ in range(p)]
    want_o = [torch.zeros(b * n, dim, device=DEV, dtype=torch.bfloat16) for _ in range(p)]
    for j in range(p):
        rv = recv[j]
        q, k, v = rv[:, :dp], rv[:, dp:2 * dp], rv[:, 2 * dp:3 * dp]
        g = rv[:, 3 * dp:3 * dp + hp] if gated else None
        o = torch.empty(b * t_full, dp, device=DEV, dtype=torch.bfloat16)
        nat.attention(q, k, v, o, b, t_full, t_full, hp, hd, hd ** -0.5, g)
        for r in range(p):
            rows = [bb * t_full + r * n + t for bb in range(b) for t in range(n)]
            want_o[r][:, j * dp:(j + 1) * dp] = o[rows]
        nat.attention_scatter(q, k, v, b, t_full, hp, hd, hd ** -0.5, g, [t.data_ptr() for t in outs], dim, j * dp)
    torch.cuda.synchronize()
    assert nat.device_error_flags() == 0
    for r in range(p):
        assert torch.equal(outs[r], want_o[r]), r
