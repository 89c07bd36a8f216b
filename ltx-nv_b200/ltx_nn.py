"""B200-native neural building blocks of the LTX DiT (drop-in for lipaul/ltx-nv
standalone/ltx_nn.py).

Same module / function names, constructor arguments, parameter names and call
signatures as the reference; every forward runs libltxb200's sm_100a kernels through
_native (the reference runs cuBLAS + cuDNN SDPA + torch element-wise ops). Activations
are (B, T, D) CUDA tensors in float32 (the accuracy mode) or bfloat16.

Layout choices that differ inside (not at the API):
  * RoPE tables are kept token-major, (T, H*d/2), shared by all samples whose positions
    agree; precompute_freqs_cis returns them as (B, H, T, d/2) views of that storage so
    callers see the reference's shapes.
  * q, k, v and the gate logits of a self-attention are one packed (3D+H, D) weight:
    the module's own to_q / to_k / to_v / to_gate_logits parameters become views into
    it, so state_dict() is unchanged and nothing is stored twice.
"""

from __future__ import annotations

import functools
import math

import numpy
import torch

import _native as nat


def _rows(x: torch.Tensor) -> torch.Tensor:
    return x.reshape(-1, x.shape[-1])


def rms_norm(x: torch.Tensor, eps: float = 1e-6, weight: torch.Tensor | None = None) -> torch.Tensor:
    """ltx_nn.py:18-19. weight=None only (the learned-weight form is Attention's q/k norm)."""
    if weight is not None:
        raise NotImplementedError("rms_norm with a weight runs fused inside Attention (ltx_qk_norm_rope)")
    xr = _rows(x.contiguous())
    y = torch.empty_like(xr)
    nat.norm_modulate(xr, y, xr.shape[0], nat.LTX_NORM_RMS, eps, None)
    return y.view_as(x)


def sdpa(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mask: torch.Tensor | None = None) -> torch.Tensor:
    """ltx_nn.py:22-26: q, k, v (B, H, T, d) -> (B, H, T, d), non-causal, no mask."""
    if mask is not None:
        raise NotImplementedError("attention masks are not used by the LTX DiT path")
    b, h, tq, d = q.shape
    tk = k.shape[2]
    qt = q.transpose(1, 2).reshape(b * tq, h * d).contiguous()
    kt = k.transpose(1, 2).reshape(b * tk, h * d).contiguous()
    vt = v.transpose(1, 2).reshape(b * tk, h * d).contiguous()
    o = torch.empty_like(qt)
    nat.attention(qt, kt, vt, o, b, tq, tk, h, d, d ** -0.5, None)
    return o.view(b, tq, h, d).transpose(1, 2)


# ---------------------------------------------------------------------------------------
# RoPE (split type)
# ---------------------------------------------------------------------------------------


@functools.lru_cache(maxsize=8)
def generate_freq_grid_np(theta: float, n_axes: int, inner_dim: int) -> torch.Tensor:
    """ltx_nn.py:34-46: float64 frequency grid theta^linspace(0,1) * pi/2, as float32."""
    n_elem = 2 * n_axes
    pw = numpy.power(theta, numpy.linspace(0.0, 1.0, inner_dim // n_elem, dtype=numpy.float64))
    return torch.as_tensor(pw * math.pi / 2, dtype=torch.float32)


@functools.lru_cache(maxsize=8)
def generate_freq_grid_pytorch(theta: float, n_axes: int, inner_dim: int) -> torch.Tensor:
    """ltx_nn.py:49-60 (float32 grid)."""
    n_elem = 2 * n_axes
    idx = theta ** torch.linspace(math.log(1.0, theta), math.log(theta, theta), inner_dim // n_elem,
                                  dtype=torch.float32)
    return idx.to(torch.float32) * math.pi / 2


class RopeTables:
    """cos/sin tables (T, dim/2) per distinct sample, token-major, in the activation dtype.

    `ld_batch` is the element stride between samples (0 when every sample shares the
    same positions, the CFG case). `heads` is the head count the reference splits the
    table with (it fixes which RoPE pairs (j, j + d/2) belong together)."""

    def __init__(self, cos: torch.Tensor, sin: torch.Tensor, ld_batch: int, heads: int):
        self.cos, self.sin, self.ld_batch, self.heads = cos, sin, ld_batch, heads

    def reference_layout(self, batch: int) -> tuple[torch.Tensor, torch.Tensor]:
        """(B, H, T, d/2) views matching precompute_freqs_cis's return value."""
        t, half = self.cos.shape[-2], self.cos.shape[-1]
        h = self.heads

        def view(x):
            x = x.view(-1, t, h, half // h)
            if x.shape[0] == 1:
                x = x.expand(batch, -1, -1, -1)
            return x.permute(0, 2, 1, 3)

        return view(self.cos), view(self.sin)


def rope_tables(positions: torch.Tensor, dim: int, out_dtype: torch.dtype, theta: float, max_pos: list,
                heads: int, double_precision: bool = True) -> RopeTables:
    """Native RoPE tables for positions (B, n_axes, T, 2) (ltx_nn.py:63-96)."""
    b, n_axes, t, _ = positions.shape
    gen = generate_freq_grid_np if double_precision else generate_freq_grid_pytorch
    dev = positions.device
    freqs = gen(float(theta), n_axes, dim).to(dev)
    mp = torch.tensor([float(m) for m in max_pos[:n_axes]], dtype=torch.float32, device=dev)
    pos = positions.to(torch.float32)
    shared = b == 1 or bool((pos == pos[:1]).all())
    nb = 1 if shared else b
    cos = torch.empty(nb, t, dim // 2, device=dev, dtype=out_dtype)
    sin = torch.empty_like(cos)
    for i in range(nb):
        nat.rope_tables(pos[i].contiguous(), freqs, mp, dim, cos[i], sin[i])
    return RopeTables(cos, sin, 0 if shared else t * (dim // 2), heads)


def precompute_freqs_cis(indices_grid: torch.Tensor, dim: int, out_dtype: torch.dtype, theta: float = 10000.0,
                         max_pos: list[int] | None = None, use_middle_indices_grid: bool = True,
                         num_attention_heads: int = 32,
                         double_precision: bool = True) -> tuple[torch.Tensor, torch.Tensor]:
    """ltx_nn.py:63-96 -> (cos, sin) of shape (B, H, T, dim/2/H) (views of token-major tables)."""
    if not use_middle_indices_grid or indices_grid.ndim != 4:
        raise NotImplementedError("only the mid-point (B, n_axes, T, 2) position grid is used by LTX")
    tabs = rope_tables(indices_grid, dim, out_dtype, theta, max_pos or [20, 2048, 2048], num_attention_heads,
                       double_precision)
    return tabs.reference_layout(indices_grid.shape[0])


def _tables_from_reference_layout(freqs_cis) -> RopeTables:
    cos, sin = freqs_cis
    if isinstance(freqs_cis, RopeTables):
        return freqs_cis
    b, h, t, q = cos.shape
    base_c = cos.permute(0, 2, 1, 3)
    base_s = sin.permute(0, 2, 1, 3)
    if base_c.stride(0) == 0 or b == 1:
        c = base_c[:1].reshape(1, t, h * q).contiguous()
        s = base_s[:1].reshape(1, t, h * q).contiguous()
        return RopeTables(c, s, 0, h)
    c = base_c.reshape(b, t, h * q).contiguous()
    s = base_s.reshape(b, t, h * q).contiguous()
    return RopeTables(c, s, t * h * q, h)


def apply_split_rotary_emb(x: torch.Tensor, freqs_cis) -> torch.Tensor:
    """ltx_nn.py:99-115 (no norm): rotates pairs (j, j + d/2) of each head."""
    tabs = _tables_from_reference_layout(freqs_cis)
    if x.ndim == 4:
        b, h, t, d = x.shape
        xt = x.transpose(1, 2).reshape(b * t, h * d).contiguous()
    else:
        b, t, dd = x.shape
        xt = x.reshape(b * t, dd).contiguous()
    heads = tabs.heads
    hd = xt.shape[1] // heads
    # weight=None: rotation only (no q/k RMSNorm).
    nat.qk_norm_rope(xt, t, heads, hd, None, 0.0, tabs.cos.reshape(-1, xt.shape[1] // 2),
                     tabs.sin.reshape(-1, xt.shape[1] // 2), rope_ld_batch=tabs.ld_batch)
    if x.ndim == 4:
        return xt.view(b, t, h, d).transpose(1, 2)
    return xt.view_as(x)


# ---------------------------------------------------------------------------------------
# Timestep embedding / adaLN-single
# ---------------------------------------------------------------------------------------


class TimestepEmbedder(torch.nn.Module):
    """ltx_nn.py:123-130: linear_2(silu(linear_1(x)))."""

    def __init__(self, in_channels: int, time_embed_dim: int):
        super().__init__()
        self.linear_1 = torch.nn.Linear(in_channels, time_embed_dim)
        self.linear_2 = torch.nn.Linear(time_embed_dim, time_embed_dim)

    def forward(self, x: torch.Tensor, silu_out: torch.Tensor | None = None) -> torch.Tensor:
        h = torch.empty(x.shape[0], self.linear_1.out_features, device=x.device, dtype=x.dtype)
        nat.linear(x, self.linear_1.weight, h, nat.epilogue(nat.EPI_SILU, bias=self.linear_1.bias))
        out = torch.empty(x.shape[0], self.linear_2.out_features, device=x.device, dtype=x.dtype)
        nat.linear(h, self.linear_2.weight, out, nat.epilogue(bias=self.linear_2.bias))
        if silu_out is not None:
            nat.linear(h, self.linear_2.weight, silu_out, nat.epilogue(nat.EPI_SILU, bias=self.linear_2.bias))
        return out


class CombinedTimestepEmbeddings(torch.nn.Module):
    """ltx_nn.py:133-145: 256-dim [cos, sin] sinusoid -> TimestepEmbedder."""

    def __init__(self, embedding_dim: int):
        super().__init__()
        self.timestep_embedder = TimestepEmbedder(256, embedding_dim)

    def forward(self, timestep: torch.Tensor, hidden_dtype: torch.dtype, scale: float = 1.0,
                silu_out: torch.Tensor | None = None) -> torch.Tensor:
        t = timestep.reshape(-1).to(torch.float32).contiguous()
        proj = torch.empty(t.numel(), 256, device=t.device, dtype=hidden_dtype)
        nat.timestep_embedding(t, scale, 256, 10000.0, proj)
        return self.timestep_embedder(proj, silu_out)


class AdaLayerNormSingle(torch.nn.Module):
    """ltx_nn.py:148-158: (Linear(silu(emb)) , emb)."""

    def __init__(self, embedding_dim: int, embedding_coefficient: int = 6):
        super().__init__()
        self.emb = CombinedTimestepEmbeddings(embedding_dim)
        self.linear = torch.nn.Linear(embedding_dim, embedding_coefficient * embedding_dim, bias=True)

    def forward(self, timestep: torch.Tensor, hidden_dtype: torch.dtype,
                scale: float = 1.0) -> tuple[torch.Tensor, torch.Tensor]:
        """timestep (N,) -> (modulation (N, n*D), embedded (N, D)). `scale` multiplies
        the timestep inside the kernel (the reference's *timestep_scale_multiplier)."""
        n = timestep.numel()
        d = self.linear.in_features
        dev = timestep.device
        if n < 32:
            emb = self.emb(timestep, hidden_dtype, scale)
            mod = torch.empty(n, self.linear.out_features, device=dev, dtype=hidden_dtype)
            nat.linear(emb, self.linear.weight, mod, nat.epilogue(bias=self.linear.bias, silu_input=True))
        else:
            silu = torch.empty(n, d, device=dev, dtype=hidden_dtype)
            emb = self.emb(timestep, hidden_dtype, scale, silu_out=silu)
            mod = torch.empty(n, self.linear.out_features, device=dev, dtype=hidden_dtype)
            nat.linear(silu, self.linear.weight, mod, nat.epilogue(bias=self.linear.bias))
        return mod, emb


# ---------------------------------------------------------------------------------------
# Attention + FFN
# ---------------------------------------------------------------------------------------


def _pack(mod: torch.nn.Module, names: list[str], attr: str) -> tuple[torch.Tensor, torch.Tensor]:
    """Pack the listed Linear sub-modules' weights (and biases) into one contiguous
    buffer and re-point their parameters at views of it. Idempotent."""
    key = "_packed_" + attr
    subs = [getattr(mod, n) for n in names]
    cached = getattr(mod, key, None)
    if cached is not None:
        w, b, ptrs = cached
        if ptrs == [s.weight.data_ptr() for s in subs] and w.device == subs[0].weight.device \
                and w.dtype == subs[0].weight.dtype:
            return w, b
    rows = sum(s.weight.shape[0] for s in subs)
    pad = (-rows) % 8  # keep the packed output's row stride a multiple of 8 elements
    ref = subs[0].weight
    w = torch.zeros(rows + pad, ref.shape[1], device=ref.device, dtype=ref.dtype)
    b = torch.zeros(rows + pad, device=ref.device, dtype=ref.dtype)
    torch.cat([s.weight.detach() for s in subs], dim=0, out=w[:rows])
    torch.cat([s.bias.detach() for s in subs], dim=0, out=b[:rows])
    row = 0
    for s in subs:
        n = s.weight.shape[0]
        s.weight.data = w[row:row + n]
        s.bias.data = b[row:row + n]
        row += n
    setattr(mod, key, (w, b, [s.weight.data_ptr() for s in subs]))
    return w, b


class Attention(torch.nn.Module):
    """ltx_nn.py:166-236: gated multi-head attention with q/k RMSNorm over the inner
    dim and split RoPE. Same parameters and forward signature as the reference."""

    def __init__(self, query_dim: int, context_dim: int | None = None, heads: int = 8, dim_head: int = 64,
                 norm_eps: float = 1e-6, apply_gated_attention: bool = False):
        super().__init__()
        self.heads = heads
        self.dim_head = dim_head
        self.norm_eps = norm_eps
        inner = heads * dim_head
        context_dim = query_dim if context_dim is None else context_dim
        self.q_norm = torch.nn.RMSNorm(inner, eps=norm_eps)
        self.k_norm = torch.nn.RMSNorm(inner, eps=norm_eps)
        self.to_q = torch.nn.Linear(query_dim, inner, bias=True)
        self.to_k = torch.nn.Linear(context_dim, inner, bias=True)
        self.to_v = torch.nn.Linear(context_dim, inner, bias=True)
        self.to_gate_logits = torch.nn.Linear(query_dim, heads, bias=True) if apply_gated_attention else None
        self.to_out = torch.nn.Linear(inner, query_dim, bias=True)

    # packed weights -----------------------------------------------------------------
    def packed_self(self):
        names = ["to_q", "to_k", "to_v"] + (["to_gate_logits"] if self.to_gate_logits is not None else [])
        return _pack(self, names, "self")

    def packed_q(self):
        names = ["to_q"] + (["to_gate_logits"] if self.to_gate_logits is not None else [])
        return _pack(self, names, "q")

    def packed_kv(self):
        return _pack(self, ["to_k", "to_v"], "kv")

    # native core ----------------------------------------------------------------------
    def project_qkv(self, x2: torch.Tensor, rows_per_batch: int, pe: RopeTables | None,
                    k_pe: RopeTables | None = None, normalize: bool = True) -> torch.Tensor:
        """Self-attention projections of x2 (B*T, D) -> packed (B*T, 3I(+H)) buffer with
        q and k normalised and rotated in place (normalize=False: left as projected, for a
        caller that fuses the normalisation into its exchange)."""
        inner = self.heads * self.dim_head
        w, b = self.packed_self()
        qkv = torch.empty(x2.shape[0], w.shape[0], device=x2.device, dtype=x2.dtype)
        nat.linear(x2, w, qkv, nat.epilogue(bias=b))
        if not normalize:
            return qkv
        if k_pe is None:
            # q and k share the tables: one pass over both blocks
            if pe is None:
                nat.qk_norm_rope_pair(qkv, inner, rows_per_batch, self.heads, self.dim_head, self.q_norm.weight,
                                      self.k_norm.weight, self.norm_eps, None, None)
            else:
                rh = pe.heads
                nat.qk_norm_rope_pair(qkv, inner, rows_per_batch, rh, inner // rh, self.q_norm.weight,
                                      self.k_norm.weight, self.norm_eps,
                                      pe.cos.view(-1, inner // 2) if pe.cos.dim() == 3 else pe.cos,
                                      pe.sin.view(-1, inner // 2) if pe.sin.dim() == 3 else pe.sin,
                                      rope_ld_batch=pe.ld_batch)
            return qkv
        self._norm_rope(qkv[:, :inner], rows_per_batch, self.q_norm.weight, pe)
        self._norm_rope(qkv[:, inner:2 * inner], rows_per_batch, self.k_norm.weight, k_pe)
        return qkv

    def _norm_rope(self, view: torch.Tensor, rows_per_batch: int, weight: torch.Tensor, pe: RopeTables | None):
        inner = self.heads * self.dim_head
        if pe is None:
            nat.qk_norm_rope(view, rows_per_batch, self.heads, self.dim_head, weight, self.norm_eps, None, None)
        else:
            rh = pe.heads
            nat.qk_norm_rope(view, rows_per_batch, rh, inner // rh, weight, self.norm_eps, pe.cos.view(-1, inner // 2)
                             if pe.cos.dim() == 3 else pe.cos, pe.sin.view(-1, inner // 2) if pe.sin.dim() == 3
                             else pe.sin, rope_ld_batch=pe.ld_batch)

    def attend(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, gate: torch.Tensor | None, batch: int,
               tq: int, tk: int) -> torch.Tensor:
        o = torch.empty(q.shape[0], self.heads * self.dim_head, device=q.device, dtype=q.dtype)
        nat.attention(q, k, v, o, batch, tq, tk, self.heads, self.dim_head, self.dim_head ** -0.5, gate)
        return o

    def forward(self, x: torch.Tensor, context: torch.Tensor | None = None, mask: torch.Tensor | None = None,
                pe=None, k_pe=None, perturbation_mask: torch.Tensor | None = None,
                all_perturbed: bool = False) -> torch.Tensor:
        if mask is not None or perturbation_mask is not None or all_perturbed:
            raise NotImplementedError("attention masks / STG perturbation are not supported yet")
        b, t, _ = x.shape
        inner = self.heads * self.dim_head
        x2 = x.reshape(b * t, -1)
        pe_t = _tables_from_reference_layout(pe) if pe is not None else None
        kpe_t = _tables_from_reference_layout(k_pe) if k_pe is not None else None
        gated = self.to_gate_logits is not None
        if context is None:
            qkv = self.project_qkv(x2, t, pe_t, kpe_t)
            o = self.attend(qkv[:, :inner], qkv[:, inner:2 * inner], qkv[:, 2 * inner:3 * inner],
                            qkv[:, 3 * inner:] if gated else None, b, t, t)
        else:
            s = context.shape[1]
            c2 = context.reshape(b * s, -1)
            wq, bq = self.packed_q()
            qg = torch.empty(b * t, wq.shape[0], device=x.device, dtype=x.dtype)
            nat.linear(x2, wq, qg, nat.epilogue(bias=bq))
            wkv, bkv = self.packed_kv()
            kv = torch.empty(b * s, 2 * inner, device=x.device, dtype=x.dtype)
            nat.linear(c2, wkv, kv, nat.epilogue(bias=bkv))
            self._norm_rope(qg[:, :inner], t, self.q_norm.weight, pe_t)
            self._norm_rope(kv[:, :inner], s, self.k_norm.weight, kpe_t if kpe_t is not None else pe_t)
            o = self.attend(qg[:, :inner], kv[:, :inner], kv[:, inner:], qg[:, inner:] if gated else None, b, t, s)
        out = torch.empty(b * t, self.to_out.out_features, device=x.device, dtype=x.dtype)
        nat.linear(o, self.to_out.weight, out, nat.epilogue(bias=self.to_out.bias))
        return out.view(b, t, -1)


class FeedForward(torch.nn.Module):
    """ltx_nn.py:239-248: proj_out(gelu_tanh(proj_in(x)))."""

    def __init__(self, dim: int, dim_out: int | None = None, mult: int = 4, bias: bool = True):
        super().__init__()
        dim_out = dim if dim_out is None else dim_out
        inner = int(dim * mult)
        self.proj_in = torch.nn.Linear(dim, inner, bias=bias)
        self.proj_out = torch.nn.Linear(inner, dim_out, bias=bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        b, t, d = x.shape
        x2 = x.reshape(b * t, d)
        h = torch.empty(b * t, self.proj_in.out_features, device=x.device, dtype=x.dtype)
        nat.linear(x2, self.proj_in.weight, h, nat.epilogue(nat.EPI_GELU_TANH, bias=self.proj_in.bias))
        out = torch.empty(b * t, self.proj_out.out_features, device=x.device, dtype=x.dtype)
        nat.linear(h, self.proj_out.weight, out, nat.epilogue(bias=self.proj_out.bias))
        return out.view(b, t, -1)
