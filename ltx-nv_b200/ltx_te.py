"""Text-embedding connector of LTX-2.5 on the sm_100a kernels (drop-in for the connector
part of lipaul/ltx-nv standalone/ltx_te.py).

Embeddings1DConnector turns the feature extractor's per-token text features into the
DiT's cross-attention context: learnable registers replace padded tokens
(ltx_te.py:218-223), then `num_layers` bidirectional blocks x + attn1(rms(x)) and
x + ff(rms(x)) with 1D RoPE over token indices (ltx_te.py:187-196, 224-228), and a final
RMS norm. Same class names, constructor arguments and parameter names as the reference,
so its state dicts load unchanged.

Every op is a libltxb200 kernel: ltx_register_fill, ltx_norm_modulate (RMS, no
modulation), the packed QKV GEMM, q/k RMSNorm + RoPE, tcgen05 attention, out-projection
and FFN GEMMs whose epilogues add the residual in place.
"""

from __future__ import annotations

import torch

import _native as nat
from ltx_nn import Attention, FeedForward, rope_tables

NORM_EPS = 1e-6


class ConnectorBlock(torch.nn.Module):
    """ltx_te.py:187-196."""

    def __init__(self, dim: int, heads: int, dim_head: int, gated: bool, ff_bias: bool, norm_eps: float = NORM_EPS):
        super().__init__()
        self.attn1 = Attention(dim, None, heads, dim_head, norm_eps, apply_gated_attention=gated)
        self.ff = FeedForward(dim, dim, bias=ff_bias)

    def run(self, x: torch.Tensor, h: torch.Tensor, batch: int, s: int, pe) -> None:
        """One block on the (B*S, D) residual stream x, updated in place; h is scratch."""
        attn, ff = self.attn1, self.ff
        inner = attn.heads * attn.dim_head
        nat.norm_modulate(x, h, s, nat.LTX_NORM_RMS, NORM_EPS, None)
        qkv = attn.project_qkv(h, s, pe)
        gated = attn.to_gate_logits is not None
        o = attn.attend(qkv[:, :inner], qkv[:, inner:2 * inner], qkv[:, 2 * inner:3 * inner],
                        qkv[:, 3 * inner:3 * inner + attn.heads] if gated else None, batch, s, s)
        nat.linear(o, attn.to_out.weight, x, nat.epilogue(nat.EPI_GATE_RESIDUAL, bias=attn.to_out.bias, residual=x,
                                                          rows_per_batch=s))
        nat.norm_modulate(x, h, s, nat.LTX_NORM_RMS, NORM_EPS, None)
        f = torch.empty(x.shape[0], ff.proj_in.out_features, device=x.device, dtype=x.dtype)
        nat.linear(h, ff.proj_in.weight, f, nat.epilogue(nat.EPI_GELU_TANH, bias=ff.proj_in.bias))
        nat.linear(f, ff.proj_out.weight, x, nat.epilogue(nat.EPI_GATE_RESIDUAL, bias=ff.proj_out.bias, residual=x,
                                                          rows_per_batch=s))

    def forward(self, x: torch.Tensor, additive_mask=None, pe=None) -> torch.Tensor:
        if additive_mask is not None and bool((additive_mask != 0).any()):
            raise NotImplementedError("additive attention masks (connectors without registers)")
        b, s, d = x.shape
        xs = x.reshape(b * s, d).contiguous().clone()
        h = torch.empty_like(xs)
        self.run(xs, h, b, s, pe)
        return xs.view(b, s, d)


class Embeddings1DConnector(torch.nn.Module):
    """ltx_te.py:199-229."""

    def __init__(self, heads: int, dim_head: int, num_layers: int, max_pos: list[int], registers: int, gated: bool,
                 ff_bias: bool):
        super().__init__()
        self.inner_dim = heads * dim_head
        self.positional_max_pos = list(max_pos)
        self.blocks = torch.nn.ModuleList(
            [ConnectorBlock(self.inner_dim, heads, dim_head, gated, ff_bias) for _ in range(num_layers)])
        self.num_registers = registers
        if registers:
            self.learnable_registers = torch.nn.Parameter(torch.empty(registers, self.inner_dim))
        self._pe_cache = None

    def _pe(self, s: int, device, dtype):
        """1D RoPE over token indices 0..s-1 (no mid-point grid): the tables of bounds
        (i, i), whose mid-point is i exactly."""
        key = (s, device, dtype)
        if self._pe_cache is None or self._pe_cache[0] != key:
            grid = torch.arange(s, dtype=torch.float32, device=device)[None, None, :]
            pos = torch.stack([grid, grid], dim=-1)
            heads = self.blocks[0].attn1.heads
            self._pe_cache = (key, rope_tables(pos, self.inner_dim, dtype, 10000.0, self.positional_max_pos, heads))
        return self._pe_cache[1]

    @torch.inference_mode()
    def forward(self, hidden_states: torch.Tensor, additive_mask: torch.Tensor):
        """(B, S, D) features and a (B, 1, 1, S) additive mask -> (RMS-normed (B, S, D),
        the mask the reference returns: zeros when registers are used)."""
        b, s, d = hidden_states.shape
        x = torch.empty(b * s, d, device=hidden_states.device, dtype=hidden_states.dtype)
        if self.num_registers:
            if s % self.num_registers:
                raise ValueError("the sequence length must be a multiple of the register count")
            nat.register_fill(hidden_states.reshape(b * s, d).contiguous(),
                              additive_mask.to(hidden_states.dtype).reshape(b * s).contiguous(),
                              self.learnable_registers.to(hidden_states.dtype), s, x)
            additive_mask = torch.zeros_like(additive_mask)
        else:
            if bool((additive_mask != 0).any()):
                raise NotImplementedError("additive attention masks (connectors without registers)")
            x.copy_(hidden_states.reshape(b * s, d))
        pe = self._pe(s, hidden_states.device, hidden_states.dtype)
        h = torch.empty_like(x)
        for blk in self.blocks:
            blk.run(x, h, b, s, pe)
        out = torch.empty_like(x)
        nat.norm_modulate(x, out, s, nat.LTX_NORM_RMS, NORM_EPS, None)
        return out.view(b, s, d), additive_mask
