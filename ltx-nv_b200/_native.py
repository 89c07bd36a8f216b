"""ctypes binding of libltxb200.so (the sm_100a kernels of the DiT step).

PyTorch is used here only for device memory and streams: every wrapper takes torch
tensors, passes their data pointers, sizes and the current CUDA stream through the C
ABI declared in include/ltxb200.h, and raises LtxError when the library reports a
failure. There is no CPU or PyTorch fallback: if the library is missing or a call is
rejected, the error propagates.
"""

from __future__ import annotations

import ctypes
import os
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libltxb200.so"

LTX_F32, LTX_BF16 = 0, 1
LTX_NORM_RMS, LTX_NORM_LAYER, LTX_NORM_NONE = 0, 1, 2
EPI_NONE, EPI_GELU_TANH, EPI_SILU, EPI_GATE_RESIDUAL, EPI_ROW_MASK_ADD = 0, 1, 2, 3, 4

c_i64 = ctypes.c_int64
c_vp = ctypes.c_void_p


class LtxError(RuntimeError):
    """A libltxb200 call returned a non-zero status."""

    def __init__(self, fn: str, code: int, msg: str):
        super().__init__(f"{fn} failed with status {code}: {msg}")
        self.code = code


class Modulation(ctypes.Structure):
    """Mirror of ltx_modulation (include/ltxb200.h)."""

    _fields_ = [
        ("table", c_vp),
        ("mod", c_vp),
        ("mod_ld_batch", c_i64),
        ("mod_ld_tok", c_i64),
        ("shift_table_off", c_i64),
        ("shift_mod_off", c_i64),
        ("scale_table_off", c_i64),
        ("scale_mod_off", c_i64),
        ("has_shift", ctypes.c_int),
        ("has_scale", ctypes.c_int),
    ]


class Epilogue(ctypes.Structure):
    """Mirror of ltx_epilogue (include/ltxb200.h)."""

    _fields_ = [
        ("kind", ctypes.c_int),
        ("bias", c_vp),
        ("residual", c_vp),
        ("ld_residual", c_i64),
        ("gate", Modulation),
        ("rows_per_batch", c_i64),
        ("row_mask", c_vp),
        ("row_vec", c_vp),
        ("silu_input", ctypes.c_int),
    ]


class DitConfig(ctypes.Structure):
    """Mirror of ltx_dit_config (include/ltxb200.h)."""

    _fields_ = [
        ("num_layers", ctypes.c_int),
        ("heads", ctypes.c_int),
        ("head_dim", ctypes.c_int),
        ("in_channels", ctypes.c_int),
        ("out_channels", ctypes.c_int),
        ("cross_dim", ctypes.c_int),
        ("ffn_dim", ctypes.c_int),
        ("gated_attention", ctypes.c_int),
        ("norm_eps", ctypes.c_float),
        ("theta", ctypes.c_double),
        ("max_pos", ctypes.c_float * 3),
        ("timestep_scale_multiplier", ctypes.c_float),
        ("dtype", ctypes.c_int),
    ]


DIT_BLOCK_FIELDS = ["scale_shift_table", "attn1_qkvg_w", "attn1_qkvg_b", "attn1_q_norm", "attn1_k_norm",
                    "attn1_out_w", "attn1_out_b", "attn2_qg_w", "attn2_qg_b", "attn2_kv_w", "attn2_kv_b",
                    "attn2_q_norm", "attn2_k_norm", "attn2_out_w", "attn2_out_b", "ff_in_w", "ff_in_b", "ff_out_w",
                    "ff_out_b"]


class DitBlockWeights(ctypes.Structure):
    """Mirror of ltx_dit_block_weights (include/ltxb200.h)."""

    _fields_ = [(n, c_vp) for n in DIT_BLOCK_FIELDS]


class DitWeights(ctypes.Structure):
    """Mirror of ltx_dit_weights (include/ltxb200.h)."""

    _fields_ = [(n, c_vp) for n in ("patchify_w", "patchify_b", "keyframes_emb", "t_linear_1_w", "t_linear_1_b",
                                     "t_linear_2_w", "t_linear_2_b", "adaln_w", "adaln_b", "scale_shift_table",
                                     "proj_out_w", "proj_out_b")] + [("blocks", ctypes.POINTER(DitBlockWeights))]


class DitStepArgs(ctypes.Structure):
    """Mirror of ltx_dit_step_args (include/ltxb200.h)."""

    _fields_ = [
        ("latent", c_vp),
        ("positions", c_vp),
        ("context_pos", c_vp),
        ("context_neg", c_vp),
        ("keyframes_mask", c_vp),
        ("T", c_i64),
        ("S", c_i64),
        ("sigma", ctypes.c_float),
        ("sigma_next", ctypes.c_float),
        ("cfg_scale", ctypes.c_float),
        ("flags", ctypes.c_int),
    ]


STEP_REUSE_TEXT_KV, STEP_REUSE_ROPE = 1, 2

# name -> (restype, argtypes); the exported symbols of include/ltxb200.h (and the test
# hooks of include/ltxb200_testing.h).
_SIGNATURES = {
    "ltx_last_error": (ctypes.c_char_p, []),
    "ltx_abi_version": (ctypes.c_int, []),
    "ltx_launch_count": (ctypes.c_uint64, []),
    "ltx_device_error_flags": (ctypes.c_int, [ctypes.POINTER(ctypes.c_int), ctypes.c_int, c_vp]),
    "ltx_philox_grid": (ctypes.c_int, [ctypes.c_int, c_i64, ctypes.POINTER(ctypes.c_int)]),
    "ltx_philox_offset_increment": (c_i64, [c_i64, ctypes.c_int]),
    "ltx_philox_randn": (ctypes.c_int, [c_vp, c_i64, ctypes.c_int, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_int, c_vp]),
    "ltx_philox_raw": (ctypes.c_int, [c_vp, c_i64, c_i64, ctypes.c_uint64, ctypes.c_uint64, c_vp]),
    "ltx_norm_modulate": (ctypes.c_int, [c_vp, c_i64, c_vp, c_i64, c_i64, c_i64, ctypes.c_int, ctypes.c_int,
                                         ctypes.c_float, ctypes.POINTER(Modulation), ctypes.c_int, c_vp]),
    "ltx_qk_norm_rope": (ctypes.c_int, [c_vp, c_i64, c_i64, c_i64, ctypes.c_int, ctypes.c_int, c_vp, ctypes.c_float,
                                        c_vp, c_vp, c_i64, c_i64, ctypes.c_int, c_vp]),
    "ltx_qk_norm_rope_pair": (ctypes.c_int, [c_vp, c_i64, c_i64, c_i64, c_i64, ctypes.c_int, ctypes.c_int, c_vp, c_vp,
                                             ctypes.c_float, c_vp, c_vp, c_i64, c_i64, ctypes.c_int, c_vp]),
    "ltx_rope_tables": (ctypes.c_int, [c_vp, ctypes.c_int, c_i64, c_vp, ctypes.c_int, c_vp, ctypes.c_int, c_vp, c_vp,
                                       ctypes.c_int, c_vp]),
    "ltx_gelu_tanh": (ctypes.c_int, [c_vp, c_vp, c_i64, ctypes.c_int, c_vp]),
    "ltx_gate_residual": (ctypes.c_int, [c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_i64, c_i64, ctypes.c_int,
                                         ctypes.POINTER(Modulation), ctypes.c_int, c_vp]),
    "ltx_timestep_embedding": (ctypes.c_int, [c_vp, c_i64, ctypes.c_float, ctypes.c_int, ctypes.c_float, c_vp,
                                              ctypes.c_int, c_vp]),
    "ltx_linear": (ctypes.c_int, [c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_i64, c_i64, c_i64,
                                  ctypes.POINTER(Epilogue), ctypes.c_int, c_vp]),
    "ltx_gemm_set_tile_n": (ctypes.c_int, [ctypes.c_int]),
    "ltx_test_bounded_wait": (ctypes.c_int, [ctypes.c_ulonglong, c_vp, c_vp]),
    "ltx_test_attention_force_split": (ctypes.c_int, [ctypes.c_int]),
    "ltx_test_attention_plan": (ctypes.c_int, [c_i64, c_i64, ctypes.c_int, ctypes.POINTER(ctypes.c_int),
                                               ctypes.POINTER(ctypes.c_int)]),
    "ltx_attention": (ctypes.c_int, [c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, ctypes.c_int, c_i64, c_i64,
                                     ctypes.c_int, ctypes.c_int, ctypes.c_float, c_vp, c_i64, ctypes.c_int, c_vp]),
    "ltx_cfg_euler": (ctypes.c_int, [c_vp, c_vp, c_vp, c_i64, ctypes.c_int, ctypes.c_float, ctypes.c_float,
                                     ctypes.c_float, c_vp, c_vp, ctypes.c_int, c_vp]),
    "ltx_sp_pack": (ctypes.c_int, [c_vp, c_i64, c_i64, ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_int),
                                   ctypes.POINTER(ctypes.c_int), c_vp, ctypes.c_int, c_vp]),
    "ltx_sp_unpack": (ctypes.c_int, [c_vp, c_i64, ctypes.c_int, ctypes.c_int, c_vp, c_i64, ctypes.c_int, c_vp]),
    "ltx_peer_alloc": (ctypes.c_int, [ctypes.c_size_t, ctypes.POINTER(c_vp), c_vp]),
    "ltx_peer_open": (ctypes.c_int, [c_vp, ctypes.POINTER(c_vp)]),
    "ltx_peer_close": (ctypes.c_int, [c_vp]),
    "ltx_peer_free": (ctypes.c_int, [c_vp]),
    "ltx_qk_norm_rope_scatter": (ctypes.c_int, [c_vp, c_i64, c_i64, c_i64, ctypes.c_int, ctypes.c_int, c_vp, c_vp,
                                                ctypes.c_float, c_vp, c_vp, c_i64, c_i64, ctypes.c_int, ctypes.c_int,
                                                ctypes.c_int, ctypes.POINTER(c_vp), c_i64, c_vp]),
    "ltx_attention_scatter": (ctypes.c_int, [c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, ctypes.c_int, c_i64,
                                             ctypes.c_int, ctypes.c_int, ctypes.c_float, c_vp, c_i64, c_vp,
                                             ctypes.c_size_t, ctypes.c_int, ctypes.POINTER(c_vp), c_i64, ctypes.c_int,
                                             c_vp]),
    "ltx_sp_barrier": (ctypes.c_int, [ctypes.POINTER(c_vp), c_vp, ctypes.c_int, ctypes.c_int, ctypes.c_ulonglong,
                                      c_vp]),
    "ltx_guide": (ctypes.c_int, [c_vp, c_vp, c_vp, c_vp, c_i64, ctypes.c_float, ctypes.c_float, ctypes.c_float, c_vp,
                                 ctypes.c_int, c_vp]),
    "ltx_euler": (ctypes.c_int, [c_vp, c_vp, c_i64, ctypes.c_float, ctypes.c_float, c_vp, ctypes.c_int, c_vp]),
    "ltx_value_gate": (ctypes.c_int, [c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_i64, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_int, c_vp]),
    "ltx_x0": (ctypes.c_int, [c_vp, c_vp, c_vp, c_i64, ctypes.c_int, c_vp, ctypes.c_int, c_vp]),
    "ltx_register_fill": (ctypes.c_int, [c_vp, c_i64, c_vp, c_vp, ctypes.c_int, c_i64, c_i64, ctypes.c_int, c_vp,
                                         c_i64, ctypes.c_int, c_vp]),
    "ltx_conv3d": (ctypes.c_int, [c_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, c_vp,
                                  c_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, c_vp, c_vp, c_vp]),
    "ltx_conv3d_norm": (ctypes.c_int, [c_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                       c_vp, c_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, c_vp, ctypes.c_int,
                                       ctypes.c_float, c_vp, c_vp]),
    "ltx_pixel_norm": (ctypes.c_int, [c_vp, c_vp, c_i64, ctypes.c_int, ctypes.c_float, ctypes.c_int, c_vp]),
    "ltx_group_norm1_workspace_bytes": (c_i64, [ctypes.c_int]),
    "ltx_group_norm1": (ctypes.c_int, [c_vp, ctypes.c_int, c_i64, ctypes.c_int, c_vp, c_vp, ctypes.c_float, c_vp, c_i64,
                                       c_vp, c_vp]),
    "ltx_depth_to_space": (ctypes.c_int, [c_vp] + [ctypes.c_int] * 9 + [c_vp, c_vp]),
    "ltx_vae_latent_in": (ctypes.c_int, [c_vp] + [ctypes.c_int] * 5 + [c_vp, c_vp, c_vp, c_vp]),
    "ltx_vae_unpatchify": (ctypes.c_int, [c_vp] + [ctypes.c_int] * 7 + [c_vp, c_vp]),
    "ltx_guide_rescale_workspace_bytes": (ctypes.c_size_t, [c_i64]),
    "ltx_guide_rescale_noalloc": (ctypes.c_int, [c_vp, c_vp, c_vp, c_vp, c_i64, ctypes.c_float, ctypes.c_float,
                                                 ctypes.c_float, ctypes.c_float, c_vp, ctypes.c_int, c_vp]),
    "ltx_guide_rescale": (ctypes.c_int, [c_vp, c_vp, c_vp, c_vp, c_i64, ctypes.c_float, ctypes.c_float, ctypes.c_float,
                                         ctypes.c_float, c_vp, c_vp, ctypes.c_size_t, ctypes.c_int, c_vp]),
    "ltx_proj_out_cfg_euler": (ctypes.c_int, [c_vp, c_i64, c_vp, c_vp, c_i64, ctypes.c_int, c_i64, c_vp, c_vp,
                                              ctypes.c_float, ctypes.c_float, ctypes.c_float, c_vp, c_vp, c_vp,
                                              ctypes.c_int, c_vp]),
    "ltx_attention_workspace_bytes": (ctypes.c_size_t, [ctypes.c_int, c_i64, c_i64, ctypes.c_int, ctypes.c_int]),
    "ltx_attention_ws": (ctypes.c_int, [c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, ctypes.c_int, c_i64,
                                        c_i64, ctypes.c_int, ctypes.c_int, ctypes.c_float, c_vp, c_i64, c_vp,
                                        ctypes.c_size_t, ctypes.c_int, c_vp]),
    "ltx_attention_partial": (ctypes.c_int, [c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_vp, c_i64, c_vp, c_i64,
                                             ctypes.c_int, c_i64, c_i64, ctypes.c_int, ctypes.c_int, ctypes.c_float,
                                             c_vp]),
    "ltx_attention_merge": (ctypes.c_int, [c_vp, c_vp, ctypes.c_int, c_i64, ctypes.c_int, ctypes.c_int, c_vp, c_i64,
                                           c_vp, c_i64, c_vp]),
    "ltx_ctx_create": (ctypes.c_int, [ctypes.c_int, ctypes.POINTER(c_vp)]),
    "ltx_ctx_destroy": (ctypes.c_int, [c_vp]),
    "ltx_dit_workspace_bytes": (ctypes.c_size_t, [ctypes.POINTER(DitConfig), c_i64, c_i64]),
    "ltx_dit_reserve": (ctypes.c_int, [c_vp, ctypes.POINTER(DitConfig), c_i64, c_i64]),
    "ltx_dit_step": (ctypes.c_int, [c_vp, ctypes.POINTER(DitConfig), ctypes.POINTER(DitWeights),
                                    ctypes.POINTER(DitStepArgs), c_vp, c_vp, c_vp, c_vp]),
}

_lib = None


def load_library(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    """Load libltxb200.so (once) and bind every exported entry point's signature."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path is not None else LIB_PATH
    if not p.exists():
        raise FileNotFoundError(
            f"{p} not found: build it with `python -c 'import __graft_entry__ as g; g.build()'` "
            "(there is no fallback implementation)")
    lib = ctypes.CDLL(str(p))
    for name, (res, args) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def _check(name: str, status: int) -> None:
    if status != 0:
        msg = _lib.ltx_last_error().decode(errors="replace")
        raise LtxError(name, status, msg)


_profile: dict | None = None


class profile:
    """Context manager that brackets every library call with CUDA events on the
    launching (current) stream: {label: [(start, end), ...]}, label = entry point name
    plus the call's shape. Used by bench.py for per-kernel durations."""

    def __enter__(self):
        global _profile
        _profile = {}
        self.records = _profile
        return self

    def __exit__(self, *exc):
        global _profile
        _profile = None

    def summary(self) -> dict:
        torch.cuda.synchronize()
        out = {}
        for label, evs in self.records.items():
            ms = [s.elapsed_time(e) for s, e in evs]
            out[label] = {"launches": len(ms), "total_ms": sum(ms), "avg_ms": sum(ms) / len(ms)}
        return out


def _call(name: str, *args, label: str | None = None):
    lib = load_library()
    if _profile is None:
        _check(name, getattr(lib, name)(*args))
        return
    s = torch.cuda.Event(enable_timing=True)
    e = torch.cuda.Event(enable_timing=True)
    s.record()
    st = getattr(lib, name)(*args)
    e.record()
    _check(name, st)
    _profile.setdefault(label or name, []).append((s, e))


def _stream(t: torch.Tensor | None = None) -> int:
    dev = t.device if t is not None else torch.device("cuda")
    return torch.cuda.current_stream(dev).cuda_stream


def _dt(t: torch.Tensor) -> int:
    if t.dtype == torch.float32:
        return LTX_F32
    if t.dtype == torch.bfloat16:
        return LTX_BF16
    raise TypeError(f"unsupported dtype {t.dtype}; the kernels take float32 or bfloat16")


def _ptr(t: torch.Tensor | None) -> int | None:
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("libltxb200 kernels take CUDA tensors only")
    return t.data_ptr()


def _ld(t: torch.Tensor) -> int:
    """Leading dimension (elements between rows) of a row-major 2-D view."""
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError(f"expected a 2-D row-major view, got shape {tuple(t.shape)} stride {t.stride()}")
    return t.stride(0)


# ---------------------------------------------------------------------------------------
# Modulation descriptors
# ---------------------------------------------------------------------------------------


def modulation(table: torch.Tensor | None, mod: torch.Tensor | None, *, shift: tuple[int, int] | None,
               scale: tuple[int, int] | None, mod_ld_batch: int = 0, mod_ld_tok: int = 0) -> Modulation:
    """Describe shift/scale vectors table[t_off:] + mod[b, t, m_off:] (element offsets)."""
    m = Modulation()
    m.table = _ptr(table)
    m.mod = _ptr(mod)
    m.mod_ld_batch = mod_ld_batch
    m.mod_ld_tok = mod_ld_tok
    if shift is not None:
        m.has_shift = 1
        m.shift_table_off, m.shift_mod_off = shift
    if scale is not None:
        m.has_scale = 1
        m.scale_table_off, m.scale_mod_off = scale
    return m


# ---------------------------------------------------------------------------------------
# Wrappers
# ---------------------------------------------------------------------------------------


def abi_version() -> int:
    return load_library().ltx_abi_version()


def launch_count() -> int:
    """Kernels launched by libltxb200 in this process so far."""
    return int(load_library().ltx_launch_count())


def device_error_flags(clear: bool = True) -> int:
    flags = ctypes.c_int(0)
    _call("ltx_device_error_flags", ctypes.byref(flags), int(clear), _stream())
    return flags.value


def philox_grid(n: int, device: int | None = None) -> int:
    g = ctypes.c_int(0)
    dev = torch.cuda.current_device() if device is None else device
    _call("ltx_philox_grid", dev, n, ctypes.byref(g))
    return g.value


def philox_offset_increment(n: int, grid: int) -> int:
    return load_library().ltx_philox_offset_increment(n, grid)


def philox_randn(out: torch.Tensor, seed: int, offset: int, grid: int) -> None:
    if not out.is_contiguous():
        raise ValueError("out must be contiguous")
    _call("ltx_philox_randn", _ptr(out), out.numel(), _dt(out), seed, offset, grid, _stream(out))


def philox_raw(out: torch.Tensor, threads: int, rounds: int, seed: int, offset: int) -> None:
    if out.dtype != torch.int32 or out.numel() < threads * rounds * 4:
        raise ValueError("out must be int32 with threads*rounds*4 elements")
    _call("ltx_philox_raw", _ptr(out), threads, rounds, seed, offset, _stream(out))


def norm_modulate(x: torch.Tensor, y: torch.Tensor, rows_per_batch: int, kind: int, eps: float,
                  mod: Modulation | None) -> None:
    rows, d = x.shape
    _call("ltx_norm_modulate", _ptr(x), _ld(x), _ptr(y), _ld(y), rows, rows_per_batch, d, kind, eps,
          ctypes.byref(mod) if mod is not None else None, _dt(x), _stream(x))


def qk_norm_rope(x: torch.Tensor, rows_per_batch: int, heads: int, head_dim: int, weight: torch.Tensor, eps: float,
                 cos: torch.Tensor | None, sin: torch.Tensor | None, rope_ld_batch: int = 0) -> None:
    rows = x.shape[0]
    ld_rope = _ld(cos) if cos is not None else 0
    _call("ltx_qk_norm_rope", _ptr(x), _ld(x), rows, rows_per_batch, heads, head_dim, _ptr(weight), eps, _ptr(cos),
          _ptr(sin), ld_rope, rope_ld_batch, _dt(x), _stream(x))


def qk_norm_rope_pair(x: torch.Tensor, k_offset: int, rows_per_batch: int, heads: int, head_dim: int,
                      q_weight: torch.Tensor, k_weight: torch.Tensor, eps: float, cos: torch.Tensor | None,
                      sin: torch.Tensor | None, rope_ld_batch: int = 0) -> None:
    """q (columns [0, H*d)) and k (columns [k_offset, k_offset + H*d)) of x normalised and
    rotated in one launch; x is a row-major view whose row stride covers both blocks."""
    ld_rope = _ld(cos) if cos is not None else 0
    _call("ltx_qk_norm_rope_pair", _ptr(x), _ld(x), k_offset, x.shape[0], rows_per_batch, heads, head_dim,
          _ptr(q_weight), _ptr(k_weight), eps, _ptr(cos), _ptr(sin), ld_rope, rope_ld_batch, _dt(x), _stream(x))


def rope_tables(bounds: torch.Tensor, freqs: torch.Tensor, max_pos: torch.Tensor, dim: int, cos_out: torch.Tensor,
                sin_out: torch.Tensor) -> None:
    """bounds (n_axes, T, 2) fp32 contiguous positions of one sample -> cos/sin (T, dim/2)."""
    n_axes, t, two = bounds.shape
    if two != 2 or not bounds.is_contiguous() or bounds.dtype != torch.float32:
        raise ValueError("bounds must be a contiguous float32 (n_axes, T, 2) tensor")
    _call("ltx_rope_tables", _ptr(bounds), n_axes, t, _ptr(freqs), freqs.numel(), _ptr(max_pos), dim, _ptr(cos_out),
          _ptr(sin_out), _dt(cos_out), _stream(bounds))


def gelu_tanh(x: torch.Tensor, y: torch.Tensor) -> None:
    _call("ltx_gelu_tanh", _ptr(x), _ptr(y), x.numel(), _dt(x), _stream(x))


def gate_residual(x: torch.Tensor, y: torch.Tensor, out: torch.Tensor, rows_per_batch: int,
                  gate: Modulation | None) -> None:
    rows, d = x.shape
    _call("ltx_gate_residual", _ptr(x), _ld(x), _ptr(y), _ld(y), _ptr(out), _ld(out), rows, rows_per_batch, d,
          ctypes.byref(gate) if gate is not None else None, _dt(x), _stream(x))


def timestep_embedding(t: torch.Tensor, scale: float, dim: int, max_period: float, out: torch.Tensor) -> None:
    if t.dtype != torch.float32:
        raise TypeError("timesteps must be float32")
    _call("ltx_timestep_embedding", _ptr(t), t.numel(), scale, dim, max_period, _ptr(out), _dt(out), _stream(t))


def epilogue(kind: int = EPI_NONE, bias: torch.Tensor | None = None, residual: torch.Tensor | None = None,
             gate: Modulation | None = None, rows_per_batch: int = 1, row_mask: torch.Tensor | None = None,
             row_vec: torch.Tensor | None = None, silu_input: bool = False) -> Epilogue:
    e = Epilogue()
    e.kind = kind
    e.bias = _ptr(bias)
    if residual is not None:
        e.residual = _ptr(residual)
        e.ld_residual = _ld(residual)
    if gate is not None:
        e.gate = gate
    e.rows_per_batch = rows_per_batch
    e.row_mask = _ptr(row_mask)
    e.row_vec = _ptr(row_vec)
    e.silu_input = int(silu_input)
    return e


def linear(a: torch.Tensor, w: torch.Tensor, c: torch.Tensor, epi: Epilogue | None = None) -> None:
    """c = epilogue(a @ w.T (+ bias)); a (M, K), w (N, K), c (M, N) row-major views."""
    m, k = a.shape
    n = w.shape[0]
    if w.shape[1] != k or c.shape[0] != m or c.shape[1] != n:
        raise ValueError(f"shape mismatch a{tuple(a.shape)} w{tuple(w.shape)} c{tuple(c.shape)}")
    _call("ltx_linear", _ptr(a), _ld(a), _ptr(w), _ld(w), _ptr(c), _ld(c), m, n, k,
          ctypes.byref(epi) if epi is not None else None, _dt(a), _stream(a),
          label=f"linear M={m} N={n} K={k}" if _profile is not None else None)


def test_bounded_wait(limit_cycles: int, returned: torch.Tensor) -> None:
    """Test hook (include/ltxb200_testing.h): a bounded mbarrier wait that must expire."""
    _call("ltx_test_bounded_wait", limit_cycles, _ptr(returned), _stream(returned))


def attention_force_split(parts: int) -> None:
    """Test hook (include/ltxb200_testing.h): run every unit of the calling thread's
    attention calls as `parts` key-range parts (0: the automatic plan; -1: never split)."""
    _call("ltx_test_attention_force_split", parts)


def attention_plan(units: int, tk: int, sms: int) -> tuple[int, int]:
    """Test hook: (units run whole, parts per remaining unit) of the automatic split plan."""
    n_full, split_k = ctypes.c_int(), ctypes.c_int()
    _call("ltx_test_attention_plan", units, tk, sms, ctypes.byref(n_full), ctypes.byref(split_k))
    return n_full.value, split_k.value


def gemm_set_tile_n(bn: int) -> None:
    """Test hook (include/ltxb200_testing.h): force the calling thread's GEMM tile width."""
    _call("ltx_gemm_set_tile_n", bn)


_attn_ws: dict[tuple[int, int], torch.Tensor] = {}


def attention_workspace(batch: int, tq: int, tk: int, heads: int, head_dim: int,
                        device: torch.device) -> torch.Tensor | None:
    """The zero-filled attention workspace of the current stream on `device`, grown to
    what this shape needs (ltx_attention_workspace_bytes); None when the shape needs none.
    Calls on one stream run in order and share it; every stream has its own."""
    n = load_library().ltx_attention_workspace_bytes(batch, tq, tk, heads, head_dim)
    if n == 0:
        return None
    key = (device.index, torch.cuda.current_stream(device).cuda_stream)
    ws = _attn_ws.get(key)
    if ws is None or ws.numel() < n:
        ws = torch.zeros(n, dtype=torch.uint8, device=device)
        _attn_ws[key] = ws
    return ws


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, o: torch.Tensor, batch: int, tq: int, tk: int,
              heads: int, head_dim: int, scale: float, gate_logits: torch.Tensor | None = None,
              split_tail: bool = True) -> None:
    """q (B*Tq, >=H*d), k/v (B*Tk, >=H*d), o (B*Tq, >=H*d) row-major views; gate (B*Tq, >=H).
    bf16 runs through ltx_attention_ws with the stream's workspace; split_tail=False
    passes no workspace (the single-pass launch of ltx_attention)."""
    ws = attention_workspace(batch, tq, tk, heads, head_dim, q.device) \
        if split_tail and q.dtype == torch.bfloat16 else None
    _call("ltx_attention_ws", _ptr(q), _ld(q), _ptr(k), _ld(k), _ptr(v), _ld(v), _ptr(o), _ld(o), batch, tq, tk,
          heads, head_dim, scale, _ptr(gate_logits), _ld(gate_logits) if gate_logits is not None else 0, _ptr(ws),
          ws.numel() if ws is not None else 0, _dt(q), _stream(q),
          label=f"attention B={batch} H={heads} Tq={tq} Tk={tk} d={head_dim}" if _profile is not None else None)


def attention_partial(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, o_part: torch.Tensor, lse: torch.Tensor,
                      batch: int, tq: int, tk: int, heads: int, head_dim: int, scale: float) -> None:
    """Split-KV partial attention: o_part (B*Tq, >=H*d) fp32 = O / l over these keys,
    lse (B*Tq, >=H) fp32 = log2-sum-exp of the scaled scores (q/k/v bf16 row-major views)."""
    if o_part.dtype != torch.float32 or lse.dtype != torch.float32:
        raise TypeError("o_part and lse must be float32")
    _call("ltx_attention_partial", _ptr(q), _ld(q), _ptr(k), _ld(k), _ptr(v), _ld(v), _ptr(o_part), _ld(o_part),
          _ptr(lse), _ld(lse), batch, tq, tk, heads, head_dim, scale, _stream(q),
          label=f"attention_partial B={batch} H={heads} Tq={tq} Tk={tk} d={head_dim}" if _profile is not None else None)


def attention_merge(o_parts: torch.Tensor, lse_parts: torch.Tensor, gate_logits: torch.Tensor | None,
                    out: torch.Tensor, heads: int, head_dim: int) -> None:
    """out (rows, >=H*d) bf16 = merge of o_parts (R, rows, H*d) / lse_parts (R, rows, H) fp32
    (contiguous) with the gate 2*sigmoid(logit) applied."""
    r, rows = o_parts.shape[0], o_parts.shape[1]
    if not (o_parts.is_contiguous() and lse_parts.is_contiguous()) or o_parts.shape[2] != heads * head_dim \
            or tuple(lse_parts.shape) != (r, rows, heads):
        raise ValueError("o_parts (R, rows, H*d) and lse_parts (R, rows, H) must be contiguous")
    _call("ltx_attention_merge", _ptr(o_parts), _ptr(lse_parts), r, rows, heads, head_dim, _ptr(gate_logits),
          _ld(gate_logits) if gate_logits is not None else 0, _ptr(out), _ld(out), _stream(out))


def cfg_euler(vel: torch.Tensor, latent: torch.Tensor, timesteps: torch.Tensor, cfg_scale: float, sigma: float,
              sigma_next: float, new_latent: torch.Tensor, denoised: torch.Tensor | None = None) -> None:
    t, c = latent.shape[-2], latent.shape[-1]
    _call("ltx_cfg_euler", _ptr(vel), _ptr(latent), _ptr(timesteps), t, c, cfg_scale, sigma, sigma_next,
          _ptr(denoised), _ptr(new_latent), _dt(latent), _stream(latent))


def sp_pack(src: torch.Tensor, parts: int, segments: list[tuple[int, int]], dst: torch.Tensor) -> None:
    """dst (parts, rows, W) <- per-destination column segments (offset, width) of src (rows, ld)."""
    n = len(segments)
    off = (ctypes.c_int * n)(*[s[0] for s in segments])
    wid = (ctypes.c_int * n)(*[s[1] for s in segments])
    _call("ltx_sp_pack", _ptr(src), _ld(src), src.shape[0], parts, n, off, wid, _ptr(dst), _dt(src), _stream(src))


def sp_unpack(src: torch.Tensor, parts: int, dst: torch.Tensor) -> None:
    """dst (rows, parts*w) <- src (parts, rows, w)."""
    p, rows, w = src.shape
    _call("ltx_sp_unpack", _ptr(src), rows, parts, w, _ptr(dst), _ld(dst), _dt(src), _stream(src))


def peer_alloc(nbytes: int) -> tuple[int, bytes]:
    """A zero-filled device buffer other processes of the node can map: (pointer, 64-byte
    CUDA IPC handle). Freed with peer_free."""
    ptr = c_vp()
    handle = ctypes.create_string_buffer(64)
    _call("ltx_peer_alloc", nbytes, ctypes.byref(ptr), ctypes.cast(handle, c_vp))
    return int(ptr.value), handle.raw


def peer_open(handle: bytes) -> int:
    """Map another process's peer_alloc buffer into this one (its device pointer here)."""
    ptr = c_vp()
    buf = ctypes.create_string_buffer(handle, 64)
    _call("ltx_peer_open", ctypes.cast(buf, c_vp), ctypes.byref(ptr))
    return int(ptr.value)


def peer_close(ptr: int) -> None:
    _call("ltx_peer_close", ptr)


def peer_free(ptr: int) -> None:
    _call("ltx_peer_free", ptr)


def _ptr_array(ptrs: list[int]):
    return (c_vp * len(ptrs))(*ptrs)


def qk_norm_rope_scatter(x: torch.Tensor, rows_per_batch: int, heads: int, head_dim: int, q_weight: torch.Tensor,
                         k_weight: torch.Tensor, eps: float, cos: torch.Tensor | None, sin: torch.Tensor | None,
                         gated: bool, sp_rank: int, dst: list[int], ld_dst: int, rope_ld_batch: int = 0) -> None:
    """Self-attention q/k RMSNorm + RoPE of x (rows, [q | k | v | gate]) with the rows sent
    to the SP ranks' receive buffers (dst[j], row stride ld_dst) instead of written back."""
    _call("ltx_qk_norm_rope_scatter", _ptr(x), _ld(x), x.shape[0], rows_per_batch, heads, head_dim, _ptr(q_weight),
          _ptr(k_weight), eps, _ptr(cos), _ptr(sin), _ld(cos) if cos is not None else 0, rope_ld_batch, int(gated),
          len(dst), sp_rank, _ptr_array(dst), ld_dst, _stream(x),
          label="ltx_qk_norm_rope_scatter" if _profile is not None else None)


def attention_scatter(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, batch: int, t: int, heads: int,
                      head_dim: int, scale: float, gate_logits: torch.Tensor | None, out: list[int], out_ld: int,
                      out_col0: int) -> None:
    """Self-attention over the receive buffer (batch x t tokens) with each output row
    written to its token owner's buffer (out[j], rows t / len(out) per sample)."""
    ws = attention_workspace(batch, t, t, heads, head_dim, q.device)
    _call("ltx_attention_scatter", _ptr(q), _ld(q), _ptr(k), _ld(k), _ptr(v), _ld(v), batch, t, heads, head_dim,
          scale, _ptr(gate_logits), _ld(gate_logits) if gate_logits is not None else 0, _ptr(ws),
          ws.numel() if ws is not None else 0, len(out), _ptr_array(out), out_ld, out_col0, _stream(q),
          label=f"attention B={batch} H={heads} Tq={t} Tk={t} d={head_dim} (scatter)" if _profile is not None
          else None)


def sp_barrier(flags: list[int], counter: int, rank: int, limit_cycles: int = 4_000_000_000,
               stream: torch.cuda.Stream | None = None) -> None:
    """Flag barrier of the SP group over peer memory (see ltx_sp_barrier)."""
    s = (stream or torch.cuda.current_stream()).cuda_stream
    _call("ltx_sp_barrier", _ptr_array(flags), counter, len(flags), rank, limit_cycles, s,
          label="ltx_sp_barrier" if _profile is not None else None)


def _same_elementwise(*ts: torch.Tensor) -> None:
    """The element-wise entry points take flat buffers: every tensor must be contiguous
    and have the first one's element count, dtype and device."""
    ref = ts[0]
    for t in ts:
        if not t.is_contiguous():
            raise ValueError("element-wise operands must be contiguous")
        if t.numel() != ref.numel() or t.dtype != ref.dtype or t.device != ref.device:
            raise ValueError(f"element-wise operands differ: {tuple(t.shape)} {t.dtype} {t.device} vs "
                             f"{tuple(ref.shape)} {ref.dtype} {ref.device}")


def guide(cond: torch.Tensor, uncond: torch.Tensor, ptb: torch.Tensor, mod: torch.Tensor, cfg_scale: float,
          stg_scale: float, modality_scale: float, out: torch.Tensor) -> None:
    _same_elementwise(cond, uncond, ptb, mod, out)
    _call("ltx_guide", _ptr(cond), _ptr(uncond), _ptr(ptb), _ptr(mod), cond.numel(), cfg_scale, stg_scale,
          modality_scale, _ptr(out), _dt(cond), _stream(cond))


def value_gate(v: torch.Tensor, gate_logits: torch.Tensor | None, o: torch.Tensor, heads: int, head_dim: int) -> None:
    """o = V gated by 2*sigmoid(logit) per (row, head): the STG-perturbed attention output.
    v / o (rows, >= H*d) row-major views, gate (rows, >= H)."""
    _call("ltx_value_gate", _ptr(v), _ld(v), _ptr(gate_logits), _ld(gate_logits) if gate_logits is not None else 0,
          _ptr(o), _ld(o), v.shape[0], heads, head_dim, _dt(v), _stream(v))


def x0(latent: torch.Tensor, velocity: torch.Tensor, timesteps: torch.Tensor, out: torch.Tensor) -> None:
    """out = round(latent - velocity * timesteps) over (rows, C); timesteps fp32 (rows,)."""
    c = latent.shape[-1]
    rows = latent.numel() // c
    if timesteps.dtype != torch.float32 or not timesteps.is_contiguous() or timesteps.numel() != rows:
        raise ValueError("timesteps must be a contiguous float32 tensor with one entry per row")
    _call("ltx_x0", _ptr(latent), _ptr(velocity), _ptr(timesteps), rows, c, _ptr(out), _dt(latent), _stream(latent))


def register_fill(x: torch.Tensor, additive_mask: torch.Tensor, registers: torch.Tensor, rows_per_batch: int,
                  out: torch.Tensor) -> None:
    """out = x where the per-row additive mask is >= 0, else registers[(row % S) % R]."""
    if not additive_mask.is_contiguous() or additive_mask.numel() != x.shape[0]:
        raise ValueError("additive_mask must be contiguous with one entry per row")
    _call("ltx_register_fill", _ptr(x), _ld(x), _ptr(additive_mask), _ptr(registers.contiguous()),
          registers.shape[0], x.shape[0], rows_per_batch, x.shape[1], _ptr(out), _ld(out), _dt(x), _stream(x))


# ---------------------------------------------------------------------------------------
# Video VAE decoder (channels-last (B, F, H, W, C) bf16 activations)
# ---------------------------------------------------------------------------------------
def _cl5(t: torch.Tensor) -> tuple[int, int, int, int, int]:
    if t.dim() != 5 or not t.is_contiguous() or t.dtype != torch.bfloat16:
        raise ValueError(f"expected a contiguous (B, F, H, W, C) bf16 tensor, got {tuple(t.shape)} {t.dtype}")
    return tuple(t.shape)


def conv3d(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, out: torch.Tensor, ksize: int,
           causal: bool = False, residual: torch.Tensor | None = None, norm_silu_eps: float | None = None) -> None:
    """out (B, F, H, W, cout) = conv(x) + bias (+ residual); weight (cout, taps, cin). With
    norm_silu_eps, out = silu(PixelNorm(conv(x) + bias)) computed in the epilogue."""
    b, f, h, w, cin = _cl5(x)
    cout = _cl5(out)[4]
    if weight.shape != (cout, ksize ** 3, cin) or not weight.is_contiguous():
        raise ValueError(f"weight must be contiguous ({cout}, {ksize ** 3}, {cin}), got {tuple(weight.shape)}")
    if residual is not None and residual.shape != out.shape:
        raise ValueError("residual must have the output's shape")
    fused = norm_silu_eps is not None
    _call("ltx_conv3d_norm", _ptr(x), b, f, h, w, cin, _ptr(weight), _ptr(bias), cout, ksize, int(causal),
          _ptr(residual), int(fused), float(norm_silu_eps) if fused else 0.0, _ptr(out), _stream(x),
          label=f"conv3d k{ksize} {cin}->{cout} {b}x{f}x{h}x{w}{' +norm' if fused else ''}"
          if _profile is not None else None)


def pixel_norm(x: torch.Tensor, y: torch.Tensor, eps: float = 1e-8, silu: bool = False) -> None:
    c = x.shape[-1]
    _call("ltx_pixel_norm", _ptr(x), _ptr(y), x.numel() // c, c, eps, int(silu), _stream(x),
          label=f"pixel_norm C={c}" if _profile is not None else None)


def group_norm1(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float, y: torch.Tensor,
                workspace: torch.Tensor) -> None:
    b, c = x.shape[0], x.shape[-1]
    _call("ltx_group_norm1", _ptr(x), b, x.numel() // b, c, _ptr(weight), _ptr(bias), eps, _ptr(workspace),
          workspace.numel() * workspace.element_size(), _ptr(y), _stream(x))


def group_norm1_workspace(batch: int, device: torch.device) -> torch.Tensor:
    nbytes = int(load_library().ltx_group_norm1_workspace_bytes(batch))
    return torch.empty(nbytes // 8, dtype=torch.float64, device=device)


def depth_to_space(x: torch.Tensor, stride: tuple[int, int, int], drop_first: bool, y: torch.Tensor) -> None:
    b, f, h, w, cin = _cl5(x)
    p1, p2, p3 = stride
    c = cin // (p1 * p2 * p3)
    if y.shape != (b, f * p1 - int(drop_first), h * p2, w * p3, c):
        raise ValueError(f"output shape {tuple(y.shape)} does not match the rearrange")
    _call("ltx_depth_to_space", _ptr(x), b, f, h, w, c, p1, p2, p3, int(drop_first), _ptr(y), _stream(x))


def vae_latent_in(latent: torch.Tensor, std: torch.Tensor, mean: torch.Tensor, y: torch.Tensor) -> None:
    b, c, f, h, w = latent.shape
    _call("ltx_vae_latent_in", _ptr(latent.contiguous()), b, c, f, h, w, _ptr(std.float().contiguous()),
          _ptr(mean.float().contiguous()), _ptr(y), _stream(latent))


def vae_unpatchify(x: torch.Tensor, p: int, out: torch.Tensor, frames: bool = False) -> None:
    b, f, h, w, cin = _cl5(x)
    _call("ltx_vae_unpatchify", _ptr(x), b, f, h, w, cin // (p * p), p, int(frames), _ptr(out), _stream(x))


def guide_rescale_workspace(n: int, device: torch.device) -> torch.Tensor:
    """A zeroed device workspace for guide_rescale over n elements (reusable: every call
    leaves its completion counter at zero)."""
    nbytes = int(load_library().ltx_guide_rescale_workspace_bytes(n))
    return torch.zeros((nbytes + 15) // 16 * 16, dtype=torch.uint8, device=device)


def guide_rescale(cond: torch.Tensor, uncond: torch.Tensor, ptb: torch.Tensor, mod: torch.Tensor, cfg_scale: float,
                  stg_scale: float, modality_scale: float, rescale_scale: float, out: torch.Tensor,
                  workspace: torch.Tensor) -> None:
    _same_elementwise(cond, uncond, ptb, mod, out)
    if not workspace.is_contiguous() or workspace.dtype != torch.uint8 or workspace.device != cond.device:
        raise ValueError("workspace must be a contiguous uint8 tensor on the operands' device")
    _call("ltx_guide_rescale", _ptr(cond), _ptr(uncond), _ptr(ptb), _ptr(mod), cond.numel(), cfg_scale, stg_scale,
          modality_scale, rescale_scale, _ptr(out), _ptr(workspace), workspace.numel(), _dt(cond), _stream(cond))


def guide_rescale_noalloc(cond: torch.Tensor, uncond: torch.Tensor, ptb: torch.Tensor, mod: torch.Tensor,
                          cfg_scale: float, stg_scale: float, modality_scale: float, rescale_scale: float,
                          out: torch.Tensor) -> None:
    """guide_rescale with the library's static scratch (no workspace, n <= 1,048,576)."""
    _same_elementwise(cond, uncond, ptb, mod, out)
    _call("ltx_guide_rescale_noalloc", _ptr(cond), _ptr(uncond), _ptr(ptb), _ptr(mod), cond.numel(), cfg_scale,
          stg_scale, modality_scale, rescale_scale, _ptr(out), _dt(cond), _stream(cond))


def euler(sample: torch.Tensor, denoised: torch.Tensor, sigma: float, sigma_next: float, out: torch.Tensor) -> None:
    _same_elementwise(sample, denoised, out)
    _call("ltx_euler", _ptr(sample), _ptr(denoised), sample.numel(), sigma, sigma_next, _ptr(out), _dt(sample),
          _stream(sample))


def proj_out_cfg_euler(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor, latent: torch.Tensor,
                       timesteps: torch.Tensor, cfg_scale: float, sigma: float, sigma_next: float,
                       new_latent: torch.Tensor, denoised: torch.Tensor | None = None,
                       vel_out: torch.Tensor | None = None) -> None:
    t, c = latent.shape[-2], latent.shape[-1]
    _call("ltx_proj_out_cfg_euler", _ptr(x), _ld(x), _ptr(w), _ptr(bias), t, c, x.shape[1], _ptr(latent),
          _ptr(timesteps), cfg_scale, sigma, sigma_next, _ptr(vel_out), _ptr(denoised), _ptr(new_latent), _dt(x),
          _stream(x))


# ---------------------------------------------------------------------------------------
# Whole-step entry point (ltx_ctx / ltx_dit_step)
# ---------------------------------------------------------------------------------------
def ctx_create(device: int) -> int:
    h = c_vp()
    _call("ltx_ctx_create", device, ctypes.byref(h))
    return h.value


def ctx_destroy(ctx: int) -> None:
    _call("ltx_ctx_destroy", ctx)


def dit_workspace_bytes(cfg: DitConfig, t: int, s: int) -> int:
    return int(load_library().ltx_dit_workspace_bytes(ctypes.byref(cfg), t, s))


def dit_reserve(ctx: int, cfg: DitConfig, t: int, s: int) -> None:
    _call("ltx_dit_reserve", ctx, ctypes.byref(cfg), t, s)


def dit_step(ctx: int, cfg: DitConfig, weights: DitWeights, args: DitStepArgs, velocity: torch.Tensor | None,
             denoised: torch.Tensor | None, new_latent: torch.Tensor) -> None:
    _call("ltx_dit_step", ctx, ctypes.byref(cfg), ctypes.byref(weights), ctypes.byref(args), _ptr(velocity),
          _ptr(denoised), _ptr(new_latent), _stream(new_latent), label="ltx_dit_step" if _profile is not None else None)
