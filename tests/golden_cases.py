"""Loading helpers for the golden fixtures (tests/golden/*.pt, written by
tests/golden/make_golden.py from the reference implementation)."""

from __future__ import annotations

from pathlib import Path
from types import SimpleNamespace

import torch

from oracle import ltx_oracle

GOLDEN = Path(__file__).resolve().parent / "golden"
CASES = ["tiny_video_float32", "tiny_video_bfloat16", "tiny_av_float32", "tiny_av_bfloat16"]


def load(case: str) -> dict:
    return torch.load(GOLDEN / f"dit_{case}.pt", weights_only=False)


def cfg_of(rec: dict) -> SimpleNamespace:
    return SimpleNamespace(**rec["config"])


def weights_of(rec: dict, dtype: torch.dtype | None = None) -> dict:
    dt = dtype if dtype is not None else getattr(torch, rec["dtype"])
    return ltx_oracle.synthetic_state_dict(rec["param_shapes"], rec["weight_seed"], dtype=dt)


def modality(d: dict | None) -> ltx_oracle.Modality | None:
    if d is None:
        return None
    return ltx_oracle.Modality(**d)


GUIDED_CASES = ["guided_tiny_av_float32", "guided_tiny_av_bfloat16"]


def load_guided(case: str) -> dict:
    return torch.load(GOLDEN / f"{case}.pt", weights_only=False)
