"""Shared test helpers: the BASELINE parity gate, golden fixture loading, configs."""
from __future__ import annotations

import json
from dataclasses import dataclass
from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"

# Parity gate against the fp32 oracle: max-abs <= 2e-2,
# mean-abs <= 2e-3 over all elements, masked token rows exactly zero.
MAX_ABS_TOL = 2e-2
MEAN_ABS_TOL = 2e-3


@dataclass
class GateResult:
    max_abs: float
    mean_abs: float
    masked_rows_zero: bool
    finite: bool

    @property
    def passed(self) -> bool:
        return (self.finite and self.masked_rows_zero and self.max_abs <= MAX_ABS_TOL
                and self.mean_abs <= MEAN_ABS_TOL)


def gate(reference: torch.Tensor, candidate: torch.Tensor, mask) -> GateResult:
    ref = reference.detach().float().cpu()
    out = candidate.detach().float().cpu()
    assert ref.shape == out.shape, (ref.shape, out.shape)
    err = (out - ref).abs()
    if mask is not None:
        m = mask.detach().cpu().bool()
        masked_zero = bool((out[~m] == 0).all())
    else:
        masked_zero = True
    return GateResult(float(err.max()) if err.numel() else 0.0,
                      float(err.mean()) if err.numel() else 0.0, masked_zero,
                      bool(torch.isfinite(out).all()))


def golden_index() -> dict:
    return json.loads((GOLDEN / "index.json").read_text())


def load_golden(name: str):
    d = np.load(GOLDEN / f"{name}.npz")
    x = torch.from_numpy(d["x"])
    mask = torch.from_numpy(d["mask"]) if bool(d["has_mask"]) else None
    out = torch.from_numpy(d["out"])
    return x, mask, out


# BASELINE.json configs (C1..C5): (B, S, D, H, F, L, causal, dtype, lengths)
CONFIGS = {
    "C1": (2, 128, 256, 4, 1024, 2, False, torch.float32, (64, 128)),
    "C2": (8, 1024, 512, 8, 2048, 4, True, torch.float16, None),
    "C3": (32, 512, 256, 8, 1024, 6, False, torch.float16, (32, 512)),
    "C4": (4, 8192, 768, 12, 3072, 12, True, torch.float16, (4096, 8192)),
    "C5": (256, 256, 1024, 16, 4096, 24, True, torch.float16, (128, 256)),
}
