"""The reference's 14 implemented benchmark cases, run through the same constructor.

``IMPLEMENTED_CASES`` and ``IMPLEMENTED_CASE_LAYERS`` restate the reference's public
table (optimized_transformer.py:22-42): (batch, sequence, d_model, heads), every case
with ffn_dim == d_model, causal attention and 4 layers (2 for case 14).  The reference
builds a separate module per case; here every case goes through
``make_optimized_transformer`` and the same kernels (head_dim 8 runs on heads padded to
32 columns, head_dim 128 and 256 on their own attention variants).

``case_number_for_model`` keeps the reference's lookup and ValueError message
(optimized_transformer.py:45-66) for callers that dispatch on the case number.
``case_inputs`` draws inputs the way the reference's regression harness does
(benchmarks/regression.py:82-110 with generate_random_case,
benchmarks/torch_transformer_benchmark.py:235-272): padding ratio r gives per-sequence
valid lengths uniform in [round(S * (1 - r)), S], padded rows of x zeroed.
"""
from __future__ import annotations

import torch

from .spec import TransformerConfig, generate_inputs

IMPLEMENTED_CASES: dict[int, tuple[int, int, int, int]] = {
    1: (64, 128, 128, 4),
    2: (1, 128, 128, 4),
    3: (4, 128, 128, 4),
    4: (16, 128, 128, 4),
    5: (128, 128, 128, 4),
    6: (10000, 128, 128, 4),
    7: (64, 128, 32, 4),
    8: (64, 128, 1024, 4),
    9: (64, 128, 128, 1),
    10: (64, 128, 128, 2),
    11: (64, 128, 128, 16),
    12: (64, 32, 128, 4),
    13: (64, 1024, 128, 4),
    14: (32, 100000, 1024, 16),
}

IMPLEMENTED_CASE_LAYERS: dict[int, int] = {n: 2 if n == 14 else 4 for n in IMPLEMENTED_CASES}


def case_config(case_number: int, batch_size: int | None = None) -> TransformerConfig:
    """TransformerConfig of a reference case (``batch_size`` overrides the case's batch,
    as the reference's regression harness does for case 14)."""
    if case_number not in IMPLEMENTED_CASES:
        raise ValueError(f"unknown case {case_number}; cases are 1..14")
    b, s, d, h = IMPLEMENTED_CASES[case_number]
    return TransformerConfig(batch_size if batch_size is not None else b, s, d, h, d,
                             IMPLEMENTED_CASE_LAYERS[case_number], True)


def case_number_for_model(parameter_model) -> int:
    """The reference case whose shape ``parameter_model.config`` has; ValueError otherwise."""
    config = parameter_model.config
    shape = (config.batch_size, config.seq_len, config.d_model, config.num_heads)
    if config.ffn_dim == config.d_model and config.causal:
        for n, case_shape in IMPLEMENTED_CASES.items():
            if shape == case_shape and config.num_layers == IMPLEMENTED_CASE_LAYERS[n]:
                return n
    raise ValueError(
        "no optimized transformer is implemented for "
        f"shape={shape}, ffn_dim={config.ffn_dim}, "
        f"layers={config.num_layers}, causal={config.causal}"
    )


def case_lengths(config: TransformerConfig, padding_ratio: float) -> tuple[int, int] | None:
    """Valid-length range of the reference harness for ``padding_ratio`` (None: no padding)."""
    if padding_ratio <= 0:
        return None
    lo = max(1, int(round(config.seq_len * (1.0 - padding_ratio))))
    return lo, config.seq_len


def case_inputs(config: TransformerConfig, seed: int, padding_ratio: float,
                dtype: torch.dtype = torch.float16, device: torch.device | str = "cpu"):
    """Seeded x [B, S, D] and valid_token_mask (None without padding) for a case."""
    return generate_inputs(config, seed, dtype, case_lengths(config, padding_ratio), device)
