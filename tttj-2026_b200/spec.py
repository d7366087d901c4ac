"""Shape record and parameter container of the transformer this package accelerates.

``TransformerConfig`` mirrors the reference's frozen dataclass
(benchmarks/torch_transformer_benchmark.py:29-56) field for field, including
``validate()``.  ``TransformerParameters`` is an nn.Module with the reference
organizer model's module tree (BaselineTransformer :148-172, BaselineTransformerBlock
:125-145, BaselineSelfAttention :59-75), so ``make_optimized_transformer`` accepts it
and the reference's own ``BaselineTransformer`` interchangeably, and
``load_state_dict`` moves weights between them.  It has no forward of its own.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn as nn


@dataclass(frozen=True)
class TransformerConfig:
    batch_size: int
    seq_len: int
    d_model: int
    num_heads: int
    ffn_dim: int
    num_layers: int
    causal: bool

    def validate(self) -> None:
        # Same checks and messages as the reference (torch_transformer_benchmark.py:39-56).
        if self.batch_size <= 0:
            raise ValueError("batch_size must be positive")
        if self.seq_len <= 0:
            raise ValueError("seq_len must be positive")
        if self.d_model <= 0:
            raise ValueError("d_model must be positive")
        if self.num_heads <= 0:
            raise ValueError("num_heads must be positive")
        if self.d_model % self.num_heads != 0:
            raise ValueError(
                f"d_model ({self.d_model}) must be divisible by "
                f"num_heads ({self.num_heads})"
            )
        if self.ffn_dim <= 0:
            raise ValueError("ffn_dim must be positive")
        if self.num_layers <= 0:
            raise ValueError("num_layers must be positive")

    @property
    def head_dim(self) -> int:
        return self.d_model // self.num_heads


class _Attention(nn.Module):
    def __init__(self, d_model: int, num_heads: int) -> None:
        super().__init__()
        self.d_model = d_model
        self.num_heads = num_heads
        self.head_dim = d_model // num_heads
        self.scale = self.head_dim**-0.5
        self.q_proj = nn.Linear(d_model, d_model, bias=True)
        self.k_proj = nn.Linear(d_model, d_model, bias=True)
        self.v_proj = nn.Linear(d_model, d_model, bias=True)
        self.out_proj = nn.Linear(d_model, d_model, bias=True)


class _Block(nn.Module):
    def __init__(self, d_model: int, num_heads: int, ffn_dim: int) -> None:
        super().__init__()
        self.norm1 = nn.LayerNorm(d_model)
        self.attention = _Attention(d_model, num_heads)
        self.norm2 = nn.LayerNorm(d_model)
        self.ffn_in = nn.Linear(d_model, ffn_dim)
        self.ffn_out = nn.Linear(ffn_dim, d_model)


class TransformerParameters(nn.Module):
    """Weights of the stack, laid out exactly like the reference organizer model.

    Construction consumes the global torch RNG in the same order as the reference's
    ``BaselineTransformer(config)``, so ``torch.manual_seed(s)`` followed by either
    constructor yields identical default-initialised weights.
    """

    def __init__(self, config: TransformerConfig) -> None:
        super().__init__()
        config.validate()
        self.config = config
        self.layers = nn.ModuleList(
            [_Block(config.d_model, config.num_heads, config.ffn_dim) for _ in range(config.num_layers)]
        )
        self.final_norm = nn.LayerNorm(config.d_model)

    def forward(self, *args, **kwargs):  # pragma: no cover - container only
        raise NotImplementedError(
            "TransformerParameters only holds weights; build the executable module with "
            "make_optimized_transformer(model)"
        )


def make_parameter_model(config: TransformerConfig, seed: int, dtype: torch.dtype,
                         device: torch.device | str) -> TransformerParameters:
    """Default-initialised weights from ``torch.manual_seed(seed)`` (the reference
    harness's convention, benchmarks/regression.py:41-43), cast to ``dtype``."""
    torch.manual_seed(seed)
    model = TransformerParameters(config)
    return model.to(device=device, dtype=dtype).eval()


def generate_inputs(config: TransformerConfig, seed: int, dtype: torch.dtype,
                    lengths: tuple[int, int] | None, device: torch.device | str = "cpu"):
    """Seeded synthetic inputs: x ~ N(0, 1) [B, S, D] and a prefix valid_token_mask
    with per-sequence length uniform in ``lengths`` (inclusive), or None for no mask.
    Padded input rows are zeroed as the reference generator does
    (benchmarks/torch_transformer_benchmark.py:258-271).  Generated on the CPU so the
    same seed gives the same case on every machine."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(config.batch_size, config.seq_len, config.d_model, generator=g)
    mask = None
    if lengths is not None:
        lo, hi = lengths
        lens = torch.randint(lo, hi + 1, (config.batch_size,), generator=g)
        mask = torch.arange(config.seq_len)[None, :] < lens[:, None]
        x = x.masked_fill(~mask[..., None], 0)
    x = x.to(dtype=dtype, device=device)
    if mask is not None:
        mask = mask.to(device)
    return x, mask
