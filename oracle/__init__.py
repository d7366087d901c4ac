"""Test infrastructure: fp32 restatement of the reference transformer forward.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm may
import this package.  It is the checker the CUDA path is compared against, never a
code path of the product.
"""
from .reference_fp32 import (  # noqa: F401
    attention_fp32,
    block_fp32,
    forward_fp32,
    forward_fp32_per_sequence,
    gelu_erf,
    layer_norm,
    linear,
    state_dict_fp32,
)
