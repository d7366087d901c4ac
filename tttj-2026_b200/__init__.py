"""B200-native (sm_100a) forward path of the tttj-2026 transformer stack.

Import name ``tttj_2026_b200`` (the directory is ``tttj-2026_b200/``, which is not a
valid Python identifier; ``optimized_transformer.py`` at the repository root
registers it under this name).

Public surface:
  * make_optimized_transformer(model) -> nn.Module with forward(x, valid_token_mask)
  * TransformerConfig, TransformerParameters (weights container with the reference
    organizer model's module tree)
  * ops: per-kernel wrappers (linear, layernorm, attention)
  * cases: the reference's 14 benchmark cases (IMPLEMENTED_CASES,
    case_number_for_model), all served by make_optimized_transformer
  * sharding: batch data parallelism (LPT shards, one process per GPU or one
    process driving several GPUs)
"""
from __future__ import annotations

from . import _lib, cases, ops, sharding
from .cases import IMPLEMENTED_CASES, IMPLEMENTED_CASE_LAYERS, case_number_for_model
from .model import B200Transformer, pack_weights, validate_model_config
from .sharding import MultiDeviceTransformer, distributed_forward
from .spec import TransformerConfig, TransformerParameters, generate_inputs, make_parameter_model

__all__ = [
    "B200Transformer",
    "IMPLEMENTED_CASES",
    "IMPLEMENTED_CASE_LAYERS",
    "case_number_for_model",
    "cases",
    "MultiDeviceTransformer",
    "distributed_forward",
    "TransformerConfig",
    "TransformerParameters",
    "generate_inputs",
    "make_optimized_transformer",
    "make_parameter_model",
    "ops",
    "pack_weights",
    "sharding",
    "validate_model_config",
]


def make_optimized_transformer(parameter_model, *, verbose_build: bool = False):
    """Build the B200 module for ``parameter_model``.

    Same name, signature and error behaviour as the reference constructor
    (optimized_transformer.py:69-93): reads ``parameter_model.config`` and its layer
    weights, raises ValueError for shapes without a kernel.  Beyond the reference's 14
    cases it accepts any config with head_dim a multiple of 8 up to 256 and d_model,
    ffn_dim multiples of 32 (causal or not, ffn_dim != d_model), and fp16 or fp32
    parameters on a CUDA device.  ``verbose_build`` prints the
    library version (the library is built ahead of time, not JIT-compiled).
    """
    if verbose_build:
        print(f"[tttj_b200] {_lib.lib().tttj_version().decode()} from {_lib.LIB_PATH}")
    return B200Transformer(parameter_model)
