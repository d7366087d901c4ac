"""CPU: the drop-in boundary exercised with the reference's own classes.

The reference's organizer module (benchmarks/torch_transformer_benchmark.py of
Scallion3008/tttj-2026: TransformerConfig, BaselineTransformer, UserOptimizedTransformer,
copy_model_weights, compare_outputs) is imported unmodified from its sources when they
are present next to this repository (they are read-only and never travel to a GPU
machine, so these tests run on the CPU and are skipped elsewhere).  They check that

* make_optimized_transformer reads a reference BaselineTransformer exactly as it reads
  this package's TransformerParameters (same module tree, byte-identical packed weights),
* the reference's copy_model_weights moves weights between the two (strict state dict),
* the organizer's UserOptimizedTransformer slot, whose forward builds the B200 module
  from itself on first use (kept in the instance dict, outside the submodules), reaches
  the constructor (on a CPU model it raises the constructor's ValueError; on a
  CUDA device the same slot runs the B200 forward), and
* the reference's own regression gate, compare_outputs (rtol 0.01 / atol 0.001,
  benchmarks/torch_transformer_benchmark.py:289-330), accepts the fp32 oracle against the
  reference module on the committed golden cases.
"""
import importlib.util
import sys
from pathlib import Path

import pytest
import torch

import tttj_2026_b200 as tb
from helpers import golden_index, load_golden
from oracle import forward_fp32, state_dict_fp32
from test_oracle_golden import _model as golden_model

REFERENCE_ROOT = Path(__file__).resolve().parents[2] / "reference"
REFERENCE_MODULE = REFERENCE_ROOT / "benchmarks" / "torch_transformer_benchmark.py"

pytestmark = pytest.mark.skipif(not REFERENCE_MODULE.exists(),
                                reason="reference sources not present on this machine")


@pytest.fixture(scope="module")
def ref():
    spec = importlib.util.spec_from_file_location("_tttj_reference_organizer", REFERENCE_MODULE)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod
    spec.loader.exec_module(mod)
    return mod


CFG = dict(batch_size=2, seq_len=40, d_model=128, num_heads=2, ffn_dim=256, num_layers=2, causal=True)


def _pair(ref, seed=5):
    torch.manual_seed(seed)
    theirs = ref.BaselineTransformer(ref.TransformerConfig(**CFG)).half()
    torch.manual_seed(seed)
    ours = tb.TransformerParameters(tb.TransformerConfig(**CFG)).half()
    return theirs, ours


def test_reference_model_packs_like_the_parameter_model(ref):
    theirs, ours = _pair(ref)
    sd_t, sd_o = theirs.state_dict(), ours.state_dict()
    assert list(sd_t) == list(sd_o)
    for k in sd_t:
        assert torch.equal(sd_t[k], sd_o[k]), k
    tb.validate_model_config(theirs.config)
    assert torch.equal(tb.pack_weights(theirs, torch.device("cpu")),
                       tb.pack_weights(ours, torch.device("cpu")))


def test_reference_copy_model_weights_into_the_parameter_model(ref):
    theirs, _ = _pair(ref, seed=6)
    _, ours = _pair(ref, seed=7)
    ref.copy_model_weights(theirs, ours, strict=True)
    assert torch.equal(tb.pack_weights(theirs, torch.device("cpu")),
                       tb.pack_weights(ours, torch.device("cpu")))


def test_organizer_slot_reaches_the_constructor(ref):
    from optimized_transformer import make_optimized_transformer

    class Slot(ref.UserOptimizedTransformer):
        def forward(self, x, valid_token_mask=None):
            if "_b200" not in self.__dict__:
                self.__dict__["_b200"] = make_optimized_transformer(self)
            return self._b200(x, valid_token_mask)

    model = Slot(ref.TransformerConfig(**CFG))
    x = torch.zeros(2, 40, 128)
    with pytest.raises(ValueError, match="CUDA"):
        model(x, None)
    # Shapes without a kernel raise the reference constructor's ValueError as well.
    bad = Slot(ref.TransformerConfig(2, 16, 48, 4, 64, 1, True))  # head_dim 12
    with pytest.raises(ValueError, match="head_dim=12"):
        tb.validate_model_config(bad.config)


@pytest.mark.parametrize("name", sorted(golden_index()))
def test_reference_regression_gate_accepts_the_oracle(ref, name):
    entry = golden_index()[name]
    cfg, model = golden_model(entry)
    x, mask, ref_out = load_golden(name)
    out = forward_fp32(state_dict_fp32(model, "cpu"), cfg, x.float(), mask)
    result = ref.compare_outputs(ref_out, out, rtol=0.01, atol=0.001)
    assert result.passed, result
