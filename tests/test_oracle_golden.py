"""CPU: pin the fp32 oracle against golden outputs of the unmodified reference module.

The fixtures under tests/golden/ were produced by tests/golden/make_golden.py, which
runs the reference's BaselineTransformer (benchmarks/torch_transformer_benchmark.py
:148-172) in fp32.  The weights are rebuilt here from the same seed through
TransformerParameters; the stored checksum proves they are the reference's weights.
"""
import importlib.util

import pytest
import torch

import tttj_2026_b200 as tb
from helpers import GOLDEN, golden_index, load_golden
from oracle import forward_fp32, forward_fp32_per_sequence, state_dict_fp32

_spec = importlib.util.spec_from_file_location("_make_golden", GOLDEN / "make_golden.py")
make_golden = importlib.util.module_from_spec(_spec)
_spec.loader.exec_module(make_golden)

INDEX = golden_index()


def _model(entry):
    cfg = tb.TransformerConfig(**entry["config"])
    torch.manual_seed(entry["model_seed"])
    model = tb.TransformerParameters(cfg).eval()
    if entry["perturbed_norms"]:
        make_golden.perturb_norms(model, entry["model_seed"] + 1000)
    return cfg, model


@pytest.mark.parametrize("name", sorted(INDEX))
def test_parameter_model_matches_reference_init(name):
    entry = INDEX[name]
    _, model = _model(entry)
    assert make_golden.weights_checksum(model) == pytest.approx(entry["weights_checksum"], rel=1e-12, abs=1e-9)


@pytest.mark.parametrize("name", sorted(INDEX))
def test_oracle_matches_reference_outputs(name):
    entry = INDEX[name]
    cfg, model = _model(entry)
    x, mask, ref_out = load_golden(name)
    with torch.inference_mode():
        out = forward_fp32(state_dict_fp32(model), cfg, x, mask)
    err = (out - ref_out).abs()
    assert torch.isfinite(out).all()
    assert float(err.max()) < 2e-5, float(err.max())
    if mask is not None:
        assert (out[~mask] == 0).all()


@pytest.mark.parametrize("name", ["causal_hd64_ragged", "empty_sequence"])
def test_oracle_per_sequence_equals_batched(name):
    entry = INDEX[name]
    cfg, model = _model(entry)
    x, mask, ref_out = load_golden(name)
    p = state_dict_fp32(model)
    with torch.inference_mode():
        per_seq = forward_fp32_per_sequence(p, cfg, x, mask)
    assert float((per_seq - ref_out).abs().max()) < 2e-5


def test_inputs_generator_matches_golden_case():
    """generate_inputs reproduces the fixture generator's C1 input bit for bit."""
    entry = INDEX["c1_tiny_encoder"]
    cfg = tb.TransformerConfig(**entry["config"])
    x, mask = tb.generate_inputs(cfg, entry["input_seed"], torch.float32, tuple(entry["lengths"]))
    gx, gmask, _ = load_golden("c1_tiny_encoder")
    assert torch.equal(x, gx)
    assert torch.equal(mask, gmask)
