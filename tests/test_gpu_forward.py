"""GPU: the whole forward through make_optimized_transformer -> tttj_forward, against
the golden reference outputs and the fp32 oracle at the BASELINE.json configs."""
import pytest
import torch

import tttj_2026_b200 as tb
from helpers import CONFIGS, gate, golden_index, load_golden
from oracle import forward_fp32, forward_fp32_per_sequence, state_dict_fp32
from test_oracle_golden import _model as golden_model

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


@pytest.fixture(autouse=True, scope="module")
def _no_tf32():
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32 = prev


@pytest.mark.parametrize("name", sorted(golden_index()))
def test_golden_cases_fp32_model(name):
    """fp32 parameter model (weights cast to fp16 inside), fp32 input and output."""
    entry = golden_index()[name]
    cfg, model = golden_model(entry)
    x, mask, ref_out = load_golden(name)
    opt = tb.make_optimized_transformer(model.to(DEV))
    with torch.inference_mode():
        out = opt(x.to(DEV), None if mask is None else mask.to(DEV))
    torch.cuda.synchronize()
    assert out.dtype == torch.float32 and out.shape == x.shape
    r = gate(ref_out, out, mask)
    assert r.passed, r


def _case(name, seed=0):
    B, S, D, H, F, L, causal, dtype, lengths = CONFIGS[name]
    cfg = tb.TransformerConfig(B, S, D, H, F, L, causal)
    model = tb.make_parameter_model(cfg, seed, dtype, DEV)
    x, mask = tb.generate_inputs(cfg, seed + 1, dtype, lengths, DEV)
    return cfg, model, x, mask


@pytest.mark.parametrize("name", ["C1", "C2", "C3", "C5"])
def test_baseline_config_vs_oracle(name):
    cfg, model, x, mask = _case(name)
    opt = tb.make_optimized_transformer(model)
    with torch.inference_mode():
        out = opt(x, mask)
        ref = forward_fp32(state_dict_fp32(model, DEV), cfg, x.float(), mask)
    torch.cuda.synchronize()
    assert out.dtype == x.dtype
    r = gate(ref, out, mask)
    print(name, r)
    assert r.passed, r


@pytest.mark.parametrize("batch", [4, 1])
def test_c2_per_rank_shapes_vs_oracle(batch):
    """C2's batch sharded over 2 and 8 GPUs (distributed_forward / MultiDeviceTransformer
    give each GPU an LPT share of the sequences): fewer rows change the tile choices (at 2 GPUs ffn_out runs CTA-pair 256 x 128 tiles and
    out_proj 64-wide ones, so the two LayerNorms read different statistics partial
    counts; at 8 GPUs both run 64-wide tiles)."""
    B, S, D, H, F, L, causal, dtype, lengths = CONFIGS["C2"]
    cfg = tb.TransformerConfig(batch, S, D, H, F, L, causal)
    model = tb.make_parameter_model(cfg, 0, dtype, DEV)
    x, mask = tb.generate_inputs(cfg, 1, dtype, lengths, DEV)
    opt = tb.make_optimized_transformer(model)
    with torch.inference_mode():
        out = opt(x, mask)
        again = opt(x, mask)
        ref = forward_fp32(state_dict_fp32(model, DEV), cfg, x.float(), mask)
    torch.cuda.synchronize()
    assert torch.equal(out, again)
    r = gate(ref, out, mask)
    print("C2 batch", batch, r)
    assert r.passed, r
    assert opt.device_status() == 0


def test_organizer_slot_pattern():
    """The organizer harness's slot (UserOptimizedTransformer.forward building the B200
    module from itself on its first call and keeping it outside the module's
    submodules; the reference's class itself is
    exercised on the CPU by tests/test_reference_classes.py): the output matches the
    oracle, a second call reuses the module, and the model's state_dict still works."""
    cfg = tb.TransformerConfig(4, 200, 256, 4, 512, 2, True)

    class Slot(tb.TransformerParameters):
        def forward(self, x, valid_token_mask=None):
            if "_b200" not in self.__dict__:
                self.__dict__["_b200"] = tb.make_optimized_transformer(self)
            return self._b200(x, valid_token_mask)

    torch.manual_seed(3)
    model = Slot(cfg).to(device=DEV, dtype=torch.float16).eval()
    x, mask = tb.generate_inputs(cfg, 4, torch.float16, (50, 200), DEV)
    with torch.inference_mode():
        out = model(x, mask)
        again = model(x, mask)
        ref = forward_fp32(state_dict_fp32(model, DEV), cfg, x.float(), mask)
    torch.cuda.synchronize()
    assert torch.equal(out, again)
    r = gate(ref, out, mask)
    assert r.passed, r
    assert set(model.state_dict()) == set(tb.TransformerParameters(cfg).state_dict())


def test_c3_padding_075_vs_oracle():
    """C3's shape with lengths in [128, 512] (padding ratio 0.75, the third ratio of the
    reference's gate, profiling/validate_fused_gate.py:17-20)."""
    B, S, D, H, F, L, causal, dtype, _ = CONFIGS["C3"]
    cfg = tb.TransformerConfig(B, S, D, H, F, L, causal)
    model = tb.make_parameter_model(cfg, 0, dtype, DEV)
    x, mask = tb.generate_inputs(cfg, 31, dtype, (128, 512), DEV)
    opt = tb.make_optimized_transformer(model)
    with torch.inference_mode():
        out = opt(x, mask)
        ref = forward_fp32(state_dict_fp32(model, DEV), cfg, x.float(), mask)
    torch.cuda.synchronize()
    r = gate(ref, out, mask)
    print("C3 padding 0.75", r)
    assert r.passed, r


def test_c4_long_sequence_vs_oracle():
    cfg, model, x, mask = _case("C4")
    opt = tb.make_optimized_transformer(model)
    with torch.inference_mode():
        out = opt(x, mask)
        ref = forward_fp32_per_sequence(state_dict_fp32(model, DEV), cfg, x.float(), mask)
    torch.cuda.synchronize()
    r = gate(ref, out, mask)
    print("C4", r)
    assert r.passed, r


def test_repeat_is_bit_identical_and_mask_none_equals_all_valid():
    cfg, model, x, _ = _case("C2")
    opt = tb.make_optimized_transformer(model)
    with torch.inference_mode():
        a = opt(x, None)
        b = opt(x, None)
        c = opt(x, torch.ones(x.shape[:2], dtype=torch.bool, device=DEV))
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert torch.equal(a, c)


def test_sequences_are_independent():
    """Changing one sequence's tokens leaves every other sequence's output unchanged
    (padding and packing never leak across sequences)."""
    cfg, model, x, mask = _case("C3")
    opt = tb.make_optimized_transformer(model)
    x2 = x.clone()
    x2[5] = torch.randn_like(x2[5].float()).half() * 10
    with torch.inference_mode():
        a = opt(x, mask)
        b = opt(x2, mask)
    torch.cuda.synchronize()
    keep = torch.ones(cfg.batch_size, dtype=torch.bool)
    keep[5] = False
    assert torch.equal(a[keep.to(DEV)], b[keep.to(DEV)])
    assert not torch.equal(a[5], b[5])


def test_other_batch_shapes_and_no_device_error():
    """A sub-batch gives the same rows.  Across batch shapes the GEMM tile width may
    differ, which regroups the LayerNorm statistics' partial sums, so rows agree to
    fp32 rounding rather than bit for bit (same-shape repeats are bit-identical)."""
    cfg, model, x, mask = _case("C3")
    opt = tb.make_optimized_transformer(model)
    with torch.inference_mode():
        full = opt(x, mask)
        part = opt(x[3:9].contiguous(), mask[3:9].contiguous())
        again = opt(x[3:9].contiguous(), mask[3:9].contiguous())
    torch.cuda.synchronize()
    assert torch.equal(part, again)
    # fp16 output: allow about two ulps of the value (an ulp is 2^-10 of |y| at most).
    ref = full[3:9].float()
    assert bool(((ref - part.float()).abs() <= 2e-3 + 2e-3 * ref.abs()).all())
    assert opt.device_status() == 0


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_multi_device_matches_single_device():
    cfg, model, x, mask = _case("C3")
    single = tb.make_optimized_transformer(model)
    with torch.inference_mode():
        ref = single(x, mask)
        multi = tb.MultiDeviceTransformer(model, [0, 1])
        out = multi(x, mask)
    torch.cuda.synchronize()
    # Each device runs a sub-batch, whose GEMM tile width (hence the grouping of the
    # LayerNorm statistics) may differ from the full batch's: rows agree to about two
    # fp16 ulps, and padded rows stay exactly zero.
    r = ref.float()
    assert bool(((out.float() - r).abs() <= 2e-3 + 2e-3 * r.abs()).all())
    assert bool((out[~mask] == 0).all())
