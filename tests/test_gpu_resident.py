"""GPU: the resident-stack kernel (one launch for the whole forward of sequences of
<= 128 tokens) against the fp32 oracle and against the layer-by-layer kernels, on
BASELINE config C1 and the reference's resident cases (kernels/sequence_resident.py,
optimized_transformer.py:22-42), with ragged, non-prefix and empty masks."""
import pytest
import torch

import tttj_2026_b200 as tb
from helpers import gate
from oracle import forward_fp32, state_dict_fp32

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


@pytest.fixture(autouse=True, scope="module")
def _no_tf32():
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32 = prev


# name: (B, S, D, H, F, L, causal, dtype, mask kind)
SHAPES = {
    "C1": (2, 128, 256, 4, 1024, 2, False, torch.float32, "prefix"),
    "case1": (64, 128, 128, 4, 128, 4, True, torch.float16, None),
    "case2": (1, 128, 128, 4, 128, 4, True, torch.float16, "prefix"),
    "case7_hd8_d32": (64, 128, 32, 4, 32, 4, True, torch.float16, "prefix"),
    "case9_hd128": (64, 128, 128, 1, 128, 4, True, torch.float16, "prefix"),
    "case10_hd64": (64, 128, 128, 2, 128, 4, True, torch.float16, None),
    "case11_hd8_h16": (8, 128, 128, 16, 128, 4, True, torch.float16, "prefix"),
    "case12_s32": (64, 32, 128, 4, 128, 4, True, torch.float16, "prefix"),
    "holes_f192": (6, 100, 128, 2, 192, 2, False, torch.float16, "holes"),
    "empty_seq": (3, 64, 64, 2, 160, 2, True, torch.float16, "empty"),
    # odd head count: one head per attention step (even counts of 32-wide heads pair up)
    "odd_heads_d96": (4, 100, 96, 3, 96, 2, True, torch.float16, "prefix"),
}


def _inputs(name, cfg, dtype):
    B, S = cfg.batch_size, cfg.seq_len
    kind = SHAPES[name][-1]
    g = torch.Generator().manual_seed(len(name) * 7919 + B)
    x = torch.randn(B, S, cfg.d_model, generator=g)
    if kind is None:
        mask = None
    elif kind == "prefix":
        lens = torch.randint(max(1, S // 2), S + 1, (B,), generator=g)
        mask = torch.arange(S)[None, :] < lens[:, None]
    elif kind == "holes":
        mask = torch.rand(B, S, generator=g) > 0.35
    else:  # one sequence without any valid token, one full, one short
        mask = torch.zeros(B, S, dtype=torch.bool)
        mask[1] = True
        mask[2, :5] = True
    if mask is not None:
        x = x.masked_fill(~mask[..., None], 0)
        mask = mask.to(DEV)
    return x.to(dtype=dtype, device=DEV), mask


@pytest.mark.parametrize("name", sorted(SHAPES))
def test_resident_matches_oracle_and_layerwise(name):
    B, S, D, H, F, L, causal, dtype, _ = SHAPES[name]
    cfg = tb.TransformerConfig(B, S, D, H, F, L, causal)
    model = tb.make_parameter_model(cfg, 3, dtype, DEV)
    x, mask = _inputs(name, cfg, dtype)
    opt = tb.make_optimized_transformer(model)
    opt.set_path("resident")
    assert opt.uses_resident(B, S), name
    assert opt.launches_per_forward(B, S) == 1
    with torch.inference_mode():
        res = opt(x, mask)
        res2 = opt(x, mask)
        opt.set_path("layerwise")
        assert not opt.uses_resident(B, S)
        lw = opt(x, mask)
        opt.set_path("auto")
        ref = forward_fp32(state_dict_fp32(model, DEV), cfg, x.float(), mask)
    torch.cuda.synchronize()
    assert res.dtype == x.dtype and res.shape == x.shape
    assert torch.equal(res, res2)
    r = gate(ref, res, mask)
    print(name, "resident", r)
    assert r.passed, r
    # Both paths approximate the same fp32 result; they differ in accumulation order.
    assert float((res.float() - lw.float()).abs().max()) <= 1e-2
    assert opt.device_status() == 0


def test_long_sequences_keep_the_layerwise_path():
    cfg = tb.TransformerConfig(2, 129, 128, 4, 128, 1, True)
    model = tb.make_parameter_model(cfg, 0, torch.float16, DEV)
    opt = tb.make_optimized_transformer(model)
    assert not opt.uses_resident(2, 129)
    assert opt.launches_per_forward(2, 129) == 5 * 1 + 3
    with pytest.raises(ValueError, match="does not fit"):
        opt.set_path("resident")
    assert not opt.uses_resident(2, 129)  # the failed switch changed nothing


def test_auto_path_choice():
    """Auto takes the resident kernel for the reference's small cases and keeps the
    layer-by-layer kernels where those measured faster (C1: 1.6 MB of weights per layer)."""
    def auto(B, S, D, H, F, L, causal):
        cfg = tb.TransformerConfig(B, S, D, H, F, L, causal)
        opt = tb.make_optimized_transformer(tb.make_parameter_model(cfg, 0, torch.float16, DEV))
        return opt.uses_resident(B, S)

    assert auto(64, 128, 128, 4, 128, 4, True)        # case 1
    assert auto(64, 128, 128, 1, 128, 4, True)        # case 9
    assert auto(64, 128, 128, 16, 128, 4, True)       # case 11 (8 head pairs)
    assert not auto(2, 128, 256, 4, 1024, 2, False)   # C1
