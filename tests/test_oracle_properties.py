"""CPU: size-independent properties of the fp32 oracle on random small shapes -- the
semantics the CUDA path is held to (benchmarks/torch_transformer_benchmark.py:97-172):
masked rows exactly zero, sequences independent of one another, causal outputs
independent of later tokens, padded tokens without influence on valid ones, and
mask=None equal to an all-valid mask."""
import torch
from hypothesis import given, settings
from hypothesis import strategies as st

import tttj_2026_b200 as tb
from oracle import forward_fp32, state_dict_fp32

shapes = st.tuples(
    st.integers(1, 3),                 # batch
    st.integers(1, 12),                # sequence length
    st.sampled_from([(32, 2), (32, 4), (64, 2), (64, 8)]),  # (d_model, heads)
    st.sampled_from([32, 96]),         # ffn_dim
    st.integers(1, 2),                 # layers
    st.booleans(),                     # causal
    st.integers(0, 2**31 - 1),         # seed
)


def _setup(shape):
    B, S, (D, H), F, L, causal, seed = shape
    cfg = tb.TransformerConfig(B, S, D, H, F, L, causal)
    torch.manual_seed(seed)
    params = state_dict_fp32(tb.TransformerParameters(cfg))
    g = torch.Generator().manual_seed(seed + 1)
    x = torch.randn(B, S, D, generator=g)
    lens = torch.randint(0, S + 1, (B,), generator=g)
    mask = torch.arange(S)[None, :] < lens[:, None]
    return cfg, params, x, mask, g


@settings(max_examples=25, deadline=None)
@given(shapes)
def test_masked_rows_are_exactly_zero(shape):
    cfg, p, x, mask, _ = _setup(shape)
    with torch.inference_mode():
        y = forward_fp32(p, cfg, x, mask)
    assert bool((y[~mask] == 0).all())
    assert bool(torch.isfinite(y).all())


@settings(max_examples=25, deadline=None)
@given(shapes)
def test_padded_tokens_do_not_influence_valid_ones(shape):
    cfg, p, x, mask, g = _setup(shape)
    noise = torch.randn(x.shape, generator=g) * 100
    x2 = torch.where(mask[..., None], x, noise)
    with torch.inference_mode():
        a = forward_fp32(p, cfg, x, mask)
        b = forward_fp32(p, cfg, x2, mask)
    assert torch.equal(a[mask], b[mask])


@settings(max_examples=25, deadline=None)
@given(shapes)
def test_sequences_are_independent(shape):
    cfg, p, x, mask, _ = _setup(shape)
    with torch.inference_mode():
        full = forward_fp32(p, cfg, x, mask)
        for b in range(cfg.batch_size):
            one = tb.TransformerConfig(1, cfg.seq_len, cfg.d_model, cfg.num_heads, cfg.ffn_dim,
                                       cfg.num_layers, cfg.causal)
            yb = forward_fp32(p, one, x[b:b + 1], mask[b:b + 1])
            assert torch.allclose(yb[0], full[b], rtol=1e-5, atol=1e-5)


@settings(max_examples=25, deadline=None)
@given(shapes)
def test_causal_outputs_ignore_later_tokens(shape):
    cfg, p, x, mask, g = _setup(shape)
    if not cfg.causal or cfg.seq_len < 2:
        return
    t = cfg.seq_len // 2
    x2 = x.clone()
    x2[:, t:] = torch.randn(x2[:, t:].shape, generator=g)
    with torch.inference_mode():
        a = forward_fp32(p, cfg, x, None)
        b = forward_fp32(p, cfg, x2, None)
    assert torch.allclose(a[:, :t], b[:, :t], rtol=1e-5, atol=1e-5)


@settings(max_examples=15, deadline=None)
@given(shapes)
def test_mask_none_equals_all_valid(shape):
    cfg, p, x, _, _ = _setup(shape)
    ones = torch.ones(x.shape[:2], dtype=torch.bool)
    with torch.inference_mode():
        a = forward_fp32(p, cfg, x, None)
        b = forward_fp32(p, cfg, x, ones)
    assert torch.equal(a, b)
