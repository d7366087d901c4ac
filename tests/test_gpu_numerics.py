"""GPU: numerics and isolation of the forward beyond N(0, 1) inputs.

* Input scale and DC-offset sweeps against the fp32 oracle, on the layer-by-layer path
  and on the resident-stack path: x = s * N(0, 1) + mu.  Rows whose mean is large
  against their spread are where a one-pass sum-of-squares variance, or an fp16 copy of
  the uncentred residual, loses the LayerNorm input; the kernels keep every LayerNorm's
  statistics and its fp16 GEMM operand relative to a per-row pivot instead.  The
  reference validated its fused paths over input scales 1e-4 .. 1000 at padding 0,
  0.25 and 0.75 (llm-scratchpad/h100_ncu_optimization_results.md:107-110,
  profiling/validate_fused_gate.py:17-20); the same matrix runs here.
* Sequence isolation: NaN / Inf in one sequence's tokens leave every other sequence's
  output bit-identical, also when the NaN rows stay behind in the workspace for a
  later call with fewer valid tokens.
* Device errors surface on the next forward without a synchronisation; forwards of one
  shape on two streams; the bounded plan cache.
"""
import pytest
import torch

import tttj_2026_b200 as tb
from helpers import gate
from oracle import forward_fp32, state_dict_fp32
from tttj_2026_b200 import cases

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


@pytest.fixture(autouse=True, scope="module")
def _no_tf32():
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32 = prev


def _inputs(cfg, seed, scale, offset, padding):
    """x = scale * N(0, 1) + offset in fp16 (generated in fp32 on the host, then cast),
    a prefix mask with lengths in [round(S (1 - padding)), S] (or None at padding 0),
    padded rows zero (the reference generator's convention,
    benchmarks/torch_transformer_benchmark.py:234-272)."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(cfg.batch_size, cfg.seq_len, cfg.d_model, generator=g) * scale + offset
    mask = None
    if padding > 0:
        lo = max(1, round(cfg.seq_len * (1.0 - padding)))
        lens = torch.randint(lo, cfg.seq_len + 1, (cfg.batch_size,), generator=g)
        mask = torch.arange(cfg.seq_len)[None, :] < lens[:, None]
        x = x.masked_fill(~mask[..., None], 0)
        mask = mask.to(DEV)
    return x.half().to(DEV), mask


# Layer by layer: hd 64, causal, S not a multiple of 128 (partial tiles everywhere).
LAYERWISE_CFG = tb.TransformerConfig(4, 320, 256, 4, 1024, 2, True)
# Resident stack: the reference's case-1 layer shape (D = F = 128, 4 heads), 8 sequences.
RESIDENT_CFG = tb.TransformerConfig(8, 128, 128, 4, 128, 4, True)


def _check(cfg, opt, model, x, mask, label):
    with torch.inference_mode():
        out = opt(x, mask)
        again = opt(x, mask)
        ref = forward_fp32(state_dict_fp32(model, DEV), cfg, x.float(), mask)
    torch.cuda.synchronize()
    assert torch.equal(out, again), label
    r = gate(ref, out, mask)
    print(label, r)
    assert r.passed, (label, r)


@pytest.mark.parametrize("path,cfg", [("layerwise", LAYERWISE_CFG), ("resident", RESIDENT_CFG)])
def test_scale_and_offset_sweep(path, cfg):
    model = tb.make_parameter_model(cfg, 11, torch.float16, DEV)
    # Non-trivial LayerNorm affines, so the folded weights and biases are exercised.
    with torch.no_grad():
        g = torch.Generator().manual_seed(5)
        for m in model.modules():
            if isinstance(m, torch.nn.LayerNorm):
                m.weight.copy_((1 + 0.2 * torch.randn(m.weight.shape, generator=g)).half())
                m.bias.copy_((0.1 * torch.randn(m.bias.shape, generator=g)).half())
    opt = tb.make_optimized_transformer(model)
    opt.set_path(path)
    assert opt.uses_resident(cfg.batch_size, cfg.seq_len) == (path == "resident")
    for scale in (1e-3, 1.0, 10.0, 100.0):
        for offset in (0.0, 10.0, 100.0):
            x, mask = _inputs(cfg, 7, scale, offset, 0.25)
            _check(cfg, opt, model, x, mask, f"{path} scale={scale} offset={offset}")
    assert opt.device_status() == 0


@pytest.mark.parametrize("padding", [0.0, 0.25, 0.75])
@pytest.mark.parametrize("n", [1, 13])
def test_reference_scale_matrix(n, padding):
    """The reference's validation matrix: input scales 1e-4 .. 1000 at padding 0, 0.25
    and 0.75, on case 1 (resident path) and case 13 (layer by layer, S = 1024)."""
    cfg = cases.case_config(n, 16 if n == 1 else 4)
    model = tb.make_parameter_model(cfg, 1234, torch.float16, DEV)
    opt = tb.make_optimized_transformer(model)
    for scale in (1e-4, 1e-3, 3e-3, 1e-2, 0.1, 1.0, 10.0, 100.0, 1000.0):
        x, mask = _inputs(cfg, 4000 + round(100 * padding), scale, 0.0, padding)
        _check(cfg, opt, model, x, mask, f"case {n} padding={padding} scale={scale}")


def _poison(x, mask, b):
    """Copy of x with NaN and +Inf in two valid tokens of sequence b."""
    y = x.clone()
    n = int(mask[b].sum()) if mask is not None else x.shape[1]
    y[b, n // 2, 3] = float("nan")
    y[b, n - 1, :7] = float("inf")
    return y


@pytest.mark.parametrize("label,cfg,lengths", [
    ("C3-like hd32 non-causal", tb.TransformerConfig(12, 512, 256, 8, 1024, 2, False), (32, 512)),
    ("hd64 causal", tb.TransformerConfig(6, 700, 256, 4, 512, 2, True), (100, 700)),
    ("hd128", tb.TransformerConfig(5, 300, 256, 2, 512, 1, False), (60, 300)),
    ("resident", RESIDENT_CFG, (40, 128)),
])
def test_non_finite_sequence_does_not_leak(label, cfg, lengths):
    model = tb.make_parameter_model(cfg, 3, torch.float16, DEV)
    x, mask = tb.generate_inputs(cfg, 4, torch.float16, lengths, DEV)
    opt = tb.make_optimized_transformer(model)
    for b in (0, cfg.batch_size // 2, cfg.batch_size - 1):
        bad = _poison(x, mask, b)
        with torch.inference_mode():
            clean = opt(x, mask)
            dirty = opt(bad, mask)
        torch.cuda.synchronize()
        keep = torch.ones(cfg.batch_size, dtype=torch.bool, device=DEV)
        keep[b] = False
        assert torch.equal(clean[keep], dirty[keep]), (label, b)
        assert not bool(torch.isfinite(dirty[b][mask[b]]).all()), (label, b)
        assert bool((dirty[~mask] == 0).all()), (label, b)
    assert opt.device_status() == 0


def test_stale_non_finite_rows_do_not_reach_a_later_call():
    """A forward with NaN tokens leaves NaN rows in the workspace just past the valid
    tokens of a later forward with shorter sequences (packed rows 880.. here, inside the
    key tile that holds the later call's last sequence end); the later forward equals a
    fresh module's."""
    cfg = tb.TransformerConfig(4, 384, 256, 4, 512, 2, True)
    model = tb.make_parameter_model(cfg, 8, torch.float16, DEV)
    x, _ = tb.generate_inputs(cfg, 9, torch.float16, None, DEV)
    full = torch.ones(cfg.batch_size, cfg.seq_len, dtype=torch.bool, device=DEV)
    short = torch.arange(cfg.seq_len, device=DEV)[None, :] < torch.tensor([300, 250, 200, 130],
                                                                          device=DEV)[:, None]
    x_short = x.masked_fill(~short[..., None], 0)
    used = tb.make_optimized_transformer(model)
    fresh = tb.make_optimized_transformer(model)
    bad = x.clone()
    # With every token valid, packed row b * 384 + s: rows 868..1067 are sequence 2's
    # tokens 100..299.  The later call has 880 valid rows; its sequence 3 (130 tokens,
    # rows 750..879) streams key tile 878..1005.
    bad[2, 100:300, :] = float("nan")
    with torch.inference_mode():
        used(bad, full)
        out = used(x_short, short)
        ref = fresh(x_short, short)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    assert bool(torch.isfinite(out).all())


def test_device_timeout_surfaces_on_next_forward():
    """A bounded device wait that gives up is reported by the next forward of the
    shape (RuntimeError, nothing launched), without a host synchronisation in the
    forward; the forward after that runs normally."""
    cfg = tb.TransformerConfig(2, 256, 256, 4, 512, 2, True)
    model = tb.make_parameter_model(cfg, 1, torch.float16, DEV)
    x, mask = tb.generate_inputs(cfg, 2, torch.float16, (100, 256), DEV)
    opt = tb.make_optimized_transformer(model)
    with torch.inference_mode():
        good = opt(x, mask)
        opt.selftest_device_timeout(cfg.batch_size, cfg.seq_len, limit_ns=2_000_000)
        torch.cuda.synchronize()
        with pytest.raises(RuntimeError, match="timed out"):
            opt(x, mask)
        again = opt(x, mask)
    torch.cuda.synchronize()
    assert torch.equal(good, again)
    assert opt.device_status() == 0


def test_two_streams_share_one_plan():
    """Forwards of one shape enqueued on two streams: the plan orders them (its
    workspace is shared), and every output equals the single-stream result."""
    cfg = tb.TransformerConfig(6, 512, 256, 8, 1024, 2, False)
    model = tb.make_parameter_model(cfg, 5, torch.float16, DEV)
    xs, masks = [], []
    for seed in range(4):
        x, m = tb.generate_inputs(cfg, 20 + seed, torch.float16, (32, 512), DEV)
        xs.append(x)
        masks.append(m)
    opt = tb.make_optimized_transformer(model)
    with torch.inference_mode():
        expected = [opt(x, m) for x, m in zip(xs, masks)]
    torch.cuda.synchronize()
    s1, s2 = torch.cuda.Stream(DEV), torch.cuda.Stream(DEV)
    outs = []
    with torch.inference_mode():
        for rep in range(3):
            for i, (x, m) in enumerate(zip(xs, masks)):
                s = s1 if (i + rep) % 2 == 0 else s2
                s.wait_stream(torch.cuda.current_stream(DEV))
                with torch.cuda.stream(s):
                    outs.append((i, opt(x, m)))
    torch.cuda.synchronize()
    for i, out in outs:
        assert torch.equal(out, expected[i]), i
    assert opt.device_status() == 0


def test_plan_cache_is_bounded():
    cfg = tb.TransformerConfig(4, 256, 256, 4, 512, 2, True)
    model = tb.make_parameter_model(cfg, 6, torch.float16, DEV)
    x, mask = tb.generate_inputs(cfg, 7, torch.float16, (64, 256), DEV)
    opt = tb.make_optimized_transformer(model)
    opt.max_plans = 2
    with torch.inference_mode():
        first = opt(x[:2], mask[:2])
        for b in (3, 4, 1, 2):
            opt(x[:b], mask[:b])
        assert len(opt.cached_shapes()) == 2
        assert opt.cached_shapes()[-1] == (2, 256)
        opt(x[:3], mask[:3])  # evicts (1, 256)
        assert opt.cached_shapes() == [(2, 256), (3, 256)]
        again = opt(x[:2], mask[:2])
    torch.cuda.synchronize()
    assert torch.equal(first, again)
