"""GPU: the reference's 14 benchmark cases (optimized_transformer.py:22-42) through
make_optimized_transformer, against the fp32 oracle, at the padding ratios of the
reference's regression harness (benchmarks/regression.py:56-60: 0.0 and 0.25) and
of its fused-path gate (profiling/validate_fused_gate.py:17-20: 0.75 as well).

Case 14 runs one 100k-token sequence, as the reference's harness does
(benchmarks/regression.py:86-97), with the oracle's attention chunked over queries
(benchmarks/benchmark_step_8.py:33-87)."""
import pytest
import torch

import tttj_2026_b200 as tb
from helpers import gate
from oracle import forward_fp32, state_dict_fp32
from tttj_2026_b200 import cases

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
SEED = 1234


@pytest.fixture(autouse=True, scope="module")
def _no_tf32():
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32 = prev


def _run(n: int, padding: float, batch=None, query_chunk: int = 4096):
    cfg = cases.case_config(n, batch)
    model = tb.make_parameter_model(cfg, SEED, torch.float16, DEV)
    if batch is None:
        assert cases.case_number_for_model(model) == n
    x, mask = cases.case_inputs(cfg, SEED + 100_000 * n + round(100 * padding), padding,
                                torch.float16, DEV)
    opt = tb.make_optimized_transformer(model)
    with torch.inference_mode():
        out = opt(x, mask)
        again = opt(x, mask)
        ref = forward_fp32(state_dict_fp32(model, DEV), cfg, x.float(), mask, query_chunk)
    torch.cuda.synchronize()
    assert out.dtype == torch.float16 and out.shape == x.shape
    assert torch.equal(out, again)
    r = gate(ref, out, mask)
    print(f"case {n} padding {padding}", r)
    assert r.passed, r
    assert opt.device_status() == 0


@pytest.mark.parametrize("padding", [0.0, 0.25, 0.75])
@pytest.mark.parametrize("n", list(range(1, 14)))
def test_reference_case(n, padding):
    """Padding 0.75 is the third ratio of the reference's fused-path gate
    (profiling/validate_fused_gate.py:17-20)."""
    _run(n, padding)


@pytest.mark.parametrize("padding", [0.0, 0.25])
def test_reference_case_14_one_sequence(padding):
    _run(14, padding, batch=1, query_chunk=512)
