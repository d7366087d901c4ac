"""CPU: bench.py's host-side accounting -- the algorithmic work per forward and per
kernel launch that roofline fractions divide by, the DRAM traffic lookup in the
committed ncu summaries, and the workload labels.  No GPU is touched."""
import importlib.util
from pathlib import Path

import pytest
import torch

import tttj_2026_b200 as tb

REPO = Path(__file__).resolve().parent.parent


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", REPO / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _cfg(bench, name):
    B, S, D, H, F, L, causal, _, _ = bench.CONFIGS[name]
    return tb.TransformerConfig(B, S, D, H, F, L, causal)


def test_c2_forward_flops_match_the_formula(bench):
    """C2 (mask=None): 2 T (4 D^2 + 2 D F) L GEMM FLOPs plus 4 hd H P L attention FLOPs
    with P = B S (S + 1) / 2 causal pairs -- 240.6 GFLOP per forward."""
    cfg = _cfg(bench, "C2")
    Tv, pairs, per_launch, flops = bench.useful_work(cfg, None, 2)
    assert Tv == 8 * 1024
    assert pairs == 8 * 1024 * 1025 // 2
    assert flops == pytest.approx(240.6e9, rel=1e-3)
    launches = (per_launch["gemm_qkv"][1] + per_launch["gemm_out_proj"][1]
                + per_launch["gemm_ffn_in_gelu"][1] + per_launch["gemm_ffn_out"][1]
                + per_launch["attention"][1])
    assert launches * cfg.num_layers == pytest.approx(flops, rel=1e-12)
    assert per_launch["resident_stack"] == ("tensor", flops)


def test_masked_work_counts_valid_tokens_only(bench):
    cfg = tb.TransformerConfig(3, 16, 64, 2, 128, 1, False)
    mask = torch.zeros(3, 16, dtype=torch.bool)
    mask[0, :5] = True
    mask[2, :16] = True
    Tv, pairs, _, _ = bench.useful_work(cfg, mask, 2)
    assert Tv == 21
    assert pairs == 5 * 5 + 16 * 16  # non-causal: len^2 per sequence


@pytest.mark.parametrize("x_bytes", [2, 4])
def test_layernorm_bytes(bench, x_bytes):
    """Gather: x in, fp32 residual + fp16 copy out; final: fp32 residual in, every
    output row (padded rows too) out in x's dtype."""
    cfg = _cfg(bench, "C2")
    Tv, _, per_launch, _ = bench.useful_work(cfg, None, x_bytes)
    D = cfg.d_model
    assert per_launch["layernorm"] == ("hbm", (x_bytes + 6.0) * Tv * D)
    assert per_launch["final_layernorm_scatter"] == ("hbm", 4.0 * Tv * D + 8 * 1024 * D * x_bytes)


def test_traffic_lookup_reads_the_committed_summaries(bench):
    assert bench._profile_traffic("gemm_ffn_in_gelu", "C2") == 11144960.0
    assert bench._profile_traffic("resident_stack", "R5") == 5126912.0
    assert bench._profile_traffic("gemm_ffn_in_gelu", "C3") is None


def test_workload_labels(bench):
    assert bench.workload_desc("C2").startswith("C2: L4 D512 H8 hd64 F2048 B8 S1024 causal, mask=None")
    assert "reference case 5" in bench.workload_desc("R5")


def _run_bench(args, env_extra=None, timeout=300):
    import json
    import os
    import subprocess
    import sys
    env = dict(os.environ)
    env.update(env_extra or {})
    r = subprocess.run([sys.executable, str(REPO / "bench.py"), *args], cwd=REPO, env=env,
                       capture_output=True, text=True, timeout=timeout)
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    return r.returncode, [json.loads(l) for l in lines], r.stdout


def test_reference_arm_prints_one_contract_line():
    """`bench.py --impl reference` (the CPU arm the driver runs beside ours): one JSON
    line with the metric, a cpu_baseline block and a zero-copy e2e block."""
    rc, lines, _ = _run_bench(["--impl", "reference", "--config", "C1", "--steps", "2",
                               "--warmup", "1"])
    assert rc == 0 and len(lines) == 1
    d = lines[0]
    assert d["impl"] == "reference" and d["metric"] == "forward tokens/sec"
    assert d["unit"] == "tokens/s" and d["higher_is_better"] is True and d["value"] > 0
    assert d["steps"] == 2 and d["warmup"] == 1 and d["n_gpus"] == 1
    assert d["cpu_baseline"]["kind"] == "port" and d["cpu_baseline"]["value"] == d["value"]
    assert d["e2e"] == {"value": d["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}


def test_reference_arm_other_ranks_stay_silent():
    rc, lines, out = _run_bench(["--impl", "reference", "--config", "C1", "--steps", "1",
                                 "--warmup", "0"], {"RANK": "1", "WORLD_SIZE": "2"})
    assert rc == 0 and lines == [] and out.strip() == ""


def test_reference_arm_without_a_bounded_sample_says_unavailable():
    rc, lines, _ = _run_bench(["--impl", "reference", "--config", "R14", "--steps", "1",
                               "--warmup", "0"])
    assert rc == 0 and len(lines) == 1
    assert lines[0]["impl"] == "reference" and "unavailable" in lines[0]
