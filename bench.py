#!/usr/bin/env python3
"""Forward tokens/s of the B200 transformer path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C5] [--impl b200|reference]

A step is one forward of the whole stack (L blocks + final LayerNorm + masking)
over one batch of the chosen BASELINE.json configuration.  The default is C5
(configs[4]: L24 D1024 H16 F4096, batch 256 x seq 256, causal + prefix padding, fp16),
the largest configuration that fits one GPU.  With N > 1 the script runs under
torchrun, one process per GPU, and the configuration's batch is split across the
ranks (strong scaling: the same 256 sequences in total, each rank an LPT share by
predicted cost, tttj_2026_b200.sharding.local_shard); no collective runs on the data
path and the reported time is the max over ranks.

--impl b200 (default): the CUDA path through make_optimized_transformer.
  value      tokens/s of the whole batch, each rank's shard resident in its HBM,
             L2 flushed between steps
  e2e        the same through the public module call with pinned host buffers:
             H2D of each rank's x and mask + forward + D2H of its output every step,
             run as a serving loop runs it (the next step's H2D and the previous
             step's D2H on a copy stream, overlapping the current forward; the L2
             flush between forwards stays inside the timed span)
  gather_to_rank0  (N > 1) distributed_forward with the whole batch on every rank:
             shard select + forward + NCCL gather of the outputs to rank 0
  roofline   the dominant kernel class, timed with CUDA events inside real forwards
  cpu_baseline  the fp32 oracle (op-for-op restatement of the reference module's
             PyTorch eager forward) on the host cores, bounded sample (rank 0, N=1)
--impl reference: the reference's CPU path (the fp32 oracle port, all host threads)
  on a bounded sample of the same workload; rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from datetime import timedelta
from pathlib import Path

REPO = Path(__file__).resolve().parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

# (B, S, D, H, F, L, causal, dtype name, prefix-length range or None)
CONFIGS = {
    "C1": (2, 128, 256, 4, 1024, 2, False, "float32", (64, 128)),
    "C2": (8, 1024, 512, 8, 2048, 4, True, "float16", None),
    "C3": (32, 512, 256, 8, 1024, 6, False, "float16", (32, 512)),
    "C4": (4, 8192, 768, 12, 3072, 12, True, "float16", (4096, 8192)),
    "C5": (256, 256, 1024, 16, 4096, 24, True, "float16", (128, 256)),
}
# Bounded CPU sample per config: (sequences, layers) of the workload per step.
CPU_SAMPLE = {"C1": (2, 2), "C2": (1, 4), "C3": (4, 6), "C4": (1, 1), "C5": (1, 24)}

# The reference's own 14 cases (optimized_transformer.py:22-42: F = D, causal, 4 layers,
# 2 for case 14) as workloads R1..R14, all tokens valid and fp16 as in the reference's
# published timings (benchmarks/benchmark_compile_comparison.py:146-160), with those
# published H200 forward times (README.md:164-177) for vs_baseline.
REF_CASES = {
    1: (64, 128, 128, 4), 2: (1, 128, 128, 4), 3: (4, 128, 128, 4), 4: (16, 128, 128, 4),
    5: (128, 128, 128, 4), 6: (10000, 128, 128, 4), 7: (64, 128, 32, 4), 8: (64, 128, 1024, 4),
    9: (64, 128, 128, 1), 10: (64, 128, 128, 2), 11: (64, 128, 128, 16), 12: (64, 32, 128, 4),
    13: (64, 1024, 128, 4), 14: (32, 100000, 1024, 16),
}
PUBLISHED_H200_MS = {
    1: 0.169280, 2: 0.114272, 3: 0.109408, 4: 0.109664, 5: 0.262880, 6: 12.374400,
    7: 0.095456, 8: 1.065472, 9: 0.158224, 10: 0.155680, 11: 0.220128, 12: 0.104352,
    13: 4.443712, 14: 2927.799072,
}
for _n, (_b, _s, _d, _h) in REF_CASES.items():
    CONFIGS[f"R{_n}"] = (_b, _s, _d, _h, _d, 2 if _n == 14 else 4, True, "float16", (_s, _s))
    # One sequence, one layer per CPU rep; a 100k-token sequence is out of reach.
    CPU_SAMPLE[f"R{_n}"] = None if _n == 14 else (1, 1)
METRIC = "forward tokens/sec"
UNIT = "tokens/s"
L2_FLUSH_BYTES = 256 << 20  # > 126 MB L2


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description="B200 transformer forward benchmark")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="C5", choices=list(CONFIGS))
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--path", default="auto", choices=["auto", "layerwise", "resident"],
                    help="auto: the library picks (the resident whole-stack kernel for short "
                         "sequences of small layers); layerwise / resident: force one path")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="CPU baseline time budget")
    ap.add_argument("--cp", type=int, default=1,
                    help="context parallelism: groups of CP ranks each split one sequence at a "
                         "time (tttj_2026_b200.context_parallel); for batches smaller than the "
                         "GPU count, e.g. --config C4 --gpus 8 --cp 2")
    return ap.parse_args(argv)


def workload_desc(name: str) -> str:
    B, S, D, H, F, L, causal, dt, lens = CONFIGS[name]
    if lens is None:
        mask = "mask=None"
    elif lens[0] == lens[1] == S:
        mask = "all-valid mask"
    else:
        mask = f"prefix mask len~U[{lens[0]},{lens[1]}]"
    case = f" (reference case {name[1:]})" if name.startswith("R") else ""
    return (f"{name}{case}: L{L} D{D} H{H} hd{D // H} F{F} B{B} S{S} "
            f"{'causal' if causal else 'non-causal'}, {mask}, {dt}")


def make_case(name: str, seed: int, device):
    """Weights and the whole batch of inputs (the same seeds on every rank)."""
    import torch

    import optimized_transformer  # noqa: F401
    import tttj_2026_b200 as tb

    B, S, D, H, F, L, causal, dt, lens = CONFIGS[name]
    dtype = getattr(torch, dt)
    cfg = tb.TransformerConfig(B, S, D, H, F, L, causal)
    model = tb.make_parameter_model(cfg, seed, dtype, device)
    x, mask = tb.generate_inputs(cfg, seed + 1, dtype, lens, device)
    return cfg, model, x, mask


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def useful_work(cfg, mask, x_bytes: int = 2):
    """Valid tokens, attention pairs and per-class FLOPs / bytes of one forward."""
    import torch

    B, S = cfg.batch_size, cfg.seq_len
    if mask is None:
        lengths = [S] * B
    else:
        lengths = mask.sum(1).tolist()
    Tv = sum(lengths)
    if cfg.causal:
        pairs = sum(l * (l + 1) // 2 for l in lengths)
    else:
        pairs = sum(l * l for l in lengths)
    D, F, H = cfg.d_model, cfg.ffn_dim, cfg.num_heads
    hd = D // H
    per_launch = {
        "gemm_qkv": ("tensor", 2.0 * Tv * 3 * D * D),
        "gemm_out_proj": ("tensor", 2.0 * Tv * D * D),
        "gemm_ffn_in_gelu": ("tensor", 2.0 * Tv * F * D),
        "gemm_ffn_out": ("tensor", 2.0 * Tv * D * F),
        "attention": ("tensor", 4.0 * hd * H * pairs),
        # bytes.  Gather: x row in (x's dtype), fp32 residual row + its fp16 copy out.
        # Final: fp32 residual row in, every [B, S] output row out (zeros included).
        "layernorm": ("hbm", (x_bytes + 4.0 + 2.0) * Tv * D),
        "final_layernorm_scatter": ("hbm", 4.0 * Tv * D + B * S * D * x_bytes),
        "plan_tokens": ("hbm", float(B * S)),
    }
    flops = (2.0 * Tv * (4 * D * D + 2 * D * F) + 4.0 * hd * H * pairs) * cfg.num_layers
    # The resident path runs the whole stack (every layer) in one launch.
    per_launch["resident_stack"] = ("tensor", flops)
    return Tv, pairs, per_launch, flops


def load_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "tflops": float(d["bf16_tflops"]),
                "tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "tflops": 1590.0, "tflops_sustained": 1400.0, "source": "fallback"}


# Steps at least this long keep the GPU at its power limit for the whole timed region
# (sw_power_cap, SM clock near 1.4 GHz on a 1 kW B200): their tensor kernels are
# compared with the sustained GEMM peak, shorter steps with the burst peak.
LONG_STEP_MS = 5.0


class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling while GPU work runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        import torch

        self.proc = None
        self.path = None
        self.out = None
        try:
            props = torch.cuda.get_device_properties(device_index)
            self.bus = f"{props.pci_domain_id:08X}:{props.pci_bus_id:02X}:{props.pci_device_id:02X}.0"
        except Exception:
            self.bus = None

    def start(self):
        self.out = None
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            cmd = ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "50"]
            if self.bus:
                cmd += ["-i", self.bus]
            self.out = open(self.path, "w")
            self.proc = subprocess.Popen(cmd, stdout=self.out, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
            self._cleanup()
        return self

    def _cleanup(self):
        if self.out is not None:
            self.out.close()
            self.out = None
        if self.path is not None:
            try:
                os.unlink(self.path)
            except OSError:
                pass

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
            self.proc.wait()
        self.out.close()
        self.out = None
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        self._cleanup()
        if not rows:
            return None
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, r in rows for i, v in enumerate(r) if v.lower() == "active"})
        busy = [sm for sm, _, _ in rows]
        return {"sm_mhz": statistics.median(busy), "sm_max_mhz": max(m for _, m, _ in rows),
                "reasons": reasons, "samples": len(rows)}


def cpu_oracle_rate(name: str, seed: int, seconds: float, threads: int):
    """Time the fp32 oracle (the reference module's math in PyTorch eager fp32) on
    the host cores over a bounded sample of the workload.  Returns tokens/s scaled
    to the full stack, plus a description."""
    import torch

    import optimized_transformer  # noqa: F401
    import tttj_2026_b200 as tb
    from oracle import forward_fp32, state_dict_fp32

    torch.set_num_threads(threads)
    B, S, D, H, F, L, causal, dt, lens = CONFIGS[name]
    if CPU_SAMPLE[name] is None:
        return None, "no bounded CPU sample for this workload", None
    n_seq, n_layers = CPU_SAMPLE[name]
    full = tb.TransformerConfig(B, S, D, H, F, L, causal)
    torch.manual_seed(seed)
    params = tb.TransformerParameters(full).to(getattr(torch, dt))
    p = state_dict_fp32(params, "cpu")
    cfg = tb.TransformerConfig(n_seq, S, D, H, F, n_layers, causal)
    x, mask = tb.generate_inputs(full, seed + 1, getattr(torch, dt), lens, "cpu")
    x = x[:n_seq].float()
    mask = None if mask is None else mask[:n_seq]
    with torch.inference_mode():
        forward_fp32(p, cfg, x, mask)  # warm-up
        reps, t0 = 0, time.perf_counter()
        while True:
            forward_fp32(p, cfg, x, mask)
            reps += 1
            el = time.perf_counter() - t0
            if el >= seconds or reps >= 1000:
                break
    per_step_full = el / reps * (L / n_layers)  # seconds for n_seq sequences, all layers
    value = n_seq * S / per_step_full
    sample = (f"{n_seq} of {B} sequences x {n_layers} of {L} layers per rep, {reps} reps in {el:.1f} s; "
              f"time scaled x{L / n_layers:g} to the full stack")
    return value, sample, el / reps


def run_reference(args, rank: int, world: int):
    if rank != 0:
        return 0
    import torch

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    name = args.config
    B, S, D, H, F, L, causal, dt, lens = CONFIGS[name]
    if CPU_SAMPLE[name] is None:
        print(json.dumps({"impl": "reference", "unavailable":
                          f"{name}: one CPU forward of a {S}-token sequence exceeds the bench's time bound"}),
              flush=True)
        return 0
    n_seq, n_layers = CPU_SAMPLE[name]

    import optimized_transformer  # noqa: F401
    import tttj_2026_b200 as tb
    from oracle import forward_fp32, state_dict_fp32

    full = tb.TransformerConfig(B, S, D, H, F, L, causal)
    torch.manual_seed(args.seed)
    params = tb.TransformerParameters(full).to(getattr(torch, dt))
    p = state_dict_fp32(params, "cpu")
    cfg = tb.TransformerConfig(n_seq, S, D, H, F, n_layers, causal)
    x, mask = tb.generate_inputs(full, args.seed + 1, getattr(torch, dt), lens, "cpu")
    x = x[:n_seq].float()
    mask = None if mask is None else mask[:n_seq]
    times = []
    with torch.inference_mode():
        for i in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            forward_fp32(p, cfg, x, mask)
            if i >= args.warmup:
                times.append(time.perf_counter() - t0)
    scale = L / n_layers
    step_s = statistics.fmean(times) * scale
    value = n_seq * S / step_s
    sample = f"{n_seq} of {B} sequences x {n_layers} of {L} layers per step, time scaled x{scale:g}"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": step_s * 1e3,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic",
        "config": {"workload": workload_desc(name), "global_batch": B, "seq_len": S,
                   "parallelism": "cpu"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "cpu_model": cpu_model(), "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_cp(args, rank: int, world: int, local_rank: int):
    """--cp K: the ranks form world / K groups of K; each group takes its LPT share of the
    batch's sequences and runs them one after another, each split across the group's
    ranks (ContextParallelTransformer: token-sliced GEMMs, one q|k|v all-gather per
    layer).  value = B * S * steps / max-over-ranks time; e2e adds, per sequence, the
    H2D of its input and the D2H of the rank's output rows."""
    import torch
    import torch.distributed as dist

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    import optimized_transformer  # noqa: F401
    import tttj_2026_b200 as tb
    from tttj_2026_b200 import sharding
    from tttj_2026_b200.context_parallel import ContextParallelTransformer

    name, K = args.config, args.cp
    if world % K:
        raise SystemExit(f"--cp {K} must divide the number of ranks ({world})")
    B, S = CONFIGS[name][0], CONFIGS[name][1]
    cfg, model, x_full, mask_full = make_case(name, args.seed, dev)
    groups = [dist.new_group(list(range(g * K, (g + 1) * K))) for g in range(world // K)]
    gi = rank // K
    lengths = sharding.lengths_of(mask_full, B, S)
    mine = sharding.local_shard(lengths, cfg, gi, world // K)  # this group's sequences
    # Each sequence's split forward is captured once into a CUDA graph and replayed; its
    # valid length is known on the host (no read-back of the mask per call).
    cp = ContextParallelTransformer(model, groups[gi], graphs=True)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    seqs = [(x_full[b:b + 1].contiguous(),
             None if mask_full is None else mask_full[b:b + 1].contiguous()) for b in mine]
    lens = [int(lengths[b]) for b in mine]

    def step():
        for (xs, ms), n in zip(seqs, lens):
            cp(xs, ms, gather=False, length=n)

    def max_over_ranks(v: float) -> float:
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    clocks = ClockSampler(local_rank).start()
    with torch.inference_mode():
        for _ in range(args.warmup):
            step()
            flush.zero_()
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
              for _ in range(args.steps)]
        dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize(dev)
        for a, b in ev:
            a.record(stream)
            step()
            b.record(stream)
            flush.zero_()
        torch.cuda.synchronize(dev)
        dist.barrier(device_ids=[local_rank])
        total_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in ev))
        # e2e: each rank copies its own rows of every sequence in from pinned host memory
        # and its output rows out to pinned host memory (the valid lengths are known on
        # the host, so the mask itself is not needed).
        dev_x, host_x, host_out, spans = [], [], [], []
        for (xs, _), n in zip(seqs, lens):
            lo, hi = cp.shares(n)[cp.rank]
            spans.append((lo, hi))
            dev_x.append(torch.zeros_like(xs))
            host_x.append(xs[0, lo:hi].cpu().pin_memory())
            host_out.append(torch.empty((hi - lo, xs.shape[2]), dtype=xs.dtype).pin_memory())
        h2d = sum(h.numel() * h.element_size() for h in host_x)
        d2h = sum(h.numel() * h.element_size() for h in host_out)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize(dev)
        t0.record(stream)
        for _ in range(args.steps):
            for i, n in enumerate(lens):
                lo, hi = spans[i]
                dev_x[i][0, lo:hi].copy_(host_x[i], non_blocking=True)
                _, _, rows = cp(dev_x[i], None, gather=False, length=n)
                host_out[i].copy_(rows, non_blocking=True)
            flush.zero_()
        t1.record(stream)
        torch.cuda.synchronize(dev)
        e2e_ms = max_over_ranks(t0.elapsed_time(t1))
        nb = torch.tensor([h2d, d2h], dtype=torch.float64, device=dev)
        dist.all_reduce(nb)
        launches = (5 * cfg.num_layers + 2) * len(seqs)
    cp.close()  # the graphs hold NCCL calls: released before the process group
    clk = clocks.stop()
    if rank != 0:
        return 0
    value = B * S * args.steps / (total_ms / 1e3)
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "fp16", "data": "synthetic",
        "config": {"workload": workload_desc(name), "global_batch": B, "seq_len": S,
                   "parallelism": f"cp{K} x dp{world // K} (each sequence split across {K} ranks, "
                                  f"one q|k|v all-gather per layer, each sequence's split "
                                  f"forward replayed from a CUDA graph; groups take LPT shares "
                                  f"of the batch)",
                   "l2": "flushed between steps (256 MiB write)",
                   "weights": f"default nn.Linear/LayerNorm init, torch.manual_seed({args.seed})",
                   "inputs": f"x~N(0,1), input seed {args.seed + 1}"},
        "e2e": {"value": B * S * args.steps / (e2e_ms / 1e3), "unit": UNIT,
                "h2d_bytes_per_step": int(nb[0].item()), "d2h_bytes_per_step": int(nb[1].item()),
                "copies": "each rank copies its own rows of its group's sequences in and its "
                          "output rows out (pinned buffers, bytes summed over ranks)"},
        "roofline": None, "cpu_baseline": None, "clocks": clk,
        "gpu_launches": launches * args.steps, "launches_per_step": launches,
    }
    print(json.dumps(line), flush=True)
    return 0


def run_b200(args, rank: int, world: int, local_rank: int):
    import torch
    import torch.distributed as dist

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    import optimized_transformer  # noqa: F401
    import tttj_2026_b200 as tb
    from tttj_2026_b200 import sharding

    name = args.config
    B, S = CONFIGS[name][0], CONFIGS[name][1]
    cfg_full, model, x_full, mask_full = make_case(name, args.seed, dev)
    # This rank's LPT share of the batch (every sequence at N = 1), resident in HBM.
    lengths = sharding.lengths_of(mask_full, B, S)
    mine = sharding.local_shard(lengths, cfg_full, rank, world)
    sel = torch.as_tensor(mine, device=dev, dtype=torch.long)
    x = x_full.index_select(0, sel).contiguous()
    mask = None if mask_full is None else mask_full.index_select(0, sel).contiguous()
    b_local = len(mine)  # 0 when the batch has fewer sequences than ranks (the rank idles)
    cfg = tb.TransformerConfig(max(b_local, 1), S, cfg_full.d_model, cfg_full.num_heads, cfg_full.ffn_dim,
                               cfg_full.num_layers, cfg_full.causal)
    opt = tb.make_optimized_transformer(model)
    opt.set_path(args.path)
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    clocks = ClockSampler(local_rank).start()
    with torch.inference_mode():
        # ---- device-resident timed loop ----
        for _ in range(args.warmup):
            opt(x, mask)
            flush.zero_()
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        barrier()
        torch.cuda.synchronize(dev)
        for i in range(args.steps):
            starts[i].record(stream)
            opt(x, mask)
            ends[i].record(stream)
            flush.zero_()  # L2 flush between timed steps (outside the events)
        torch.cuda.synchronize(dev)
        barrier()
        step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
        total_ms = max_over_ranks(sum(step_ms))

        # ---- end to end through the public call with host buffers ----
        x_host = x.cpu().pin_memory()
        m_host = None if mask is None else mask.cpu().pin_memory()
        out_host = torch.empty(x.shape, dtype=x.dtype).pin_memory()
        h2d = x_host.numel() * x_host.element_size() + (0 if m_host is None else m_host.numel())
        d2h = out_host.numel() * out_host.element_size()
        x_dev = [torch.empty_like(x) for _ in range(2)]
        m_dev = [None if mask is None else torch.empty_like(mask) for _ in range(2)]
        out_hosts = [out_host, torch.empty(x.shape, dtype=x.dtype).pin_memory()]
        copy_stream = torch.cuda.Stream(device=dev)

        def e2e_run(n_steps):
            """n_steps forwards through the module call, inputs copied in and outputs
            copied out every step; returns the elapsed ms of the whole span (events on
            the copy stream: first H2D issued .. last D2H done)."""
            t0 = torch.cuda.Event(enable_timing=True)
            t1 = torch.cuda.Event(enable_timing=True)
            copy_stream.wait_stream(stream)
            with torch.cuda.stream(copy_stream):
                t0.record(copy_stream)
                x_dev[0].copy_(x_host, non_blocking=True)
                if m_dev[0] is not None:
                    m_dev[0].copy_(m_host, non_blocking=True)
                ready = torch.cuda.Event()
                ready.record(copy_stream)
            done_prev = None
            for i in range(n_steps):
                b = i & 1
                stream.wait_event(ready)  # step i's inputs have landed
                out = opt(x_dev[b], m_dev[b])
                done = torch.cuda.Event()
                done.record(stream)
                out.record_stream(copy_stream)
                flush.zero_()  # L2 flush between forwards (inside the timed span)
                with torch.cuda.stream(copy_stream):
                    if i + 1 < n_steps:
                        if done_prev is not None:  # buffer b^1 was read by forward i-1
                            copy_stream.wait_event(done_prev)
                        x_dev[b ^ 1].copy_(x_host, non_blocking=True)
                        if m_dev[b ^ 1] is not None:
                            m_dev[b ^ 1].copy_(m_host, non_blocking=True)
                        ready = torch.cuda.Event()
                        ready.record(copy_stream)
                    copy_stream.wait_event(done)
                    out_hosts[b].copy_(out, non_blocking=True)
                done_prev = done
            t1.record(copy_stream)
            torch.cuda.synchronize(dev)
            return t0.elapsed_time(t1), out_hosts[(n_steps - 1) & 1]

        e2e_run(args.warmup)
        barrier()
        torch.cuda.synchronize(dev)
        e2e_span_ms, out_last = e2e_run(args.steps)
        barrier()
        e2e_total_ms = max_over_ranks(e2e_span_ms)
        ok_e2e = torch.equal(out_last, opt(x, mask).cpu())
        if world > 1:  # bytes copied per step by all ranks together
            nb = torch.tensor([h2d, d2h], dtype=torch.float64, device=dev)
            dist.all_reduce(nb)
            h2d, d2h = int(nb[0].item()), int(nb[1].item())

        # ---- N > 1: the whole batch on every rank, gathered to rank 0 ----
        gathered = None
        if world > 1:
            def gather_step():
                out, _ = sharding.distributed_forward(opt, x_full, mask_full, dst=0)
                return out

            for _ in range(args.warmup):
                gather_step()
                flush.zero_()
            g0 = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
            g1 = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
            barrier()
            torch.cuda.synchronize(dev)
            for i in range(args.steps):
                g0[i].record(stream)
                out_full = gather_step()
                g1[i].record(stream)
                flush.zero_()
            torch.cuda.synchronize(dev)
            barrier()
            g_ms = max_over_ranks(sum(a.elapsed_time(b_) for a, b_ in zip(g0, g1)))
            gathered = {"value": B * S * args.steps / (g_ms / 1e3), "unit": UNIT,
                        "ms_per_step": g_ms / args.steps,
                        "what": "distributed_forward(module, x, mask, dst=0): every rank holds "
                                "the whole batch, runs its LPT shard, NCCL gather to rank 0"}
            if rank == 0:
                gathered["output_matches_local_shard"] = bool(torch.equal(
                    out_full.index_select(0, sel), opt(x, mask)))

        # ---- per-kernel-class timing inside real forwards ----
        ktimes, launches = {}, 0
        if b_local:
            opt.set_kernel_timing(b_local, S, True)
            for _ in range(args.steps):
                opt(x, mask)
                flush.zero_()
            ktimes = opt.kernel_times(b_local, S)
            opt.set_kernel_timing(b_local, S, False)
            launches = opt.launches_per_forward(b_local, S)
        opt.device_status()
    clk = clocks.stop()

    if rank != 0:
        return 0

    tokens = B * S  # the whole batch, all ranks together
    value = tokens * args.steps / (total_ms / 1e3)
    e2e_value = tokens * args.steps / (e2e_total_ms / 1e3)
    Tv, pairs, per_launch, flops_local = useful_work(cfg, mask, x.element_size())
    Tv_full, _, _, flops_full = useful_work(cfg_full, mask_full, x.element_size())
    peaks = load_peaks()
    ms_per_step = total_ms / args.steps
    long_step = ms_per_step >= LONG_STEP_MS
    tensor_peak = peaks["tflops_sustained"] if long_step else peaks["tflops"]
    tensor_src = "bf16_tflops_sustained" if long_step else "bf16_tflops burst"
    kernels = {}
    for cls, (ms, n) in ktimes.items():
        if n == 0:
            continue
        bound, work = per_launch[cls]
        avg_ms = ms / n
        if bound == "tensor":
            achieved = work / (avg_ms * 1e-3) / 1e12
            peak, unit = tensor_peak, "TFLOP/s"
        else:
            achieved = work / (avg_ms * 1e-3) / 1e9
            peak, unit = peaks["hbm_gbs"], "GB/s"
        kernels[cls] = {"launches": n, "total_ms": round(ms, 4), "avg_us": round(avg_ms * 1e3, 2),
                        "share": None, "bound": "hbm" if bound == "hbm" else "tensor",
                        "achieved": round(achieved, 2), "unit": unit, "frac": round(achieved / peak, 4)}
    ksum = sum(v["total_ms"] for v in kernels.values())
    for v in kernels.values():
        v["share"] = round(v["total_ms"] / ksum, 4) if ksum else None
    dom = max(kernels, key=lambda k: kernels[k]["total_ms"])
    dk = kernels[dom]
    traffic = _profile_traffic(dom, name) if world == 1 else None
    roofline = {"kernel": dom, "bound": dk["bound"], "achieved": dk["achieved"],
                "peak": tensor_peak if dk["bound"] == "tensor" else peaks["hbm_gbs"],
                "unit": dk["unit"], "frac": dk["frac"], "traffic": traffic,
                "peak_source": f"{peaks['source']} ({tensor_src if dk['bound'] == 'tensor' else 'hbm_gbs'})"}

    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        threads = os.cpu_count() or 1
        cval, sample, _ = cpu_oracle_rate(name, args.seed, args.cpu_seconds, threads)
        if cval is not None:
            cpu = {"value": cval, "unit": UNIT, "cores": threads, "kind": "port",
                   "cpu_model": cpu_model(), "sample": sample}

    vs_baseline = None
    if name.startswith("R") and world == 1:
        # Published H200 forward time of the same case (tokens/s = B*S / time).
        vs_baseline = value / (tokens / (PUBLISHED_H200_MS[int(name[1:])] * 1e-3))
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_per_step, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": vs_baseline, "dtype": "fp16", "data": "synthetic",
        "config": {"workload": workload_desc(name), "global_batch": B, "seq_len": S,
                   "parallelism": f"dp{world} (batch split, LPT by predicted cost; "
                                  f"rank 0 runs {b_local} of {B} sequences)",
                   "l2": "flushed between steps (256 MiB write)",
                   "path": ("resident stack (1 launch per forward)" if opt.uses_resident(b_local, S)
                            else f"layer by layer ({launches} launches per forward)"),
                   "weights": f"default nn.Linear/LayerNorm init, torch.manual_seed({args.seed})",
                   "inputs": f"x~N(0,1), input seed {args.seed + 1}"},
        "p50_ms": statistics.median(step_ms),
        "valid_tokens_per_s": Tv_full * args.steps / (total_ms / 1e3),
        "useful_tflops_per_gpu": flops_full / world / (ms_per_step * 1e-3) / 1e12,
        "useful_frac_of_peak": flops_full / world / (ms_per_step * 1e-3) / 1e12 / tensor_peak,
        "roofline": roofline,
        "kernels": kernels,
        "cpu_baseline": cpu,
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "ms_per_step": e2e_total_ms / args.steps, "output_matches_device_path": ok_e2e,
                "copies": "each rank copies its own shard in and its output shard out "
                          "(bytes summed over ranks)"},
        "gather_to_rank0": gathered,
        "clocks": clk,
        "gpu_launches": launches * args.steps,
        "launches_per_step": launches,
    }
    print(json.dumps(line), flush=True)
    return 0


def _profile_traffic(kernel_class: str, config: str):
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary
    (a line `traffic_bytes_per_launch <class> <config> <bytes>`), else None."""
    for f in sorted((REPO / "profiles").glob("*.md")):
        for line in f.read_text().splitlines():
            parts = line.strip().strip("`").split()
            if len(parts) == 4 and parts[0] == "traffic_bytes_per_launch" and parts[1] == kernel_class \
                    and parts[2] == config:
                try:
                    return float(parts[3])
                except ValueError:
                    return None
    return None


def main(argv=None) -> int:
    args = parse_args(argv)
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if world > 1:
        # Keep rank 0's stdout to the one JSON line (no NCCL version banner).
        os.environ.setdefault("NCCL_DEBUG", "WARN")
        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.cp > 1:
            return run_cp(args, rank, world, local_rank)
        return run_b200(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    sys.exit(main())
