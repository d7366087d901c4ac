"""Run a few forwards of one configuration, for profiling the kernels under ncu.

    python tttj-2026_b200/profile_case.py --config C5 [--layers 2] [--forwards 2]

Builds the seeded model and inputs of a BASELINE.json configuration (C1..C5, see
bench.py) or of a reference case (R1..R14), optionally with fewer layers (every layer
of the stack has the same shapes, so one or two layers show every kernel at full
batch size with a fraction of the device memory and launches), runs ``--forwards``
forwards on cuda:0 and exits 0 when the device status is clean.  Nothing is timed:
``ncu -k <kernel> -s <skip> -c <count>`` picks the launches.
"""
from __future__ import annotations

import argparse
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))


def main(argv=None) -> int:
    import torch

    import bench
    import optimized_transformer  # noqa: F401
    import tttj_2026_b200 as tb

    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--config", default="C5", choices=list(bench.CONFIGS))
    ap.add_argument("--layers", type=int, default=None, help="override the number of layers")
    ap.add_argument("--batch", type=int, default=None, help="override the batch size")
    ap.add_argument("--forwards", type=int, default=2)
    ap.add_argument("--path", default="auto", choices=["auto", "layerwise", "resident"])
    ap.add_argument("--seed", type=int, default=0)
    args = ap.parse_args(argv)

    B, S, D, H, F, L, causal, dt, lens = bench.CONFIGS[args.config]
    B = args.batch or B
    L = args.layers or L
    dtype = getattr(torch, dt)
    dev = torch.device("cuda", 0)
    cfg = tb.TransformerConfig(B, S, D, H, F, L, causal)
    model = tb.make_parameter_model(cfg, args.seed, dtype, dev)
    x, mask = tb.generate_inputs(cfg, args.seed + 1, dtype, lens, dev)
    opt = tb.make_optimized_transformer(model)
    opt.set_path(args.path)
    with torch.inference_mode():
        for _ in range(args.forwards):
            out = opt(x, mask)
    torch.cuda.synchronize(dev)
    opt.device_status()
    print(f"[profile_case] {args.config} B{B} S{S} L{L}: {args.forwards} forwards, "
          f"{opt.launches_per_forward(B, S)} launches each, finite={bool(torch.isfinite(out).all())}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
