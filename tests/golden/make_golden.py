"""Generate the golden vectors that pin the fp32 oracle to the real reference.

Runs the UNMODIFIED reference organizer module (``BaselineTransformer`` from
benchmarks/torch_transformer_benchmark.py of Scallion3008/tttj-2026) in fp32 on the
CPU and stores, per case, the input, the mask, the output and a checksum of the
default-initialised weights.  The weights themselves are not stored: the test
rebuilds them with ``torch.manual_seed(model_seed)`` and this package's
TransformerParameters (same module tree, same RNG consumption order) and checks the
checksum first.

Usage (needs the reference sources, read-only):
    python tests/golden/make_golden.py --reference /path/to/tttj-2026
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

# name: (batch, seq, d_model, heads, ffn, layers, causal, model_seed, input_seed, lengths)
# lengths: None = valid_token_mask None; list = explicit per-sequence prefix lengths;
# (lo, hi) tuple = uniform in [lo, hi] drawn from the input generator.
CASES = {
    # BASELINE.json configs[0] exactly (the reference's own CPU-runnable case).
    "c1_tiny_encoder": (2, 128, 256, 4, 1024, 2, False, 0, 1, (64, 128)),
    # causal, hd64, ragged lengths incl. a length-1 sequence
    "causal_hd64_ragged": (3, 40, 128, 2, 256, 2, True, 11, 12, [40, 1, 17]),
    # non-causal hd32 with a partial last key tile
    "enc_hd32_ragged": (2, 70, 128, 4, 512, 2, False, 21, 22, [70, 33]),
    # mask=None, causal, single head
    "causal_nomask": (2, 33, 64, 1, 128, 1, True, 31, 32, None),
    # a fully padded sequence next to a valid one
    "empty_sequence": (2, 24, 64, 2, 192, 2, False, 41, 42, [0, 20]),
    # head widths of the reference's own cases (optimized_transformer.py:22-42),
    # F = D and causal like them, at small batch and sequence:
    # case 7 (d_model 32, 4 heads of 8)
    "case7_hd8": (2, 48, 32, 4, 32, 2, True, 51, 52, [48, 30]),
    # case 11 (d_model 128, 16 heads of 8)
    "case11_hd8_h16": (2, 40, 128, 16, 128, 1, True, 81, 82, [40, 9]),
    # case 9 (one head of 128)
    "case9_hd128": (2, 140, 128, 1, 128, 2, True, 61, 62, [140, 25]),
    # case 8's head width 256 (2 heads at d_model 512 keep the fixture small)
    "case8_hd256": (2, 36, 512, 2, 512, 1, True, 71, 72, [36, 20]),
}


def load_reference(ref_root: Path):
    path = ref_root / "benchmarks" / "torch_transformer_benchmark.py"
    spec = importlib.util.spec_from_file_location("_tttj_reference_bench", path)
    mod = importlib.util.module_from_spec(spec)
    sys.modules[spec.name] = mod
    spec.loader.exec_module(mod)
    return mod


def weights_checksum(model: torch.nn.Module) -> float:
    """Order-sensitive checksum of every parameter (float64)."""
    total = 0.0
    for i, (_, t) in enumerate(sorted(model.state_dict().items())):
        flat = t.detach().double().reshape(-1)
        w = torch.arange(1, flat.numel() + 1, dtype=torch.float64) / flat.numel()
        total += float((flat * w).sum()) * (i + 1)
    return total


def perturb_norms(model: torch.nn.Module, seed: int) -> None:
    """Replace every LayerNorm's default (1, 0) affine with seeded values, so the
    golden outputs also pin the oracle's use of gamma and beta.  Iterates modules
    in registration order, which is the same for the reference module and
    TransformerParameters."""
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for mod in model.modules():
            if isinstance(mod, torch.nn.LayerNorm):
                n = mod.weight.numel()
                mod.weight.copy_(1.0 + 0.2 * torch.randn(n, generator=g))
                mod.bias.copy_(0.2 * torch.randn(n, generator=g))


def make_inputs(B, S, D, input_seed, lengths):
    g = torch.Generator().manual_seed(input_seed)
    x = torch.randn(B, S, D, generator=g)
    if lengths is None:
        return x, None
    if isinstance(lengths, tuple):
        lo, hi = lengths
        lens = torch.randint(lo, hi + 1, (B,), generator=g)
    else:
        lens = torch.tensor(lengths)
    mask = torch.arange(S)[None, :] < lens[:, None]
    x = x.masked_fill(~mask[..., None], 0)
    return x, mask


def main(argv=None) -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, required=True)
    ap.add_argument("--only", nargs="+", choices=sorted(CASES),
                    help="regenerate these cases only (the index keeps the others)")
    args = ap.parse_args(argv)
    ref = load_reference(args.reference)
    torch.set_num_threads(8)
    index_path = HERE / "index.json"
    index = json.loads(index_path.read_text()) if args.only and index_path.exists() else {}
    for name, (B, S, D, H, F, L, causal, mseed, iseed, lengths) in CASES.items():
        if args.only and name not in args.only:
            continue
        cfg = ref.TransformerConfig(B, S, D, H, F, L, causal)
        torch.manual_seed(mseed)
        model = ref.BaselineTransformer(cfg).eval()
        if name != "c1_tiny_encoder":  # C1 keeps the default init of BASELINE configs[0]
            perturb_norms(model, mseed + 1000)
        x, mask = make_inputs(B, S, D, iseed, lengths)
        with torch.inference_mode():
            out = model(x, mask)
        np.savez_compressed(
            HERE / f"{name}.npz",
            x=x.numpy().astype(np.float32),
            mask=(mask.numpy() if mask is not None else np.zeros((0,), dtype=bool)),
            has_mask=np.array(mask is not None),
            out=out.numpy().astype(np.float32),
        )
        index[name] = {
            "config": dict(batch_size=B, seq_len=S, d_model=D, num_heads=H, ffn_dim=F,
                           num_layers=L, causal=causal),
            "model_seed": mseed,
            "input_seed": iseed,
            "lengths": list(lengths) if lengths is not None else None,
            "perturbed_norms": name != "c1_tiny_encoder",
            "weights_checksum": weights_checksum(model),
            "out_abs_sum": float(out.abs().sum()),
        }
        print(f"{name}: out |sum| = {index[name]['out_abs_sum']:.6f}")
    index_path.write_text(json.dumps(index, indent=1, sort_keys=True) + "\n")
    return 0


if __name__ == "__main__":
    sys.exit(main())
