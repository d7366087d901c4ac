"""GPU: the per-stage capture (tttj_forward_debug / B200Transformer.run(capture_debug=True))
against the same stages of the fp32 oracle -- the reference's capture_debug stages
(kernels/sequence_resident.py:28-46) for a chosen sequence and layer."""
import math

import pytest
import torch

import tttj_2026_b200 as tb
from oracle import attention_fp32, block_fp32, gelu_erf, layer_norm, linear, state_dict_fp32

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


@pytest.fixture(autouse=True, scope="module")
def _no_tf32():
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32 = prev


def _oracle_stages(p, cfg, x, mask, layer, b):
    """fp32 stages of block `layer` for batch index b (the reference module's math)."""
    xs = x.float()
    for i in range(layer):
        xs = block_fp32(xs, p, i, cfg.num_heads, mask, cfg.causal)
    pre = f"layers.{layer}."
    h = layer_norm(xs, p[pre + "norm1.weight"], p[pre + "norm1.bias"])
    q = linear(h, p[pre + "attention.q_proj.weight"], p[pre + "attention.q_proj.bias"])
    k = linear(h, p[pre + "attention.k_proj.weight"], p[pre + "attention.k_proj.bias"])
    v = linear(h, p[pre + "attention.v_proj.weight"], p[pre + "attention.v_proj.bias"])
    B, S, D = xs.shape
    H, hd = cfg.num_heads, D // cfg.num_heads
    qh = q[b].view(S, H, hd).transpose(0, 1)
    kh = k[b].view(S, H, hd).transpose(0, 1)
    vh = v[b].view(S, H, hd).transpose(0, 1)
    scores = qh @ kh.transpose(-1, -2) / math.sqrt(hd)
    valid = torch.ones(S, dtype=torch.bool, device=DEV) if mask is None else mask[b]
    masked = ~valid[None, :].expand(S, S)
    if cfg.causal:
        masked = masked | torch.ones(S, S, dtype=torch.bool, device=DEV).triu(1)
    scores = scores.masked_fill(masked[None], float("-inf"))
    probs = torch.softmax(scores, -1)
    pv = (probs @ vh).transpose(0, 1).reshape(S, D)
    attn = attention_fp32(h, p, pre + "attention.", cfg.num_heads, mask, cfg.causal)
    x2 = xs + attn
    h2 = layer_norm(x2, p[pre + "norm2.weight"], p[pre + "norm2.bias"])
    ffn = linear(gelu_erf(linear(h2, p[pre + "ffn_in.weight"], p[pre + "ffn_in.bias"])),
                 p[pre + "ffn_out.weight"], p[pre + "ffn_out.bias"])
    if mask is not None:
        ffn = ffn.masked_fill(~mask[..., None], 0)
    z = ~valid[:, None]
    return {"layernorm": h[b].masked_fill(z, 0), "qkv.q": q[b].masked_fill(z, 0),
            "qkv.k": k[b].masked_fill(z, 0), "qkv.v": v[b].masked_fill(z, 0),
            "scores": scores.masked_fill(~valid[None, :, None], 0),
            "softmax": probs.masked_fill(~valid[None, :, None], 0),
            "pv": pv.masked_fill(z, 0), "output_projection": attn[b], "ffn": ffn[b]}


@pytest.mark.parametrize("shape,layer,b", [
    ((3, 40, 64, 2, 96, 2, True), 0, 0),     # the reference's choice: layer 0, sequence 0
    ((3, 40, 64, 2, 96, 2, True), 1, 2),
    ((2, 70, 128, 16, 128, 1, False), 0, 1),  # head_dim 8 (padded heads)
])
def test_capture_matches_oracle_stages(shape, layer, b):
    cfg = tb.TransformerConfig(*shape)
    model = tb.make_parameter_model(cfg, 5, torch.float32, DEV)
    g = torch.Generator().manual_seed(6)
    S = cfg.seq_len
    lens = torch.tensor([S, S // 2 + 3, 9][: cfg.batch_size])
    mask = (torch.arange(S)[None, :] < lens[:, None]).to(DEV)
    x = torch.randn(cfg.batch_size, S, cfg.d_model, generator=g).to(DEV)
    x = x.masked_fill(~mask[..., None], 0)
    opt = tb.make_optimized_transformer(model)
    with torch.inference_mode():
        out, st = opt.run(x, mask, capture_debug=True, debug_layer=layer, debug_sequence=b)
        plain = opt(x, mask)
        ref = _oracle_stages(state_dict_fp32(model, DEV), cfg, x, mask, layer, b)
    torch.cuda.synchronize()
    assert set(st) == set(ref)
    # The captured forward is the layer-by-layer forward itself.
    opt.set_path("layerwise")
    with torch.inference_mode():
        lw = opt(x, mask)
    torch.cuda.synchronize()
    assert torch.equal(out, lw)
    for name, r in ref.items():
        c = st[name]
        assert c.shape == r.shape, name
        if name == "scores":  # compare finite entries; masked ones must be -inf in both
            fin = torch.isfinite(r)
            assert torch.equal(fin, torch.isfinite(c)), name
            c, r = c[fin], r[fin]
        err = (c - r).abs().max().item() if c.numel() else 0.0
        tol = 2e-2 + 2e-2 * r.abs().max().item()
        assert err <= tol, (name, err, tol)
