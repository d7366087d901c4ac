"""GPU: forwards without a mask reuse the all-valid token plan of the previous mask-free
forward (the gather kernel that opens each forward zeroes the attention work counters),
and a masked forward in between rebuilds it (kernels/sequence_resident.py:173-192 caches
the all-valid case the same way)."""
import pytest
import torch

import tttj_2026_b200 as tb
from helpers import gate
from oracle import forward_fp32, state_dict_fp32

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


@pytest.mark.parametrize("shape", [(8, 256, 128, 4, 256, 2, True), (3, 300, 256, 2, 512, 3, False)])
def test_mask_free_forwards_reuse_the_plan(shape):
    B, S, D, H, F, L, causal = shape
    cfg = tb.TransformerConfig(B, S, D, H, F, L, causal)
    model = tb.make_parameter_model(cfg, 5, torch.float16, DEV)
    opt = tb.make_optimized_transformer(model)
    assert not opt.uses_resident(B, S)
    full = opt.launches_per_forward(B, S)
    g = torch.Generator().manual_seed(B * S)
    x = torch.randn(B, S, D, generator=g).to(torch.float16)
    lens = torch.randint(1, S + 1, (B,), generator=g)
    mask = (torch.arange(S)[None, :] < lens[:, None])
    xm = x.masked_fill(~mask[..., None], 0).to(DEV)
    x, mask = x.to(DEV), mask.to(DEV)
    with torch.inference_mode():
        first = opt(x, None)
        assert opt.launches_per_forward(B, S) == full - 1
        again = [opt(x, None) for _ in range(3)]
        masked = opt(xm, mask)
        assert opt.launches_per_forward(B, S) == full
        after = opt(x, None)
        masked_again = opt(xm, mask)
        sd = state_dict_fp32(model, DEV)
        ref = forward_fp32(sd, cfg, x.float(), None)
        ref_m = forward_fp32(sd, cfg, xm.float(), mask)
    torch.cuda.synchronize()
    for y in again + [after]:
        assert torch.equal(y, first)
    assert torch.equal(masked, masked_again)
    r = gate(ref, first, None)
    assert r.passed, r
    r = gate(ref_m, masked, mask)
    assert r.passed, r
    assert opt.device_status() == 0
