"""GPU: each kernel through the C ABI against a plain PyTorch fp32 computation of
the same op on the same fp16 inputs."""
import pytest
import torch

import tttj_2026_b200 as tb
from tttj_2026_b200 import ops

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def _close(out, ref, atol, rtol):
    err = (out.float() - ref).abs()
    bound = atol + rtol * ref.abs()
    bad = err > bound
    assert not bad.any(), f"max err {err.max().item():.3e}, {int(bad.sum())} elements out of tolerance"


@pytest.mark.parametrize("M,N,K", [(128, 128, 64), (300, 768, 256), (1000, 512, 512),
                                   (4096, 2048, 512), (2048, 1024, 4096), (77, 1536, 1024),
                                   (8192, 4096, 1024)])  # CTA pairs, 12 epilogue warps (gelu)
@pytest.mark.parametrize("epilogue", ["bias", "gelu", "residual", "residual_f32"])
def test_linear_matches_torch(M, N, K, epilogue):
    g = torch.Generator(device=DEV).manual_seed(M * 7 + N * 3 + K)
    a = torch.randn(M, K, device=DEV, generator=g).half()
    w = (torch.randn(N, K, device=DEV, generator=g) / K**0.5).half()
    b = torch.randn(N, device=DEV, generator=g) * 0.1
    ref = a.float() @ w.float().t() + b
    res = None
    if epilogue == "gelu":
        ref = torch.nn.functional.gelu(ref)
    elif epilogue == "residual":
        res = torch.randn(M, N, device=DEV, generator=g).half()
        ref = ref + res.float()
    elif epilogue == "residual_f32":
        res = torch.randn(M, N, device=DEV, generator=g) * 4
        ref = ref + res
    out = ops.linear(a, w, b, epilogue=epilogue, residual=res)
    torch.cuda.synchronize()
    if epilogue == "residual_f32":
        assert out.dtype == torch.float32
        _close(out, ref, atol=2e-4, rtol=2e-5)  # fp32 store: only the fp16 operands round
    else:
        _close(out, ref, atol=2e-3, rtol=2e-3)


def test_gelu_epilogue_accuracy_over_a_dense_range():
    """Drive the GELU epilogue through an identity GEMM: every pre-activation in
    [-12, 12] (step ~1e-3) must come out as fp16(GELU(x)) up to fp16 rounding,
    comparing with torch's exact-erf GELU in fp32."""
    N = 256
    vals = torch.linspace(-12, 12, 128 * 100 * N // 4, device=DEV)
    M = vals.numel() // N
    x = vals[: M * N].view(M, N).half()
    eye = torch.eye(N, device=DEV).half()
    zero = torch.zeros(N, device=DEV)
    out = ops.linear(x, eye, zero, epilogue="gelu")
    torch.cuda.synchronize()
    ref = torch.nn.functional.gelu(x.float())
    err = (out.float() - ref).abs()
    ulp = torch.clamp(ref.abs(), min=2.0**-14) * 2.0**-10  # one fp16 ulp (or subnormal step)
    assert bool((err <= 0.5 * ulp + 1e-6).all()), float((err / ulp).max())


def test_linear_residual_in_place_and_device_row_count():
    M, N, K = 640, 512, 256
    g = torch.Generator(device=DEV).manual_seed(3)
    a = torch.randn(M, K, device=DEV, generator=g).half()
    w = (torch.randn(N, K, device=DEV, generator=g) / K**0.5).half()
    b = torch.randn(N, device=DEV, generator=g)
    x = torch.randn(M, N, device=DEV, generator=g).half()
    x0 = x.clone()
    rows = torch.tensor([333], dtype=torch.int32, device=DEV)
    ops.linear(a, w, b, epilogue="residual", residual=x, out=x, rows_dev=rows)
    torch.cuda.synchronize()
    ref = a.float() @ w.float().t() + b + x0.float()
    _close(x[:333], ref[:333], atol=2e-3, rtol=2e-3)
    assert torch.equal(x[333:], x0[333:])  # rows past the device count untouched


@pytest.mark.parametrize("rows,d", [(1, 256), (1000, 512), (4097, 768), (64, 1024), (33, 2048), (10, 136)])
def test_layernorm_matches_torch(rows, d):
    g = torch.Generator(device=DEV).manual_seed(rows + d)
    x = (torch.randn(rows, d, device=DEV, generator=g) * 3 + 1).half()
    w = torch.randn(d, device=DEV, generator=g)
    b = torch.randn(d, device=DEV, generator=g)
    out = ops.layernorm(x, w, b)
    ref = torch.nn.functional.layer_norm(x.float(), (d,), w, b, 1e-5)
    _close(out, ref, atol=4e-3, rtol=4e-3)


def _attention_ref(qkv, lengths, H, causal):
    """fp32 attention per sequence over the packed layout."""
    D = qkv.shape[1] // 3
    hd = D // H
    outs = []
    off = 0
    for L in lengths:
        if L == 0:
            continue
        t = qkv[off : off + L].float()
        q, k, v = t[:, :D], t[:, D : 2 * D], t[:, 2 * D :]
        q = q.view(L, H, hd).transpose(0, 1)
        k = k.view(L, H, hd).transpose(0, 1)
        v = v.view(L, H, hd).transpose(0, 1)
        s = q @ k.transpose(-1, -2) * hd**-0.5
        if causal:
            s = s.masked_fill(torch.ones(L, L, dtype=torch.bool, device=qkv.device).triu(1), float("-inf"))
        p = torch.softmax(s, -1)
        outs.append((p @ v).transpose(0, 1).reshape(L, D))
        off += L
    return torch.cat(outs, 0)


@pytest.mark.parametrize("hd", [32, 64, 128, 256])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("lengths,S", [([128], 128), ([1, 64, 65, 200, 0, 127], 200),
                                       ([513, 1000, 7], 1000), ([300, 300], 300)])
def test_attention_matches_torch(hd, causal, lengths, S):
    H = {32: 8, 64: 4, 128: 2, 256: 1}[hd]
    D = H * hd
    B = len(lengths)
    mask = torch.arange(S, device=DEV)[None, :] < torch.tensor(lengths, device=DEV)[:, None]
    Tv = sum(lengths)
    g = torch.Generator(device=DEV).manual_seed(Tv + hd)
    qkv = (torch.randn(Tv, 3 * D, device=DEV, generator=g) * 1.5).half()
    ctx = ops.attention(qkv, mask, B, S, H, causal)
    ref = _attention_ref(qkv, lengths, H, causal)
    _close(ctx, ref, atol=3e-3, rtol=3e-3)


def test_attention_non_prefix_mask():
    """A mask with holes: packing keeps token order, so causal masking stays exact."""
    B, S, H, hd = 2, 96, 2, 64
    D = H * hd
    g = torch.Generator(device=DEV).manual_seed(9)
    mask = torch.rand(B, S, device=DEV, generator=g) > 0.4
    lengths = mask.sum(1).tolist()
    qkv = torch.randn(sum(lengths), 3 * D, device=DEV, generator=g).half()
    for causal in (False, True):
        ctx = ops.attention(qkv, mask, B, S, H, causal)
        _close(ctx, _attention_ref(qkv, lengths, H, causal), atol=3e-3, rtol=3e-3)


def test_bounded_wait_reports_timeout_and_context_survives():
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    ops.selftest_wait_timeout(status, limit_ns=2_000_000)  # 2 ms
    torch.cuda.synchronize()
    assert int(status.item()) == 0x1FF
    # the context is still usable
    x = torch.ones(4, device=DEV)
    assert float((x * 2).sum().item()) == 8.0
