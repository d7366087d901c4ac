"""GPU: the allocation-free attention entry point, tttj_attention_noalloc.

It serves callers that cannot allocate device memory when they call attention (code
inside an allocator or memory-pool callback, hosts that forbid cudaMalloc after
start-up, runtimes that pass only pre-placed buffers).  Instead of a caller
workspace it uses a fixed scratch array inside the library.  These tests call it
through the C ABI and check that two calls in a row -- different shapes and masks,
so the second call runs over the first call's leftovers in the shared scratch --
give the same output as tttj_attention with a caller-provided workspace, and, so that
a fault shared by both entry points cannot pass, the same output as an fp32 attention
computed by torch, within the attention tolerance of tests/test_gpu_kernels.py.

This file is named so that pytest collects it last.
"""
import ctypes

import pytest
import torch

import tttj_2026_b200 as tb  # noqa: F401  (package registration via conftest)
from tttj_2026_b200 import _lib, ops
from test_gpu_kernels import _attention_ref

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
ATOL, RTOL = 3e-3, 3e-3  # the attention tolerance used by tests/test_gpu_kernels.py


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _case(lengths, S, H, hd, seed):
    D = H * hd
    mask = torch.arange(S, device=DEV)[None, :] < torch.tensor(lengths, device=DEV)[:, None]
    g = torch.Generator(device=DEV).manual_seed(seed)
    qkv = (torch.randn(sum(lengths), 3 * D, device=DEV, generator=g) * 1.5).half()
    return qkv, mask


def _noalloc(qkv, mask, B, S, H, causal):
    D = qkv.shape[1] // 3
    # Poison the output so a row the kernel fails to write cannot pass.
    ctx = torch.full((qkv.shape[0], D), float("nan"), dtype=torch.float16, device=DEV)
    m = None if mask is None else mask.contiguous().view(torch.uint8)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = _lib.lib().tttj_attention_noalloc(_ptr(qkv), _ptr(ctx), qkv.shape[0], _ptr(m), B, S, D,
                                           H, 1 if causal else 0, stream)
    _lib.check(rc, "attention_noalloc")
    return ctx


def _close(out, ref):
    err = (out.float() - ref.float()).abs()
    bad = ~(err <= ATOL + RTOL * ref.float().abs())  # NaN counts as bad
    assert not bad.any(), f"max err {err.max().item():.3e}, {int(bad.sum())} elements out of tolerance"


def test_noalloc_matches_workspace_entry_on_two_calls_in_a_row():
    # Call 1: causal, head_dim 64, ragged lengths (incl. a length-1 sequence).
    # Call 2: non-causal, head_dim 32, a different batch and sequence length.
    cases = [
        dict(lengths=[300, 1, 129, 256], S=300, H=4, hd=64, causal=True, seed=1),
        dict(lengths=[77, 512, 5], S=512, H=8, hd=32, causal=False, seed=2),
    ]
    for c in cases:
        qkv, mask = _case(c["lengths"], c["S"], c["H"], c["hd"], c["seed"])
        B = len(c["lengths"])
        ref = ops.attention(qkv, mask, B, c["S"], c["H"], c["causal"])
        out = _noalloc(qkv, mask, B, c["S"], c["H"], c["causal"])
        torch.cuda.synchronize()
        _close(out, ref)
        _close(out, _attention_ref(qkv, c["lengths"], c["H"], c["causal"]))


def test_noalloc_repeat_and_mask_none():
    qkv, _ = _case([128, 128], 128, 2, 64, 3)
    ref = ops.attention(qkv, None, 2, 128, 2, True)
    first = _noalloc(qkv, None, 2, 128, 2, True)
    second = _noalloc(qkv, None, 2, 128, 2, True)
    torch.cuda.synchronize()
    _close(first, ref)
    assert torch.equal(first, second)


def test_noalloc_rejects_shapes_beyond_the_scratch():
    L = _lib.lib()
    # 4096 x 8192 tokens need ~270 MB of plan; nothing may be launched.
    rc = L.tttj_attention_noalloc(ctypes.c_void_p(256), ctypes.c_void_p(256), 4096 * 8192, None,
                                  4096, 8192, 512, 8, 1, None)
    assert rc == _lib.TTTJ_ERR_INVALID
    msg = L.tttj_last_error().decode()
    assert "scratch" in msg and "tttj_attention" in msg
