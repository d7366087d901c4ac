"""Thin torch-tensor wrappers over the per-kernel C entry points.

Each wrapper checks dtype, shape, contiguity and device (the reference's
TORCH_CHECK conventions, kernels/csrc/case14_softmax.cpp:18-35) and launches on the
current CUDA stream.  They exist for parity tests and for callers composing their
own layer; the forward of ``B200Transformer`` runs the same kernels from C.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from . import _lib


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _need(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


def linear(a: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, *, epilogue: str = "bias",
           residual: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
           rows_dev: Optional[torch.Tensor] = None, status: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out = epi(a @ weight.T + bias) on the tcgen05 GEMM.

    epilogue: "bias", "gelu" (exact erf GELU), "residual" (out = residual + ...;
    ``out`` may be ``residual`` itself; fp16) or "residual_f32" (fp32 residual and
    out, the forward's residual stream).  a [M, K] fp16, weight [N, K] fp16,
    bias [N] fp32.
    """
    epi = {"bias": _lib.EPI_BIAS, "gelu": _lib.EPI_BIAS_GELU, "residual": _lib.EPI_BIAS_RESIDUAL,
           "residual_f32": _lib.EPI_BIAS_RESIDUAL_F32}[epilogue]
    _need(a.dtype == torch.float16 and weight.dtype == torch.float16, "linear: a and weight must be fp16")
    _need(bias.dtype == torch.float32, "linear: bias must be fp32")
    _need(a.dim() == 2 and weight.dim() == 2 and a.shape[1] == weight.shape[1], "linear: shape mismatch")
    _need(a.stride(1) == 1 and weight.stride(1) == 1 and bias.is_contiguous(), "linear: inner dims must be contiguous")
    M, K = a.shape
    N = weight.shape[0]
    out_dtype = torch.float32 if epi == _lib.EPI_BIAS_RESIDUAL_F32 else torch.float16
    if out is None:
        out = torch.empty(M, N, dtype=out_dtype, device=a.device)
    _need(out.dtype == out_dtype and out.stride(1) == 1, f"linear: out must be {out_dtype} [M, N]")
    if epi in (_lib.EPI_BIAS_RESIDUAL, _lib.EPI_BIAS_RESIDUAL_F32):
        _need(residual is not None and residual.shape == (M, N) and residual.dtype == out_dtype,
              f"linear: residual must be {out_dtype} [M, N]")
    rc = _lib.lib().tttj_linear(
        _ptr(a), a.stride(0), _ptr(weight), weight.stride(0), _ptr(bias), _ptr(out), out.stride(0),
        _ptr(residual), residual.stride(0) if residual is not None else 0, M, _ptr(rows_dev), N, K, epi,
        _ptr(status), _stream(a.device))
    _lib.check(rc, "linear")
    return out


def layernorm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float = 1e-5,
              out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """nn.LayerNorm over the last dim of a contiguous fp16 [rows, d] tensor."""
    _need(x.dtype == torch.float16 and x.is_contiguous() and x.dim() == 2, "layernorm: x must be contiguous fp16 [rows, d]")
    _need(weight.dtype == torch.float32 and bias.dtype == torch.float32, "layernorm: weight/bias must be fp32")
    if out is None:
        out = torch.empty_like(x)
    rc = _lib.lib().tttj_layernorm(_ptr(x), _ptr(out), x.shape[0], x.shape[1], _ptr(weight), _ptr(bias),
                                   float(eps), _stream(x.device))
    _lib.check(rc, "layernorm")
    return out


def attention_workspace_bytes(batch: int, seq_len: int, num_heads: int) -> int:
    return int(_lib.lib().tttj_attention_workspace_bytes(batch, seq_len, num_heads))


def attention(qkv: torch.Tensor, valid_token_mask: Optional[torch.Tensor], batch: int, seq_len: int,
              num_heads: int, causal: bool, workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Attention over the packed valid-token layout: qkv [Tv, 3D] fp16 -> ctx [Tv, D]."""
    _need(qkv.dtype == torch.float16 and qkv.is_contiguous() and qkv.dim() == 2, "attention: qkv must be contiguous fp16 [Tv, 3D]")
    D = qkv.shape[1] // 3
    ctx = torch.zeros(qkv.shape[0], D, dtype=torch.float16, device=qkv.device)
    nbytes = attention_workspace_bytes(batch, seq_len, num_heads)
    if workspace is None:
        workspace = torch.empty(nbytes, dtype=torch.uint8, device=qkv.device)
    mask = None
    if valid_token_mask is not None:
        mask = valid_token_mask.to(torch.bool).contiguous().view(torch.uint8)
    rc = _lib.lib().tttj_attention(_ptr(qkv), _ptr(ctx), qkv.shape[0], _ptr(mask), batch, seq_len, D, num_heads,
                                   1 if causal else 0, _ptr(workspace), workspace.numel(),
                                   _stream(qkv.device))
    _lib.check(rc, "attention")
    return ctx


def selftest_wait_timeout(status: torch.Tensor, limit_ns: int) -> None:
    """Launch the bounded-wait self test (writes 0x1ff into ``status`` on timeout)."""
    _need(status.dtype == torch.int32 and status.is_cuda, "selftest: status must be a CUDA int32 tensor")
    _lib.check(_lib.lib().tttj_selftest_wait_timeout(_ptr(status), int(limit_ns), _stream(status.device)), "selftest")
