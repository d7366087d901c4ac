"""The nn.Module returned by ``make_optimized_transformer``.

It packs the parameter model's weights once into the library's device layout
(fp16 matrices in nn.Linear's [out, in] layout, fp32 vectors; see
include/tttj_b200.h), folds the LayerNorm affines into copies of the QKV / ffn_in
weights once, and runs every forward as one ``tttj_forward`` call on the caller's
current CUDA stream.  Replaces the reference adapters
SequenceResidentTransformer (kernels/sequence_resident.py:125-233),
Case8OptimizedTransformer (kernels/layerwise_hybrid.py:449-465), GraphedCase13Hybrid
(kernels/case13_hybrid.py:641-748) and Case14OptimizedTransformer
(kernels/case14_hybrid.py:774-849) for every supported shape.
"""
from __future__ import annotations

import ctypes
from collections import OrderedDict
from typing import Optional

import torch
import torch.nn as nn

from . import _lib

_SUPPORTED_INPUT = {torch.float16: _lib.DTYPE_F16, torch.float32: _lib.DTYPE_F32}


def validate_model_config(cfg) -> None:
    """Raise ValueError (the reference constructor's convention,
    optimized_transformer.py:62-66) when the library has no kernel for ``cfg``."""
    if hasattr(cfg, "validate"):
        cfg.validate()
    c = _lib.TttjConfig.from_config(cfg)
    _lib.check(_lib.lib().tttj_validate_config(ctypes.byref(c)), "make_optimized_transformer")


def pack_weights(parameter_model: nn.Module, device: torch.device) -> torch.Tensor:
    """Pack the parameter model into the library's weight buffer on ``device``.

    Reads the same attributes the reference packer reads
    (kernels/sequence_resident.py:98-108): layers[i].norm1, attention.{q,k,v,out}_proj,
    norm2, ffn_in, ffn_out, and final_norm.  Weights of any float dtype are accepted
    and stored as fp16 matrices / fp32 vectors.
    """
    cfg = parameter_model.config
    L = _lib.lib()
    c = _lib.TttjConfig.from_config(cfg)
    nbytes = L.tttj_weights_bytes(ctypes.byref(c))
    if nbytes == 0:
        _lib.check(L.tttj_validate_config(ctypes.byref(c)), "pack_weights")
    buf = torch.zeros(nbytes, dtype=torch.uint8, device=device)

    def put(layer: int, field: int, tensor: torch.Tensor, dtype: torch.dtype) -> None:
        off = ctypes.c_size_t()
        size = ctypes.c_size_t()
        _lib.check(
            L.tttj_weight_offset(ctypes.byref(c), layer, field, ctypes.byref(off), ctypes.byref(size)),
            "pack_weights",
        )
        src = tensor.detach().to(device=device, dtype=dtype).contiguous().reshape(-1)
        if src.numel() * src.element_size() != size.value:
            raise ValueError(f"weight field {field} of layer {layer}: size mismatch")
        buf[off.value : off.value + size.value].view(dtype).copy_(src)

    with torch.no_grad():
        for i, blk in enumerate(parameter_model.layers):
            att = blk.attention
            put(i, _lib.W_QKV, torch.cat([att.q_proj.weight, att.k_proj.weight, att.v_proj.weight], 0),
                torch.float16)
            put(i, _lib.W_OUT, att.out_proj.weight, torch.float16)
            put(i, _lib.W_FFN_IN, blk.ffn_in.weight, torch.float16)
            put(i, _lib.W_FFN_OUT, blk.ffn_out.weight, torch.float16)
            put(i, _lib.B_QKV, torch.cat([att.q_proj.bias, att.k_proj.bias, att.v_proj.bias], 0),
                torch.float32)
            put(i, _lib.B_OUT, att.out_proj.bias, torch.float32)
            put(i, _lib.B_FFN_IN, blk.ffn_in.bias, torch.float32)
            put(i, _lib.B_FFN_OUT, blk.ffn_out.bias, torch.float32)
            put(i, _lib.LN1_W, blk.norm1.weight, torch.float32)
            put(i, _lib.LN1_B, blk.norm1.bias, torch.float32)
            put(i, _lib.LN2_W, blk.norm2.weight, torch.float32)
            put(i, _lib.LN2_B, blk.norm2.bias, torch.float32)
        n = len(parameter_model.layers)
        put(n, _lib.LNF_W, parameter_model.final_norm.weight, torch.float32)
        put(n, _lib.LNF_B, parameter_model.final_norm.bias, torch.float32)
    return buf


def fold_weights(cfg, packed: torch.Tensor) -> torch.Tensor:
    """LayerNorm-folded copies of every block's QKV / ffn_in weights (and the padded
    out_proj of narrow heads), computed once per model on the current stream
    (``tttj_fold_weights``).  They depend on the layer shapes only, so every (B, S)
    plan of the model shares them."""
    L = _lib.lib()
    c = _lib.TttjConfig.from_config(cfg)
    nbytes = L.tttj_folded_bytes(ctypes.byref(c))
    if nbytes == 0:
        _lib.check(L.tttj_validate_config(ctypes.byref(c)), "fold_weights")
    folded = torch.empty(nbytes, dtype=torch.uint8, device=packed.device)
    stream = torch.cuda.current_stream(packed.device).cuda_stream
    _lib.check(L.tttj_fold_weights(ctypes.byref(c), ctypes.c_void_p(packed.data_ptr()),
                                   ctypes.c_void_p(folded.data_ptr()), nbytes,
                                   ctypes.c_void_p(stream)), "fold_weights")
    return folded


class _Plan:
    """One C plan (TMA descriptors + workspace) for one (batch, seq_len) shape.

    Creating it launches nothing but the workspace's zero fill, on the current stream
    (the stream of the forward that needs the plan); the plan orders its own forwards
    across streams, and destroying it waits for its last forward."""

    def __init__(self, cfg, batch: int, seq_len: int, weights: torch.Tensor,
                 folded: torch.Tensor, device: torch.device):
        L = _lib.lib()
        self.c = _lib.TttjConfig.from_config(cfg, batch, seq_len)
        self.handle = ctypes.c_void_p()
        ws_bytes = L.tttj_workspace_bytes(ctypes.byref(self.c))
        if ws_bytes == 0:
            _lib.check(L.tttj_validate_config(ctypes.byref(self.c)), "plan")
        # Zero-filled once: rows a call does not write stay finite for later calls.
        self.workspace = torch.zeros(ws_bytes, dtype=torch.uint8, device=device)
        handle = ctypes.c_void_p()
        _lib.check(
            L.tttj_plan_create(ctypes.byref(self.c), device.index, ctypes.c_void_p(weights.data_ptr()),
                               ctypes.c_void_p(folded.data_ptr()),
                               ctypes.c_void_p(self.workspace.data_ptr()), ws_bytes,
                               ctypes.byref(handle)),
            "plan",
        )
        self.handle = handle

    def close(self) -> None:
        if self.handle:
            _lib.lib().tttj_plan_destroy(self.handle)
            self.handle = ctypes.c_void_p()

    def __del__(self):  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass


class B200Transformer(nn.Module):
    """Drop-in for the reference's optimized modules: ``forward(x, valid_token_mask=None)``.

    * ``x``: [B, S, d_model] fp16 or fp32 CUDA tensor on the parameter model's device
      (any B and S; a plan is built per shape on first use).
    * ``valid_token_mask``: optional bool [B, S]; None means every token is valid
      (kernels/sequence_resident.py:164-167).  Any bool mask is accepted, not only
      prefix masks.
    * returns a fresh [B, S, d_model] tensor in x's dtype; masked rows are exact zeros.
    """

    def __init__(self, parameter_model: nn.Module):
        super().__init__()
        cfg = parameter_model.config
        validate_model_config(cfg)
        params = list(parameter_model.parameters())
        if not params:
            raise ValueError("parameter model has no parameters")
        device = params[0].device
        if device.type != "cuda":
            raise ValueError("make_optimized_transformer: the parameter model must be on a CUDA device")
        if device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        self.config = cfg
        self.device = device
        # Keep a reference to the caller's model, as the reference adapter does
        # (kernels/sequence_resident.py:134-137).
        self.parameter_model = parameter_model
        with torch.cuda.device(device):
            self.register_buffer("packed_weights", pack_weights(parameter_model, device), persistent=False)
            self.register_buffer("folded_weights", fold_weights(cfg, self.packed_weights), persistent=False)
            # Plans are built on whichever stream first runs their shape: each waits
            # for the fold once (an event, no host synchronisation).
            self._weights_ready = torch.cuda.Event()
            self._weights_ready.record(torch.cuda.current_stream(device))
        self._plans: "OrderedDict[tuple[int, int], _Plan]" = OrderedDict()
        self._path = _lib.PATH_AUTO
        self.max_plans = self.DEFAULT_MAX_PLANS

    # Plans (workspace + descriptors) kept per module, least recently used evicted.
    DEFAULT_MAX_PLANS = 8

    def plan_for(self, batch: int, seq_len: int) -> _Plan:
        key = (batch, seq_len)
        plan = self._plans.get(key)
        if plan is not None:
            self._plans.move_to_end(key)
            return plan
        while len(self._plans) >= max(1, int(self.max_plans)):
            _, old = self._plans.popitem(last=False)
            old.close()  # waits for the evicted plan's last forward, then frees it
        torch.cuda.current_stream(self.device).wait_event(self._weights_ready)
        plan = _Plan(self.config, batch, seq_len, self.packed_weights, self.folded_weights, self.device)
        _lib.check(_lib.lib().tttj_plan_set_path(plan.handle, self._path), "set_path")
        self._plans[key] = plan
        return plan

    def cached_shapes(self) -> list[tuple[int, int]]:
        """(batch, seq_len) of the plans currently held, least recently used first."""
        return list(self._plans)

    def set_path(self, path: str) -> None:
        """Forward path for every shape: "auto" (default: the resident whole-stack
        kernel for short sequences of small layers, where it is faster, else layer by
        layer), "layerwise", or "resident" (whenever it fits; shapes it does not fit
        raise ValueError when their plan is built or used)."""
        if path not in _lib.PATHS:
            raise ValueError(f"path must be one of {sorted(_lib.PATHS)}, got {path!r}")
        new = _lib.PATHS[path]
        done = []
        try:
            for plan in self._plans.values():
                _lib.check(_lib.lib().tttj_plan_set_path(plan.handle, new), "set_path")
                done.append(plan)
        except Exception:
            for plan in done:  # all or nothing
                _lib.lib().tttj_plan_set_path(plan.handle, self._path)
            raise
        self._path = new

    def uses_resident(self, batch: int, seq_len: int) -> bool:
        """Whether a forward of shape [batch, seq_len] runs the resident-stack kernel."""
        return bool(_lib.lib().tttj_plan_path(self.plan_for(batch, seq_len).handle))

    def forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        if x.dim() != 3 or x.shape[-1] != self.config.d_model:
            raise ValueError(f"x must be [B, S, {self.config.d_model}], got {tuple(x.shape)}")
        if x.dtype not in _SUPPORTED_INPUT:
            raise ValueError(f"x dtype {x.dtype} unsupported (float16, float32)")
        if x.device != self.device:
            raise ValueError(f"x is on {x.device}, the model on {self.device}")
        B, S, _ = x.shape
        x = x.contiguous()
        mask_ptr = None
        mask = None
        if valid_token_mask is not None:
            if valid_token_mask.shape != (B, S):
                raise ValueError(f"valid_token_mask must be [{B}, {S}], got {tuple(valid_token_mask.shape)}")
            if valid_token_mask.device != self.device:
                raise ValueError("valid_token_mask must be on the model's device")
            mask = valid_token_mask
            if mask.dtype != torch.bool:
                mask = mask != 0
            mask = mask.contiguous().view(torch.uint8)
            mask_ptr = ctypes.c_void_p(mask.data_ptr())
        out = torch.empty_like(x)
        if B * S == 0:
            return out
        plan = self.plan_for(B, S)
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _lib.check(
            _lib.lib().tttj_forward(plan.handle, ctypes.c_void_p(x.data_ptr()), _SUPPORTED_INPUT[x.dtype],
                                    mask_ptr, ctypes.c_void_p(out.data_ptr()), ctypes.c_void_p(stream)),
            "forward",
        )
        return out

    # Stage names and shapes of the capture, as the reference's unpack_debug
    # (kernels/sequence_resident.py:28-46, 112-122) returns them.
    _DEBUG_STAGES = ("layernorm", "qkv.q", "qkv.k", "qkv.v", "scores", "softmax", "pv",
                     "output_projection", "ffn")

    def run(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None,
            capture_debug: bool = False, debug_layer: int = 0, debug_sequence: int = 0):
        """(output, stages or None), like the reference adapter's run(x, mask,
        capture_debug) (kernels/sequence_resident.py:158-225).  With capture_debug the
        forward runs layer by layer and also returns, for batch index ``debug_sequence``
        at block ``debug_layer`` (the reference: sequence 0, layer 0), a dict of fp32
        tensors: layernorm / qkv.q / qkv.k / qkv.v / pv / output_projection / ffn
        [S, D] and scores / softmax [H, S, S]; padded positions are zeros."""
        if not capture_debug:
            return self.forward(x, valid_token_mask), None
        B, S, D = x.shape
        H = self.config.num_heads
        plan = self.plan_for(B, S)
        n = int(_lib.lib().tttj_debug_floats(ctypes.byref(plan.c)))
        debug = torch.zeros(n, dtype=torch.float32, device=self.device)
        x = x.contiguous()
        mask = None
        if valid_token_mask is not None:
            mask = (valid_token_mask != 0).contiguous().view(torch.uint8)
        out = torch.empty_like(x)
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _lib.check(
            _lib.lib().tttj_forward_debug(plan.handle, ctypes.c_void_p(x.data_ptr()),
                                          _SUPPORTED_INPUT[x.dtype],
                                          None if mask is None else ctypes.c_void_p(mask.data_ptr()),
                                          ctypes.c_void_p(out.data_ptr()), int(debug_layer),
                                          int(debug_sequence), ctypes.c_void_p(debug.data_ptr()),
                                          ctypes.c_void_p(stream)),
            "forward_debug",
        )
        sizes = {"scores": (H, S, S), "softmax": (H, S, S)}
        stages, off = {}, 0
        for name in self._DEBUG_STAGES:
            shape = sizes.get(name, (S, D))
            count = 1
            for v in shape:
                count *= v
            stages[name] = debug[off:off + count].view(shape)
            off += count
        return out, stages

    def launches_per_forward(self, batch: int, seq_len: int) -> int:
        """Kernel launches one forward of shape [batch, seq_len] enqueues, given the same
        kind of mask (None or a tensor) as the last one of that shape."""
        return int(_lib.lib().tttj_plan_launch_count(self.plan_for(batch, seq_len).handle))

    def set_kernel_timing(self, batch: int, seq_len: int, enable: bool) -> None:
        """Record CUDA events around every kernel of later forwards of this shape."""
        plan = self.plan_for(batch, seq_len)
        _lib.check(_lib.lib().tttj_plan_enable_timing(plan.handle, 1 if enable else 0), "timing")

    def kernel_times(self, batch: int, seq_len: int) -> dict:
        """{kernel class: (total device ms, launches)} since timing was enabled."""
        plan = self.plan_for(batch, seq_len)
        ms = (ctypes.c_double * _lib.KCLASS_COUNT)()
        n = (ctypes.c_long * _lib.KCLASS_COUNT)()
        _lib.check(_lib.lib().tttj_plan_kernel_times(plan.handle, ms, n), "timing")
        L = _lib.lib()
        return {L.tttj_kernel_class_name(i).decode(): (float(ms[i]), int(n[i]))
                for i in range(_lib.KCLASS_COUNT)}

    def device_status(self) -> int:
        """Synchronise and read the device status word of every plan; raise
        RuntimeError if a bounded device wait gave up (returns 0 when healthy).
        Without this call, the next forward of the affected shape raises instead."""
        for plan in self._plans.values():
            v = ctypes.c_int(0)
            _lib.check(_lib.lib().tttj_plan_status(plan.handle, ctypes.byref(v)), "device status")
        return 0

    def selftest_device_timeout(self, batch: int, seq_len: int, limit_ns: int = 2_000_000) -> None:
        """Failure-detection self test: a bounded device wait on nothing gives up after
        ``limit_ns`` and reports through the plan of shape [batch, seq_len] exactly as a
        forward's kernel would, so that the next forward of that shape raises
        RuntimeError.  No GPU fault is involved."""
        plan = self.plan_for(batch, seq_len)
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _lib.check(_lib.lib().tttj_plan_selftest_timeout(plan.handle, int(limit_ns),
                                                         ctypes.c_void_p(stream)), "selftest")
