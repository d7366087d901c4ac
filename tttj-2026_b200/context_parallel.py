"""Context parallelism: one sequence split across the ranks of a process group.

Batch sharding (``sharding.py``) leaves GPUs idle when a batch has fewer sequences than
GPUs -- the north star's C4 (4 sequences of 8192 tokens) on 8 GPUs.  Here the valid
tokens of one sequence are shared out between the ranks of a group in contiguous
slices: every GEMM of the stack (QKV, out_proj, ffn_in, ffn_out), the LayerNorms, the
residual stream and the final LayerNorm run on a rank's own rows only, and one exchange
per layer -- an in-place all-gather of the ranks' q|k|v rows right after the QKV GEMM
-- gives every rank the whole sequence's keys and values for its attention (its own
queries against all keys they may see), which is therefore exact.  The reference has
no multi-GPU path; its long-sequence answer on one GPU is query-chunked attention
(kernels/case14_hybrid.py:565-630), of which this is the multi-GPU counterpart.

* ``cp_split`` chooses the slices: contiguous, each boundary on an attention work
  item (256 rows), the first slice the largest (so the all-gather of equal-sized slots
  lands every rank's rows at their sequence positions), and balanced by predicted cost
  -- projection FLOPs grow with the tokens, causal attention with their positions, so
  the first rank takes more tokens (two ranks) -- or equal slots (more ranks).
* ``allgather_shares`` is the exchange: an in-place ``all_gather_into_tensor`` of the
  ranks' slots of the plan's q|k|v buffer (NCCL over NVLink on a B200 node; any backend
  for CPU tensors), enqueued on the current stream.
* ``ContextParallelTransformer`` runs a split forward through the C ABI
  (``tttj_plan_create_cp`` / ``tttj_forward_cp``), calling the exchange once per layer.
  With ``graphs=True`` each (valid length, dtype) is captured once into a CUDA graph --
  the forward's kernels and its per-layer all-gathers -- and replayed: the eager forward
  re-enters Python at every layer's exchange, and at C4's shape (~0.1 ms of device work
  per layer and rank) that host time can set the pace instead of the GPUs.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch
import torch.nn as nn

from . import _lib


def _cost(lo: int, hi: int, length: int, d_model: int, ffn_dim: int, causal: bool,
          attention_weight: float) -> float:
    """Predicted cost of rows [lo, hi): 2 (4 D^2 + 2 D F) projection FLOPs per row plus
    4 D FLOPs per attended (query, key) pair, the latter weighted by how much slower
    the attention runs than the GEMMs."""
    rows = hi - lo
    if causal:
        pairs = (hi * (hi + 1) - lo * (lo + 1)) / 2.0
    else:
        pairs = float(rows) * length
    return 2.0 * rows * (4 * d_model * d_model + 2 * d_model * ffn_dim) + \
        attention_weight * 4.0 * d_model * pairs


def cp_split(length: int, cfg, ranks: int, item: int = 256,
             attention_weight: float = 2.0) -> list[tuple[int, int]]:
    """Contiguous shares [lo, hi) of the valid tokens [0, length) for ``ranks`` ranks.

    Every boundary is a multiple of ``item`` and the first share is the largest, which
    the in-place all-gather layout needs (rank r's slot starts at r * m, m = the first
    share's size, and must start at its rows' sequence position).  Two ranks: the split
    point that best balances the predicted cost.  More ranks: equal slots of m rows
    (the last one shorter).  Ranks without rows get an empty share (lo == hi)."""
    if ranks <= 0:
        raise ValueError("ranks must be positive")
    if length <= 0:
        return [(0, 0)] * ranks
    d, f, causal = int(cfg.d_model), int(cfg.ffn_dim), bool(cfg.causal)
    if ranks == 1:
        return [(0, length)]
    if ranks == 2:
        best, best_cost = None, None
        lo_split = -(-length // 2)  # the first share is at least half
        s = -(-lo_split // item) * item
        while s < length:
            c = max(_cost(0, s, length, d, f, causal, attention_weight),
                    _cost(s, length, length, d, f, causal, attention_weight))
            if best_cost is None or c < best_cost:
                best, best_cost = s, c
            s += item
        if best is None:  # too short to split on an item boundary: one rank runs it all
            return [(0, length), (length, length)]
        return [(0, best), (best, length)]
    m = -(-length // ranks)
    m = -(-m // item) * item
    shares = []
    for r in range(ranks):
        lo = min(r * m, length)
        shares.append((lo, min(lo + m, length)))
    return shares


def allgather_shares(buffer: torch.Tensor, offset: int, row_bytes: int, slot_rows: int,
                     group=None) -> None:
    """In-place all-gather of the ranks' q|k|v slots: rank r's ``slot_rows`` rows of
    ``row_bytes`` bytes start at byte ``offset + r * slot_rows * row_bytes`` of the uint8
    ``buffer``; afterwards every rank holds every slot.  Enqueued on the current
    stream (torch.distributed, any backend)."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    slot = slot_rows * row_bytes
    full = buffer[offset: offset + world * slot]
    dist.all_gather_into_tensor(full, full[rank * slot: (rank + 1) * slot], group=group)


class _CpPlan:
    """A split plan of the C library for one (valid length, share) of a sequence."""

    def __init__(self, cfg, length: int, lo: int, hi: int, full_rows: int,
                 weights: torch.Tensor, folded: torch.Tensor, device: torch.device):
        L = _lib.lib()
        self.c = _lib.TttjConfig.from_config(cfg, 1, hi - lo)
        self.handle = ctypes.c_void_p()
        nbytes = L.tttj_workspace_bytes_cp(ctypes.byref(self.c), full_rows)
        if nbytes == 0:
            _lib.check(L.tttj_validate_config(ctypes.byref(self.c)), "plan_cp")
        self.workspace = torch.zeros(nbytes, dtype=torch.uint8, device=device)
        handle = ctypes.c_void_p()
        _lib.check(L.tttj_plan_create_cp(ctypes.byref(self.c), device.index,
                                         ctypes.c_void_p(weights.data_ptr()),
                                         ctypes.c_void_p(folded.data_ptr()), length, lo, full_rows,
                                         ctypes.c_void_p(self.workspace.data_ptr()), nbytes,
                                         ctypes.byref(handle)), "plan_cp")
        self.handle = handle
        off, row_bytes, rows = ctypes.c_size_t(), ctypes.c_size_t(), ctypes.c_int()
        _lib.check(L.tttj_plan_cp_qkv(handle, ctypes.byref(off), ctypes.byref(row_bytes),
                                      ctypes.byref(rows)), "plan_cp")
        self.qkv_offset, self.row_bytes = off.value, row_bytes.value

    def close(self) -> None:
        if self.handle:
            _lib.lib().tttj_plan_destroy(self.handle)
            self.handle = ctypes.c_void_p()

    def __del__(self):  # pragma: no cover - interpreter shutdown order
        try:
            self.close()
        except Exception:
            pass


class ContextParallelTransformer(nn.Module):
    """One sequence per call, its valid tokens split across the ranks of ``group``.

    ``forward(x, valid_token_mask)`` takes the same [1, S, D] input (and prefix mask, or
    None) on every rank of the group and returns the whole [1, S, D] output on every
    rank (``gather=True``; padded rows exact zeros) or this rank's rows
    ``(lo, hi, rows)`` (``gather=False``).  Each rank holds the full weights (packed and
    LayerNorm-folded once, as ``make_optimized_transformer`` does).
    """

    def __init__(self, parameter_model: nn.Module, group=None, graphs: bool = False):
        super().__init__()
        import torch.distributed as dist
        from .model import B200Transformer

        self.base = B200Transformer(parameter_model)
        self.config = self.base.config
        self.device = self.base.device
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self._plans: dict[tuple[int, int, int, int], _CpPlan] = {}
        self._exchange_error: Optional[BaseException] = None
        self.graphs = graphs
        # (length, dtype) -> (graph, static input rows, static output rows);
        # ("idle", length) -> (graph, buffer) for a rank without rows
        self._graphs: dict = {}

    def close(self) -> None:
        """Release the captured graphs (they hold NCCL calls: release them before
        ``destroy_process_group``) and the split plans."""
        self._graphs.clear()
        for plan in self._plans.values():
            plan.close()
        self._plans.clear()

    def shares(self, length: int) -> list[tuple[int, int]]:
        hd = self.config.d_model // self.config.num_heads
        item = 128 if hd > 128 else 256
        return cp_split(length, self.config, self.world, item)

    def _plan(self, length: int, lo: int, hi: int, full_rows: int) -> _CpPlan:
        key = (length, lo, hi, full_rows)
        plan = self._plans.get(key)
        if plan is None:
            torch.cuda.current_stream(self.device).wait_event(self.base._weights_ready)
            plan = _CpPlan(self.config, length, lo, hi, full_rows, self.base.packed_weights,
                           self.base.folded_weights, self.device)
            self._plans[key] = plan
        return plan

    def _run(self, plan: _CpPlan, xl: torch.Tensor, out_local: torch.Tensor, slot: int) -> None:
        """One split forward of the rank's rows xl into out_local on the current stream,
        the exchange called back once per layer."""
        stream = torch.cuda.current_stream(self.device)

        def exchange(_user, _layer, _stream):
            try:
                allgather_shares(plan.workspace, plan.qkv_offset, plan.row_bytes, slot,
                                 self.group)
                return 0
            except BaseException as e:  # reported after the C call returns
                self._exchange_error = e
                return 1

        cb = _lib.EXCHANGE_FN(exchange)
        rc = _lib.lib().tttj_forward_cp(plan.handle, ctypes.c_void_p(xl.data_ptr()),
                                        _lib.DTYPE_F16 if xl.dtype == torch.float16 else _lib.DTYPE_F32,
                                        ctypes.c_void_p(out_local.data_ptr()), cb, None,
                                        ctypes.c_void_p(stream.cuda_stream))
        if self._exchange_error is not None:
            err, self._exchange_error = self._exchange_error, None
            raise RuntimeError("context-parallel exchange failed") from err
        _lib.check(rc, "forward_cp")

    def _graph(self, plan: _CpPlan, length: int, rows: int, dtype, slot: int):
        """The captured split forward for (length, dtype): on its first use an eager
        forward (it builds the split plan's token plans, which replays reuse, and brings
        up the group's communicator), then the capture."""
        key = (length, dtype)
        entry = self._graphs.get(key)
        if entry is None:
            static_x = torch.zeros((rows, self.config.d_model), dtype=dtype, device=self.device)
            static_out = torch.zeros_like(static_x)
            self._run(plan, static_x, static_out, slot)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                self._run(plan, static_x, static_out, slot)
            entry = (graph, static_x, static_out)
            self._graphs[key] = entry
        return entry

    def _idle(self, length: int, slot: int) -> None:
        """A rank without rows (a sequence shorter than one work item per rank) still
        takes part in every layer's exchange, with the same collectives in the same
        order as its peers: eagerly, or -- with graphs -- an eager pass, a captured one
        and a replay on the first call for a length (what a peer's _graph and replay
        run), a replay afterwards."""
        row_bytes = 3 * self._qkv_width() * 2
        if not self.graphs:
            buf = torch.zeros(slot * self.world * row_bytes, dtype=torch.uint8, device=self.device)
            for _ in range(self.config.num_layers):
                allgather_shares(buf, 0, row_bytes, slot, self.group)
            return
        key = ("idle", length)
        entry = self._graphs.get(key)
        if entry is None:
            buf = torch.zeros(slot * self.world * row_bytes, dtype=torch.uint8, device=self.device)
            for _ in range(self.config.num_layers):
                allgather_shares(buf, 0, row_bytes, slot, self.group)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for _ in range(self.config.num_layers):
                    allgather_shares(buf, 0, row_bytes, slot, self.group)
            entry = (graph, buf)
            self._graphs[key] = entry
        entry[0].replay()

    def forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None,
                gather: bool = True, length: Optional[int] = None):
        """``length``: the number of valid tokens when the caller knows it (skips reading
        the mask back to the host, which waits for the device)."""
        import torch.distributed as dist

        if x.dim() != 3 or x.shape[0] != 1 or x.shape[2] != self.config.d_model:
            raise ValueError(f"x must be [1, S, {self.config.d_model}], got {tuple(x.shape)}")
        S = x.shape[1]
        if length is not None:
            length = int(length)
            if not 0 <= length <= S:
                raise ValueError(f"length {length} outside [0, {S}]")
        elif valid_token_mask is None:
            length = S
        else:
            m = valid_token_mask.reshape(-1).to(torch.bool)
            length = int(m.sum())
            if not bool(m[:length].all()):
                raise ValueError("context parallelism needs a prefix valid_token_mask")
        shares = self.shares(length)
        slot = max(hi - lo for lo, hi in shares)
        lo, hi = shares[self.rank]
        if hi > lo:
            plan = self._plan(length, lo, hi, slot * self.world)
            if self.graphs:
                graph, static_x, static_out = self._graph(plan, length, hi - lo, x.dtype, slot)
                static_x.copy_(x[0, lo:hi])
                graph.replay()
                out_local = static_out.clone()
            else:
                out_local = x.new_zeros((hi - lo, x.shape[2]))
                self._run(plan, x[0, lo:hi].contiguous(), out_local, slot)
        else:
            out_local = x.new_zeros((0, x.shape[2]))
            self._idle(length, slot)
        if not gather:
            return lo, hi, out_local
        pad = x.new_zeros((slot, x.shape[2]))
        pad[: hi - lo] = out_local
        full = x.new_zeros((self.world * slot, x.shape[2]))
        dist.all_gather_into_tensor(full, pad, group=self.group)
        out = x.new_zeros(x.shape)
        for r, (a, b) in enumerate(shares):
            if b > a:
                out[0, a:b] = full[r * slot: r * slot + (b - a)]
        return out

    def _qkv_width(self) -> int:
        hd = self.config.d_model // self.config.num_heads
        hp = 32 if hd <= 32 else 64 if hd <= 64 else 128 if hd <= 128 else 256
        return self.config.num_heads * hp
