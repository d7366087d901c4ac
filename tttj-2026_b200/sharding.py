"""Batch data parallelism across the GPUs of one node.

Sequences never interact in this transformer (attention is per sequence, every other
op is per token), so the batch shards exactly: each GPU runs the whole stack on its
own sequences with its own replica of the weights, and no collective runs inside the
forward.  The reference has no multi-GPU path; this follows the batch-sharded plan of
its north star.

* ``sequence_costs`` predicts each sequence's forward cost from its valid length
  (projection FLOPs ~ len, attention FLOPs ~ len^2, causal halves the latter).
* ``lpt_partition`` assigns sequences to shards longest-processing-time first, so
  padded batches with ragged lengths still balance.
* ``shard_indices`` / ``local_shard`` / ``gather_shards`` / ``distributed_forward``: the
  one-process-per-GPU layout (torch.distributed): every rank selects its sequences,
  runs its replica, and the outputs are reassembled in the original batch order on
  the caller's request (all_gather to every rank, or a gather to one rank).
* ``MultiDeviceTransformer``: one process driving several GPUs -- replicas on each
  device, peer copies of the shards, per-device streams, gather on the caller's device.
"""
from __future__ import annotations

from typing import Optional, Sequence

import torch


def sequence_costs(lengths: Sequence[int], d_model: int, ffn_dim: int, causal: bool) -> list[float]:
    """Relative forward cost of each sequence: 2*len*(4D^2 + 2DF) projection FLOPs plus
    4*D*pairs attention FLOPs (pairs = len^2, or len(len+1)/2 when causal)."""
    out = []
    for n in lengths:
        n = int(n)
        pairs = n * (n + 1) / 2 if causal else float(n * n)
        out.append(2.0 * n * (4 * d_model * d_model + 2 * d_model * ffn_dim) + 4.0 * d_model * pairs)
    return out


def lpt_partition(costs: Sequence[float], parts: int) -> list[list[int]]:
    """Greedy longest-processing-time partition of item indices into ``parts`` bins.

    Items are taken in decreasing cost (ties by index) and each goes to the bin with
    the smallest load so far (ties by bin index).  Each bin's indices are returned in
    increasing order, so a bin's sequences keep their batch order.  Deterministic.
    """
    if parts <= 0:
        raise ValueError("parts must be positive")
    order = sorted(range(len(costs)), key=lambda i: (-float(costs[i]), i))
    load = [0.0] * parts
    bins: list[list[int]] = [[] for _ in range(parts)]
    for i in order:
        b = min(range(parts), key=lambda j: (load[j], j))
        bins[b].append(i)
        load[b] += float(costs[i])
    return [sorted(b) for b in bins]


def lengths_of(valid_token_mask: Optional[torch.Tensor], batch: int, seq_len: int) -> list[int]:
    if valid_token_mask is None:
        return [seq_len] * batch
    return [int(v) for v in valid_token_mask.sum(dim=1).tolist()]


def shard_indices(lengths: Sequence[int], cfg, world_size: int) -> list[list[int]]:
    """Per-rank sequence indices for ``world_size`` ranks (LPT by predicted cost)."""
    return lpt_partition(sequence_costs(lengths, cfg.d_model, cfg.ffn_dim, bool(cfg.causal)), world_size)


def gather_shards(shards: Sequence[torch.Tensor], indices: Sequence[Sequence[int]], batch: int) -> torch.Tensor:
    """Reassemble per-shard outputs [n_r, S, D] into [batch, S, D] in batch order."""
    ref = next(t for t in shards if t is not None)
    out = torch.empty((batch,) + tuple(ref.shape[1:]), dtype=ref.dtype, device=ref.device)
    for t, idx in zip(shards, indices):
        if len(idx) == 0:
            continue
        out[torch.as_tensor(list(idx), device=out.device)] = t.to(out.device)
    return out


def local_shard(lengths: Sequence[int], cfg, rank: int, world_size: int) -> list[int]:
    """Sequence indices rank ``rank`` of ``world_size`` runs (its LPT share, batch order).
    A serving process that feeds only its own sequences selects them with this."""
    return shard_indices(lengths, cfg, world_size)[rank]


def distributed_forward(module, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor],
                        group=None, gather: bool = True, dst: Optional[int] = None):
    """One-process-per-GPU forward: every rank holds the full batch (or the same
    seeded inputs), runs only its LPT shard on its own GPU, and -- if ``gather`` --
    collects the shard outputs into the full [B, S, D] output in batch order:
    on every rank (``dst`` None: all_gather) or on rank ``dst`` only (a gather; the
    other ranks return None for the output).  Returns (output, shard indices).

    ``module`` is this rank's B200Transformer.  The collectives move fixed-size padded
    shard buffers (torch.distributed, any backend; NCCL over NVLink on a B200 node).
    """
    import torch.distributed as dist

    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    B, S, D = x.shape
    idx = shard_indices(lengths_of(valid_token_mask, B, S), module.config, world)
    mine = idx[rank]
    if len(mine):
        sel = torch.as_tensor(mine, device=x.device)
        xm = x.index_select(0, sel).contiguous()
        mm = None if valid_token_mask is None else valid_token_mask.index_select(0, sel).contiguous()
        local = module(xm, mm)
    else:
        local = x.new_empty((0, S, D))
    if not gather:
        return local, idx
    cap = max(len(i) for i in idx)
    buf = x.new_zeros((cap, S, D)) if len(mine) < cap else local
    if len(mine) < cap and len(mine):
        buf[: len(mine)] = local
    if dst is None:
        bufs = [torch.empty_like(buf) for _ in range(world)]
        dist.all_gather(bufs, buf, group=group)
    else:
        bufs = [torch.empty_like(buf) for _ in range(world)] if rank == dst else None
        dist.gather(buf, bufs, dst=dst, group=group)
        if rank != dst:
            return None, idx
    shards = [b[: len(i)] for b, i in zip(bufs, idx)]
    return gather_shards(shards, idx, B), idx


class MultiDeviceTransformer(torch.nn.Module):
    """One process, several GPUs: a B200Transformer replica per device.

    forward(x, mask) on x resident on ``devices[0]``: the batch is split LPT across
    the devices, each shard is copied peer-to-peer to its device, every replica runs
    on its own stream, and the outputs are copied back into one tensor on
    ``devices[0]``.  Callers see a synchronous module on the caller's stream.
    """

    def __init__(self, parameter_model: torch.nn.Module, devices: Sequence[int]):
        super().__init__()
        from .model import B200Transformer

        if not devices:
            raise ValueError("devices must not be empty")
        self.devices = [torch.device("cuda", int(d)) for d in devices]
        self.config = parameter_model.config
        self.replicas = []
        for dev in self.devices:
            with torch.cuda.device(dev):
                self.replicas.append(B200Transformer(parameter_model.to(dev)))
        parameter_model.to(self.devices[0])
        self.streams = [torch.cuda.Stream(device=d) for d in self.devices]

    def forward(self, x: torch.Tensor, valid_token_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
        B, S, D = x.shape
        idx = shard_indices(lengths_of(valid_token_mask, B, S), self.config, len(self.devices))
        out = torch.empty_like(x)
        caller = torch.cuda.current_stream(x.device)
        ready = torch.cuda.Event()
        ready.record(caller)
        done = []
        for rep, dev, stream, sel in zip(self.replicas, self.devices, self.streams, idx):
            if not sel:
                continue
            with torch.cuda.device(dev), torch.cuda.stream(stream):
                stream.wait_event(ready)
                sel_t = torch.as_tensor(sel, device=x.device)
                xs = x.index_select(0, sel_t).to(dev, non_blocking=True)
                ms = None
                if valid_token_mask is not None:
                    ms = valid_token_mask.index_select(0, sel_t).to(dev, non_blocking=True)
                ys = rep(xs, ms)
                out.index_copy_(0, sel_t, ys.to(x.device, non_blocking=True))
                ev = torch.cuda.Event()
                ev.record(stream)
                done.append(ev)
        for ev in done:
            caller.wait_event(ev)
        return out
