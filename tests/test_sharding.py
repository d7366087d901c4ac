"""CPU: batch sharding across ranks (the one-process-per-GPU layout) with gloo.

The forward itself needs a B200; these tests cover the host-side logic around it --
LPT partition, shard selection, all-gather reassembly -- with the fp32 oracle standing
in for the per-rank forward, and the failure path of a rank that dies mid-step.
"""
import multiprocessing as mp
import os
import socket
import time
from datetime import timedelta

import pytest
import torch

import optimized_transformer  # noqa: F401  (registers tttj_2026_b200 in spawned ranks too)
import tttj_2026_b200 as tb
from tttj_2026_b200 import sharding
from oracle import forward_fp32, state_dict_fp32


def test_lpt_partition_covers_each_item_once_and_balances():
    costs = [10, 9, 8, 7, 6, 5, 4, 3, 2, 1]
    bins = sharding.lpt_partition(costs, 3)
    flat = sorted(i for b in bins for i in b)
    assert flat == list(range(10))
    loads = [sum(costs[i] for i in b) for b in bins]
    assert max(loads) - min(loads) <= max(costs)
    assert bins == sharding.lpt_partition(costs, 3)  # deterministic
    for b in bins:
        assert b == sorted(b)


def test_lpt_more_parts_than_items():
    bins = sharding.lpt_partition([3.0, 1.0], 4)
    assert sorted(len(b) for b in bins) == [0, 0, 1, 1]


def test_sequence_costs_grow_with_length_and_causal_is_cheaper():
    c = sharding.sequence_costs([128, 256], 512, 2048, False)
    cc = sharding.sequence_costs([128, 256], 512, 2048, True)
    assert c[1] > 2 * c[0] * 0.99
    assert cc[1] < c[1]


def test_gather_shards_restores_batch_order():
    x = torch.arange(5 * 2 * 3, dtype=torch.float32).view(5, 2, 3)
    idx = [[0, 3], [1, 2, 4]]
    shards = [x[i] for i in idx]
    assert torch.equal(sharding.gather_shards(shards, idx, 5), x)


class _OracleModule(torch.nn.Module):
    """Stands in for one rank's B200Transformer: the fp32 oracle on the CPU."""

    def __init__(self, model):
        super().__init__()
        self.config = model.config
        self.p = state_dict_fp32(model)

    def forward(self, x, mask=None):
        return forward_fp32(self.p, self.config, x, mask)


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, mode, q):
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import optimized_transformer  # noqa: F401
    import torch.distributed as dist

    import tttj_2026_b200 as tbr
    from tttj_2026_b200 import sharding as sh

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=6))
    try:
        cfg = tbr.TransformerConfig(5, 24, 64, 2, 128, 2, True)
        model = tbr.make_parameter_model(cfg, 3, torch.float32, "cpu")
        x, mask = tbr.generate_inputs(cfg, 4, torch.float32, (1, 24), "cpu")
        mod = _OracleModule(model)
        if mode == "ok":
            out, idx = sh.distributed_forward(mod, x, mask)
            full = mod(x, mask)
            q.put((rank, "ok", float((out - full).abs().max()), [len(i) for i in idx]))
        elif mode == "dst":
            # Gather to rank 0 only: rank 0 gets the whole batch, the others None.
            out, idx = sh.distributed_forward(mod, x, mask, dst=0)
            mine = sh.local_shard(sh.lengths_of(mask, 5, 24), cfg, rank, world)
            assert mine == idx[rank]
            if rank == 0:
                full = mod(x, mask)
                q.put((rank, "ok", float((out - full).abs().max()), [len(i) for i in idx]))
            else:
                q.put((rank, "none" if out is None else "output", 0.0, [len(i) for i in idx]))
        else:
            # rank 1 dies before the gather; rank 0 must get an error, not hang
            if rank == 1:
                q.put((rank, "died", 0.0, []))
                q.close()
                q.join_thread()  # flush before the abrupt exit
                os._exit(3)
            t0 = time.time()
            try:
                sh.distributed_forward(mod, x, mask)
                q.put((rank, "no-error", time.time() - t0, []))
            except Exception as e:  # gloo reports the lost peer / timeout
                q.put((rank, "error:" + type(e).__name__, time.time() - t0, []))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = []
    deadline = time.time() + 120
    while len(results) < world and time.time() < deadline:
        try:
            results.append(q.get(timeout=5))
        except Exception:
            if not any(p.is_alive() for p in procs):
                break
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    return sorted(results)


def test_distributed_forward_two_ranks_matches_single_process():
    res = _run(2, "ok")
    assert len(res) == 2, res
    for rank, status, err, sizes in res:
        assert status == "ok"
        assert err == 0.0  # sequences are independent: sharding is exact
        assert sum(sizes) == 5


def test_distributed_forward_gathers_to_one_rank():
    res = _run(2, "dst")
    assert len(res) == 2, res
    assert res[0][1] == "ok" and res[0][2] == 0.0 and sum(res[0][3]) == 5
    assert res[1][1] == "none"


def test_rank_failure_surfaces_as_error_on_the_survivor():
    res = _run(2, "fail")
    by_rank = {r: (s, t) for r, s, t, _ in res}
    assert by_rank[1][0] == "died"
    assert by_rank[0][0].startswith("error:"), by_rank
    assert by_rank[0][1] < 60
