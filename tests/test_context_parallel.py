"""Context parallelism (one sequence split across ranks).

CPU: the split rule and the per-layer exchange -- ``allgather_shares`` over gloo with
world size 2 puts every rank's q|k|v rows at their sequence positions -- and the
decomposition itself, restated on the fp32 oracle: token-sliced projections plus
attention of a rank's queries over the gathered keys equal the whole forward.
GPU (two devices, NCCL): ``ContextParallelTransformer`` against the single-GPU module
and the fp32 oracle, eager and replayed from CUDA graphs (identical outputs; the third
case leaves one rank without rows).
"""
import multiprocessing as mp
import os
import socket
import time
from datetime import timedelta

import pytest
import torch
import torch.nn.functional as F

import optimized_transformer  # noqa: F401  (registers tttj_2026_b200 in spawned ranks too)
import tttj_2026_b200 as tb
from tttj_2026_b200.context_parallel import cp_split, _cost


C4 = tb.TransformerConfig(1, 8192, 768, 12, 3072, 12, True)


@pytest.mark.parametrize("length", [8192, 6000, 4100, 300, 256, 255, 1])
@pytest.mark.parametrize("ranks", [1, 2, 4])
def test_cp_split_shares(length, ranks):
    shares = cp_split(length, C4, ranks)
    assert len(shares) == ranks
    assert shares[0][0] == 0
    for (a, b), (c, d) in zip(shares, shares[1:]):
        assert b == c  # contiguous
    assert shares[-1][1] == length or (shares[-1][0] == shares[-1][1] == length)
    sizes = [b - a for a, b in shares]
    assert sizes[0] == max(sizes)  # the all-gather slot layout
    for a, b in shares:
        assert a % 256 == 0 or a == length
        assert b % 256 == 0 or b == length


def test_cp_split_balances_causal_cost():
    (a0, b0), (a1, b1) = cp_split(8192, C4, 2)
    half = 4096
    c = lambda lo, hi: _cost(lo, hi, 8192, 768, 3072, True, 2.0)
    assert b0 > half  # the early tokens attend to fewer keys: the first rank takes more
    assert max(c(a0, b0), c(a1, b1)) < max(c(0, half), c(half, 8192))


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _attention_rows(q, k, v, H, q_lo, causal):
    """fp32 attention of query rows q (positions q_lo..) over keys k, v [len, D]."""
    n, D = q.shape
    hd = D // H
    qh = q.view(n, H, hd).transpose(0, 1)
    kh = k.view(-1, H, hd).transpose(0, 1)
    vh = v.view(-1, H, hd).transpose(0, 1)
    s = qh @ kh.transpose(-1, -2) * hd ** -0.5
    if causal:
        pos_q = torch.arange(q_lo, q_lo + n)[:, None]
        pos_k = torch.arange(k.shape[0])[None, :]
        s = s.masked_fill(pos_k > pos_q, float("-inf"))
    return (torch.softmax(s, -1) @ vh).transpose(0, 1).reshape(n, D)


def _rank_main(rank, world, port, q):
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    import optimized_transformer  # noqa: F401
    import torch.distributed as dist

    import tttj_2026_b200 as tbr
    from oracle import forward_fp32, state_dict_fp32
    from tttj_2026_b200.context_parallel import allgather_shares, cp_split as split

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    try:
        # 1) the exchange layout: rank r fills its rows (value = sequence position).
        length, row_bytes = 700, 12
        shares = split(length, tbr.TransformerConfig(1, 1024, 64, 2, 128, 1, True), world)
        slot = max(b - a for a, b in shares)
        buf = torch.zeros(16 + world * slot * row_bytes, dtype=torch.uint8)
        lo, hi = shares[rank]
        rows = buf[16:16 + world * slot * row_bytes].view(world * slot, row_bytes)
        for r in range(lo, hi):
            rows[r] = r % 251
        allgather_shares(buf, 16, row_bytes, slot, None)
        ok_layout = all(int(rows[r, 0]) == r % 251 for r in range(length))

        # 2) the decomposition on the fp32 oracle: token-sliced projections, gathered
        #    k / v, attention of this rank's queries; equals the whole forward.
        torch.set_grad_enabled(False)
        cfg = tbr.TransformerConfig(1, 600, 64, 2, 128, 2, True)
        model = tbr.make_parameter_model(cfg, 3, torch.float32, "cpu")
        x, _ = tbr.generate_inputs(cfg, 4, torch.float32, None, "cpu")
        full = forward_fp32(state_dict_fp32(model, "cpu"), cfg, x, None)[0]
        shares = split(600, cfg, world)
        lo, hi = shares[rank]
        h = x[0, lo:hi].clone()
        for blk in model.layers:
            a = blk.attention
            hn = F.layer_norm(h, (64,), blk.norm1.weight, blk.norm1.bias, 1e-5)
            qkv = torch.cat([F.linear(hn, a.q_proj.weight, a.q_proj.bias),
                             F.linear(hn, a.k_proj.weight, a.k_proj.bias),
                             F.linear(hn, a.v_proj.weight, a.v_proj.bias)], 1)
            slot = max(b - a_ for a_, b in shares)
            gathered = torch.zeros(world * slot, qkv.shape[1])
            mine = torch.zeros(slot, qkv.shape[1])
            mine[: hi - lo] = qkv
            dist.all_gather_into_tensor(gathered, mine)
            k, v = gathered[:600, 64:128], gathered[:600, 128:]
            ctx = _attention_rows(qkv[:, :64], k, v, 2, lo, True)
            h = h + F.linear(ctx, a.out_proj.weight, a.out_proj.bias)
            hn = F.layer_norm(h, (64,), blk.norm2.weight, blk.norm2.bias, 1e-5)
            h = h + F.linear(F.gelu(F.linear(hn, blk.ffn_in.weight, blk.ffn_in.bias)),
                             blk.ffn_out.weight, blk.ffn_out.bias)
        h = F.layer_norm(h, (64,), model.final_norm.weight, model.final_norm.bias, 1e-5)
        err = float((h - full[lo:hi]).abs().max())
        q.put((rank, ok_layout, err))
    finally:
        dist.destroy_process_group()


def test_exchange_and_decomposition_two_ranks_gloo():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = []
    deadline = time.time() + 120
    while len(res) < 2 and time.time() < deadline:
        try:
            res.append(q.get(timeout=5))
        except Exception:
            if not any(p.is_alive() for p in procs):
                break
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert len(res) == 2, res
    for rank, ok_layout, err in res:
        assert ok_layout
        assert err < 1e-4, (rank, err)


def _gpu_rank_main(rank, world, port, q):
    import sys

    here = os.path.dirname(os.path.abspath(__file__))
    sys.path.insert(0, os.path.dirname(here))
    sys.path.insert(0, here)
    import optimized_transformer  # noqa: F401
    import torch.distributed as dist

    import tttj_2026_b200 as tbr
    from helpers import gate
    from oracle import forward_fp32_per_sequence, state_dict_fp32
    from tttj_2026_b200.context_parallel import ContextParallelTransformer

    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=dev)
    try:
        results = []
        for causal, length, seed in ((True, 3000, 1), (False, 2500, 2), (True, 256, 3)):
            cfg = tbr.TransformerConfig(1, 3072, 768, 12, 3072, 2, causal)
            model = tbr.make_parameter_model(cfg, seed, torch.float16, dev)
            x, _ = tbr.generate_inputs(cfg, seed + 10, torch.float16, None, dev)
            mask = torch.arange(3072, device=dev)[None, :] < length
            x = x.masked_fill(~mask[..., None], 0)
            cp = ContextParallelTransformer(model, None)
            cpg = ContextParallelTransformer(model, None, graphs=True)
            single = tbr.make_optimized_transformer(model)
            with torch.inference_mode():
                out = cp(x, mask)
                again = cp(x, mask)
                # graph replays (captured on the first call), the length given by the caller
                g1 = cpg(x, mask, length=length)
                g2 = cpg(x, mask, length=length)
                ref1 = single(x, mask)
                ref = forward_fp32_per_sequence(state_dict_fp32(model, dev), cfg, x.float(), mask)
            torch.cuda.synchronize(dev)
            cpg.close()
            r = gate(ref, out, mask)
            d = float((out.float() - ref1.float()).abs().max())
            results.append((causal, length, r.passed, r.max_abs, r.mean_abs, d,
                            bool(torch.equal(out, again) and torch.equal(out, g1) and
                                 torch.equal(out, g2))))
        q.put((rank, results))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_context_parallel_two_gpus_matches_single_gpu_and_oracle():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gpu_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = []
    deadline = time.time() + 300
    while len(res) < 2 and time.time() < deadline:
        try:
            res.append(q.get(timeout=5))
        except Exception:
            if not any(p.is_alive() for p in procs):
                break
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert len(res) == 2, res
    for rank, results in res:
        for causal, length, passed, max_abs, mean_abs, diff_single, repeat_equal in results:
            assert passed, (rank, causal, length, max_abs, mean_abs)
            assert repeat_equal
            # The ranks' GEMM tiles differ from the single GPU's (fewer rows), which
            # regroups the LayerNorm statistics: agreement to about two fp16 ulps.
            assert diff_single < 2e-2, (rank, causal, length, diff_single)


def test_graph_mode_ranks_with_and_without_rows_run_the_same_collectives(monkeypatch):
    """With graphs, a rank that holds rows runs an eager forward, captures one and
    replays it on the first call for a length (a replay afterwards); a rank without rows
    must run the same exchanges in the same order, or NCCL's collectives pair up wrongly
    and the group hangs until its timeout.  Checked on the host with a fake graph that
    records the exchanges called while capturing and runs them at replay."""
    import types
    from contextlib import contextmanager
    from tttj_2026_b200 import context_parallel as cpm

    L = 3
    state = {"capture": None}

    class FakeGraph:
        def __init__(self):
            self.recorded = []

        def replay(self):
            for f in self.recorded:
                f()

    @contextmanager
    def fake_graph(g):
        state["capture"] = g
        try:
            yield
        finally:
            state["capture"] = None

    monkeypatch.setattr(torch.cuda, "CUDAGraph", FakeGraph)
    monkeypatch.setattr(torch.cuda, "graph", fake_graph)

    def make(rank, log):
        def exchange(*_a, **_k):
            if state["capture"] is not None:
                state["capture"].recorded.append(lambda: log.append("allgather"))
            else:
                log.append("allgather")

        monkeypatch.setattr(cpm, "allgather_shares", exchange)
        m = cpm.ContextParallelTransformer.__new__(cpm.ContextParallelTransformer)
        torch.nn.Module.__init__(m)
        m.config = types.SimpleNamespace(num_layers=L, d_model=64, num_heads=2, ffn_dim=128,
                                         causal=True)
        m.device, m.group, m.rank, m.world = torch.device("cpu"), None, rank, 2
        m.graphs, m._graphs, m._plans, m._exchange_error = True, {}, {}, None
        m._plan = lambda *a: types.SimpleNamespace()
        m._run = lambda plan, xl, out, slot: [exchange() for _ in range(L)]
        return m

    def calls(rank, length):
        log = []
        m = make(rank, log)
        x = torch.zeros(1, 600, 64)
        for _ in range(2):
            m(x, None, gather=False, length=length)
            log.append("|")
        return log

    # 300 tokens: one 256-row item each (rank 1 rows 256..299); 200 tokens: rank 1 has none.
    assert calls(0, 300) == calls(1, 300)
    assert calls(0, 200) == calls(1, 200)
    log = calls(0, 200)
    assert log.count("allgather") == 3 * L  # eager + replay on the first call, replay after
