"""GPU: the module's forward captured into a CUDA graph and replayed.

The forward enqueues only kernels on the caller's stream, so torch.cuda.graph can
capture it once its plan exists (made by an ordinary forward first).  A captured
forward always rebuilds its token plan from the mask it was captured with (the graph
reads that mask tensor at every replay), so new inputs and new valid lengths written
into the captured tensors give the same outputs as eager forwards, bit for bit, on the
layer-by-layer path and on the resident one.
"""
import pytest
import torch

import tttj_2026_b200 as tb

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def _inputs(cfg, seed, lengths, dtype):
    g = torch.Generator().manual_seed(seed)
    B, S = cfg.batch_size, cfg.seq_len
    mask = (torch.arange(S)[None, :] < torch.tensor(lengths)[:, None]).to(DEV)
    x = torch.randn(B, S, cfg.d_model, generator=g).to(DEV, dtype).masked_fill(~mask[..., None], 0)
    return x, mask


@pytest.mark.parametrize("shape,path", [
    ((4, 200, 256, 4, 512, 2, True), "layerwise"),
    ((3, 96, 128, 2, 256, 2, False), "resident"),
])
def test_forward_replays_from_a_cuda_graph(shape, path):
    cfg = tb.TransformerConfig(*shape)
    B, S = cfg.batch_size, cfg.seq_len
    model = tb.make_parameter_model(cfg, 21, torch.float16, DEV)
    opt = tb.make_optimized_transformer(model)
    opt.set_path(path)
    x1, m1 = _inputs(cfg, 1, [S, S // 2, 7, S - 3][:B], torch.float16)
    x2, m2 = _inputs(cfg, 2, [S // 3, S, S - 1, 40][:B], torch.float16)
    with torch.inference_mode():
        ref1 = opt(x1, m1)  # also creates the plan
        ref2 = opt(x2, m2)
        ref_free = opt(x2)
        sx, sm = x1.clone(), m1.clone()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            sout = opt(sx, sm)
        free_graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(free_graph):
            sout_free = opt(sx)
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(sout, ref1)
        sx.copy_(x2)
        sm.copy_(m2)
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(sout, ref2)
        free_graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(sout_free, ref_free)
        # eager forwards after the replays still see their own masks
        again = opt(x1, m1)
        again_free = opt(x2)
    torch.cuda.synchronize()
    assert torch.equal(again, ref1)
    assert torch.equal(again_free, ref_free)
    assert opt.device_status() == 0
