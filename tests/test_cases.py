"""CPU: the reference case table (optimized_transformer.py:22-42) and its lookup
(:45-66), and that the library accepts every case's configuration."""
import ctypes

import pytest
import torch

import tttj_2026_b200 as tb
from tttj_2026_b200 import _lib, cases


def test_case_table_shape():
    assert sorted(cases.IMPLEMENTED_CASES) == list(range(1, 15))
    assert all(cases.IMPLEMENTED_CASE_LAYERS[n] == (2 if n == 14 else 4) for n in range(1, 15))
    # Head widths the cases need: 8 (7, 11), 32, 64 (10, 14), 128 (9), 256 (8).
    hds = {n: d // h for n, (_, _, d, h) in cases.IMPLEMENTED_CASES.items()}
    assert {hds[7], hds[11], hds[9], hds[8], hds[10], hds[14], hds[1]} == {8, 128, 256, 64, 32}


@pytest.mark.parametrize("n", list(range(1, 15)))
def test_every_case_is_supported_and_looked_up(n):
    cfg = cases.case_config(n)
    c = _lib.TttjConfig.from_config(cfg)
    lib = _lib.lib()
    assert lib.tttj_validate_config(ctypes.byref(c)) == 0, lib.tttj_last_error()
    assert lib.tttj_weights_bytes(ctypes.byref(c)) > 0
    assert lib.tttj_workspace_bytes(ctypes.byref(c)) > 0
    tb.validate_model_config(cfg)

    class _M:
        config = cfg

    assert cases.case_number_for_model(_M()) == n


def test_case_lookup_rejects_other_shapes():
    class _M:
        config = tb.TransformerConfig(64, 128, 128, 4, 256, 4, True)  # F != D

    with pytest.raises(ValueError, match="no optimized transformer"):
        cases.case_number_for_model(_M())


def test_padded_heads_workspace_holds_the_padded_layout():
    """hd 8 runs on 32-column layout heads: the workspace grows by the padded q/k/v and
    context columns, the folded weights by the padded QKV rows and the padded out_proj
    weight, and nothing else changes."""
    lib = _lib.lib()
    base = tb.TransformerConfig(4, 128, 128, 4, 128, 1, True)   # hd 32, unpadded
    pad = tb.TransformerConfig(4, 128, 128, 16, 128, 1, True)   # hd 8, padded x4
    cb, cp = _lib.TttjConfig.from_config(base), _lib.TttjConfig.from_config(pad)
    ws_base = lib.tttj_workspace_bytes(ctypes.byref(cb))
    ws_pad = lib.tttj_workspace_bytes(ctypes.byref(cp))
    T, D, Q = 4 * 128, 128, 16 * 32
    extra = T * 3 * (Q - D) * 2 + T * (Q - D) * 2
    # 16 heads instead of 4 also lengthen the attention work list (8 bytes per item).
    extra += 4 * (16 - 4) * 1 * 8
    assert abs((ws_pad - ws_base) - extra) <= 8 * 256  # alignment slack
    fold_extra = 3 * (Q - D) * (D * 2 + 8) + D * Q * 2
    f_base = lib.tttj_folded_bytes(ctypes.byref(cb))
    f_pad = lib.tttj_folded_bytes(ctypes.byref(cp))
    assert abs((f_pad - f_base) - fold_extra) <= 8 * 256
    # The packed weights are the caller's unpadded layout either way.
    w_base = lib.tttj_weights_bytes(ctypes.byref(_lib.TttjConfig.from_config(base)))
    w_pad = lib.tttj_weights_bytes(ctypes.byref(_lib.TttjConfig.from_config(pad)))
    assert w_base == w_pad


def test_case_inputs_follow_the_reference_padding_rule():
    cfg = cases.case_config(1)
    x, mask = cases.case_inputs(cfg, 7, 0.25)
    lens = mask.sum(1)
    assert int(lens.min()) >= round(128 * 0.75) and int(lens.max()) <= 128
    assert bool((x[~mask] == 0).all())
    x0, m0 = cases.case_inputs(cfg, 7, 0.0)
    assert m0 is None and x0.dtype == torch.float16
