"""CPU: the C-ABI library loads, exports every symbol include/tttj_b200.h declares,
and its host-side logic (config validation, packed-weight and workspace layouts,
argument checks) behaves -- no kernel is launched here."""
import ctypes
import re
from pathlib import Path

import pytest
import torch

import tttj_2026_b200 as tb
from tttj_2026_b200 import _lib
from helpers import CONFIGS

HEADER = Path(__file__).resolve().parent.parent / "include" / "tttj_b200.h"


def declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(tttj_[a-z0-9_]+)\s*\(", text)))


def test_header_and_binding_agree():
    assert declared_functions() == sorted(_lib.exported_symbols())


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    for name in declared_functions():
        assert hasattr(L, name), name
    assert b"sm_100a" in L.tttj_version()


def _c(B, S, D, H, F, Lyr, causal):
    return _lib.TttjConfig(B, S, D, H, F, Lyr, 1 if causal else 0)


@pytest.mark.parametrize("name", sorted(CONFIGS))
def test_baseline_configs_are_supported(name):
    B, S, D, H, F, L, causal, _, _ = CONFIGS[name]
    c = _c(B, S, D, H, F, L, causal)
    assert _lib.lib().tttj_validate_config(ctypes.byref(c)) == 0
    assert _lib.lib().tttj_weights_bytes(ctypes.byref(c)) > 0
    assert _lib.lib().tttj_workspace_bytes(ctypes.byref(c)) > 0


@pytest.mark.parametrize(
    "shape,msg",
    [((2, 128, 1024, 2, 1024, 2, True), "head_dim=512"),  # wider than 256
     ((2, 128, 48, 4, 64, 4, True), "head_dim=12"),        # not a multiple of 8
     ((2, 128, 80, 2, 128, 1, False), "multiples of 32"),
     ((2, 128, 256, 3, 1024, 1, False), "divisible")],
)
def test_unsupported_configs_raise_value_error(shape, msg):
    cfg = tb.TransformerConfig(*shape)
    with pytest.raises(ValueError, match=msg):
        tb.validate_model_config(cfg)


def test_weight_layout_fields_disjoint_and_aligned():
    B, S, D, H, F, L, causal, _, _ = CONFIGS["C3"]
    c = _c(B, S, D, H, F, L, causal)
    lib = _lib.lib()
    total = lib.tttj_weights_bytes(ctypes.byref(c))
    spans = []
    for layer in range(L + 1):
        fields = range(12) if layer < L else (12, 13)
        for f in fields:
            off, size = ctypes.c_size_t(), ctypes.c_size_t()
            assert lib.tttj_weight_offset(ctypes.byref(c), layer, f, ctypes.byref(off), ctypes.byref(size)) == 0
            assert off.value % 256 == 0
            spans.append((off.value, off.value + size.value))
    spans.sort()
    for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
        assert a1 <= b0
    assert spans[-1][1] <= total
    # per-layer weight bytes: fp16 matrices 4D^2 + 2DF, fp32 vectors
    off, size = ctypes.c_size_t(), ctypes.c_size_t()
    lib.tttj_weight_offset(ctypes.byref(c), 0, 0, ctypes.byref(off), ctypes.byref(size))
    assert size.value == 3 * D * D * 2
    assert lib.tttj_weight_offset(ctypes.byref(c), L, 0, ctypes.byref(off), ctypes.byref(size)) == 1


def test_pack_weights_places_every_parameter():
    """pack_weights on the CPU: each field holds the parameter it should."""
    cfg = tb.TransformerConfig(2, 16, 64, 2, 128, 2, True)
    torch.manual_seed(5)
    model = tb.TransformerParameters(cfg)
    buf = tb.pack_weights(model, torch.device("cpu"))
    c = _lib.TttjConfig.from_config(cfg)
    lib = _lib.lib()

    def field(layer, f, dtype):
        off, size = ctypes.c_size_t(), ctypes.c_size_t()
        lib.tttj_weight_offset(ctypes.byref(c), layer, f, ctypes.byref(off), ctypes.byref(size))
        return buf[off.value : off.value + size.value].view(dtype)

    for i, blk in enumerate(model.layers):
        a = blk.attention
        wqkv = torch.cat([a.q_proj.weight, a.k_proj.weight, a.v_proj.weight]).half().reshape(-1)
        assert torch.equal(field(i, _lib.W_QKV, torch.float16), wqkv)
        assert torch.equal(field(i, _lib.W_FFN_OUT, torch.float16), blk.ffn_out.weight.half().reshape(-1))
        assert torch.equal(field(i, _lib.B_FFN_IN, torch.float32), blk.ffn_in.bias.float())
        assert torch.equal(field(i, _lib.LN2_W, torch.float32), blk.norm2.weight.float())
    assert torch.equal(field(2, _lib.LNF_B, torch.float32), model.final_norm.bias.float())


def test_constructor_rejects_cpu_model():
    cfg = tb.TransformerConfig(2, 16, 64, 1, 128, 1, False)
    model = tb.TransformerParameters(cfg)
    with pytest.raises(ValueError, match="CUDA"):
        tb.make_optimized_transformer(model)


def test_plan_create_rejects_bad_arguments():
    lib = _lib.lib()
    c = _c(2, 16, 64, 1, 128, 1, False)
    out = ctypes.c_void_p()
    assert lib.tttj_plan_create(ctypes.byref(c), 0, None, None, 0, ctypes.byref(out)) == _lib.TTTJ_ERR_INVALID
    assert b"null" in lib.tttj_last_error()
    bad = _c(2, 16, 64, 1, 128, 0, False)
    assert lib.tttj_validate_config(ctypes.byref(bad)) == _lib.TTTJ_ERR_INVALID


def test_linear_argument_checks_do_not_launch():
    lib = _lib.lib()
    # n not a multiple of 32 -> rejected before any CUDA call.
    rc = lib.tttj_linear(ctypes.c_void_p(16), 64, ctypes.c_void_p(16), 64, ctypes.c_void_p(16),
                         ctypes.c_void_p(16), 40, None, 0, 8, None, 40, 64, 0, None, None)
    assert rc == _lib.TTTJ_ERR_INVALID
    assert b"multiple of 32" in lib.tttj_last_error()
    assert lib.tttj_attention_workspace_bytes(4, 300, 3) > 0
