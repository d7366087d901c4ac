"""ctypes binding of libtttj_b200.so (declared in include/tttj_b200.h).

The library is the product: every forward, linear, layernorm and attention call of
this package goes through it.  There is no Python or PyTorch fallback; if the
shared library is missing, :func:`lib` raises.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "libtttj_b200.so"

TTTJ_OK = 0
TTTJ_ERR_INVALID = 1
TTTJ_ERR_CUDA = 2
TTTJ_ERR_DEVICE_TIMEOUT = 3

DTYPE_F16 = 0
DTYPE_F32 = 1

EPI_BIAS = 0
EPI_BIAS_GELU = 1
EPI_BIAS_RESIDUAL = 2
EPI_BIAS_RESIDUAL_F32 = 3

# Packed weight fields (include/tttj_b200.h).
W_QKV, W_OUT, W_FFN_IN, W_FFN_OUT = 0, 1, 2, 3
B_QKV, B_OUT, B_FFN_IN, B_FFN_OUT = 4, 5, 6, 7
LN1_W, LN1_B, LN2_W, LN2_B = 8, 9, 10, 11
LNF_W, LNF_B = 12, 13

# int exchange(void* user, int layer, void* stream) -- see tttj_forward_cp.
EXCHANGE_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p)

# Every symbol include/tttj_b200.h declares, with (restype, argtypes).
_c = ctypes
_vp = _c.c_void_p
_SIGNATURES = {
    "tttj_last_error": (_c.c_char_p, []),
    "tttj_version": (_c.c_char_p, []),
    "tttj_validate_config": (_c.c_int, [_vp]),
    "tttj_weights_bytes": (_c.c_size_t, [_vp]),
    "tttj_weight_offset": (
        _c.c_int,
        [_vp, _c.c_int, _c.c_int, _c.POINTER(_c.c_size_t), _c.POINTER(_c.c_size_t)],
    ),
    "tttj_folded_bytes": (_c.c_size_t, [_vp]),
    "tttj_fold_weights": (_c.c_int, [_vp, _vp, _vp, _c.c_size_t, _vp]),
    "tttj_workspace_bytes": (_c.c_size_t, [_vp]),
    "tttj_plan_create": (_c.c_int, [_vp, _c.c_int, _vp, _vp, _vp, _c.c_size_t, _c.POINTER(_vp)]),
    "tttj_plan_destroy": (_c.c_int, [_vp]),
    "tttj_forward": (_c.c_int, [_vp, _vp, _c.c_int, _vp, _vp, _vp]),
    "tttj_plan_status": (_c.c_int, [_vp, _c.POINTER(_c.c_int)]),
    "tttj_linear": (
        _c.c_int,
        [_vp, _c.c_int, _vp, _c.c_int, _vp, _vp, _c.c_int, _vp, _c.c_int, _c.c_int, _vp,
         _c.c_int, _c.c_int, _c.c_int, _vp, _vp],
    ),
    "tttj_layernorm": (
        _c.c_int, [_vp, _vp, _c.c_int, _c.c_int, _vp, _vp, _c.c_float, _vp]
    ),
    "tttj_attention_workspace_bytes": (_c.c_size_t, [_c.c_int, _c.c_int, _c.c_int]),
    "tttj_path_choice": (
        _c.c_int, [_vp, _c.POINTER(_c.c_int), _c.POINTER(_c.c_int), _c.POINTER(_c.c_int)]
    ),
    "tttj_gemm_tile": (
        _c.c_int,
        [_c.c_int, _c.c_int, _c.c_int, _c.c_int, _c.c_int, _c.POINTER(_c.c_int),
         _c.POINTER(_c.c_int)],
    ),
    "tttj_attention": (
        _c.c_int,
        [_vp, _vp, _c.c_int, _vp, _c.c_int, _c.c_int, _c.c_int, _c.c_int, _c.c_int, _vp,
         _c.c_size_t, _vp],
    ),
    "tttj_attention_noalloc": (
        _c.c_int, [_vp, _vp, _c.c_int, _vp, _c.c_int, _c.c_int, _c.c_int, _c.c_int, _c.c_int, _vp]
    ),
    "tttj_selftest_wait_timeout": (_c.c_int, [_vp, _c.c_uint64, _vp]),
    "tttj_plan_selftest_timeout": (_c.c_int, [_vp, _c.c_uint64, _vp]),
    "tttj_workspace_bytes_cp": (_c.c_size_t, [_vp, _c.c_int]),
    "tttj_plan_create_cp": (
        _c.c_int,
        [_vp, _c.c_int, _vp, _vp, _c.c_int, _c.c_int, _c.c_int, _vp, _c.c_size_t, _c.POINTER(_vp)],
    ),
    "tttj_plan_cp_qkv": (
        _c.c_int, [_vp, _c.POINTER(_c.c_size_t), _c.POINTER(_c.c_size_t), _c.POINTER(_c.c_int)]
    ),
    "tttj_forward_cp": (_c.c_int, [_vp, _vp, _c.c_int, _vp, EXCHANGE_FN, _vp, _vp]),
    "tttj_device_sm_count": (_c.c_int, [_c.c_int]),
    "tttj_plan_launch_count": (_c.c_int, [_vp]),
    "tttj_plan_enable_timing": (_c.c_int, [_vp, _c.c_int]),
    "tttj_plan_kernel_times": (_c.c_int, [_vp, _c.POINTER(_c.c_double), _c.POINTER(_c.c_long)]),
    "tttj_kernel_class_name": (_c.c_char_p, [_c.c_int]),
    "tttj_plan_set_path": (_c.c_int, [_vp, _c.c_int]),
    "tttj_debug_floats": (_c.c_size_t, [_c.c_void_p]),
    "tttj_forward_debug": (
        _c.c_int, [_vp, _vp, _c.c_int, _vp, _vp, _c.c_int, _c.c_int, _vp, _vp]
    ),
    "tttj_plan_path": (_c.c_int, [_vp]),
}

KCLASS_COUNT = 9
PATH_AUTO = 0
PATH_LAYERWISE = 1
PATH_RESIDENT = 2
PATHS = {"auto": PATH_AUTO, "layerwise": PATH_LAYERWISE, "resident": PATH_RESIDENT}


class TttjConfig(ctypes.Structure):
    """C mirror of TransformerConfig (reference benchmarks/torch_transformer_benchmark.py:29-56)."""

    _fields_ = [
        ("batch_size", ctypes.c_int32),
        ("seq_len", ctypes.c_int32),
        ("d_model", ctypes.c_int32),
        ("num_heads", ctypes.c_int32),
        ("ffn_dim", ctypes.c_int32),
        ("num_layers", ctypes.c_int32),
        ("causal", ctypes.c_int32),
    ]

    @classmethod
    def from_config(cls, cfg, batch_size: int | None = None, seq_len: int | None = None):
        return cls(
            int(cfg.batch_size if batch_size is None else batch_size),
            int(cfg.seq_len if seq_len is None else seq_len),
            int(cfg.d_model),
            int(cfg.num_heads),
            int(cfg.ffn_dim),
            int(cfg.num_layers),
            1 if cfg.causal else 0,
        )


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    """Load libtttj_b200.so (once) and attach the C signatures."""
    global _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH} is missing: build it with `python tttj-2026_b200/build_lib.py` "
                    "(there is no fallback implementation)"
                )
            handle = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
        return _lib


def exported_symbols() -> list[str]:
    return list(_SIGNATURES)


def check(rc: int, what: str = "tttj") -> None:
    """Turn a C return code into the reference's Python exception conventions."""
    if rc == TTTJ_OK:
        return
    msg = lib().tttj_last_error().decode(errors="replace")
    if rc == TTTJ_ERR_INVALID:
        raise ValueError(f"{what}: {msg}")
    raise RuntimeError(f"{what}: {msg} (code {rc})")
