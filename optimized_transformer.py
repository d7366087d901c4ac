"""Public construction API, at the same path and with the same name as the
reference's (optimized_transformer.py:69-93 in Scallion3008/tttj-2026):

    from optimized_transformer import make_optimized_transformer
    optimized = make_optimized_transformer(model)      # model: BaselineTransformer-like
    y = optimized(x, valid_token_mask)

Importing this module also registers the package directory ``tttj-2026_b200/`` as
the importable package ``tttj_2026_b200``.
"""
from __future__ import annotations

import importlib.util
import sys
from pathlib import Path

_PKG_NAME = "tttj_2026_b200"
_PKG_DIR = Path(__file__).resolve().parent / "tttj-2026_b200"


def _register_package():
    mod = sys.modules.get(_PKG_NAME)
    if mod is not None:
        return mod
    spec = importlib.util.spec_from_file_location(
        _PKG_NAME, _PKG_DIR / "__init__.py", submodule_search_locations=[str(_PKG_DIR)]
    )
    mod = importlib.util.module_from_spec(spec)
    sys.modules[_PKG_NAME] = mod
    try:
        spec.loader.exec_module(mod)
    except BaseException:
        sys.modules.pop(_PKG_NAME, None)
        raise
    return mod


_pkg = _register_package()

make_optimized_transformer = _pkg.make_optimized_transformer
TransformerConfig = _pkg.TransformerConfig
TransformerParameters = _pkg.TransformerParameters
IMPLEMENTED_CASES = _pkg.IMPLEMENTED_CASES
IMPLEMENTED_CASE_LAYERS = _pkg.IMPLEMENTED_CASE_LAYERS
case_number_for_model = _pkg.case_number_for_model

__all__ = ["make_optimized_transformer", "TransformerConfig", "TransformerParameters",
           "IMPLEMENTED_CASES", "IMPLEMENTED_CASE_LAYERS", "case_number_for_model"]
