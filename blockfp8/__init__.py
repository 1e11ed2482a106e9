"""Drop-in name for blockfp8_b200: code written against the reference's
`import blockfp8` (and blockfp8.layout / .quant / .reference / .gemm) runs
unchanged on the B200 implementation."""

import sys as _sys

import blockfp8_b200 as _impl
from blockfp8_b200 import *  # noqa: F401,F403
from blockfp8_b200 import __all__  # noqa: F401
from blockfp8_b200 import gemm as _gemm_mod  # noqa: F401  (the submodule, below)

for _name in ("layout", "quant", "reference", "gemm"):
    _sys.modules[f"{__name__}.{_name}"] = _sys.modules[f"blockfp8_b200.{_name}"]
gemm = _impl.gemm  # the function, as in the reference's package namespace
del _sys, _name
