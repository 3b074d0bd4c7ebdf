"""``flex_gemm``-compatible sparse operators on the B200 kernels.

The reference picks its sparse-operator provider purely by import name (promptmoge/model.py:27-30: the bundled
fallback is used only when no ``flex_gemm`` package is importable).  ``install()`` registers this package under that
name, so the refiner's modules (flex_sparse_blocks.py:8-12, sparse_unet.py:14, qat.py:126) bind to these classes
without any change to the reference code:

    import promptmoge_b200.flex_gemm
    promptmoge_b200.flex_gemm.install()      # before the reference's model modules are imported
"""
from __future__ import annotations

import sys

from . import nn, ops

__version__ = "0.1.0+b200"
__all__ = ["ops", "nn", "install"]


def install(force: bool = False) -> None:
    """Make ``import flex_gemm`` (and ``flex_gemm.nn`` / ``flex_gemm.ops``) resolve to this package.  An already
    imported ``flex_gemm`` is replaced only with ``force=True``."""
    current = sys.modules.get("flex_gemm")
    if current is not None and current is not sys.modules[__name__] and not force:
        raise RuntimeError(f"a flex_gemm module is already imported ({current!r}); pass force=True to replace it")
    pkg = sys.modules[__name__]
    sys.modules["flex_gemm"] = pkg
    sys.modules["flex_gemm.nn"] = nn
    sys.modules["flex_gemm.ops"] = ops
