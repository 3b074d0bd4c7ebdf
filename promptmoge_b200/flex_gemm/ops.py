"""Functional operators and caches, under the names the refiner imports (``from flex_gemm.ops import
NeighborCache``; reference promptmoge/_fallback/flex_gemm/ops/__init__.py)."""
from ._core import (  # noqa: F401
    NeighborCache,
    NeighborCacheT,
    build_pool_cache,
    build_submanifold_cache,
    make_conv_kernel_delta,
    sparse_pool,
    sparse_upsample,
    submanifold_conv,
)

__all__ = ["NeighborCache", "NeighborCacheT", "build_submanifold_cache", "build_pool_cache", "submanifold_conv",
           "sparse_pool", "sparse_upsample", "make_conv_kernel_delta"]
