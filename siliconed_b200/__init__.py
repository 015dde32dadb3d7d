"""siliconed_b200: a B200 (sm_100a) implementation of Siliconed's quantized linear stage.

The product is ``libsiliconed_cuda.so`` (C ABI: include/siliconed_cuda.h), built from
``siliconed_b200/csrc`` by ``siliconed_b200.build``.  This package adds the host-side mirror of the
reference's interface (``WeightProducts``, ``QuantizedWeight``) and the multi-GPU helpers.
"""
from .abi import SiliconedError, load, header_functions  # noqa: F401
from . import abi  # noqa: F401

__all__ = ["SiliconedError", "load", "header_functions", "abi", "Context", "QuantizedWeight", "WeightProducts"]


def __getattr__(name):
    if name in ("Context", "QuantizedWeight", "WeightProducts"):
        from . import products
        return getattr(products, name)
    raise AttributeError(name)
