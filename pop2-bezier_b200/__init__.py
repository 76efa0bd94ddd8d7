"""pop2-bezier B200 int8 historical-KV decode engine.

The product is libpp_b200.so (CUDA kernels for sm_100a behind the C ABI in
include/pp_b200.h).  This package is its Python binding: ctypes over the ABI,
with torch providing device memory and streams.  Importing it loads the
library and fails if it is missing; nothing here computes on the CPU.
"""
from . import _native  # noqa: F401  (loads libpp_b200.so or raises)
from . import int8_kv_ops  # noqa: F401
from . import kv_cache  # noqa: F401
from . import decoder  # noqa: F401
from . import sampling  # noqa: F401
from . import fused_attention  # noqa: F401
from . import sched  # noqa: F401
from ._native import (  # noqa: F401
    ExecutionUncertainError,
    InvalidOutputError,
    PreconditionError,
    abi_version,
)

__all__ = ["int8_kv_ops", "kv_cache", "decoder", "sampling", "fused_attention", "sched", "abi_version", "PreconditionError", "InvalidOutputError",
           "ExecutionUncertainError"]
