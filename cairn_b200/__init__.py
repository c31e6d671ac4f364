"""cairn_b200: CAIRN's data-parallel hot path (the tensor-core multiply, `parallel` regions and `reduce +`) as
hand-written sm_100a CUDA behind a flat C ABI (include/cairn_b200.h, libcairn_b200.so).

The C ABI is the product; this package builds it (cairn_b200.build), loads it (cairn_b200._lib) and offers
torch-facing forms of its entries (cairn_b200.ops) and the range-sharded multi-GPU forms (cairn_b200.shard).
"""

from ._lib import CairnError, LIB_PATH, header_symbols, lib
from .host import HostGemm, HostSaxpy
from .ops import gemm, mma_unordered, reduce_sum, saxpy, stream_status, watchdog_selftest

__all__ = [
    "CairnError",
    "HostGemm",
    "HostSaxpy",
    "LIB_PATH",
    "gemm",
    "header_symbols",
    "lib",
    "mma_unordered",
    "reduce_sum",
    "saxpy",
    "stream_status",
    "watchdog_selftest",
]
__version__ = "0.1.0"
