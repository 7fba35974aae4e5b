"""tensorrs_b200 -- B200 (sm_100a) broadcast-elementwise / axis-reduction path
of tensorrs (GooseKIller/Tensors).

The product is libtrs_b200.so, a C ABI (include/trs.h) over hand-written CUDA
kernels.  `abi` binds it with ctypes; `device` wraps torch CUDA tensors as
trs_views for callers that manage device memory with PyTorch.
"""
from . import abi  # noqa: F401

__all__ = ["abi"]
