"""spmv_decode_b200 -- B200-native (sm_100a) N:M sparse GEMV decode engine.

Drop-in for the reference's decode path (xinwei-niu/SpMV_decode):
``torch.ops.nmsparse.gemv``, ``NmSparseLinear``, ``swap_to_nmsparse`` and a
gpt-fast-style decode step, backed by hand-written CUDA kernels in
libnmsparse_b200.so (C ABI: include/nmsparse_b200.h).
"""
from .nmsparse_linear import NmSparseLinear, make_sparse, swap_to_nmsparse  # noqa: F401
from . import nmsparse_op  # noqa: F401

__all__ = ["NmSparseLinear", "swap_to_nmsparse", "make_sparse", "nmsparse_op"]
