"""B200 (sm_100a) NVFP4 Gated DeltaNet state update.

Python front end of libgdn_b200.so (C ABI: include/gdn_b200.h) and of the
torch custom ops in the reference's `gdn_sm120` namespace
(libgdn_sm120_op.so).  All compute runs in CUDA kernels; there is no CPU path.
"""
from ._capi import SCALE_FN448, SCALE_REF240, GdnError, version  # noqa: F401
from . import ops  # noqa: F401
from .pool import NVFP4StatePool  # noqa: F401
