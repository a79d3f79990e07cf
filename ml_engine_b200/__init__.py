"""B200-native (sm_100a) implementation of ML_Engine's training hot path.

The product is native code: ml_engine_b200/lib/libmle_kernels.so (the C ABI of
include/mle_kernels.h) and ml_engine_b200/lib/libmle_engine.so (the C++
NodeBackProp / GraphOperations / AdamParameter runtime and the C ABI of
include/mle_engine.h).  This package only builds and binds them.
"""
from ._lib import MLEError, engine, kernels  # noqa: F401

__all__ = ["MLEError", "kernels", "engine"]
