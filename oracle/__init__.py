"""CPU oracle of ML_Engine's training hot path -- TEST INFRASTRUCTURE ONLY.

`oracle.ops` wraps the C restatement in mle_oracle.c (numpy arrays in, numpy
arrays out); `oracle.graphs` composes those ops into the reference's graphs
node by node; `oracle.ref` binds the reference's own CUDA kernels compiled
from source (oracle/_ref, GPU only).  Only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg may import this package.
"""
from . import ops  # noqa: F401
