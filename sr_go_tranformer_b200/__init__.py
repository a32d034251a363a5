"""sr_go_tranformer_b200 -- B200 (sm_100a) engine step for sr_go_tranformer.

The product is libsrstep.so (C ABI in include/srstep.h): the reference Go
engine's continuous-batching prefill/decode step (cmd/monolith/monolith.go,
Model.prefillSelected) on hand-written CUDA kernels.  This package holds its
sources (csrc/), the in-tree build (build.py), ctypes bindings (_abi.py) and a
host-side mirror of the reference's step/engine API (step.py, engine.py).
"""

from . import _abi
from ._abi import SRError, lib

__all__ = ["SRError", "lib", "_abi"]
