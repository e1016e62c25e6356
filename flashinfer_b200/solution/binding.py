"""CUDA solution slot of the fused MoE definition (packed at the solution's root).

The harness's CUDA slot (reference ``solution/cuda/binding.py:11-25``) is a TVM-FFI global function
``flashinfer.kernel`` taking the definition's arguments in destination-passing style. Importing this
module builds the packed sm_100a sources next to it (nvcc, once: the library is kept in
``flashinfer_b200/_lib``), registers ``flashinfer.kernel`` and exposes the same function as
``kernel`` (the entry point named in config.toml).
"""
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
if HERE not in sys.path:
    sys.path.insert(0, HERE)

from flashinfer_b200 import build as _build  # noqa: E402

_build.build()

from flashinfer_b200.tvm_binding import NAME, kernel, register  # noqa: E402,F401

register()
