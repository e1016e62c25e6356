"""TVM-FFI binding: this build as the reference's CUDA solution slot.

The reference's CUDA slot (``solution/cuda/binding.py:11-25``) registers a TVM-FFI global
function ``flashinfer.kernel`` that the benchmark harness calls with the definition's eleven
arguments (``kernel.py:600-613``: nine tensors, ``local_expert_offset``,
``routed_scaling_factor``) in destination-passing style. ``register()`` installs that function
over ``flashinfer_b200.run``: tensors arrive as DLPack-capable objects (``tvm_ffi.Tensor``),
are viewed as torch tensors without copies, and the operator writes ``output`` in place on
torch's current stream. Errors surface as the same Python exceptions ``run`` raises.
"""
from __future__ import annotations

import torch

from .moe import run

NAME = "flashinfer.kernel"


def _as_torch(x) -> torch.Tensor:
    return x if isinstance(x, torch.Tensor) else torch.from_dlpack(x)


def kernel(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
           gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, local_expert_offset,
           routed_scaling_factor, output) -> None:
    """The slot's function: the reference's argument order, ``output`` written in place."""
    t = [_as_torch(x) for x in (routing_logits, routing_bias, hidden_states, hidden_states_scale,
                                gemm1_weights, gemm1_weights_scale, gemm2_weights,
                                gemm2_weights_scale, output)]
    run(*t[:8], int(local_expert_offset), float(routed_scaling_factor), t[8])


def register(name: str = NAME, override: bool = True):
    """Registers ``kernel`` as the TVM-FFI global function ``name``; returns the tvm_ffi
    Function the harness would look up. Needs the ``tvm_ffi`` package (apache-tvm-ffi)."""
    import tvm_ffi
    tvm_ffi.register_global_func(name, kernel, override=override)
    return tvm_ffi.get_global_func(name)
