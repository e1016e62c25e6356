"""flashinfer_b200 -- B200-native (sm_100a) fused FP8 block-scale MoE with DeepSeek-V3 routing.

Drop-in for the reference operator ``solution/triton/kernel.py::run`` of the
FlashInfer-Bench ``fused_moe`` solution
(``moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048``). The compute
path is hand-written CUDA behind the C ABI of ``include/fmoe.h``; expert
parallelism over several GPUs is in ``flashinfer_b200.ep``.
"""
from .moe import run, route, quantize_activations, read_status, workspace_for, WorkspaceView  # noqa: F401,E501

__all__ = ["run", "route", "read_status", "workspace_for", "WorkspaceView"]
