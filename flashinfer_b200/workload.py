"""Seeded synthetic workloads for the fused FP8 block-scale MoE operator.

The FlashInfer-Trace dataset the reference is benchmarked on
(`README.md:33-44` of the reference: ``flashinfer-ai/mlsys26-contest``) is not
available, so every test, smoke run and bench line draws its inputs from the
recipe below instead. Shapes, dtypes and value distributions follow the
operator definition ``moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048``
(reference ``config.toml:3``; tensor axes as in ``solution/triton/kernel.py:600-625``):

* ``routing_logits``  fp32 ``[T, 256]`` ~ N(0, 1) (optionally +skew on a slice)
* ``routing_bias``    bf16 ``[256]``    ~ N(0, 0.1)
* ``hidden_states``   e4m3 ``[T, 7168]`` from bf16 N(0, 1), one fp32 scale per
  token per 128 columns (``amax / 448``), scales laid out ``[56, T]``
* ``gemm1_weights``   e4m3 ``[E, 4096, 7168]`` from 0.02·N(0, 1), one fp32 scale
  per 128x128 block, scales ``[E, 32, 56]``
* ``gemm2_weights``   e4m3 ``[E, 7168, 2048]``, scales ``[E, 56, 16]``, same scheme

Draw order is fixed: one CPU ``torch.Generator`` seeded with the config seed
draws logits, then bias, then hidden states. Each expert's weights come from
their own generator seeded ``1000 + global_expert_id`` (W1 first, then W2), so
a single-GPU run and any expert-parallel shard see identical weights for the
same global expert, and a CPU check can regenerate only the experts it needs.
CPU generators make the draws reproducible on any host with the same torch.
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict, Iterable, Optional

import torch

HIDDEN = 7168
INTER = 2048
E_GLOBAL = 256
N_GROUP = 8
TOPK_GROUP = 4
TOP_K = 8
BLOCK = 128
FP8_MAX = 448.0
E_LOCAL_DEFAULT = 32
RSF_DEFAULT = 2.5

FP8 = torch.float8_e4m3fn


def _quantize_blocks_2d(x: torch.Tensor):
    """Per-128x128-block e4m3 quantisation of a 2-D fp32 matrix.

    Returns (q [R, C] e4m3, scale [R/128, C/128] fp32) with scale = amax/448.
    """
    r, c = x.shape
    blocks = x.view(r // BLOCK, BLOCK, c // BLOCK, BLOCK)
    amax = blocks.abs().amax(dim=(1, 3))
    scale = torch.clamp(amax, min=1e-30) / FP8_MAX
    q = (blocks / scale[:, None, :, None]).to(FP8).view(r, c)
    return q, scale.contiguous()


def quantize_activations(x_bf16: torch.Tensor):
    """Per-token, per-128-column e4m3 quantisation of bf16 activations.

    Returns (q [T, H] e4m3, scale [H/128, T] fp32) -- the transposed scale
    layout the operator consumes (reference ``kernel.py:169`` indexes it as
    ``scale[kb, token]``).
    """
    t, h = x_bf16.shape
    x = x_bf16.float().view(t, h // BLOCK, BLOCK)
    amax = x.abs().amax(dim=2)
    scale = torch.clamp(amax, min=1e-30) / FP8_MAX
    q = (x / scale[:, :, None]).to(FP8).view(t, h)
    return q, scale.t().contiguous()


def expert_weights(global_expert: int, hidden: int = HIDDEN, inter: int = INTER,
                   device: str = "cpu"):
    """Quantised (W1, S1, W2, S2) for one global expert, seeded 1000+id.

    With a CUDA ``device`` the draws come from that device's generator: same distributions,
    different values than the CPU draws (used where only timing matters, never for parity).
    """
    g = torch.Generator(device=device).manual_seed(1000 + int(global_expert))
    w1 = torch.randn(2 * inter, hidden, generator=g, device=device) * 0.02
    q1, s1 = _quantize_blocks_2d(w1)
    del w1
    w2 = torch.randn(hidden, inter, generator=g, device=device) * 0.02
    q2, s2 = _quantize_blocks_2d(w2)
    return q1, s1, q2, s2


class WeightBank:
    """Process-wide cache of per-expert quantised weights (CPU tensors)."""

    _cache: Dict[int, tuple] = {}

    @classmethod
    def get(cls, global_expert: int):
        w = cls._cache.get(global_expert)
        if w is None:
            w = expert_weights(global_expert)
            cls._cache[global_expert] = w
        return w

    @classmethod
    def stacked(cls, experts: Iterable[int]):
        ws = [cls.get(e) for e in experts]
        return (torch.stack([w[0] for w in ws]), torch.stack([w[1] for w in ws]),
                torch.stack([w[2] for w in ws]), torch.stack([w[3] for w in ws]))


@dataclass
class Activations:
    routing_logits: torch.Tensor
    routing_bias: torch.Tensor
    hidden_states: torch.Tensor
    hidden_states_scale: torch.Tensor


def make_activations(T: int, seed: int, skew_experts: Optional[range] = None,
                     skew: float = 0.0, hot_group: Optional[int] = None,
                     hot: float = 0.0, hidden: int = HIDDEN) -> Activations:
    """Seeded routing logits, bias and quantised hidden states (CPU)."""
    g = torch.Generator().manual_seed(int(seed))
    logits = torch.randn(T, E_GLOBAL, generator=g)
    if skew_experts is not None and skew != 0.0:
        logits[:, skew_experts.start:skew_experts.stop] += skew
    if hot_group is not None and hot != 0.0:
        gs = E_GLOBAL // N_GROUP
        logits[:, hot_group * gs:(hot_group + 1) * gs] += hot
    bias = (torch.randn(E_GLOBAL, generator=g) * 0.1).to(torch.bfloat16)
    hs = torch.randn(T, hidden, generator=g).to(torch.bfloat16)
    q, s = quantize_activations(hs)
    return Activations(logits.contiguous(), bias.contiguous(), q.contiguous(), s)


@dataclass
class Config:
    """One named workload from the operator's benchmark plan."""
    name: str
    T: int
    seed: int
    skew: float = 0.0          # added to logits of experts [0, 32)
    hot: float = 0.0           # added to logits of group 0
    local_expert_offset: int = 0
    e_local: int = E_LOCAL_DEFAULT
    rsf: float = RSF_DEFAULT
    extra: dict = field(default_factory=dict)

    def activations(self) -> Activations:
        return make_activations(self.T, self.seed,
                                skew_experts=range(0, 32) if self.skew else None,
                                skew=self.skew, hot_group=0 if self.hot else None,
                                hot=self.hot)


# The single-GPU workloads: config 0 (T=16), 1 (decode), 2 (batched decode, +
# skewed variants), 3 (prefill).
CONFIGS = {
    "t16_s0": Config("t16_s0", 16, 0),
    "t1_s1": Config("t1_s1", 1, 1),
    "t8_s2": Config("t8_s2", 8, 2),
    "t32_s3": Config("t32_s3", 32, 3),
    "t64_s4": Config("t64_s4", 64, 4),
    "t256_s5": Config("t256_s5", 256, 5),
    "t256_s5_skew": Config("t256_s5_skew", 256, 5, skew=2.0),
    "t1024_s6": Config("t1024_s6", 1024, 6),
    "t1024_s6_skew": Config("t1024_s6_skew", 1024, 6, skew=2.0),
    "t4096_s7": Config("t4096_s7", 4096, 7),
    "t8192_s8": Config("t8192_s8", 8192, 8),
    "t16384_s9": Config("t16384_s9", 16384, 9),
}


def local_weights(e_local: int = E_LOCAL_DEFAULT, local_expert_offset: int = 0):
    """Stacked quantised weights for experts [offset, offset+e_local) (CPU)."""
    return WeightBank.stacked(range(local_expert_offset, local_expert_offset + e_local))


def flops_per_pair(hidden: int = HIDDEN, inter: int = INTER) -> int:
    """Algorithmic FLOPs per routed (token, local expert) pair."""
    return 2 * (hidden * 2 * inter + inter * hidden)


def bytes_per_expert(hidden: int = HIDDEN, inter: int = INTER) -> int:
    """Weight + weight-scale bytes streamed per active local expert."""
    w = hidden * 2 * inter + inter * hidden
    s = (2 * inter // BLOCK) * (hidden // BLOCK) * 4 + (hidden // BLOCK) * (inter // BLOCK) * 4
    return w + s


def bytes_per_token(hidden: int = HIDDEN, e_global: int = E_GLOBAL) -> int:
    """Logits (fp32) + fp8 hidden row + its scales + the bf16 output row."""
    return e_global * 4 + hidden + (hidden // BLOCK) * 4 + hidden * 2
