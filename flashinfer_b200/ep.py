"""Expert parallelism for the fused MoE over ``torch.distributed`` (NCCL on GPUs).

The operator contract already describes one expert-parallel rank: ``run`` computes the
routing-weighted sum over the local experts ``[local_expert_offset, local_expert_offset + E_local)``
only (reference ``solution/triton/kernel.py:448-452``). With R ranks and 256 experts, rank r owns
experts ``[r*256/R, (r+1)*256/R)``. One layer call on rank r:

1. route its own T_r tokens (``fmoe_route``: global top-8 ids, bit-exact with every other rank);
2. dispatch: each token goes once to every rank that owns at least one of its 8 picks
   (deduplicated per destination; with R=8 at most 4 ranks, one per kept group). A token
   travels as one packed record: fp32 logits (1024 B), the e4m3 row (H B) and its H/128 fp32
   scales, so the receiver can run the unchanged operator on it. Counts go first in a small
   all-to-all, then the records in one variable-split ``all_to_all_single``;
3. the receiver runs the fused operator on everything it received, with its own
   ``local_expert_offset``, re-deriving the same routing, and keeps the result in fp32;
4. combine: a second all-to-all returns each fp32 partial row to its source, which adds the
   partials of the destination ranks in ascending rank order (deterministic; the same expert
   order as the single-GPU sum) and rounds once to bf16.

``route_fn`` and ``local_fn`` are injectable so the index logic can be tested on CPU ranks
(gloo) with the numpy oracle standing in for the CUDA kernels.
"""
from __future__ import annotations

from typing import Callable, List, Optional, Tuple

import torch
import torch.distributed as dist

E_GLOBAL = 256
BLOCK = 128


def plan_dispatch(ids: torch.Tensor, experts_per_rank: int, world: int
                  ) -> Tuple[torch.Tensor, torch.Tensor]:
    """Tokens to send to each rank: (token indices grouped by destination rank ascending, tokens
    ascending within a rank; per-rank counts int64 [world])."""
    T = ids.shape[0]
    owner = (ids.long() // experts_per_rank).clamp_(0, world - 1)
    dest = torch.zeros((T, world), dtype=torch.bool, device=ids.device)
    if T:
        dest.scatter_(1, owner, True)
    pairs = dest.t().nonzero()              # (rank, token), rank-major, tokens ascending
    send_tok = pairs[:, 1].contiguous()
    counts = torch.bincount(pairs[:, 0], minlength=world).to(torch.int64)
    return send_tok, counts


def record_bytes(hidden: int) -> int:
    return E_GLOBAL * 4 + hidden + (hidden // BLOCK) * 4


def pack_records(send_tok: torch.Tensor, logits: torch.Tensor, hidden_u8: torch.Tensor,
                 hidden_scale: torch.Tensor) -> torch.Tensor:
    """One uint8 record per (token, destination): logits | e4m3 row | 128-column scales."""
    H = hidden_u8.shape[1]
    n = send_tok.numel()
    buf = torch.empty((n, record_bytes(H)), dtype=torch.uint8, device=logits.device)
    if n:
        buf[:, :E_GLOBAL * 4] = logits.float().index_select(0, send_tok).view(torch.uint8)
        buf[:, E_GLOBAL * 4:E_GLOBAL * 4 + H] = hidden_u8.index_select(0, send_tok)
        buf[:, E_GLOBAL * 4 + H:] = hidden_scale.index_select(1, send_tok).t().contiguous() \
            .view(torch.uint8)
    return buf


def unpack_records(buf: torch.Tensor, hidden: int):
    """Inverse of pack_records: (logits fp32 [n,256], e4m3 [n,H], scales fp32 [H/128, n])."""
    n = buf.shape[0]
    logits = buf[:, :E_GLOBAL * 4].contiguous().view(torch.float32).view(n, E_GLOBAL)
    hs = buf[:, E_GLOBAL * 4:E_GLOBAL * 4 + hidden].contiguous().view(torch.float8_e4m3fn)
    sc = buf[:, E_GLOBAL * 4 + hidden:].contiguous().view(torch.float32).view(n, hidden // BLOCK)
    return logits, hs, sc.t().contiguous()


def _default_route(logits, bias, rsf):
    from .moe import route
    ids, _ = route(logits, bias, rsf)
    return ids


def _default_local(logits, bias, hs, sc, w1, s1, w2, s2, local_offset, rsf, out_f32):
    from .moe import _launch
    _launch(logits, bias, hs, sc, w1, s1, w2, s2, local_offset, rsf, out_f32)


class ExpertParallelMoE:
    """Expert-parallel fused MoE layer for one rank of ``group``."""

    def __init__(self, group=None, route_fn: Optional[Callable] = None,
                 local_fn: Optional[Callable] = None):
        self.group = group
        single = not (dist.is_available() and dist.is_initialized())
        self.world = 1 if single else dist.get_world_size(group)
        self.rank = 0 if single else dist.get_rank(group)
        if E_GLOBAL % self.world:
            raise ValueError(f"{E_GLOBAL} experts do not split evenly over {self.world} ranks")
        self.experts_per_rank = E_GLOBAL // self.world
        self.local_offset = self.rank * self.experts_per_rank
        self.route_fn = route_fn or _default_route
        self.local_fn = local_fn or _default_local
        self.last_counts: Optional[Tuple[List[int], List[int]]] = None

    def _all_to_all(self, out, inp, out_splits=None, in_splits=None):
        if self.world == 1:
            out.copy_(inp)
        else:
            dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    @torch.no_grad()
    def forward(self, routing_logits, routing_bias, hidden_states, hidden_states_scale,
                gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
                routed_scaling_factor: float, output: Optional[torch.Tensor] = None
                ) -> torch.Tensor:
        """This rank's tokens in, this rank's bf16 output rows out (weights: local experts)."""
        if gemm1_weights.shape[0] != self.experts_per_rank:
            raise ValueError(f"rank {self.rank} needs {self.experts_per_rank} local experts, "
                             f"got {gemm1_weights.shape[0]}")
        T, H = hidden_states.shape
        dev = hidden_states.device
        ids = self.route_fn(routing_logits, routing_bias, routed_scaling_factor)
        send_tok, send_counts = plan_dispatch(ids, self.experts_per_rank, self.world)
        recv_counts = torch.empty_like(send_counts)
        self._all_to_all(recv_counts, send_counts)
        sc_list, rc_list = send_counts.tolist(), recv_counts.tolist()
        self.last_counts = (sc_list, rc_list)

        send_buf = pack_records(send_tok, routing_logits, hidden_states.view(torch.uint8),
                                hidden_states_scale)
        recv_buf = torch.empty((sum(rc_list), send_buf.shape[1]), dtype=torch.uint8, device=dev)
        self._all_to_all(recv_buf, send_buf, rc_list, sc_list)

        n_recv = recv_buf.shape[0]
        partial = torch.empty((n_recv, H), dtype=torch.float32, device=dev)
        if n_recv:
            lg_r, hs_r, sc_r = unpack_records(recv_buf, H)
            self.local_fn(lg_r, routing_bias, hs_r, sc_r, gemm1_weights, gemm1_weights_scale,
                          gemm2_weights, gemm2_weights_scale, self.local_offset,
                          routed_scaling_factor, partial)

        back = torch.empty((send_tok.numel(), H), dtype=torch.float32, device=dev)
        self._all_to_all(back, partial, sc_list, rc_list)

        acc = torch.zeros((T, H), dtype=torch.float32, device=dev)
        start = 0
        for d in range(self.world):          # ascending rank = ascending expert order
            n = sc_list[d]
            if n:
                acc.index_add_(0, send_tok[start:start + n], back[start:start + n])
            start += n
        if output is None:
            output = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
        output.copy_(acc)
        return output
