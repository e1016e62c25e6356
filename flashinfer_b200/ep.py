"""Expert parallelism for the fused MoE: one rank per GPU, 256 experts split contiguously.

The operator contract already describes one expert-parallel rank: ``run`` computes the
routing-weighted sum over the local experts ``[local_expert_offset, local_expert_offset + E_local)``
only (reference ``solution/triton/kernel.py:448-452``). With R ranks, rank r owns experts
``[r*256/R, (r+1)*256/R)`` and its own T_r tokens. One layer call on rank r:

1. route its tokens (``fmoe_route``: global top-8 ids and weights, bit-exact on every rank);
2. dispatch: each token goes once to every rank owning at least one of its picks (with R=8 at
   most 4 ranks, one per kept group). Its slot at rank d is its position among r's tokens sent
   to d (tokens ascending), and it travels as a record: the e4m3 row, its 128-column scales and
   the 8 picks with their weights (the receiver needs no routing of its own);
3. the receiver runs the operator pre-routed on everything it received (``run_routed``) and
   produces one partial row per received token (fp16 with a power-of-two scale per 256 columns);
4. combine: the sender adds the partial rows of its destinations in ascending rank order (the
   same expert order as the single-GPU sum) in fp32 and rounds once to bf16.

Two transports move the records and the partial rows:

* ``PeerTransport`` (GPUs, R >= 2): every rank allocates one exportable buffer and maps every
  other rank's buffer through CUDA IPC. The dispatch kernel stores the records straight into the
  destinations' receive regions and the receiver's combine kernel stores its partial rows
  straight into the senders' return regions -- plain stores over NVLink, no multicast, no TMA or
  library kernel reading another GPU's memory. Two one-element NCCL all-reduces order every
  rank's consumers after every rank's producers. Counts stay on the device: no host
  synchronisation, so a layer call can be captured in a CUDA graph.
* ``CollectiveTransport`` (any backend, gloo included): the same records and partial rows through
  ``all_to_all_single`` with host-side split sizes; used by the CPU tests with injectable
  routing and local compute (the numpy oracle standing in for the CUDA kernels).

``plan_dispatch`` restates the dispatch plan of the CUDA kernel (``k_ep_plan``) in torch.
"""
from __future__ import annotations

import ctypes
from typing import Callable, List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from . import _lib

E_GLOBAL = 256
TOP_K = 8
BLOCK = 128


def plan_dispatch(ids: torch.Tensor, experts_per_rank: int, world: int
                  ) -> Tuple[torch.Tensor, torch.Tensor]:
    """Slot of each token at each rank (int32 [T, world], -1 = not sent) and the per-rank counts
    (int64 [world]): a token is sent to rank d when one of its picks lies in d's experts, and
    its slot there is the number of earlier tokens sent to d."""
    T = ids.shape[0]
    owner = (ids.long() // experts_per_rank).clamp_(0, world - 1)
    dest = torch.zeros((T, world), dtype=torch.bool, device=ids.device)
    if T:
        dest.scatter_(1, owner, True)
    ranks = torch.cumsum(dest.to(torch.int64), dim=0) - 1
    slots = torch.where(dest, ranks, torch.full_like(ranks, -1)).to(torch.int32)
    return slots, dest.sum(dim=0).to(torch.int64)


def _device_view(addr: int, nbytes: int, device: torch.device) -> torch.Tensor:
    """A uint8 tensor over device memory this module owns (no copy, no ownership)."""

    class _Iface:
        __cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (addr, False),
                                    "version": 3, "strides": None}

    return torch.as_tensor(_Iface(), device=device)


class PeerTransport:
    """Per-rank receive/return buffer shared with every other rank through CUDA IPC."""

    def __init__(self, group, world: int, rank: int, capacity: int, hidden: int,
                 device: torch.device):
        self.world, self.rank, self.capacity, self.hidden, self.device = (world, rank, capacity,
                                                                           hidden, device)
        self.lib = _lib.load()
        self.lay = _lib.ep_layout(world, capacity, hidden)
        with torch.cuda.device(device):
            ptr = ctypes.c_void_p()
            _lib.check(self.lib.fmoe_ep_alloc(self.lay.total_bytes, ctypes.byref(ptr)),
                       "fmoe_ep_alloc")
            self.base = ptr.value
            handle = (ctypes.c_uint8 * 64)()
            _lib.check(self.lib.fmoe_ipc_get_handle(ctypes.c_void_p(self.base), handle),
                       "fmoe_ipc_get_handle")
            handles: List[Optional[bytes]] = [None] * world
            dist.all_gather_object(handles, bytes(handle), group=group)
            self.peers: List[int] = []
            self._opened: List[int] = []
            for d in range(world):
                if d == rank:
                    self.peers.append(self.base)
                    continue
                p = ctypes.c_void_p()
                h = (ctypes.c_uint8 * 64).from_buffer_copy(handles[d])
                _lib.check(self.lib.fmoe_ipc_open(h, ctypes.byref(p)), "fmoe_ipc_open")
                self.peers.append(p.value)
                self._opened.append(p.value)
        self.peer_array = (ctypes.c_void_p * world)(*self.peers)
        lay, n = self.lay, world * capacity
        buf = _device_view(self.base, lay.total_bytes, device)
        self.recv_hidden = buf[lay.recv_hidden:lay.recv_hidden + n * hidden] \
            .view(torch.float8_e4m3fn).view(n, hidden)
        nkb = hidden // BLOCK
        self.recv_scale = buf[lay.recv_scale:lay.recv_scale + nkb * n * 4] \
            .view(torch.float32).view(nkb, n)
        self.recv_ids = buf[lay.recv_ids:lay.recv_ids + n * TOP_K * 4].view(torch.int32) \
            .view(n, TOP_K)
        self.recv_weights = buf[lay.recv_weights:lay.recv_weights + n * TOP_K * 4] \
            .view(torch.float32).view(n, TOP_K)
        self.recv_counts = buf[lay.recv_counts:lay.recv_counts + world * 4].view(torch.int32)
        # rank d writes its partial rows for our tokens at region d of our ret_rows; we write
        # ours for rank s's tokens at region `rank` of s's ret_rows
        self.region_output = [self.peers[s] + lay.ret_rows + rank * capacity * lay.row_bytes
                              for s in range(world)]
        self.token_dest_slot = torch.empty((capacity, world), dtype=torch.int32, device=device)
        self._buf = buf

    def dispatch(self, ids, wts, hidden_states, hidden_states_scale):
        T = hidden_states.shape[0]
        stream = torch.cuda.current_stream(self.device).cuda_stream
        p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
        _lib.check(self.lib.fmoe_ep_dispatch(
            p(ids), p(wts), p(hidden_states), p(hidden_states_scale), T, self.capacity,
            self.hidden, self.world, self.rank, self.peer_array, p(self.token_dest_slot),
            ctypes.c_void_p(stream)), "fmoe_ep_dispatch")

    def reduce(self, T: int, out: torch.Tensor):
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _lib.check(self.lib.fmoe_ep_reduce(
            ctypes.c_void_p(self.token_dest_slot.data_ptr()), ctypes.c_void_p(self.base), T,
            self.capacity, self.hidden, self.world, ctypes.c_void_p(out.data_ptr()),
            ctypes.c_void_p(stream)), "fmoe_ep_reduce")

    def close(self, group=None):
        """Unmaps the other ranks' buffers, waits until every rank has done the same (collective:
        all ranks call it together), then frees this rank's buffer."""
        torch.cuda.synchronize(self.device)
        for p in self._opened:
            self.lib.fmoe_ipc_close(ctypes.c_void_p(p))
        self._opened = []
        if dist.is_available() and dist.is_initialized():
            dist.barrier(group=group)
        if self.base:
            self.lib.fmoe_ep_free(ctypes.c_void_p(self.base))
            self.base = 0


def _default_route(logits, bias, rsf):
    from .moe import route
    return route(logits, bias, rsf)


def _default_local(ids, wts, hs, sc, w1, s1, w2, s2, local_offset, out_f32):
    from .moe import run_routed
    run_routed(ids, wts, hs, sc, w1, s1, w2, s2, local_offset, out_f32)


class ExpertParallelMoE:
    """Expert-parallel fused MoE layer for one rank of ``group``.

    ``capacity``: the most tokens any rank passes to one ``forward`` (the peer transport's
    buffers are sized for it; every rank must use the same value). ``transport``: "peer" (CUDA
    IPC, the default on GPUs with more than one rank), "collective" (all_to_all_single; any
    backend) or "local" (one rank: the operator directly).
    """

    def __init__(self, group=None, capacity: int = 16384, hidden: int = 7168,
                 transport: Optional[str] = None, route_fn: Optional[Callable] = None,
                 local_fn: Optional[Callable] = None):
        self.group = group
        single = not (dist.is_available() and dist.is_initialized())
        self.world = 1 if single else dist.get_world_size(group)
        self.rank = 0 if single else dist.get_rank(group)
        if E_GLOBAL % self.world or self.world > _lib.EP_MAX_RANKS:
            raise ValueError(f"{E_GLOBAL} experts do not split evenly over {self.world} ranks "
                             f"(at most {_lib.EP_MAX_RANKS})")
        self.experts_per_rank = E_GLOBAL // self.world
        self.local_offset = self.rank * self.experts_per_rank
        self.capacity, self.hidden = int(capacity), int(hidden)
        self.route_fn = route_fn or _default_route
        self.local_fn = local_fn or _default_local
        if transport is None:
            transport = "local" if self.world == 1 else (
                "peer" if torch.cuda.is_available() and route_fn is None and local_fn is None
                else "collective")
        self.transport = transport
        self._peer: Optional[PeerTransport] = None
        self._flag: Optional[torch.Tensor] = None
        self.last_counts: Optional[Tuple[List[int], List[int]]] = None
        # optional CUDA events recorded between the phases (peer transport): route, dispatch,
        # barrier, local operator, barrier, reduce (7 events); and inside the local operator
        # (6 events, FmoeArgs.phase_events)
        self.phase_events: Optional[Sequence[torch.cuda.Event]] = None
        self.local_phase_events: Optional[Sequence[torch.cuda.Event]] = None

    # ------------------------------------------------------------------ peer transport
    def _peer_for(self, device):
        if self._peer is None:
            self._peer = PeerTransport(self.group, self.world, self.rank, self.capacity,
                                       self.hidden, device)
            self._flag = torch.zeros(1, dtype=torch.int32, device=device)
        return self._peer

    def _barrier(self):
        # orders every rank's consumers after every rank's producers (stream-ordered; a rank's
        # kernels before the collective have finished when any rank's collective completes)
        dist.all_reduce(self._flag, group=self.group)

    def _mark(self, i):
        if self.phase_events is not None and i < len(self.phase_events):
            self.phase_events[i].record()

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
        if T > self.capacity:
            raise ValueError(f"{T} tokens exceed the layer's capacity of {self.capacity}")
        dev = hidden_states.device
        if output is None:
            output = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
        if self.transport == "local":
            from .moe import run
            return run(routing_logits, routing_bias, hidden_states, hidden_states_scale,
                       gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
                       self.local_offset, routed_scaling_factor, output)
        if self.transport == "peer":
            return self._forward_peer(routing_logits, routing_bias, hidden_states,
                                      hidden_states_scale, gemm1_weights, gemm1_weights_scale,
                                      gemm2_weights, gemm2_weights_scale, routed_scaling_factor,
                                      output)
        return self._forward_collective(routing_logits, routing_bias, hidden_states,
                                        hidden_states_scale, gemm1_weights, gemm1_weights_scale,
                                        gemm2_weights, gemm2_weights_scale,
                                        routed_scaling_factor, output)

    def _forward_peer(self, logits, bias, hs, sc, w1, s1, w2, s2, rsf, output):
        from .moe import route, run_routed
        T, H = hs.shape
        if H != self.hidden:
            raise ValueError(f"hidden size {H} differs from the layer's {self.hidden}")
        peer = self._peer_for(hs.device)
        self._mark(0)
        ids, wts = route(logits, bias, rsf)
        self._mark(1)
        peer.dispatch(ids, wts, hs, sc)
        self._mark(2)
        self._barrier()
        self._mark(3)
        run_routed(peer.recv_ids, peer.recv_weights, peer.recv_hidden, peer.recv_scale, w1, s1,
                   w2, s2, self.local_offset, region_counts=peer.recv_counts,
                   region_tokens=self.capacity, region_output=peer.region_output,
                   phase_events=self.local_phase_events)
        self._mark(4)
        self._barrier()
        self._mark(5)
        peer.reduce(T, output)
        self._mark(6)
        return output

    def counts(self) -> List[int]:
        """Tokens this rank received from each rank in the last peer-transport call (syncs)."""
        return self._peer.recv_counts.tolist() if self._peer is not None else []

    def close(self):
        """Releases the peer transport's buffers (every rank of the group calls it together)."""
        if self._peer is not None:
            self._peer.close(self.group)
            self._peer = None

    # ------------------------------------------------------------------ collective transport
    def _all_to_all(self, out, inp, out_splits=None, in_splits=None):
        dist.all_to_all_single(out, inp, out_splits, in_splits, group=self.group)

    def _forward_collective(self, logits, bias, hs, sc, w1, s1, w2, s2, rsf, output):
        T, H = hs.shape
        dev = hs.device
        ids, wts = self.route_fn(logits, bias, rsf)
        slots, send_counts = plan_dispatch(ids, self.experts_per_rank, self.world)
        recv_counts = torch.empty_like(send_counts)
        self._all_to_all(recv_counts, send_counts)
        sc_list, rc_list = send_counts.tolist(), recv_counts.tolist()
        self.last_counts = (sc_list, rc_list)
        # tokens grouped by destination rank (ascending), tokens ascending within a rank = slots
        order = [torch.nonzero(slots[:, d] >= 0).flatten() for d in range(self.world)]
        send_tok = torch.cat(order) if order else torch.empty(0, dtype=torch.long)
        nkb = H // BLOCK
        rec = H + nkb * 4 + TOP_K * 8
        buf = torch.empty((send_tok.numel(), rec), dtype=torch.uint8, device=dev)
        if send_tok.numel():
            buf[:, :H] = hs.view(torch.uint8).index_select(0, send_tok)
            buf[:, H:H + nkb * 4] = sc.index_select(1, send_tok).t().contiguous().view(torch.uint8)
            buf[:, H + nkb * 4:H + nkb * 4 + TOP_K * 4] = \
                ids.to(torch.int32).index_select(0, send_tok).contiguous().view(torch.uint8)
            buf[:, H + nkb * 4 + TOP_K * 4:] = \
                wts.float().index_select(0, send_tok).contiguous().view(torch.uint8)
        recv = torch.empty((sum(rc_list), rec), dtype=torch.uint8, device=dev)
        self._all_to_all(recv, buf, rc_list, sc_list)
        n = recv.shape[0]
        partial = torch.empty((n, H), dtype=torch.float32, device=dev)
        if n:
            r_hs = recv[:, :H].contiguous().view(torch.float8_e4m3fn)
            r_sc = recv[:, H:H + nkb * 4].contiguous().view(torch.float32).view(n, nkb).t() \
                .contiguous()
            r_ids = recv[:, H + nkb * 4:H + nkb * 4 + TOP_K * 4].contiguous().view(torch.int32) \
                .view(n, TOP_K)
            r_w = recv[:, H + nkb * 4 + TOP_K * 4:].contiguous().view(torch.float32).view(n, TOP_K)
            self.local_fn(r_ids, r_w, r_hs, r_sc, w1, s1, w2, s2, self.local_offset, partial)
        back = torch.empty((send_tok.numel(), H), dtype=torch.float32, device=dev)
        self._all_to_all(back, partial, sc_list, rc_list)
        acc = torch.zeros((T, H), dtype=torch.float32, device=dev)
        start = 0
        for d in range(self.world):          # ascending rank = ascending expert order
            n_d = sc_list[d]
            if n_d:
                acc.index_add_(0, send_tok[start:start + n_d], back[start:start + n_d])
            start += n_d
        output.copy_(acc)
        return output
