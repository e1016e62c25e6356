"""Drop-in operator entry point: ``run(...)`` with the reference's signature and layouts.

Mirrors ``solution/triton/kernel.py:600-825`` of the reference: same argument
order and meaning, same tensor layouts and dtypes, bf16 ``[T, 7168]`` output
written in place when ``output`` is given (destination-passing, as the
benchmark harness calls it). ``output`` may be omitted, in which case a new
tensor is returned -- the 10-argument form.

Underneath, one C-ABI call (``fmoe_run``) launches the sm_100a kernels on the
caller's current CUDA stream; there is no host synchronisation, no per-call
device allocation once the per-stream workspace exists, and no CPU fallback.
"""
from __future__ import annotations

import ctypes
from typing import Dict, Optional, Sequence, Tuple

import torch

from . import _lib
from ._lib import FmoeArgs

E_GLOBAL, TOP_K, N_GROUP, TOPK_GROUP, BLOCK = 256, 8, 8, 4, 128

_WORKSPACES: Dict[Tuple[int, int], torch.Tensor] = {}


def _dtype_tag(t: torch.Tensor, name: str) -> int:
    if t.dtype == torch.float32:
        return _lib.DTYPE_F32
    if t.dtype == torch.bfloat16:
        return _lib.DTYPE_BF16
    raise TypeError(f"{name} must be float32 or bfloat16, got {t.dtype}")


def _expect(t: torch.Tensor, name: str, shape, dtype) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (this operator has no CPU path)")
    if dtype is not None and t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if tuple(t.shape) != tuple(shape):
        raise ValueError(f"{name} must have shape {tuple(shape)}, got {tuple(t.shape)}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def workspace_for(device: torch.device, T: int, e_local: int, hidden: int, inter: int,
                  stream: Optional[torch.cuda.Stream] = None) -> Tuple[torch.Tensor, "_lib.FmoeLayout"]:
    """Per-(device, stream) workspace, grown on demand and reused across calls."""
    lay = _lib.workspace_layout(T, e_local, hidden, inter)
    stream = stream or torch.cuda.current_stream(device)
    key = (device.index if device.index is not None else torch.cuda.current_device(),
           stream.cuda_stream)
    ws = _WORKSPACES.get(key)
    if ws is None or ws.numel() < lay.total_bytes:
        _WORKSPACES.pop(key, None)
        ws = torch.empty(max(int(lay.total_bytes), 256), dtype=torch.uint8, device=device)
        _WORKSPACES[key] = ws
    return ws, lay


def _launch(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
            gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, local_expert_offset,
            routed_scaling_factor, output, stop_after: int = _lib.STOP_NONE,
            workspace: Optional[torch.Tensor] = None,
            routing_method: int = _lib.ROUTING_DEEPSEEK_V3, top_k: int = TOP_K,
            gemm_path: int = _lib.PATH_AUTO):
    T = int(routing_logits.shape[0])
    e_local = int(gemm1_weights.shape[0])
    hidden = int(hidden_states.shape[1])
    inter = int(gemm2_weights.shape[2])
    _expect(routing_logits, "routing_logits", (T, E_GLOBAL), None)
    _expect(routing_bias, "routing_bias", (E_GLOBAL,), None)
    _expect(hidden_states, "hidden_states", (T, hidden), torch.float8_e4m3fn)
    _expect(hidden_states_scale, "hidden_states_scale", (hidden // BLOCK, T), torch.float32)
    _expect(gemm1_weights, "gemm1_weights", (e_local, 2 * inter, hidden), torch.float8_e4m3fn)
    _expect(gemm1_weights_scale, "gemm1_weights_scale",
            (e_local, 2 * inter // BLOCK, hidden // BLOCK), torch.float32)
    _expect(gemm2_weights, "gemm2_weights", (e_local, hidden, inter), torch.float8_e4m3fn)
    _expect(gemm2_weights_scale, "gemm2_weights_scale",
            (e_local, hidden // BLOCK, inter // BLOCK), torch.float32)
    device = hidden_states.device
    for name, t in (("routing_logits", routing_logits), ("routing_bias", routing_bias),
                    ("hidden_states_scale", hidden_states_scale), ("gemm1_weights", gemm1_weights),
                    ("gemm1_weights_scale", gemm1_weights_scale), ("gemm2_weights", gemm2_weights),
                    ("gemm2_weights_scale", gemm2_weights_scale)):
        if t.device != device:
            raise ValueError(f"{name} is on {t.device}, hidden_states on {device}")
    if output is None:
        output = torch.empty((T, hidden), dtype=torch.bfloat16, device=device)
    _expect(output, "output", (T, hidden), None)
    if output.dtype not in (torch.bfloat16, torch.float32):
        raise TypeError(f"output must be bfloat16 (or float32 for partial sums), got {output.dtype}")

    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device)
        if workspace is None:
            ws, lay = workspace_for(device, T, e_local, hidden, inter, stream)
        else:
            lay = _lib.workspace_layout(T, e_local, hidden, inter)
            ws = workspace
        a = FmoeArgs()
        a.routing_logits = routing_logits.data_ptr()
        a.logits_dtype = _dtype_tag(routing_logits, "routing_logits")
        a.routing_bias = routing_bias.data_ptr()
        a.bias_dtype = _dtype_tag(routing_bias, "routing_bias")
        a.hidden_states = hidden_states.data_ptr()
        a.hidden_states_scale = hidden_states_scale.data_ptr()
        a.gemm1_weights = gemm1_weights.data_ptr()
        a.gemm1_weights_scale = gemm1_weights_scale.data_ptr()
        a.gemm2_weights = gemm2_weights.data_ptr()
        a.gemm2_weights_scale = gemm2_weights_scale.data_ptr()
        a.output = output.data_ptr()
        a.num_tokens = T
        a.hidden_size = hidden
        a.intermediate_size = inter
        a.num_experts = E_GLOBAL
        a.num_local_experts = e_local
        a.top_k = int(top_k)
        a.n_group = N_GROUP
        a.topk_group = TOPK_GROUP
        a.local_expert_offset = int(local_expert_offset)
        a.routed_scaling_factor = float(routed_scaling_factor)
        a.workspace = ws.data_ptr()
        a.workspace_bytes = ws.numel()
        a.stop_after = int(stop_after)
        a.gemm_path = int(gemm_path)
        a.output_dtype = _lib.OUT_F32 if output.dtype == torch.float32 else _lib.OUT_BF16
        a.routing_method = int(routing_method)
        rc = _lib.load().fmoe_run(ctypes.byref(a), ctypes.c_void_p(stream.cuda_stream))
    _lib.check(rc, "fmoe_run")
    return output, ws, lay


@torch.no_grad()
def run(routing_logits: torch.Tensor, routing_bias: torch.Tensor, hidden_states: torch.Tensor,
        hidden_states_scale: torch.Tensor, gemm1_weights: torch.Tensor,
        gemm1_weights_scale: torch.Tensor, gemm2_weights: torch.Tensor,
        gemm2_weights_scale: torch.Tensor, local_expert_offset: int,
        routed_scaling_factor: float, output: Optional[torch.Tensor] = None, *,
        routing_method: int = _lib.ROUTING_DEEPSEEK_V3, top_k: int = TOP_K) -> torch.Tensor:
    """Fused FP8 block-scale MoE with DeepSeek-V3 routing (reference ``kernel.py:600``).

    Tensor contract (all CUDA, contiguous):
      routing_logits       fp32 (or bf16)   [T, 256]
      routing_bias         bf16 (or fp32)   [256]
      hidden_states        float8_e4m3fn    [T, H]
      hidden_states_scale  fp32             [H/128, T]
      gemm1_weights        float8_e4m3fn    [E_local, 2I, H]   rows [0, I) gate, [I, 2I) up
      gemm1_weights_scale  fp32             [E_local, 2I/128, H/128]
      gemm2_weights        float8_e4m3fn    [E_local, H, I]
      gemm2_weights_scale  fp32             [E_local, H/128, I/128]
      output               bf16             [T, H]  (written in place; allocated if None)
    Experts [local_expert_offset, local_expert_offset + E_local) are local; the output holds
    the routing-weighted sum of the local experts only, like the reference.

    Keyword-only, beyond the reference's signature: ``routing_method`` (``_lib.ROUTING_*``) picks
    another routing of the same definition family (softmax/top-k variants, Llama4 top-1,
    uniform top-k; ``include/fmoe.h`` lists them) with ``top_k`` experts per token (1..8;
    DeepSeek-V3 uses 8, Llama4 1).
    """
    out, _, _ = _launch(routing_logits, routing_bias, hidden_states, hidden_states_scale,
                        gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
                        local_expert_offset, routed_scaling_factor, output,
                        routing_method=routing_method, top_k=top_k)
    return out


@torch.no_grad()
def run_routed(topk_ids: torch.Tensor, topk_weights: torch.Tensor, hidden_states: torch.Tensor,
               hidden_states_scale: torch.Tensor, gemm1_weights: torch.Tensor,
               gemm1_weights_scale: torch.Tensor, gemm2_weights: torch.Tensor,
               gemm2_weights_scale: torch.Tensor, local_expert_offset: int,
               output: Optional[torch.Tensor] = None, *,
               region_counts: Optional[torch.Tensor] = None, region_tokens: int = 0,
               region_output: Optional[Sequence[int]] = None,
               workspace: Optional[torch.Tensor] = None,
               phase_events: Optional[Sequence[torch.cuda.Event]] = None):
    """The operator on tokens routed elsewhere: the receiving side of expert parallelism.

    ``topk_ids`` int32 [T, 8] holds GLOBAL expert ids (-1 = no pick) and ``topk_weights`` fp32
    [T, 8] their routing weights, as the sending rank's routing produced them; the local experts
    are [local_expert_offset, local_expert_offset + E_local). With ``region_counts`` (int32 [R],
    on the device) the T tokens are R regions of ``region_tokens`` and token j of region r takes
    part only if j < region_counts[r]. ``output`` is bf16 or fp32 [T, H]; or, with
    ``region_output`` (R device addresses), each taking-part token's partial row is written as
    fp16 + power-of-two scales to region_output[r] + j * FMOE_EP_ROW_BYTES(H) (the address may be
    another GPU's memory mapped into this process) and nothing is returned. ``phase_events``
    (six CUDA events) are recorded at the operator's phase boundaries (``FmoeArgs.phase_events``).
    """
    T = int(topk_ids.shape[0])
    e_local = int(gemm1_weights.shape[0])
    hidden = int(hidden_states.shape[1])
    inter = int(gemm2_weights.shape[2])
    _expect(topk_ids, "topk_ids", (T, TOP_K), torch.int32)
    _expect(topk_weights, "topk_weights", (T, TOP_K), torch.float32)
    _expect(hidden_states, "hidden_states", (T, hidden), torch.float8_e4m3fn)
    _expect(hidden_states_scale, "hidden_states_scale", (hidden // BLOCK, T), torch.float32)
    _expect(gemm1_weights, "gemm1_weights", (e_local, 2 * inter, hidden), torch.float8_e4m3fn)
    _expect(gemm1_weights_scale, "gemm1_weights_scale",
            (e_local, 2 * inter // BLOCK, hidden // BLOCK), torch.float32)
    _expect(gemm2_weights, "gemm2_weights", (e_local, hidden, inter), torch.float8_e4m3fn)
    _expect(gemm2_weights_scale, "gemm2_weights_scale",
            (e_local, hidden // BLOCK, inter // BLOCK), torch.float32)
    device = hidden_states.device
    if region_output is None:
        if output is None:
            output = torch.empty((T, hidden), dtype=torch.bfloat16, device=device)
        _expect(output, "output", (T, hidden), None)
        if output.dtype not in (torch.bfloat16, torch.float32):
            raise TypeError(f"output must be bfloat16 or float32, got {output.dtype}")
    elif output is not None:
        raise ValueError("give either output or region_output")
    if region_counts is not None:
        _expect(region_counts, "region_counts", (region_counts.numel(),), torch.int32)
        if region_tokens <= 0 or T % region_tokens or T // region_tokens > _lib.EP_MAX_RANKS:
            raise ValueError(f"{T} tokens do not form at most {_lib.EP_MAX_RANKS} regions of "
                             f"{region_tokens}")
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device)
        if workspace is None:
            ws, lay = workspace_for(device, T, e_local, hidden, inter, stream)
        else:
            lay = _lib.workspace_layout(T, e_local, hidden, inter)
            ws = workspace
        a = FmoeArgs()
        a.hidden_states = hidden_states.data_ptr()
        a.hidden_states_scale = hidden_states_scale.data_ptr()
        a.gemm1_weights = gemm1_weights.data_ptr()
        a.gemm1_weights_scale = gemm1_weights_scale.data_ptr()
        a.gemm2_weights = gemm2_weights.data_ptr()
        a.gemm2_weights_scale = gemm2_weights_scale.data_ptr()
        a.num_tokens, a.hidden_size, a.intermediate_size = T, hidden, inter
        a.num_experts, a.num_local_experts = E_GLOBAL, e_local
        a.top_k, a.n_group, a.topk_group = TOP_K, N_GROUP, TOPK_GROUP
        a.local_expert_offset = int(local_expert_offset)
        a.routed_scaling_factor = 1.0
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
        a.topk_ids, a.topk_weights = topk_ids.data_ptr(), topk_weights.data_ptr()
        if region_counts is not None:
            a.region_counts, a.region_tokens = region_counts.data_ptr(), int(region_tokens)
        if phase_events is not None:
            handles = (ctypes.c_void_p * len(phase_events))(*[e.cuda_event for e in phase_events])
            a.phase_events = ctypes.cast(handles, ctypes.c_void_p)
            a.num_phase_events = len(phase_events)
        if region_output is not None:
            a.output_dtype = _lib.OUT_F16S
            for r, addr in enumerate(region_output):
                a.region_output[r] = int(addr)
        else:
            a.output = output.data_ptr()
            a.output_dtype = _lib.OUT_F32 if output.dtype == torch.float32 else _lib.OUT_BF16
        rc = _lib.load().fmoe_run(ctypes.byref(a), ctypes.c_void_p(stream.cuda_stream))
    _lib.check(rc, "fmoe_run (pre-routed)")
    return output


@torch.no_grad()
def route(routing_logits: torch.Tensor, routing_bias: torch.Tensor,
          routed_scaling_factor: float) -> Tuple[torch.Tensor, torch.Tensor]:
    """DeepSeek-V3 routing only: (global ids int32 [T, 8], weights fp32 [T, 8]).

    Ids come in selection order (descending biased score); the weights are the un-biased
    sigmoid scores normalised over the 8 picks and scaled by ``routed_scaling_factor``.
    """
    T = int(routing_logits.shape[0])
    _expect(routing_logits, "routing_logits", (T, E_GLOBAL), None)
    _expect(routing_bias, "routing_bias", (E_GLOBAL,), None)
    device = routing_logits.device
    ids = torch.empty((T, TOP_K), dtype=torch.int32, device=device)
    w = torch.empty((T, TOP_K), dtype=torch.float32, device=device)
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device)
        rc = _lib.load().fmoe_route(
            ctypes.c_void_p(routing_logits.data_ptr()), _dtype_tag(routing_logits, "routing_logits"),
            ctypes.c_void_p(routing_bias.data_ptr()), _dtype_tag(routing_bias, "routing_bias"),
            T, E_GLOBAL, TOP_K, N_GROUP, TOPK_GROUP, float(routed_scaling_factor),
            ctypes.c_void_p(ids.data_ptr()), ctypes.c_void_p(w.data_ptr()),
            ctypes.c_void_p(stream.cuda_stream))
    _lib.check(rc, "fmoe_route")
    return ids, w


@torch.no_grad()
def quantize_activations(x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """bf16 activations [T, H] (CUDA, contiguous) -> (e4m3 [T, H], fp32 scales [H/128, T]).

    The operator's input format: one scale per token and 128 columns, ``max(amax, 1e-30) / 448``,
    and the values divided by it and rounded to the nearest e4m3 (ties to even). The scales come
    transposed, as ``hidden_states_scale`` is consumed. Runs on the current stream.
    """
    if x.dim() != 2 or x.dtype != torch.bfloat16 or not x.is_cuda or not x.is_contiguous():
        raise TypeError("x must be a contiguous CUDA bfloat16 tensor of shape [T, H]")
    T, H = int(x.shape[0]), int(x.shape[1])
    if H % BLOCK != 0:
        raise ValueError(f"hidden size {H} is not a multiple of {BLOCK}")
    q = torch.empty((T, H), dtype=torch.float8_e4m3fn, device=x.device)
    scale = torch.empty((H // BLOCK, T), dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        rc = _lib.load().fmoe_quantize_activations(
            ctypes.c_void_p(x.data_ptr()), T, H, ctypes.c_void_p(q.data_ptr()),
            ctypes.c_void_p(scale.data_ptr()),
            ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream))
    _lib.check(rc, "fmoe_quantize_activations")
    return q, scale


def read_status(workspace: torch.Tensor) -> int:
    """Device status word of the last call on this workspace (synchronises the stream)."""
    st = ctypes.c_int32(0)
    with torch.cuda.device(workspace.device):
        rc = _lib.load().fmoe_read_status(ctypes.c_void_p(workspace.data_ptr()),
                                          ctypes.c_void_p(torch.cuda.current_stream().cuda_stream),
                                          ctypes.byref(st))
    _lib.check(rc, "fmoe_read_status")
    return st.value


class WorkspaceView:
    """Typed views of the workspace regions a staged call leaves behind (tests, tools)."""

    def __init__(self, ws: torch.Tensor, lay, T: int, e_local: int, hidden: int, inter: int):
        self.ws, self.lay, self.T, self.E, self.H, self.I = ws, lay, T, e_local, hidden, inter
        self.cap = int(lay.cap_slots)

    def _view(self, off: int, n: int, dtype: torch.dtype) -> torch.Tensor:
        nbytes = n * torch.empty((), dtype=dtype).element_size()
        return self.ws[off:off + nbytes].view(dtype)

    def plan(self):
        return self._view(self.lay.plan, 16, torch.int32)

    def topk(self):
        return (self._view(self.lay.topk_ids, self.T * TOP_K, torch.int32).view(self.T, TOP_K),
                self._view(self.lay.topk_weights, self.T * TOP_K, torch.float32).view(self.T, TOP_K))

    def expert_count(self):
        return self._view(self.lay.expert_count, self.E, torch.int32)

    def expert_base(self):
        return self._view(self.lay.expert_base, self.E + 1, torch.int32)

    def slot_token(self):
        return self._view(self.lay.slot_token, self.cap, torch.int32)

    def slot_weight(self):
        return self._view(self.lay.slot_weight, self.cap, torch.float32)

    def token_slot(self):
        return self._view(self.lay.token_slot, self.T * TOP_K, torch.int32).view(self.T, TOP_K)

    def intermediate(self):
        hi = self._view(self.lay.h_hi, self.cap * self.I, torch.uint8).view(self.cap, self.I)
        lo = self._view(self.lay.h_lo, self.cap * self.I, torch.uint8).view(self.cap, self.I)
        sc = self._view(self.lay.h_scale_t, (self.I // BLOCK) * self.cap,
                        torch.float32).view(self.I // BLOCK, self.cap)
        return hi, lo, sc

    def y_rows(self):
        """Per-slot GEMM2 rows decoded to fp32 (fp16 payload times its per-tile scale)."""
        y = self._view(self.lay.y_rows, self.cap * self.H, torch.float16).view(self.cap, self.H)
        sc = self._view(self.lay.y_scale, self.cap * (self.H // 256),
                        torch.float32).view(self.cap, self.H // 256)
        return y.float() * sc.repeat_interleave(256, dim=1)
