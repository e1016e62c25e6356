"""ctypes binding of the C ABI declared in ``include/fmoe.h``.

The library is the in-tree ``flashinfer_b200/_lib/libfmoe.so`` built by
``flashinfer_b200.build``. There is no fallback: if it is missing or does not
load, importing the operator raises, so a silent CPU or library path can never
stand in for the CUDA kernels.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, Structure, byref, c_char_p, c_float, c_int32, c_int64, c_size_t, c_void_p

# FLASHINFER_B200_LIB points at another build of the same library (A/B timing of two builds);
# a process that loads one says so on stderr, so a run on another build never passes unnoticed.
DEFAULT_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "libfmoe.so")
LIB_PATH = os.environ.get("FLASHINFER_B200_LIB") or DEFAULT_LIB_PATH

FMOE_OK = 0
ERRORS = {
    -1: "FMOE_ERR_NULL: a required pointer is NULL",
    -2: "FMOE_ERR_SHAPE: unsupported hidden/intermediate/expert/top-k sizes",
    -3: "FMOE_ERR_ALIGN: a pointer is not 16-byte aligned",
    -4: "FMOE_ERR_OFFSET: local_expert_offset + num_local_experts exceeds the expert count",
    -5: "FMOE_ERR_WORKSPACE: workspace missing or too small",
    -6: "FMOE_ERR_DTYPE: unsupported routing logits / bias dtype",
    -7: "FMOE_ERR_CUDA: a CUDA runtime or driver call failed",
    -8: "FMOE_ERR_DEVICE: the current device is not sm_100 (B200)",
    -9: "FMOE_ERR_NOALLOC_LIMIT: more tokens than fmoe_route_permute_noalloc supports (4096)",
}
NOALLOC_MAX_TOKENS = 4096
DTYPE_F32 = 0
DTYPE_BF16 = 1
OUT_BF16 = 0
OUT_F32 = 1
OUT_F16S = 2
EP_MAX_RANKS = 8


def ep_row_bytes(hidden: int) -> int:
    """FMOE_EP_ROW_BYTES: an fp16 partial row plus its power-of-two scale per 256 columns,
    padded to a multiple of 32 bytes."""
    return (hidden * 2 + hidden // 256 * 4 + 31) // 32 * 32
STOP_NONE, STOP_ROUTE, STOP_GATHER, STOP_GEMM1, STOP_GEMM2 = 0, 1, 2, 3, 4
PATH_AUTO, PATH_GEMM = 0, 1
GEMV_MAX_T = 2  # calls of at most this many tokens take the matrix-vector path (PATH_AUTO)
# FMOE_ROUTING_* (include/fmoe.h)
(ROUTING_DEEPSEEK_V3, ROUTING_DEFAULT, ROUTING_RENORMALIZE, ROUTING_LLAMA4,
 ROUTING_RENORMALIZE_NAIVE, ROUTING_TOPK) = range(6)
STATUS_TIMEOUT_GEMM1 = 0x1
STATUS_TIMEOUT_GEMM2 = 0x2

EXPORTS = ("fmoe_workspace_size", "fmoe_workspace_layout", "fmoe_run", "fmoe_route",
           "fmoe_read_status", "fmoe_device_sm_count", "fmoe_version",
           "fmoe_route_permute_noalloc", "fmoe_quantize_activations", "fmoe_ep_layout",
           "fmoe_ep_alloc", "fmoe_ep_free", "fmoe_ipc_get_handle", "fmoe_ipc_open",
           "fmoe_ipc_close", "fmoe_ep_dispatch", "fmoe_ep_reduce", "fmoe_fp8_mma_peak",
           "fmoe_debug_arm_timeout")


class FmoeArgs(Structure):
    _fields_ = [
        ("routing_logits", c_void_p),
        ("logits_dtype", c_int32),
        ("routing_bias", c_void_p),
        ("bias_dtype", c_int32),
        ("hidden_states", c_void_p),
        ("hidden_states_scale", c_void_p),
        ("gemm1_weights", c_void_p),
        ("gemm1_weights_scale", c_void_p),
        ("gemm2_weights", c_void_p),
        ("gemm2_weights_scale", c_void_p),
        ("output", c_void_p),
        ("num_tokens", c_int32),
        ("hidden_size", c_int32),
        ("intermediate_size", c_int32),
        ("num_experts", c_int32),
        ("num_local_experts", c_int32),
        ("top_k", c_int32),
        ("n_group", c_int32),
        ("topk_group", c_int32),
        ("local_expert_offset", c_int32),
        ("routed_scaling_factor", c_float),
        ("workspace", c_void_p),
        ("workspace_bytes", c_size_t),
        ("stop_after", c_int32),
        ("phase_events", c_void_p),
        ("num_phase_events", c_int32),
        ("output_dtype", c_int32),
        ("routing_method", c_int32),
        ("topk_ids", c_void_p),
        ("topk_weights", c_void_p),
        ("region_counts", c_void_p),
        ("region_tokens", c_int32),
        ("region_output", c_void_p * EP_MAX_RANKS),
        ("gemm_path", c_int32),
    ]


class FmoeEpLayout(Structure):
    _fields_ = [(n, c_size_t) for n in ("total_bytes", "recv_hidden", "recv_scale", "recv_ids",
                                        "recv_weights", "recv_counts", "ret_rows")] + \
        [("cap", c_int64), ("row_bytes", c_size_t)]


class FmoeLayout(Structure):
    _fields_ = [(n, c_size_t) for n in (
        "total_bytes", "status", "plan", "topk_ids", "topk_weights", "expert_count",
        "expert_base", "slot_token", "slot_weight", "token_slot", "token_weight", "a_perm",
        "a_scale_t", "h_hi", "h_lo", "h_scale_t", "y_rows", "y_scale", "partials", "counters",
        "block_hist", "block_off")] + [
        ("cap_slots", c_int64), ("max_units", c_int64), ("tokens_per_block", c_int64),
        ("num_blocks", c_int64)]


_lib = None


def load() -> ctypes.CDLL:
    """Loads the library once; raises if it is absent (build it with flashinfer_b200.build)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build the CUDA library with `python -m flashinfer_b200.build`")
    if LIB_PATH != DEFAULT_LIB_PATH:
        import sys
        print(f"flashinfer_b200: loading {LIB_PATH} (FLASHINFER_B200_LIB), not the in-tree build",
              file=sys.stderr)
    lib = ctypes.CDLL(LIB_PATH)
    lib.fmoe_workspace_size.argtypes = [c_int32, c_int32, c_int32, c_int32, POINTER(c_size_t)]
    lib.fmoe_workspace_layout.argtypes = [c_int32, c_int32, c_int32, c_int32, POINTER(FmoeLayout)]
    lib.fmoe_run.argtypes = [POINTER(FmoeArgs), c_void_p]
    lib.fmoe_route.argtypes = [c_void_p, c_int32, c_void_p, c_int32, c_int32, c_int32, c_int32,
                               c_int32, c_int32, c_float, c_void_p, c_void_p, c_void_p]
    lib.fmoe_read_status.argtypes = [c_void_p, c_void_p, POINTER(c_int32)]
    lib.fmoe_route_permute_noalloc.argtypes = [c_void_p, c_int32, c_void_p, c_int32, c_int32,
                                               c_int32, c_int32, c_float, c_void_p, c_void_p,
                                               c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]
    lib.fmoe_device_sm_count.argtypes = [POINTER(c_int32)]
    lib.fmoe_quantize_activations.argtypes = [c_void_p, c_int32, c_int32, c_void_p, c_void_p,
                                              c_void_p]
    lib.fmoe_ep_layout.argtypes = [c_int32, c_int32, c_int32, POINTER(FmoeEpLayout)]
    lib.fmoe_ep_alloc.argtypes = [c_size_t, POINTER(c_void_p)]
    lib.fmoe_ep_free.argtypes = [c_void_p]
    lib.fmoe_ipc_get_handle.argtypes = [c_void_p, c_void_p]
    lib.fmoe_ipc_open.argtypes = [c_void_p, POINTER(c_void_p)]
    lib.fmoe_ipc_close.argtypes = [c_void_p]
    lib.fmoe_ep_dispatch.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p, c_int32, c_int32,
                                     c_int32, c_int32, c_int32, c_void_p, c_void_p, c_void_p]
    lib.fmoe_ep_reduce.argtypes = [c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int32,
                                   c_void_p, c_void_p]
    lib.fmoe_fp8_mma_peak.argtypes = [c_int32, c_void_p, POINTER(ctypes.c_double), c_void_p]
    lib.fmoe_debug_arm_timeout.argtypes = [c_int32, ctypes.c_uint64]
    lib.fmoe_version.restype = c_char_p
    for name in EXPORTS:
        if name != "fmoe_version":
            getattr(lib, name).restype = c_int32
    _lib = lib
    return lib


def check(rc: int, what: str) -> None:
    if rc != FMOE_OK:
        raise RuntimeError(f"{what} failed: {ERRORS.get(rc, f'error {rc}')}")


def workspace_layout(T: int, e_local: int, hidden: int, inter: int) -> FmoeLayout:
    lay = FmoeLayout()
    check(load().fmoe_workspace_layout(T, e_local, hidden, inter, byref(lay)), "fmoe_workspace_layout")
    return lay


def ep_layout(world: int, capacity: int, hidden: int) -> FmoeEpLayout:
    lay = FmoeEpLayout()
    check(load().fmoe_ep_layout(world, capacity, hidden, byref(lay)), "fmoe_ep_layout")
    return lay
