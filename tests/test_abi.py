"""The C-ABI library loads, exports every entry point ``include/fmoe.h`` declares, agrees
with the ctypes mirror on struct layout, and rejects bad arguments on the host. No GPU."""
import ctypes
import os
import re
import subprocess
import tempfile

import pytest

from flashinfer_b200 import _lib
from tests.conftest import ROOT

HEADER = os.path.join(ROOT, "include", "fmoe.h")


def declared_functions():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"FMOE_API\s+[\w\s\*]+?\b(fmoe_\w+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_functions()
    assert set(names) == set(_lib.EXPORTS)
    out = subprocess.run(["nm", "-D", "--defined-only", _lib.LIB_PATH], check=True,
                         capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (fmoe_\w+)", out))
    for n in names:
        assert n in exported, n
        assert hasattr(lib, n)
    assert b"sm_100a" in lib.fmoe_version()


def test_struct_layout_matches_c():
    fields_args = [f for f, _ in _lib.FmoeArgs._fields_]
    fields_lay = [f for f, _ in _lib.FmoeLayout._fields_]
    prog = ["#include <stdio.h>", "#include <stddef.h>", f'#include "{HEADER}"', "int main(void){",
            'printf("%zu\\n", sizeof(FmoeArgs));']
    prog += [f'printf("%zu\\n", offsetof(FmoeArgs, {f}));' for f in fields_args]
    prog += ['printf("%zu\\n", sizeof(FmoeLayout));']
    prog += [f'printf("%zu\\n", offsetof(FmoeLayout, {f}));' for f in fields_lay]
    prog += ["return 0;}"]
    with tempfile.TemporaryDirectory() as d:
        c = os.path.join(d, "l.c")
        exe = os.path.join(d, "l")
        open(c, "w").write("\n".join(prog))
        subprocess.run(["gcc", "-std=c99", c, "-o", exe], check=True)
        vals = [int(x) for x in subprocess.run([exe], check=True, capture_output=True,
                                               text=True).stdout.split()]
    expect = [ctypes.sizeof(_lib.FmoeArgs)] + [getattr(_lib.FmoeArgs, f).offset for f in fields_args]
    expect += [ctypes.sizeof(_lib.FmoeLayout)] + [getattr(_lib.FmoeLayout, f).offset for f in fields_lay]
    assert vals == expect


def test_workspace_layout_is_consistent():
    for T in (1, 16, 1024, 16384):
        lay = _lib.workspace_layout(T, 32, 7168, 2048)
        offs = [getattr(lay, f) for f, t in _lib.FmoeLayout._fields_[1:] if t is ctypes.c_size_t]
        assert lay.status == 0
        assert all(o % 256 == 0 for o in offs)
        assert offs == sorted(offs)
        assert lay.total_bytes >= offs[-1]
        assert lay.cap_slots % 128 == 0
        assert lay.cap_slots >= T * 8 + 127 * min(32, T * 8)
        size = ctypes.c_size_t()
        assert _lib.load().fmoe_workspace_size(T, 32, 7168, 2048, ctypes.byref(size)) == 0
        assert size.value == lay.total_bytes


def test_bad_arguments_are_rejected_on_host():
    lib = _lib.load()
    assert lib.fmoe_run(None, None) == -1
    a = _lib.FmoeArgs()
    a.num_tokens, a.hidden_size, a.intermediate_size = 4, 7168, 2048
    a.num_experts, a.num_local_experts, a.top_k, a.n_group, a.topk_group = 256, 32, 8, 8, 4
    a.logits_dtype, a.bias_dtype = 0, 1
    assert lib.fmoe_run(ctypes.byref(a), None) == -1          # NULL tensors
    a.hidden_size = 7000
    assert lib.fmoe_run(ctypes.byref(a), None) == -2          # H not a multiple of 256
    a.hidden_size = 7168
    a.local_expert_offset = 240
    assert lib.fmoe_run(ctypes.byref(a), None) == -4          # 240 + 32 > 256
    a.local_expert_offset = 0
    a.logits_dtype = 7
    assert lib.fmoe_run(ctypes.byref(a), None) == -6
    a.logits_dtype = 0
    a.top_k = 6
    assert lib.fmoe_run(ctypes.byref(a), None) == -2          # DeepSeek-V3 needs top_k 8
    for method, top_k, rc in ((_lib.ROUTING_DEFAULT, 6, -1),   # valid: stops at the NULLs
                              (_lib.ROUTING_TOPK, 1, -1),
                              (_lib.ROUTING_LLAMA4, 2, -2),     # Llama4 is top-1
                              (_lib.ROUTING_RENORMALIZE, 9, -2),
                              (_lib.ROUTING_RENORMALIZE_NAIVE, 0, -2),
                              (6, 8, -2)):                      # no such method
        a.routing_method, a.top_k = method, top_k
        assert lib.fmoe_run(ctypes.byref(a), None) == rc, (method, top_k)
    a.routing_method, a.top_k = _lib.ROUTING_DEEPSEEK_V3, 8
    size = ctypes.c_size_t()
    assert lib.fmoe_workspace_size(16, 0, 7168, 2048, ctypes.byref(size)) == -2
    assert lib.fmoe_workspace_size(16, 32, 7168, 2048, None) == -1


def test_run_requires_cuda_tensors():
    import torch
    from flashinfer_b200 import run
    T = 2
    with pytest.raises(ValueError, match="CUDA"):
        run(torch.zeros(T, 256), torch.zeros(256, dtype=torch.bfloat16),
            torch.zeros(T, 7168).to(torch.float8_e4m3fn), torch.zeros(56, T),
            torch.zeros(1, 4096, 7168, dtype=torch.float8_e4m3fn), torch.zeros(1, 32, 56),
            torch.zeros(1, 7168, 2048, dtype=torch.float8_e4m3fn), torch.zeros(1, 56, 16), 0, 2.5)


def test_ep_layout_and_host_checks():
    """Expert-parallel buffer layout (256-byte aligned regions in order, rows of fp16 + scales)
    and the host-side argument checks of the dispatch and reduction entry points."""
    lib = _lib.load()
    for world, cap in ((2, 8192), (8, 2048), (4, 1)):
        lay = _lib.ep_layout(world, cap, 7168)
        offs = [lay.recv_hidden, lay.recv_scale, lay.recv_ids, lay.recv_weights, lay.recv_counts,
                lay.ret_rows]
        assert offs == sorted(offs) and all(o % 256 == 0 for o in offs)
        n = world * cap
        assert lay.recv_scale >= n * 7168 and lay.cap == cap
        assert lay.row_bytes == _lib.ep_row_bytes(7168) == 14464  # 7168 * 2 + 28 * 4, to 32 B
        assert lay.row_bytes % 32 == 0 and lay.ret_rows % 32 == 0
        assert lay.total_bytes >= lay.ret_rows + n * lay.row_bytes
    peers = (ctypes.c_void_p * 2)(None, None)
    H = 7168
    assert lib.fmoe_ep_dispatch(None, None, None, None, 4, 4, H, 3, 0, peers, None, None) == -2
    assert lib.fmoe_ep_dispatch(None, None, None, None, 8, 4, H, 2, 0, peers, None, None) == -2
    assert lib.fmoe_ep_dispatch(None, None, None, None, 4, 4, H, 2, 2, peers, None, None) == -2
    assert lib.fmoe_ep_dispatch(None, None, None, None, 4, 4, H, 2, 0, peers, None, None) == -1
    assert lib.fmoe_ep_reduce(None, None, 4, 2, H, 2, None, None) == -2
    assert lib.fmoe_ep_reduce(None, None, 2, 2, H, 9, None, None) == -2
    assert lib.fmoe_ep_layout(9, 16, H, ctypes.byref(_lib.FmoeEpLayout())) == -2


def test_pre_routed_argument_checks():
    """Partial-row output and token regions are only accepted for pre-routed calls, and the
    regions must tile the tokens (at most one region per rank)."""
    lib = _lib.load()
    a = _lib.FmoeArgs()
    a.num_tokens, a.hidden_size, a.intermediate_size = 8, 7168, 2048
    a.num_experts, a.num_local_experts, a.top_k, a.n_group, a.topk_group = 256, 32, 8, 8, 4
    a.logits_dtype, a.bias_dtype = 0, 1
    a.output_dtype = _lib.OUT_F16S
    assert lib.fmoe_run(ctypes.byref(a), None) == -6        # partial rows need given picks
    a.output_dtype = _lib.OUT_BF16
    a.region_counts, a.region_tokens = 16, 4                # any non-NULL address
    assert lib.fmoe_run(ctypes.byref(a), None) == -2        # regions need given picks
    a.topk_ids, a.topk_weights = 16, 16
    a.region_tokens = 3
    assert lib.fmoe_run(ctypes.byref(a), None) == -2        # 8 tokens are not regions of 3
    a.region_tokens, a.num_tokens = 1, 9
    assert lib.fmoe_run(ctypes.byref(a), None) == -2        # 9 regions > 8 ranks
