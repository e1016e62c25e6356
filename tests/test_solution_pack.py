"""The harness packaging of this build as a CUDA solution (flashinfer_b200/solution): the
Solution JSON carries the fields the reference's pack_solution.py writes, every source the slot
needs, and unpacks into a tree that builds (nvcc) and, on a GPU, serves flashinfer.kernel with
results bit-identical to run()."""
import ctypes
import json
import os
import re
import subprocess
import sys
import textwrap

import pytest

from flashinfer_b200 import solution as sol
from tests.conftest import ROOT


def test_manifest_fields_and_sources(tmp_path):
    out = tmp_path / "solution.json"
    s = sol.pack(str(out))
    on_disk = json.loads(out.read_text())
    assert on_disk == s
    cfg = sol.load_config()
    assert s["name"] == cfg["solution"]["name"]
    assert s["definition"] == "moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048"
    assert s["spec"]["language"] == "cuda" and s["spec"]["target_hardware"] == ["cuda"]
    entry_mod, entry_fn = s["spec"]["entry_point"].split("::")
    paths = [x["path"] for x in s["sources"]]
    assert entry_mod in paths and entry_fn == "kernel"
    csrc = os.path.join(ROOT, "flashinfer_b200", "csrc")
    for f in os.listdir(csrc):
        if f.endswith((".cu", ".h", ".cuh")):
            rel = f"flashinfer_b200/csrc/{f}"
            assert rel in paths, rel
            got = next(x["content"] for x in s["sources"] if x["path"] == rel)
            assert got == open(os.path.join(csrc, f)).read()
    assert "include/fmoe.h" in paths


def test_unpacked_solution_builds_and_exports_the_abi(tmp_path):
    """The unpacked tree compiles on its own (nvcc cross-compiles without a GPU) into a library
    that exports every entry point the packed header declares."""
    entry = sol.unpack(sol.pack(), str(tmp_path))
    assert os.path.exists(entry)
    code = textwrap.dedent(f"""
        import sys
        sys.path.insert(0, {str(tmp_path)!r})
        from flashinfer_b200 import build
        print(build.build())
    """)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, cwd=tmp_path)
    assert r.returncode == 0, r.stderr[-2000:]
    lib = r.stdout.strip().splitlines()[-1]
    assert lib.startswith(str(tmp_path))
    header = open(tmp_path / "include" / "fmoe.h").read()
    declared = set(re.findall(r"FMOE_API\s+[\w\s\*]+?\b(fmoe_\w+)\s*\(", header))
    loaded = ctypes.CDLL(lib)
    for name in declared:
        assert hasattr(loaded, name), name


@pytest.mark.gpu
def test_unpacked_slot_matches_run(tmp_path):
    """A fresh interpreter imports the unpacked binding.py (which builds and registers
    flashinfer.kernel) and calls the slot through TVM-FFI; its output equals run() bit for bit."""
    pytest.importorskip("tvm_ffi")
    import torch
    from flashinfer_b200 import moe as fmoe
    from flashinfer_b200 import workload as wl
    sol.unpack(sol.pack(), str(tmp_path / "sol"))
    cfg = wl.CONFIGS["t8_s2"]
    act = cfg.activations()
    ins = [act.routing_logits, act.routing_bias, act.hidden_states, act.hidden_states_scale]
    w = list(wl.local_weights(32, 0))
    in_file, out_file = tmp_path / "slot_in.pt", tmp_path / "slot_out.pt"
    torch.save({"ins": ins, "w": w, "rsf": cfg.rsf}, in_file)
    code = textwrap.dedent(f"""
        import sys
        sys.path.insert(0, {str(tmp_path / 'sol')!r})
        import torch, tvm_ffi
        import binding
        f = tvm_ffi.get_global_func("flashinfer.kernel")
        d = torch.load({str(in_file)!r})
        ts = [t.cuda() for t in d["ins"] + d["w"]]
        out = torch.full((ts[0].shape[0], ts[2].shape[1]), 7.0, dtype=torch.bfloat16, device="cuda")
        f(*[tvm_ffi.from_dlpack(t) for t in ts], 0, d["rsf"], tvm_ffi.from_dlpack(out))
        torch.cuda.synchronize()
        torch.save(out.cpu(), {str(out_file)!r})
        print(binding.__file__)
    """)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True,
                       cwd=tmp_path, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    assert str(tmp_path / "sol") in r.stdout
    ref = fmoe.run(*[t.cuda() for t in ins], *[t.cuda() for t in w], 0, cfg.rsf)
    got = torch.load(out_file)
    assert torch.equal(got.view(torch.int16), ref.cpu().view(torch.int16))
