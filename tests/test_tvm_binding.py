"""The TVM-FFI slot binding (flashinfer_b200/tvm_binding.py): registration on the host, and a
call through the registered global function against the direct Python entry point."""
import pytest
import torch

from flashinfer_b200 import moe as fmoe
from flashinfer_b200 import workload as wl

tvm_ffi = pytest.importorskip("tvm_ffi")


def test_registers_the_slot_function():
    from flashinfer_b200 import tvm_binding
    f = tvm_binding.register()
    assert f is not None
    assert tvm_ffi.get_global_func("flashinfer.kernel") is not None


@pytest.mark.gpu
def test_slot_call_matches_run():
    from flashinfer_b200 import tvm_binding
    f = tvm_binding.register()
    cfg = wl.CONFIGS["t8_s2"]
    act = cfg.activations()
    ins = [t.cuda() for t in (act.routing_logits, act.routing_bias, act.hidden_states,
                              act.hidden_states_scale)]
    w = [t.cuda() for t in wl.local_weights(32, 0)]
    ref = fmoe.run(*ins, *w, 0, cfg.rsf)
    out = torch.full((cfg.T, wl.HIDDEN), 7.0, dtype=torch.bfloat16, device="cuda")
    f(*[tvm_ffi.from_dlpack(t) for t in ins + w], 0, cfg.rsf, tvm_ffi.from_dlpack(out))
    torch.cuda.synchronize()
    assert torch.equal(out.view(torch.int16), ref.view(torch.int16))
