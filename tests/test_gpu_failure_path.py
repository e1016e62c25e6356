"""The GEMMs' bounded waits: a wait that runs out ends the kernel with an error status instead of
a hang, and leaves the context usable. fmoe_debug_arm_timeout makes one GEMM of the next call wait
on a barrier nothing arrives on, with a 5 ms limit (no fault, no trap: the failure is a wait that
expires); the call must return promptly with the GEMM's timeout bit set, and the next call --
which needs the tensor memory the aborted CTAs held -- must run normally and match the oracle."""
import time

import numpy as np
import pytest
import torch

from flashinfer_b200 import _lib
from flashinfer_b200 import moe as fmoe
from flashinfer_b200 import workload as wl
from oracle import moe as omoe
from oracle import routing as orouting
from tests.conftest import oracle_weights_for


def test_arm_rejects_bad_arguments():
    lib = _lib.load()
    assert lib.fmoe_debug_arm_timeout(3, 5_000_000) == -2
    assert lib.fmoe_debug_arm_timeout(1, 10) == -2             # below 100 us
    assert lib.fmoe_debug_arm_timeout(2, 3_000_000_000) == -2  # above 2 s


def _call(act, gpu_weights, cfg):
    lg, b, hs, sc = (t.cuda() for t in (act.routing_logits, act.routing_bias, act.hidden_states,
                                        act.hidden_states_scale))
    out, ws, _ = fmoe._launch(lg, b, hs, sc, *gpu_weights, 0, cfg.rsf, None)
    torch.cuda.synchronize()
    return out, ws


@pytest.mark.gpu
@pytest.mark.parametrize("name,gemm", [("t256_s5", 1), ("t256_s5", 2), ("t64_s4", 2)])
def test_bounded_wait_runs_out_and_the_next_call_recovers(name, gemm, gpu_weights, cpu_weights):
    cfg = wl.CONFIGS[name]
    act = cfg.activations()
    _call(act, gpu_weights, cfg)                       # workspace and tensor maps exist
    lib = _lib.load()
    assert lib.fmoe_debug_arm_timeout(gemm, 5_000_000) == 0
    t0 = time.perf_counter()
    _, ws = _call(act, gpu_weights, cfg)
    elapsed = time.perf_counter() - t0
    status = fmoe.read_status(ws)
    bit = _lib.STATUS_TIMEOUT_GEMM1 if gemm == 1 else _lib.STATUS_TIMEOUT_GEMM2
    assert status & bit, status
    assert elapsed < 1.0, elapsed                      # the 5 ms limit, not the 2 s default
    # one-shot: the next call runs normally, on the same workspace, with correct output
    out, ws = _call(act, gpu_weights, cfg)
    assert fmoe.read_status(ws) == 0
    rows = np.array([0, 1, cfg.T // 2, cfg.T - 1])
    ids, w = orouting.route(act.routing_logits.numpy(), act.routing_bias.float().numpy(), cfg.rsf)
    ids, w = ids[rows], w[rows]
    active = sorted({int(e) for e in ids.reshape(-1) if 0 <= e < 32})
    W1, s1, W2, s2 = oracle_weights_for(cpu_weights, active)
    ref = omoe.moe_reference(act.hidden_states.view(torch.uint8).numpy()[rows],
                             act.hidden_states_scale.numpy()[:, rows], W1, s1, W2, s2, ids, w, 0)
    bits = out.view(torch.int16).cpu().numpy().view(np.uint16)[rows]
    frac, err = omoe.allclose_report(bits, ref, atol=1e-2, rtol=1e-2)
    assert frac == 1.0, (frac, err)
