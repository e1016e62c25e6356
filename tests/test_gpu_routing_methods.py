"""The definition family's other routing methods on the GPU (FmoeArgs.routing_method) against
the numpy oracle: selected experts exact, weights to 1e-5 relative (softmax and exp differ from
numpy's by an ulp or two), outputs within the operator's 1e-2."""
import numpy as np
import pytest
import torch

from flashinfer_b200 import _lib
from flashinfer_b200 import moe as fmoe
from flashinfer_b200 import workload as wl
from oracle import moe as omoe
from oracle import routing as orouting
from tests.conftest import oracle_weights_for
from tests.test_oracle_pins import METHOD_CASES, _by_id

pytestmark = pytest.mark.gpu


def _gpu(act):
    return (act.routing_logits.cuda(), act.routing_bias.cuda(), act.hidden_states.cuda(),
            act.hidden_states_scale.cuda())


@pytest.mark.parametrize("method,top_k", METHOD_CASES)
def test_method_routing_and_counts(method, top_k, gpu_weights):
    cfg = wl.CONFIGS["t64_s4"]
    act = cfg.activations()
    out, ws, lay = fmoe._launch(*_gpu(act), *gpu_weights, 0, cfg.rsf, None,
                                stop_after=_lib.STOP_ROUTE, routing_method=method, top_k=top_k)
    torch.cuda.synchronize()
    assert fmoe.read_status(ws) == 0
    view = fmoe.WorkspaceView(ws, lay, cfg.T, 32, wl.HIDDEN, wl.INTER)
    ids, w = (t.cpu().numpy() for t in view.topk())
    oids, ow = orouting.route_method(act.routing_logits.numpy(),
                                     act.routing_bias.float().numpy(), cfg.rsf, method, top_k)
    assert np.all(ids[:, top_k:] == -1)
    for (a_ids, a_w), (b_ids, b_w) in zip(_by_id(ids, w), _by_id(oids, ow)):
        np.testing.assert_array_equal(a_ids, b_ids)
        np.testing.assert_allclose(a_w, b_w, rtol=1e-5, atol=1e-9)
    lid = np.where((oids >= 0) & (oids < 32), oids, -1)
    counts = np.bincount(lid[lid >= 0].ravel(), minlength=32)
    np.testing.assert_array_equal(view.expert_count().cpu().numpy(), counts)


@pytest.mark.parametrize("T", [16, 2])  # T=2: the matrix-vector path
@pytest.mark.parametrize("method,top_k", [(1, 8), (3, 1), (5, 3)])
def test_method_output_matches_oracle(method, top_k, T, gpu_weights, cpu_weights):
    cfg = wl.CONFIGS["t16_s0"] if T == 16 else wl.Config("t2_s2006", 2, 2006)
    act = cfg.activations()
    out = fmoe.run(*_gpu(act), *gpu_weights, 0, cfg.rsf, routing_method=method, top_k=top_k)
    bits = out.view(torch.int16).cpu().numpy().view(np.uint16)
    ids, w = orouting.route_method(act.routing_logits.numpy(), act.routing_bias.float().numpy(),
                                   cfg.rsf, method, top_k)
    ids_k, w_k = ids[:, :top_k], w[:, :top_k]
    active = sorted({int(e) for e in ids_k.reshape(-1) if 0 <= int(e) < 32})
    W1, s1, W2, s2 = oracle_weights_for(cpu_weights, active)
    ref = omoe.moe_reference(act.hidden_states.view(torch.uint8).numpy(),
                             act.hidden_states_scale.numpy(), W1, s1, W2, s2, ids_k, w_k, 0)
    frac, err = omoe.allclose_report(bits, ref, atol=1e-2, rtol=1e-2)
    assert frac == 1.0, (frac, err)


def test_unsupported_method_arguments_are_rejected(gpu_weights):
    cfg = wl.CONFIGS["t8_s2"]
    act = cfg.activations()
    for method, top_k in ((3, 2), (1, 9), (1, 0), (0, 4), (6, 8)):
        with pytest.raises(Exception):
            fmoe.run(*_gpu(act), *gpu_weights, 0, cfg.rsf, routing_method=method, top_k=top_k)
