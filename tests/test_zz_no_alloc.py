"""The allocation-free routing + permutation entry point agrees with the workspace-based one.

``fmoe_route_permute_noalloc`` is for callers that cannot allocate device memory where they
enqueue work (pre-planned inference engines, graph capture with a fixed pool, hosts bound to
the C ABI without a device allocator): its scratch is a static device array inside the
library. Its tables must equal the ones ``fmoe_run`` leaves in the caller's workspace before
its GEMMs -- bit for bit, since this is integer and index work plus identical fp32 weights.
This file is named so that pytest collects it after every other test file.
"""
import ctypes

import pytest
import torch

from flashinfer_b200 import _lib
from flashinfer_b200 import moe as fmoe
from flashinfer_b200 import workload as wl


def _noalloc(act, rsf, local_start, e_local, cap):
    """Calls the entry point through the C ABI; the test allocates the output tables."""
    dev = torch.device("cuda:0")
    T = act.routing_logits.shape[0]
    lg = act.routing_logits.to(dev)
    b = act.routing_bias.to(dev)
    out = {
        "expert_count": torch.full((e_local,), -7, dtype=torch.int32, device=dev),
        "expert_base": torch.full((e_local + 1,), -7, dtype=torch.int32, device=dev),
        "slot_token": torch.full((cap,), -7, dtype=torch.int32, device=dev),
        "slot_weight": torch.full((cap,), -7.0, dtype=torch.float32, device=dev),
        "token_slot": torch.full((T, 8), -7, dtype=torch.int32, device=dev),
        "token_weight": torch.full((T, 8), -7.0, dtype=torch.float32, device=dev),
    }
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    rc = _lib.load().fmoe_route_permute_noalloc(
        p(lg), _lib.DTYPE_F32, p(b), _lib.DTYPE_BF16, T, e_local, local_start, float(rsf),
        p(out["expert_count"]), p(out["expert_base"]), p(out["slot_token"]),
        p(out["slot_weight"]), p(out["token_slot"]), p(out["token_weight"]),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _lib.check(rc, "fmoe_route_permute_noalloc")
    torch.cuda.synchronize()
    return out


def _route_only_weights(e_local):
    """Weight tensors of the right shapes for a call that stops after the permutation (their
    contents are never read before that stop point)."""
    dev = torch.device("cuda:0")
    H, I = wl.HIDDEN, wl.INTER
    return (torch.empty((e_local, 2 * I, H), dtype=torch.float8_e4m3fn, device=dev),
            torch.empty((e_local, 2 * I // 128, H // 128), dtype=torch.float32, device=dev),
            torch.empty((e_local, H, I), dtype=torch.float8_e4m3fn, device=dev),
            torch.empty((e_local, H // 128, I // 128), dtype=torch.float32, device=dev))


def _workspace_tables(act, rsf, local_start, gpu_weights):
    dev = torch.device("cuda:0")
    w1, s1, w2, s2 = gpu_weights
    _, ws, lay = fmoe._launch(act.routing_logits.to(dev), act.routing_bias.to(dev),
                              act.hidden_states.to(dev), act.hidden_states_scale.to(dev),
                              w1, s1, w2, s2, local_start, rsf, None, stop_after=_lib.STOP_ROUTE)
    torch.cuda.synchronize()
    T = act.routing_logits.shape[0]
    v = fmoe.WorkspaceView(ws, lay, T, w1.shape[0], wl.HIDDEN, wl.INTER)
    padded = int(v.plan()[1])
    return {
        "expert_count": v.expert_count().clone(),
        "expert_base": v.expert_base().clone(),
        "slot_token": v.slot_token()[:padded].clone(),
        "slot_weight": v.slot_weight()[:padded].clone(),
        "token_slot": v.token_slot().clone(),
        "token_weight": v._view(lay.token_weight, T * 8, torch.float32).view(T, 8).clone(),
    }, int(lay.cap_slots), padded


@pytest.mark.gpu
def test_noalloc_tables_match_workspace_entry_point(gpu_weights):
    # Two calls in a row on different inputs (and local ranges): the second must not see the
    # first's leftovers in the shared static scratch.
    cases = []
    for name, local_start in (("t1024_s6_skew", 0), ("t64_s4", 96)):
        cfg = wl.CONFIGS[name]
        act = cfg.activations()
        ref, cap, padded = _workspace_tables(act, cfg.rsf, local_start, gpu_weights)
        cases.append((name, cfg, act, local_start, ref, cap, padded))
    results = [_noalloc(act, cfg.rsf, ls, 32, cap) for _, cfg, act, ls, _, cap, _ in cases]
    for (name, cfg, act, local_start, ref, cap, padded), got in zip(cases, results):
        _check(name, ref, got, padded)


def _check(name, ref, got, padded):
    for key in ("expert_count", "expert_base", "token_slot"):
        assert torch.equal(got[key], ref[key]), (name, key)
    assert torch.equal(got["slot_token"][:padded], ref["slot_token"]), name
    # fp32 weights are copied, not recomputed differently: compare their bits
    assert torch.equal(got["slot_weight"][:padded].view(torch.int32),
                       ref["slot_weight"].view(torch.int32)), name
    assert torch.equal(got["token_weight"].view(torch.int32),
                       ref["token_weight"].view(torch.int32)), name
    # nothing written past the padded slot range
    assert torch.all(got["slot_token"][padded:] == -7), name


@pytest.mark.gpu
@pytest.mark.parametrize("e_local", [32, 256])
def test_noalloc_at_its_token_limit(e_local):
    """The largest accepted call (T = 4096: the top-k regions of the scratch are filled exactly;
    with 256 local experts the per-block histogram reaches its 8192-count capacity), then a
    T = 4095 call right after it on the same stream, both against the workspace tables."""
    weights = _route_only_weights(e_local)
    cases = []
    for T, seed in ((_lib.NOALLOC_MAX_TOKENS, 41), (_lib.NOALLOC_MAX_TOKENS - 1, 42)):
        act = wl.make_activations(T, seed)
        ref, cap, padded = _workspace_tables(act, wl.RSF_DEFAULT, 0, weights)
        cases.append((T, act, ref, cap, padded))
    results = [_noalloc(act, wl.RSF_DEFAULT, 0, e_local, cap) for _, act, _, cap, _ in cases]
    for (T, act, ref, cap, padded), got in zip(cases, results):
        _check(f"T={T} E={e_local}", ref, got, padded)


def test_noalloc_rejects_more_tokens_than_its_scratch_holds():
    lib = _lib.load()
    rc = lib.fmoe_route_permute_noalloc(None, 0, None, 1, _lib.NOALLOC_MAX_TOKENS + 1, 32, 0,
                                        2.5, None, None, None, None, None, None, None)
    assert rc == -9
    assert "4096" in _lib.ERRORS[rc]
