"""Pins the CPU oracle to the operator's own PyTorch reference (golden vectors), no GPU.

The golden files come from running the definition reference
(``flashinfer/trace/templates/moe.py:109-184``) on the seeded workloads; see
``tests/golden/make_golden.py``.
"""
import numpy as np
import pytest
import torch

from flashinfer_b200 import workload as wl
from oracle import moe as omoe
from oracle import routing as orouting
from oracle.fp8 import bf16_round, bf16_to_f32, e4m3_to_f32, round_e4m3
from tests.conftest import bank_weights_for, oracle_weights_for
from tests.golden.make_golden import EP_CONFIGS, FULL_OUTPUT, SAMPLED

ALL = dict(wl.CONFIGS)
ALL.update(EP_CONFIGS)


@pytest.mark.parametrize("name", sorted(ALL))
def test_oracle_routing_matches_reference(name, golden_routing):
    cfg = ALL[name]
    act = cfg.activations()
    ids, w = orouting.route(act.routing_logits.numpy(), act.routing_bias.float().numpy(), cfg.rsf)
    order = np.argsort(ids, axis=1, kind="stable")
    sid = np.take_along_axis(ids, order, 1)
    gid = golden_routing[f"{name}/ids"].astype(np.int32)
    assert sid.shape == gid.shape
    np.testing.assert_array_equal(sid, gid)  # bit-exact per-token id sets
    key = f"{name}/weights"
    if key in golden_routing:
        sw = np.take_along_axis(w, order, 1)
        # the reference sums the 8 scores in torch's reduction order: weights agree to ~2 ulp
        np.testing.assert_allclose(sw, golden_routing[key], rtol=1e-6, atol=0)


def test_oracle_permutation_is_canonical():
    cfg = wl.CONFIGS["t256_s5_skew"]
    act = cfg.activations()
    ids, w = orouting.route(act.routing_logits.numpy(), act.routing_bias.float().numpy(), cfg.rsf)
    lid, lw = orouting.local_view(ids, w, 0, 32)
    counts, offsets, stoks, sw = orouting.permute(lid, lw, 32)
    assert counts.sum() == (lid >= 0).sum() == stoks.size
    for e in range(32):
        seg = stoks[offsets[e]:offsets[e + 1]]
        assert np.all(np.diff(seg) > 0)  # ascending tokens within each expert
        assert np.all((lid[seg] == e).any(axis=1))


@pytest.mark.parametrize("name", sorted(FULL_OUTPUT))
def test_oracle_forward_matches_reference(name, golden_outputs, cpu_weights):
    cfg = wl.CONFIGS[name]
    rows = FULL_OUTPUT[name]
    act = cfg.activations()
    ids, w = orouting.route(act.routing_logits.numpy(), act.routing_bias.float().numpy(), cfg.rsf)
    if rows is not None:
        ids, w = ids[:rows], w[:rows]
    active = sorted({int(e) for e in ids.reshape(-1) if 0 <= e < 32})
    W1, s1, W2, s2 = oracle_weights_for(cpu_weights, active)
    hs = act.hidden_states.view(torch.uint8).numpy()
    sc = act.hidden_states_scale.numpy()
    if rows is not None:
        hs, sc = hs[:rows], sc[:, :rows]
    got = omoe.moe_reference(hs, sc, W1, s1, W2, s2, ids, w, 0)
    ref = golden_outputs[f"{name}/out"]
    # Same fp32 algorithm; only BLAS summation order differs, so every element agrees to
    # within one bf16 ulp (relative 2^-8..2^-7) and almost all agree exactly.
    frac, maxerr = omoe.allclose_report(got, ref, atol=1e-5, rtol=2.0 ** -7)
    assert frac == 1.0, (frac, maxerr)
    assert np.mean(got == ref) > 0.99


class _DenseScales(dict):
    """Per-expert scale lookup that reports the local range size (the oracle takes len())."""

    def __init__(self, d, n):
        super().__init__(d)
        self.n = n

    def __len__(self):
        return self.n


@pytest.mark.parametrize("name", ["t1024_s6_skew", "t16384_s9", "ep_t16384_s10"])
def test_oracle_matches_reference_sampled_rows(name, golden_sampled):
    """The oracle against the reference's own output rows for sampled tokens of large configs
    (the first three sampled tokens; the expert-parallel config over all 256 experts)."""
    cfg = ALL[name]
    start, e_local, _ = SAMPLED[name]
    tok = golden_sampled[f"{name}/tokens"][:3]
    gold = golden_sampled[f"{name}/out"][:3]
    act = cfg.activations()
    ids, w = orouting.route(act.routing_logits.numpy()[tok], act.routing_bias.float().numpy(),
                            cfg.rsf)
    need = sorted({int(e) for e in ids.reshape(-1) if start <= e < start + e_local})
    W1, S1, W2, S2 = bank_weights_for(need)
    hs = act.hidden_states.view(torch.uint8).numpy()[tok]
    sc = act.hidden_states_scale.numpy()[:, tok]
    got = omoe.moe_reference(hs, sc, W1, _DenseScales(S1, e_local), W2, _DenseScales(S2, e_local),
                             ids, w, start)
    frac, maxerr = omoe.allclose_report(got, gold, atol=1e-5, rtol=2.0 ** -7)
    assert frac == 1.0, (frac, maxerr)


def test_e4m3_codec_roundtrip():
    raw = np.arange(256, dtype=np.uint8)
    vals = e4m3_to_f32(raw)
    finite = ~np.isnan(vals)
    np.testing.assert_array_equal(round_e4m3(vals[finite]), vals[finite])
    ref = torch.from_numpy(raw).view(torch.float8_e4m3fn).float().numpy()
    np.testing.assert_array_equal(vals[finite], ref[finite])
    x = np.random.default_rng(0).standard_normal(10000).astype(np.float32) * 100
    ours = round_e4m3(x)
    theirs = torch.from_numpy(np.clip(x, -448, 448)).to(torch.float8_e4m3fn).float().numpy()
    np.testing.assert_array_equal(ours, theirs)


def test_bf16_rounding_matches_torch():
    x = np.random.default_rng(1).standard_normal(10000).astype(np.float32) * 3
    ours = bf16_round(x)
    theirs = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    np.testing.assert_array_equal(ours, theirs)
    np.testing.assert_array_equal(bf16_to_f32(ours), torch.from_numpy(x).bfloat16().float().numpy())


def test_two_term_intermediate_meets_tolerance(golden_outputs, cpu_weights):
    """The device arithmetic (two-term e4m3 intermediate, bf16 Y rows) stays within
    atol=rtol=1e-2 of the reference at T=16; a single e4m3 term would not."""
    cfg = wl.CONFIGS["t16_s0"]
    act = cfg.activations()
    ids, w = orouting.route(act.routing_logits.numpy(), act.routing_bias.float().numpy(), cfg.rsf)
    active = sorted({int(e) for e in ids.reshape(-1) if 0 <= e < 32})
    W1, s1, W2, s2 = oracle_weights_for(cpu_weights, active)
    hs = act.hidden_states.view(torch.uint8).numpy()
    sc = act.hidden_states_scale.numpy()
    ref = golden_outputs["t16_s0/out"]
    dev = omoe.moe_device_numerics(hs, sc, W1, s1, W2, s2, ids, w, 0)
    frac, _ = omoe.allclose_report(dev, ref)
    assert frac == 1.0
    single = omoe.moe_device_numerics(hs, sc, W1, s1, W2, s2, ids, w, 0, two_term=False)
    frac1, _ = omoe.allclose_report(single, ref)
    assert frac1 < 0.95


def _quant_inputs(T: int, H: int, seed: int) -> torch.Tensor:
    """Seeded bf16 activations whose rows span 12 decades, with the edge blocks the quantiser
    must handle: an all-zero block, a lone spike, negative zeros and bf16 subnormals."""
    g = torch.Generator().manual_seed(seed)
    mag = torch.pow(10.0, torch.empty(T, 1).uniform_(-6, 6, generator=g))
    x = (torch.randn(T, H, generator=g) * mag).to(torch.bfloat16)
    if T >= 4 and H >= 512:
        x[0, :128] = 0.0
        x[1, 128:256] = 0.0
        x[1, 200] = -3.0e4
        x[2, 256:384] = -0.0
        x[3, 384:512] = torch.full((128,), 1.0e-39).to(torch.bfloat16)
    return x


def test_quant_oracle_matches_torch_cast():
    """oracle/quant.py against torch's float8_e4m3fn conversion (the benchmark inputs' rule)."""
    from oracle import quant as oquant
    x = _quant_inputs(64, 1024, 3)
    q_t, s_t = wl.quantize_activations(x)
    q_o, s_o = oquant.quantize_activations(x.float().numpy())
    np.testing.assert_array_equal(s_o.view(np.uint32), s_t.numpy().view(np.uint32))
    np.testing.assert_array_equal(q_o, e4m3_to_f32(q_t.view(torch.uint8).numpy()))


METHOD_CASES = [(1, 8), (1, 4), (2, 8), (2, 2), (3, 1), (4, 8), (4, 6), (5, 8), (5, 3)]


def _reference_method_routing(logits: torch.Tensor, bias: torch.Tensor, rsf: float, method: int,
                              top_k: int):
    """The routing lines of the definition's references (flashinfer/trace/templates/moe.py:
    205-209, 245-249, 285-288, 321-326, 370-378), in torch, as they are written there."""
    lg = logits.to(torch.float32) + bias.to(torch.float32).reshape(-1)
    if method == 1:
        s = torch.softmax(lg, dim=-1)
        _, idx = torch.topk(s, k=top_k, dim=1, largest=True, sorted=False)
        w = s.gather(1, idx) * rsf
    elif method == 2:
        _, idx = torch.topk(lg, k=top_k, dim=1, largest=True, sorted=False)
        w = torch.softmax(lg.gather(1, idx), dim=-1) * rsf
    elif method == 3:
        idx = lg.argmax(dim=-1, keepdim=True)
        w = (1.0 / (1.0 + torch.exp(-lg.gather(1, idx)))) * rsf
    elif method == 4:
        s = torch.softmax(lg, dim=-1)
        _, idx = torch.topk(s, k=top_k, dim=1, largest=True, sorted=False)
        g = s.gather(1, idx)
        w = g / (g.sum(dim=1, keepdim=True) + 1e-20) * rsf
    else:
        _, idx = torch.topk(lg, k=top_k, dim=1, largest=True, sorted=False)
        w = torch.full((lg.shape[0], top_k), rsf / top_k, dtype=torch.float32)
    return idx.numpy(), w.numpy()


def _by_id(ids: np.ndarray, w: np.ndarray):
    """Per token: (sorted ids, their weights) with the -1 padding dropped."""
    out = []
    for r in range(ids.shape[0]):
        keep = ids[r] >= 0
        o = np.argsort(ids[r][keep], kind="stable")
        out.append((ids[r][keep][o], w[r][keep][o]))
    return out


@pytest.mark.parametrize("method,top_k", METHOD_CASES)
def test_oracle_routing_methods_match_reference(method, top_k):
    cfg = wl.CONFIGS["t64_s4"]
    act = cfg.activations()
    ids, w = orouting.route_method(act.routing_logits.numpy(), act.routing_bias.float().numpy(),
                                   cfg.rsf, method, top_k)
    rid, rw = _reference_method_routing(act.routing_logits, act.routing_bias, cfg.rsf, method,
                                        top_k)
    for (a_ids, a_w), (b_ids, b_w) in zip(_by_id(ids, w), _by_id(rid.astype(np.int32), rw)):
        np.testing.assert_array_equal(a_ids, b_ids)
        np.testing.assert_allclose(a_w, b_w, rtol=1e-6, atol=1e-9)
