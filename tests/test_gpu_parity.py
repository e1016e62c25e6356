"""GPU parity of the sm_100a path (through the C ABI) against the CPU oracle.

Bars (from the operator's benchmark contract):
  * routing ids and the permutation: bit-exact;
  * routing weights: bit-exact against the oracle (same arithmetic), <= 1e-6 relative
    against the reference's golden weights;
  * bf16 output: atol = rtol = 1e-2 against the fp32 oracle, on every element.
"""
import numpy as np
import pytest
import torch

from flashinfer_b200 import _lib
from flashinfer_b200 import moe as fmoe
from flashinfer_b200 import workload as wl
from oracle import moe as omoe
from oracle import routing as orouting
from tests.conftest import bank_weights_for, oracle_weights_for
from tests.golden.make_golden import EP_CONFIGS, FULL_OUTPUT, SAMPLED

pytestmark = pytest.mark.gpu

ATOL = 1e-2
RTOL = 1e-2
ALL = dict(wl.CONFIGS)
ALL.update(EP_CONFIGS)


def to_gpu(act):
    return (act.routing_logits.cuda(), act.routing_bias.cuda(), act.hidden_states.cuda(),
            act.hidden_states_scale.cuda())


def oracle_rows(act, cfg, rows, cpu_weights, local_start=0, e_local=32):
    ids, w = orouting.route(act.routing_logits.numpy(), act.routing_bias.float().numpy(), cfg.rsf)
    ids, w = ids[rows], w[rows]
    active = sorted({int(e) - local_start for e in ids.reshape(-1)
                     if 0 <= int(e) - local_start < e_local})
    W1, s1, W2, s2 = oracle_weights_for(cpu_weights, active)
    hs = act.hidden_states.view(torch.uint8).numpy()[rows]
    sc = act.hidden_states_scale.numpy()[:, rows]
    return omoe.moe_reference(hs, sc, W1, s1, W2, s2, ids, w, local_start)


def run_gpu(act, gpu_weights, cfg, local_start=0, stop=_lib.STOP_NONE, path=_lib.PATH_AUTO):
    lg, b, hs, sc = to_gpu(act)
    w1, s1, w2, s2 = gpu_weights
    out, ws, lay = fmoe._launch(lg, b, hs, sc, w1, s1, w2, s2, local_start, cfg.rsf, None,
                                stop_after=stop, gemm_path=path)
    torch.cuda.synchronize()
    assert fmoe.read_status(ws) == 0
    return out, ws, lay


@pytest.mark.parametrize("name", sorted(ALL))
def test_routing_bit_exact(name, golden_routing):
    cfg = ALL[name]
    act = cfg.activations()
    ids, w = fmoe.route(act.routing_logits.cuda(), act.routing_bias.cuda(), cfg.rsf)
    ids, w = ids.cpu().numpy(), w.cpu().numpy()
    oids, ow = orouting.route(act.routing_logits.numpy(), act.routing_bias.float().numpy(), cfg.rsf)
    np.testing.assert_array_equal(ids, oids)
    np.testing.assert_array_equal(w.view(np.uint32), ow.view(np.uint32))
    np.testing.assert_array_equal(np.sort(ids, axis=1), golden_routing[f"{name}/ids"].astype(np.int32))


def test_routing_bf16_logits_and_fp32_bias():
    cfg = wl.CONFIGS["t1024_s6"]
    act = cfg.activations()
    lg = act.routing_logits.to(torch.bfloat16)
    b = act.routing_bias.float()
    ids, w = fmoe.route(lg.cuda(), b.cuda(), cfg.rsf)
    oids, ow = orouting.route(lg.float().numpy(), b.numpy(), cfg.rsf)
    np.testing.assert_array_equal(ids.cpu().numpy(), oids)
    np.testing.assert_array_equal(w.cpu().numpy().view(np.uint32), ow.view(np.uint32))


@pytest.mark.parametrize("name,local_start", [("t16_s0", 0), ("t32_s3", 0), ("t64_s4", 0),
                                              ("t256_s5_skew", 0), ("t1024_s6", 0),
                                              ("t16384_s9", 0), ("ep_t16384_s10", 96)])
def test_permutation_bit_exact(name, local_start, gpu_weights):
    cfg = ALL[name]
    act = cfg.activations()
    _, ws, lay = run_gpu(act, gpu_weights, cfg, local_start=local_start, stop=_lib.STOP_ROUTE)
    view = fmoe.WorkspaceView(ws, lay, cfg.T, 32, wl.HIDDEN, wl.INTER)
    oids, ow = orouting.route(act.routing_logits.numpy(), act.routing_bias.float().numpy(), cfg.rsf)
    lid, lw = orouting.local_view(oids, ow, local_start, 32)
    counts, offsets, stoks, sw = orouting.permute(lid, lw, 32)
    np.testing.assert_array_equal(view.expert_count().cpu().numpy(), counts)
    base = view.expert_base().cpu().numpy()
    slot_tok = view.slot_token().cpu().numpy()
    slot_w = view.slot_weight().cpu().numpy()
    plan = view.plan().cpu().numpy()
    assert plan[0] == counts.sum()
    assert plan[1] == base[-1] == sum((c + 127) // 128 * 128 for c in counts)
    for e in range(32):
        seg = slice(base[e], base[e] + counts[e])
        np.testing.assert_array_equal(slot_tok[seg], stoks[offsets[e]:offsets[e + 1]])
        np.testing.assert_array_equal(slot_w[seg].view(np.uint32),
                                      sw[offsets[e]:offsets[e + 1]].view(np.uint32))
        assert np.all(slot_tok[base[e] + counts[e]:base[e + 1]] == -1)
    # token -> slot map: local picks in ascending expert order, -1 afterwards
    ts = view.token_slot().cpu().numpy()
    for t in range(0, cfg.T, max(1, cfg.T // 257)):
        exp = sorted(int(e) for e in lid[t] if e >= 0)
        got = [int(s) for s in ts[t] if s >= 0]
        assert len(got) == len(exp)
        for s, e in zip(got, exp):
            assert base[e] <= s < base[e] + counts[e] and slot_tok[s] == t


# The smallest calls run the matrix-vector path by default; PATH_GEMM keeps the grouped
# tensor-core GEMMs covered at the same sizes.
SMALL_PATHS = [(n, p) for n in sorted(FULL_OUTPUT) for p in
               ([_lib.PATH_AUTO, _lib.PATH_GEMM] if wl.CONFIGS[n].T <= _lib.GEMV_MAX_T
                else [_lib.PATH_AUTO])]


@pytest.mark.parametrize("name,path", SMALL_PATHS)
def test_output_matches_oracle_and_golden(name, path, gpu_weights, cpu_weights, golden_outputs):
    cfg = wl.CONFIGS[name]
    act = cfg.activations()
    out, _, _ = run_gpu(act, gpu_weights, cfg, path=path)
    bits = out.view(torch.int16).cpu().numpy().view(np.uint16)
    rows = FULL_OUTPUT[name] or cfg.T
    sel = np.arange(rows)
    ref = oracle_rows(act, cfg, sel, cpu_weights)
    frac, err = omoe.allclose_report(bits[sel], ref, atol=ATOL, rtol=RTOL)
    assert frac == 1.0, (frac, err)
    gold = golden_outputs[f"{name}/out"]
    frac, err = omoe.allclose_report(bits[:gold.shape[0]], gold, atol=ATOL, rtol=RTOL)
    assert frac == 1.0, (frac, err)


@pytest.mark.parametrize("name", ["t32_s3", "t256_s5", "t1024_s6", "t1024_s6_skew", "t4096_s7",
                                  "t8192_s8", "t16384_s9"])
def test_output_sampled_rows(name, gpu_weights, cpu_weights):
    """Large T: every token's output depends only on its own row and routing, so the oracle
    checks a seeded sample of rows (plus the first and last token)."""
    cfg = wl.CONFIGS[name]
    act = cfg.activations()
    out, _, _ = run_gpu(act, gpu_weights, cfg)
    bits = out.view(torch.int16).cpu().numpy().view(np.uint16)
    rng = np.random.default_rng(cfg.seed)
    sel = np.unique(np.concatenate([[0, cfg.T - 1], rng.choice(cfg.T, size=min(cfg.T, 24),
                                                                replace=False)]))
    ref = oracle_rows(act, cfg, sel, cpu_weights)
    frac, err = omoe.allclose_report(bits[sel], ref, atol=ATOL, rtol=RTOL)
    assert frac == 1.0, (frac, err)
    assert np.isfinite(out.float().cpu().numpy()).all()


@pytest.mark.parametrize("name", sorted(n for n, v in SAMPLED.items() if v[1] == 32))
def test_output_matches_reference_golden_rows(name, gpu_weights, golden_sampled):
    """Every larger single-GPU config against the reference's own output rows (sampled tokens,
    produced by tests/golden/make_golden.py from the operator's PyTorch definition)."""
    cfg = wl.CONFIGS[name]
    act = cfg.activations()
    out, _, _ = run_gpu(act, gpu_weights, cfg)
    bits = out.view(torch.int16).cpu().numpy().view(np.uint16)
    tok = golden_sampled[f"{name}/tokens"]
    frac, err = omoe.allclose_report(bits[tok], golden_sampled[f"{name}/out"], atol=ATOL, rtol=RTOL)
    assert frac == 1.0, (frac, err)


def _weights_256(experts):
    """Stacked weights of all 256 experts on the GPU, with the seeded values for ``experts`` and
    zeros elsewhere (only the tokens whose picks are all in ``experts`` are checked)."""
    H, I = wl.HIDDEN, wl.INTER
    dev = torch.device("cuda:0")
    w1 = torch.zeros((256, 2 * I, H), dtype=torch.uint8, device=dev)
    s1 = torch.zeros((256, 2 * I // 128, H // 128), dtype=torch.float32, device=dev)
    w2 = torch.zeros((256, H, I), dtype=torch.uint8, device=dev)
    s2 = torch.zeros((256, H // 128, I // 128), dtype=torch.float32, device=dev)
    for e in experts:
        q1, a1, q2, a2 = wl.WeightBank.get(int(e))
        w1[e].copy_(q1.view(torch.uint8))
        s1[e].copy_(a1)
        w2[e].copy_(q2.view(torch.uint8))
        s2[e].copy_(a2)
    return (w1.view(torch.float8_e4m3fn), s1, w2.view(torch.float8_e4m3fn), s2)


@pytest.mark.parametrize("name", sorted(EP_CONFIGS))
def test_all_256_experts_on_one_gpu(name, golden_sampled):
    """configs[4]'s global batch (T=16384) with all 256 experts local on one GPU -- the
    single-GPU point of the expert-parallel scaling run -- against the reference's rows and the
    oracle for the sampled tokens."""
    cfg = EP_CONFIGS[name]
    act = cfg.activations()
    tok = golden_sampled[f"{name}/tokens"]
    ids, w = orouting.route(act.routing_logits.numpy()[tok], act.routing_bias.float().numpy(),
                            cfg.rsf)
    need = sorted({int(e) for e in ids.reshape(-1)})
    weights = _weights_256(need)
    out, _, _ = run_gpu(act, weights, cfg)
    bits = out.view(torch.int16).cpu().numpy().view(np.uint16)
    frac, err = omoe.allclose_report(bits[tok], golden_sampled[f"{name}/out"], atol=ATOL, rtol=RTOL)
    assert frac == 1.0, (frac, err)
    W1, S1, W2, S2 = bank_weights_for(need)

    class Dense(dict):
        def __len__(self):
            return 256

    ref = omoe.moe_reference(act.hidden_states.view(torch.uint8).numpy()[tok],
                             act.hidden_states_scale.numpy()[:, tok], W1, Dense(S1), W2,
                             Dense(S2), ids, w, 0)
    frac, err = omoe.allclose_report(bits[tok], ref, atol=ATOL, rtol=RTOL)
    assert frac == 1.0, (frac, err)


def test_deterministic_bits(gpu_weights):
    cfg = wl.CONFIGS["t1024_s6_skew"]
    act = cfg.activations()
    a, _, _ = run_gpu(act, gpu_weights, cfg)
    a = a.clone()
    b, _, _ = run_gpu(act, gpu_weights, cfg)
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))


def test_intermediate_two_term_encoding(gpu_weights, cpu_weights):
    """GEMM1 + SwiGLU output, decoded as (hi + lo) * scale, against the oracle's fp32 h."""
    cfg = wl.CONFIGS["t64_s4"]
    act = cfg.activations()
    _, ws, lay = run_gpu(act, gpu_weights, cfg, stop=_lib.STOP_GEMM1)
    view = fmoe.WorkspaceView(ws, lay, cfg.T, 32, wl.HIDDEN, wl.INTER)
    hi, lo, sc = (t.cpu() for t in view.intermediate())
    slot_tok = view.slot_token().cpu().numpy()
    base = view.expert_base().cpu().numpy()
    from oracle.fp8 import e4m3_to_f32
    A = omoe.dequant_activations(act.hidden_states.view(torch.uint8).numpy(),
                                 act.hidden_states_scale.numpy())
    checked = 0
    for e in range(32):
        slots = [s for s in range(base[e], base[e + 1]) if slot_tok[s] >= 0][:4]
        if not slots:
            continue
        W1, s1, _, _ = oracle_weights_for(cpu_weights, [e])
        W13 = omoe.dequant_weight(W1[e], s1[e])
        g1 = A[slot_tok[slots]] @ W13.T
        gate, up = g1[:, :wl.INTER], g1[:, wl.INTER:]
        h = up / (1 + np.exp(-up)) * gate
        dec = (e4m3_to_f32(hi[slots].numpy()) + e4m3_to_f32(lo[slots].numpy())) * \
            np.repeat(sc[:, slots].numpy().T, 128, axis=1)
        amax = np.abs(h).max()
        np.testing.assert_allclose(dec, h, rtol=2e-2, atol=2e-3 * amax)
        checked += 1
        if checked >= 4:
            break
    assert checked > 0


def test_no_local_pairs_gives_zeros(gpu_weights):
    """All picks outside the local range: P = 0, output zero-filled (kernel.py:692-695)."""
    act = wl.make_activations(8, 123)
    act.routing_logits[:, 64:96] -= 30.0  # sigmoid ~ 0: the local range can never win
    cfg = wl.Config("nolocal", 8, 123)
    out, ws, lay = run_gpu(act, gpu_weights, cfg, local_start=64)
    view = fmoe.WorkspaceView(ws, lay, 8, 32, wl.HIDDEN, wl.INTER)
    assert int(view.plan()[0]) == 0
    assert torch.count_nonzero(out.float()) == 0


def test_all_tokens_on_one_expert(gpu_weights, cpu_weights):
    """300 tokens all select local expert 5 (3 m-tiles, the last one ragged)."""
    T = 300
    act = wl.make_activations(T, 77)
    act.routing_logits[:, 5] += 30.0      # sigmoid ~ 1 ...
    act.routing_bias[5] = 1.0             # ... and a bias no other expert can reach
    cfg = wl.Config("hot5", T, 77)
    out, ws, lay = run_gpu(act, gpu_weights, cfg)
    view = fmoe.WorkspaceView(ws, lay, T, 32, wl.HIDDEN, wl.INTER)
    assert int(view.expert_count()[5]) == T
    bits = out.view(torch.int16).cpu().numpy().view(np.uint16)
    sel = np.array([0, 1, 127, 128, 255, 256, 299])
    ref = oracle_rows(act, cfg, sel, cpu_weights)
    frac, err = omoe.allclose_report(bits[sel], ref, atol=ATOL, rtol=RTOL)
    assert frac == 1.0, (frac, err)


@pytest.mark.parametrize("T", [33, 40, 63, 64])
def test_small_batch_one_hot_expert(T, gpu_weights, cpu_weights):
    """Every token picks local expert 7: one tile holds all T slots. Covers the two-CTA routing
    cluster (T > 32: the second CTA's ranks start after the first CTA's count) and GEMM2's packed
    hi/lo tile up to its full 64 rows, across the 32-row lane-quarter boundary."""
    act = wl.make_activations(T, 500 + T)
    act.routing_logits[:, 7] += 30.0
    act.routing_bias[7] = 1.0
    cfg = wl.Config(f"hot7_t{T}", T, 500 + T)
    out, ws, lay = run_gpu(act, gpu_weights, cfg)
    view = fmoe.WorkspaceView(ws, lay, T, 32, wl.HIDDEN, wl.INTER)
    oids, ow = orouting.route(act.routing_logits.numpy(), act.routing_bias.float().numpy(), cfg.rsf)
    lid, lw = orouting.local_view(oids, ow, 0, 32)
    counts, offsets, stoks, sw = orouting.permute(lid, lw, 32)
    assert counts[7] == T
    np.testing.assert_array_equal(view.expert_count().cpu().numpy(), counts)
    base = view.expert_base().cpu().numpy()
    slot_tok = view.slot_token().cpu().numpy()
    for e in range(32):
        np.testing.assert_array_equal(slot_tok[base[e]:base[e] + counts[e]],
                                      stoks[offsets[e]:offsets[e + 1]])
        assert np.all(slot_tok[base[e] + counts[e]:base[e + 1]] == -1)
    bits = out.view(torch.int16).cpu().numpy().view(np.uint16)
    sel = np.array(sorted({0, 1, 31, 32, T // 2, T - 2, T - 1}))
    ref = oracle_rows(act, cfg, sel, cpu_weights)
    frac, err = omoe.allclose_report(bits[sel], ref, atol=ATOL, rtol=RTOL)
    assert frac == 1.0, (frac, err)


@pytest.mark.parametrize("T,path", [(4, _lib.PATH_GEMM), (8, _lib.PATH_GEMM), (1, _lib.PATH_AUTO),
                                    (2, _lib.PATH_AUTO), (2, _lib.PATH_GEMM)])
def test_split_tiles_with_several_rows(T, path, gpu_weights, cpu_weights):
    """Every token picks local experts 5, 6, 7 and global experts 40-44 (outside the 32 local
    ones): T routed rows per active expert. Grouped GEMMs: GEMM1 has 48 tiles of T rows each,
    fewer than the SMs, so the plan splits their K range and k_split_finish sums T-row partial
    tiles. Matrix-vector path (T <= 2): a token sum over three experts in k_gemv2. Every
    output row against the oracle."""
    act = wl.make_activations(T, 700 + T)
    act.routing_logits[:, 5:8] += 30.0
    act.routing_logits[:, 40:45] += 30.0
    act.routing_bias[5:8] = 1.0
    act.routing_bias[40:45] = 1.0
    cfg = wl.Config(f"split_t{T}", T, 700 + T)
    out, ws, lay = run_gpu(act, gpu_weights, cfg, path=path)
    view = fmoe.WorkspaceView(ws, lay, T, 32, wl.HIDDEN, wl.INTER)
    counts = view.expert_count().cpu().numpy()
    assert list(np.nonzero(counts)[0]) == [5, 6, 7] and np.all(counts[5:8] == T)
    plan = view.plan().cpu().numpy()
    assert plan[3] > 1, plan  # plan word 3: GEMM1's K splits per tile (split-K for T <= 8)
    bits = out.view(torch.int16).cpu().numpy().view(np.uint16)
    ref = oracle_rows(act, cfg, np.arange(T), cpu_weights)
    frac, err = omoe.allclose_report(bits, ref, atol=ATOL, rtol=RTOL)
    assert frac == 1.0, (frac, err)


@pytest.mark.parametrize("name,logits_bf16", [("t1_s1", False), ("t1_s1", True)])
def test_small_batch_paths_agree_and_repeat(name, logits_bf16, gpu_weights):
    """The matrix-vector path against the grouped GEMMs on the same call (both are within the
    oracle tolerance elsewhere; here within 1e-2 of each other), and bit-identical on a rerun;
    also with bf16 logits and an fp32 bias."""
    cfg = wl.CONFIGS[name]
    act = cfg.activations()
    if logits_bf16:
        act.routing_logits = act.routing_logits.to(torch.bfloat16)
        act.routing_bias = act.routing_bias.float()
    gemv, _, _ = run_gpu(act, gpu_weights, cfg)
    gemv = gemv.clone()
    again, _, _ = run_gpu(act, gpu_weights, cfg)
    assert torch.equal(gemv.view(torch.int16), again.view(torch.int16))
    tc, _, _ = run_gpu(act, gpu_weights, cfg, path=_lib.PATH_GEMM)
    torch.testing.assert_close(gemv.float(), tc.float(), atol=1e-2, rtol=1e-2)


def test_output_written_in_place(gpu_weights):
    cfg = wl.CONFIGS["t8_s2"]
    act = cfg.activations()
    lg, b, hs, sc = to_gpu(act)
    w1, s1, w2, s2 = gpu_weights
    out = torch.full((cfg.T, wl.HIDDEN), 7.0, dtype=torch.bfloat16, device="cuda")
    ret = fmoe.run(lg, b, hs, sc, w1, s1, w2, s2, 0, cfg.rsf, out)
    assert ret.data_ptr() == out.data_ptr()
    assert not torch.any(out == 7.0)
