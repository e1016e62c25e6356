"""Generate the golden vectors in this folder by running the operator's own PyTorch reference.

The reference repository's tests delegate correctness to the definition
reference of ``moe_fp8_block_scale_ds_routing_topk8_ng8_kg4_e32_h7168_i2048``.
Its installed copy is ``flashinfer.trace.templates.moe._trtllm_fp8_block_scale_moe_ds_routing_reference``
(flashinfer-python 0.6.11.post2, ``flashinfer/trace/templates/moe.py:109-184``),
the "fp32-dequantise-and-loop-experts" path. This script feeds it the seeded
workloads of ``flashinfer_b200.workload`` on the CPU and records:

* ``routing.npz``  for every config: per-token ascending global expert ids
  (uint8 ``[T, 8]``), and for T <= 1024 the matching weights (fp32), captured
  by intercepting the arguments the reference passes to its expert loop
  (``moe.py:172-184``);
* ``outputs.npz``  the reference's bf16 output rows (uint16 bit patterns) for the
  small configs (all rows for T <= 16, the first 16 rows for T = 64 and the
  skewed T = 256 case);
* ``sampled_rows.npz`` the reference's bf16 output rows for a seeded sample of
  tokens of every larger config (``SAMPLED``): tokens are independent (a token's
  output depends only on its own logits row, activation row and the weights of
  its picks), so the reference runs its routing on just those rows and then its
  expert loop (``moe.py:28-100``) once per token over the token's own picks in
  the config's local expert range -- the experts it needs, in a compact stack,
  with the pick ids renumbered to index that stack. The expert-parallel configs
  are recorded over all 256 experts (the sum every rank's partial adds up to).
  ``python tests/golden/make_golden.py --sampled`` rebuilds only this file.

Run it where the installed reference is importable (not needed on the GPU box):
``python tests/golden/make_golden.py``. Takes a few minutes on 8 cores.
"""
from __future__ import annotations

import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.abspath(os.path.join(HERE, "..", "..")))

from flashinfer_b200 import workload as wl  # noqa: E402

EP_CONFIGS = {
    # Expert-parallel global workloads: uniform and hot-group logits.
    "ep_t16384_s10": wl.Config("ep_t16384_s10", 16384, 10),
    "ep_t16384_s11_hot": wl.Config("ep_t16384_s11_hot", 16384, 11, hot=1.5),
}
FULL_OUTPUT = {"t16_s0": None, "t1_s1": None, "t8_s2": None, "t64_s4": 16, "t256_s5_skew": 16}
# Sampled-token golden rows: config -> (local expert range start, size, tokens to sample).
SAMPLED = {
    "t32_s3": (0, 32, 8), "t256_s5": (0, 32, 10), "t1024_s6": (0, 32, 12),
    "t1024_s6_skew": (0, 32, 12), "t4096_s7": (0, 32, 12), "t8192_s8": (0, 32, 12),
    "t16384_s9": (0, 32, 12), "ep_t16384_s10": (0, 256, 8), "ep_t16384_s11_hot": (0, 256, 8),
}


def sampled_tokens(cfg, n):
    """The seeded token sample of a config: first, last and n more (sorted, distinct)."""
    rng = np.random.default_rng(1000 + cfg.seed)
    pick = rng.choice(cfg.T, size=min(cfg.T, n), replace=False)
    return np.unique(np.concatenate([[0, cfg.T - 1], pick])).astype(np.int64)


def reference_module():
    import flashinfer.trace.templates.moe as m
    return m


def reference_routing(m, act, rsf):
    captured = {}

    def capture(hidden_states, hidden_states_scale, g1w, g1s, g2w, g2s, weights, topk_idx,
                local_expert_offset, E_global):
        captured["w"] = weights.clone()
        captured["idx"] = topk_idx.clone()
        return None

    orig = m._fp8_moe_run_experts
    m._fp8_moe_run_experts = capture
    try:
        dummy = torch.zeros(1)
        m._trtllm_fp8_block_scale_moe_ds_routing_reference(
            act.routing_logits, act.routing_bias, act.hidden_states, act.hidden_states_scale,
            dummy, dummy, dummy, dummy, 8, 8, 4, 0, rsf)
    finally:
        m._fp8_moe_run_experts = orig
    idx = captured["idx"].numpy()
    w = captured["w"].numpy()
    order = np.argsort(idx, axis=1, kind="stable")
    return np.take_along_axis(idx, order, 1), np.take_along_axis(w, order, 1)


def reference_token_rows(m, act, rsf, tokens, local_start, e_local):
    """Reference bf16 output rows (uint16 bits) of the given tokens, local experts only."""
    sub = wl.Activations(act.routing_logits[tokens].contiguous(), act.routing_bias,
                         act.hidden_states[tokens].contiguous(),
                         act.hidden_states_scale[:, tokens].contiguous())
    ids, w = reference_routing(m, sub, rsf)
    rows = []
    for i in range(len(tokens)):
        mine = [int(e) for e in ids[i] if local_start <= int(e) < local_start + e_local]
        if not mine:
            rows.append(np.zeros(wl.HIDDEN, dtype=np.uint16))
            continue
        w1, s1, w2, s2 = wl.WeightBank.stacked(mine)
        remap = {e: j for j, e in enumerate(mine)}
        idx = torch.tensor([[remap.get(int(e), -1) for e in ids[i]]], dtype=torch.int64)
        out = m._fp8_moe_run_experts(sub.hidden_states[i:i + 1], sub.hidden_states_scale[:, i:i + 1],
                                     w1, s1, w2, s2, torch.from_numpy(w[i:i + 1].copy()), idx,
                                     0, wl.E_GLOBAL)
        rows.append(out.view(torch.int16).numpy().view(np.uint16)[0])
    return np.stack(rows)


def make_sampled(m):
    all_cfgs = dict(wl.CONFIGS)
    all_cfgs.update(EP_CONFIGS)
    rows = {}
    for name, (start, e_local, n) in SAMPLED.items():
        cfg = all_cfgs[name]
        act = cfg.activations()
        tok = sampled_tokens(cfg, n)
        t0 = time.time()
        rows[f"{name}/tokens"] = tok
        rows[f"{name}/out"] = reference_token_rows(m, act, cfg.rsf, tok, start, e_local)
        print(name, "sampled rows", len(tok), f"{time.time() - t0:.1f}s", flush=True)
        # each expert's weights are only needed by this config's sample
        wl.WeightBank._cache.clear()
    rows["meta/torch"] = np.array(torch.__version__)
    np.savez_compressed(os.path.join(HERE, "sampled_rows.npz"), **rows)


def main():
    torch.set_num_threads(os.cpu_count() or 8)
    if "--sampled" in sys.argv:
        make_sampled(reference_module())
        return
    m = reference_module()
    routing = {}
    all_cfgs = dict(wl.CONFIGS)
    all_cfgs.update(EP_CONFIGS)
    for name, cfg in all_cfgs.items():
        act = cfg.activations()
        ids, w = reference_routing(m, act, cfg.rsf)
        routing[f"{name}/ids"] = ids.astype(np.uint8)
        if cfg.T <= 1024:
            routing[f"{name}/weights"] = w.astype(np.float32)
        print(name, "routed", flush=True)
    np.savez_compressed(os.path.join(HERE, "routing.npz"), **routing)

    w1, s1, w2, s2 = wl.local_weights(32, 0)
    outputs = {}
    for name, rows in FULL_OUTPUT.items():
        cfg = wl.CONFIGS[name]
        act = cfg.activations()
        t0 = time.time()
        out = m._trtllm_fp8_block_scale_moe_ds_routing_reference(
            act.routing_logits, act.routing_bias, act.hidden_states, act.hidden_states_scale,
            w1, s1, w2, s2, 8, 8, 4, cfg.local_expert_offset, cfg.rsf)
        bits = out.view(torch.int16).numpy().view(np.uint16)
        if rows is not None:
            bits = bits[:rows]
        outputs[f"{name}/out"] = bits
        print(name, "reference output", f"{time.time() - t0:.1f}s", flush=True)
    outputs["meta/torch"] = np.array(torch.__version__)
    np.savez_compressed(os.path.join(HERE, "outputs.npz"), **outputs)


if __name__ == "__main__":
    main()
