"""Expert parallelism on real GPUs at the operator's shapes (H=7168, I=2048): the configs[4]
global batch (T=16384) split over 2 ranks of 128 experts, tokens and partial rows moved by the
peer transport (CUDA IPC stores over NVLink, NCCL all-reduces as barriers). Checked on the
reference-run golden rows of the sampled tokens and against the oracle over all 256 experts.
Only the experts those tokens pick get their seeded weights (the rest are zeros, which only the
unchecked tokens see), so the weights need not all be drawn on the CPU. Needs 2 GPUs."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch

from flashinfer_b200 import workload as wl
from oracle import moe as omoe
from oracle import routing as orouting
from tests.conftest import GOLDEN, bank_weights_for
from tests.golden.make_golden import EP_CONFIGS

pytestmark = pytest.mark.gpu

H, I = wl.HIDDEN, wl.INTER


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_weights(experts, need, dev):
    n = len(experts)
    w1 = torch.zeros((n, 2 * I, H), dtype=torch.uint8, device=dev)
    s1 = torch.zeros((n, 2 * I // 128, H // 128), dtype=torch.float32, device=dev)
    w2 = torch.zeros((n, H, I), dtype=torch.uint8, device=dev)
    s2 = torch.zeros((n, H // 128, I // 128), dtype=torch.float32, device=dev)
    for j, e in enumerate(experts):
        if e in need:
            q1, a1, q2, a2 = wl.WeightBank.get(e)
            w1[j].copy_(q1.view(torch.uint8))
            s1[j].copy_(a1)
            w2[j].copy_(q2.view(torch.uint8))
            s2[j].copy_(a2)
    return w1.view(torch.float8_e4m3fn), s1, w2.view(torch.float8_e4m3fn), s2


def _worker(rank, world, port, name, tokens, need, q):
    import torch.distributed as dist
    from flashinfer_b200.ep import ExpertParallelMoE
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    ep = None
    try:
        dev = torch.device("cuda", rank)
        cfg = EP_CONFIGS[name]
        act = cfg.activations()
        per = cfg.T // world
        rows = slice(rank * per, (rank + 1) * per)
        epr = 256 // world
        w = _rank_weights(list(range(rank * epr, (rank + 1) * epr)), need, dev)
        ep = ExpertParallelMoE(capacity=per)
        assert ep.transport == "peer"
        ins = [act.routing_logits[rows].contiguous().to(dev), act.routing_bias.to(dev),
               act.hidden_states[rows].contiguous().to(dev),
               act.hidden_states_scale[:, rows].contiguous().to(dev)]
        out = ep.forward(*ins, *w, cfg.rsf).clone()
        again = ep.forward(*ins, *w, cfg.rsf)
        torch.cuda.synchronize()
        mine = [t - rank * per for t in tokens if rank * per <= t < (rank + 1) * per]
        q.put((rank, mine, out[mine].view(torch.int16).cpu().numpy().copy(),
               bool(torch.equal(again.view(torch.int16), out.view(torch.int16)))))
    finally:
        if ep is not None:
            ep.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("name", sorted(EP_CONFIGS))
def test_ep_two_gpus_real_shapes(name):
    import torch.multiprocessing as mp
    world = 2
    gold = np.load(os.path.join(GOLDEN, "sampled_rows.npz"))
    tokens = [int(t) for t in gold[f"{name}/tokens"]]
    cfg = EP_CONFIGS[name]
    act = cfg.activations()
    ids, w = orouting.route(act.routing_logits.numpy()[tokens], act.routing_bias.float().numpy(),
                            cfg.rsf)
    need = sorted({int(e) for e in ids.reshape(-1)})
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, name, tokens, need, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, mine, bits, same = q.get()
        res[r] = (mine, bits, same)
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    assert all(res[r][2] for r in range(world)), "EP output not deterministic across calls"
    got = np.concatenate([res[r][1] for r in range(world)]).view(np.uint16)
    frac, err = omoe.allclose_report(got, gold[f"{name}/out"], atol=1e-2, rtol=1e-2)
    assert frac == 1.0, (frac, err)
    W1, S1, W2, S2 = bank_weights_for(need)

    class Dense(dict):
        def __len__(self):
            return 256

    ref = omoe.moe_reference(act.hidden_states.view(torch.uint8).numpy()[tokens],
                             act.hidden_states_scale.numpy()[:, tokens], W1, Dense(S1), W2,
                             Dense(S2), ids, w, 0)
    frac, err = omoe.allclose_report(got, ref, atol=1e-2, rtol=1e-2)
    assert frac == 1.0, (frac, err)
