"""Expert parallelism on real GPUs: NCCL dispatch/combine around the CUDA operator, checked
against the CPU oracle over all 256 experts. Needs at least 2 GPUs (skipped otherwise).
Hidden/intermediate sizes are reduced (1024/512) so all 256 experts' weights stay small."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch

from flashinfer_b200 import workload as wl
from oracle import moe as omoe
from oracle import routing as orouting

pytestmark = pytest.mark.gpu

H, I, T_GLOBAL, SEED, RSF = 1024, 512, 512, 41, 2.5


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _weights(experts):
    ws = [wl.expert_weights(e, hidden=H, inter=I) for e in experts]
    return [torch.stack([w[i] for w in ws]) for i in range(4)]


def _worker(rank, world, port, hot, q):
    import torch.distributed as dist
    from flashinfer_b200.ep import ExpertParallelMoE
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120),
                            device_id=torch.device("cuda", rank))
    try:
        dev = torch.device("cuda", rank)
        act = wl.make_activations(T_GLOBAL, SEED, hot_group=0 if hot else None, hot=hot, hidden=H)
        per = T_GLOBAL // world
        rows = slice(rank * per, (rank + 1) * per)
        epr = 256 // world
        w = [t.to(dev) for t in _weights(range(rank * epr, (rank + 1) * epr))]
        ep = ExpertParallelMoE()
        out = ep.forward(act.routing_logits[rows].contiguous().to(dev), act.routing_bias.to(dev),
                         act.hidden_states[rows].contiguous().to(dev),
                         act.hidden_states_scale[:, rows].contiguous().to(dev), *w, RSF)
        a = ep.forward(act.routing_logits[rows].contiguous().to(dev), act.routing_bias.to(dev),
                       act.hidden_states[rows].contiguous().to(dev),
                       act.hidden_states_scale[:, rows].contiguous().to(dev), *w, RSF)
        torch.cuda.synchronize()
        q.put((rank, out.view(torch.int16).cpu().numpy().copy(), bool(torch.equal(a, out))))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("hot", [0.0, 1.5])
def test_ep_two_gpus_matches_oracle(hot):
    import torch.multiprocessing as mp
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, hot, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, bits, same = q.get()
        res[r] = (bits, same)
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    assert all(res[r][1] for r in range(world)), "EP output not deterministic across calls"
    got = np.concatenate([res[r][0] for r in range(world)]).view(np.uint16)
    act = wl.make_activations(T_GLOBAL, SEED, hot_group=0 if hot else None, hot=hot, hidden=H)
    ids, w = orouting.route(act.routing_logits.numpy(), act.routing_bias.float().numpy(), RSF)
    w1, s1, w2, s2 = _weights(range(256))
    W1 = {e: w1[e].view(torch.uint8).numpy() for e in range(256)}
    W2 = {e: w2[e].view(torch.uint8).numpy() for e in range(256)}
    ref = omoe.moe_reference(act.hidden_states.view(torch.uint8).numpy(),
                             act.hidden_states_scale.numpy(), W1, s1.numpy(), W2, s2.numpy(),
                             ids, w, 0)
    frac, err = omoe.allclose_report(got, ref, atol=1e-2, rtol=1e-2)
    assert frac == 1.0, (frac, err)
