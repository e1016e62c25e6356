"""Expert-parallel dispatch/combine on CPU ranks (gloo, the collective transport), the numpy
oracle standing in for the CUDA kernels: the gathered EP output must equal the single-process
oracle over all 256 experts. Small hidden/intermediate sizes keep all 256 experts' weights cheap;
routing is the real one. The dispatch plan (``plan_dispatch``) is the restatement the CUDA dispatch
kernel is checked against on the GPU."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from flashinfer_b200 import workload as wl
from flashinfer_b200.ep import ExpertParallelMoE, plan_dispatch
from oracle import moe as omoe
from oracle import routing as orouting

H, I, T_GLOBAL, SEED, RSF = 256, 128, 24, 31, 2.5


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _weights(experts):
    ws = [wl.expert_weights(e, hidden=H, inter=I) for e in experts]
    return [torch.stack([w[i] for w in ws]) for i in range(4)]


def _np_weights(w1, s1, w2, s2):
    n = w1.shape[0]
    return ({e: w1[e].view(torch.uint8).numpy() for e in range(n)}, s1.numpy(),
            {e: w2[e].view(torch.uint8).numpy() for e in range(n)}, s2.numpy())


def _route_oracle(logits, bias, rsf):
    ids, w = orouting.route(logits.float().numpy(), bias.float().numpy(), rsf)
    return torch.from_numpy(ids), torch.from_numpy(w)


def _local_oracle(ids, w, hs, sc, w1, s1, w2, s2, local_offset, out):
    """The receiver's pre-routed operator: the sender's picks and weights, local experts only."""
    W1, S1, W2, S2 = _np_weights(w1, s1, w2, s2)
    res = omoe.moe_reference(hs.view(torch.uint8).numpy(), sc.numpy(), W1, S1, W2, S2,
                             ids.numpy(), w.numpy(), local_offset, return_f32=True)
    out.copy_(torch.from_numpy(res))


def _worker(rank, world, port, hot, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        act = wl.make_activations(T_GLOBAL, SEED, hot_group=0 if hot else None, hot=hot, hidden=H)
        per = T_GLOBAL // world
        rows = slice(rank * per, (rank + 1) * per)
        epr = 256 // world
        w1, s1, w2, s2 = _weights(range(rank * epr, (rank + 1) * epr))
        ep = ExpertParallelMoE(transport="collective", hidden=H, route_fn=_route_oracle,
                           local_fn=_local_oracle)
        out = ep.forward(act.routing_logits[rows].contiguous(), act.routing_bias,
                         act.hidden_states[rows].contiguous(),
                         act.hidden_states_scale[:, rows].contiguous(), w1, s1, w2, s2, RSF)
        q.put((rank, out.view(torch.int16).numpy().copy(), ep.last_counts))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,hot", [(2, 0.0), (4, 0.0), (4, 1.5)])
def test_ep_matches_single_process_oracle(world, hot):
    ctx = mp.get_context("spawn")
    q = ctx.SimpleQueue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, hot, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        r, bits, counts = q.get()
        results[r] = (bits, counts)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    got = np.concatenate([results[r][0] for r in range(world)]).view(np.uint16)

    act = wl.make_activations(T_GLOBAL, SEED, hot_group=0 if hot else None, hot=hot, hidden=H)
    ids, w = orouting.route(act.routing_logits.numpy(), act.routing_bias.float().numpy(), RSF)
    W1, S1, W2, S2 = _np_weights(*_weights(range(256)))
    ref = omoe.moe_reference(act.hidden_states.view(torch.uint8).numpy(),
                             act.hidden_states_scale.numpy(), W1, S1, W2, S2, ids, w, 0)
    # same fp32 algorithm; partial sums are added per rank, so only the association of the
    # fp32 sum differs from the single-process loop: at most one bf16 ulp
    frac, err = omoe.allclose_report(got, ref, atol=1e-6, rtol=2.0 ** -7)
    assert frac == 1.0, (frac, err)
    # every routed (token, owner rank) pair was sent exactly once
    sent = sum(sum(results[r][1][0]) for r in range(world))
    owners = {(t, int(e) // (256 // world)) for t in range(T_GLOBAL) for e in ids[t]}
    assert sent == len(owners)


def test_dispatch_plan_slots():
    ids = torch.tensor([[0, 40, 200, 255, 1, 2, 3, 4]] * 10, dtype=torch.int32)
    ids[3] = torch.tensor([64, 65, 66, 67, 68, 69, 70, 71])
    slots, counts = plan_dispatch(ids, 64, 4)
    assert counts.tolist() == [9, 1, 0, 9]
    # rank 0 and 3 receive every token but token 3, in token order; rank 1 only token 3
    assert slots[:, 0].tolist() == [0, 1, 2, -1, 3, 4, 5, 6, 7, 8]
    assert slots[:, 1].tolist() == [-1, -1, -1, 0, -1, -1, -1, -1, -1, -1]
    assert slots[:, 2].tolist() == [-1] * 10
    assert slots[:, 3].tolist() == slots[:, 0].tolist()


def test_dispatch_plan_matches_definition_on_real_routing():
    """Every (token, owner rank) pair once; slots are ranks among the tokens sent there."""
    act = wl.make_activations(300, 9)
    ids, _ = orouting.route(act.routing_logits.numpy(), act.routing_bias.float().numpy(), RSF)
    for world in (2, 4, 8):
        epr = 256 // world
        slots, counts = plan_dispatch(torch.from_numpy(ids), epr, world)
        for d in range(world):
            sent = [t for t in range(300) if any(int(e) // epr == d for e in ids[t])]
            assert counts[d] == len(sent)
            assert [int(slots[t, d]) for t in sent] == list(range(len(sent)))
            assert all(int(slots[t, d]) == -1 for t in set(range(300)) - set(sent))
