"""The expert-parallel kernels on one GPU: R ranks emulated as R sets of buffers in one process.

fmoe_ep_dispatch stores each rank's records into the receive regions of the "destination"
buffers, the pre-routed operator runs on each buffer and stores its partial rows into the
"senders'" return regions, and fmoe_ep_reduce sums them -- the same kernels and index arithmetic
as across GPUs, with device addresses of this GPU where other ranks would pass their IPC mappings.
No kernel waits on another, so running the ranks one after the other is exact. Checked against
the dispatch plan restated on the CPU and the oracle over all 256 experts (hidden/intermediate
reduced to 1024/512 so that all 256 experts' weights are cheap to draw)."""
import ctypes

import numpy as np
import pytest
import torch

from flashinfer_b200 import _lib
from flashinfer_b200 import moe as fmoe
from flashinfer_b200 import workload as wl
from flashinfer_b200.ep import plan_dispatch
from oracle import moe as omoe
from oracle import routing as orouting

pytestmark = pytest.mark.gpu

H, I, RSF = 1024, 512, 2.5


def _weights(experts, dev):
    ws = [wl.expert_weights(e, hidden=H, inter=I) for e in experts]
    return [torch.stack([w[i] for w in ws]).to(dev) for i in range(4)]


@pytest.fixture(scope="module")
def all_weights():
    return _weights(range(256), torch.device("cuda:0"))


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _emulate(world, act, T_rank, weights, cap):
    dev = torch.device("cuda:0")
    lib = _lib.load()
    lay = _lib.ep_layout(world, cap, H)
    bufs = [torch.zeros(lay.total_bytes, dtype=torch.uint8, device=dev) for _ in range(world)]
    peers = (ctypes.c_void_p * world)(*[b.data_ptr() for b in bufs])
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    epr = 256 // world
    tds, ids_all = [], []
    for r in range(world):
        rows = slice(r * T_rank, (r + 1) * T_rank)
        lg = act.routing_logits[rows].contiguous().to(dev)
        hs = act.hidden_states[rows].contiguous().to(dev)
        sc = act.hidden_states_scale[:, rows].contiguous().to(dev)
        ids, w = fmoe.route(lg, act.routing_bias.to(dev), RSF)
        t = torch.full((cap, world), -7, dtype=torch.int32, device=dev)
        _lib.check(lib.fmoe_ep_dispatch(_p(ids), _p(w), _p(hs), _p(sc), T_rank, cap, H, world, r,
                                        peers, _p(t), stream), "fmoe_ep_dispatch")
        tds.append(t)
        ids_all.append(ids)
    n = world * cap
    for r in range(world):
        b = bufs[r]
        view = lambda off, nbytes: b[off:off + nbytes]  # noqa: E731
        recv_hidden = view(lay.recv_hidden, n * H).view(torch.float8_e4m3fn).view(n, H)
        recv_scale = view(lay.recv_scale, (H // 128) * n * 4).view(torch.float32).view(H // 128, n)
        recv_ids = view(lay.recv_ids, n * 32).view(torch.int32).view(n, 8)
        recv_w = view(lay.recv_weights, n * 32).view(torch.float32).view(n, 8)
        counts = view(lay.recv_counts, world * 4).view(torch.int32)
        w1, s1, w2, s2 = (x[r * epr:(r + 1) * epr] for x in weights)
        region_out = [bufs[s].data_ptr() + lay.ret_rows + r * cap * lay.row_bytes
                      for s in range(world)]
        fmoe.run_routed(recv_ids, recv_w, recv_hidden, recv_scale, w1, s1, w2, s2, r * epr,
                        region_counts=counts, region_tokens=cap, region_output=region_out)
    outs = []
    for r in range(world):
        out = torch.full((T_rank, H), 7.0, dtype=torch.bfloat16, device=dev)
        _lib.check(lib.fmoe_ep_reduce(_p(tds[r]), _p(bufs[r]), T_rank, cap, H, world, _p(out),
                                      stream), "fmoe_ep_reduce")
        outs.append(out)
    torch.cuda.synchronize()
    return outs, tds, ids_all, bufs, lay


@pytest.mark.parametrize("world,hot,T_rank,cap", [(2, 0.0, 192, 192), (4, 1.5, 96, 128),
                                                  (8, 0.0, 48, 48)])
def test_emulated_ranks_match_oracle(world, hot, T_rank, cap, all_weights):
    act = wl.make_activations(world * T_rank, 61 + world, hot_group=0 if hot else None, hot=hot,
                              hidden=H)
    outs, tds, ids_all, bufs, lay = _emulate(world, act, T_rank, all_weights, cap)
    epr = 256 // world
    # dispatch plan: the kernel's slots and counts equal the CPU restatement
    for r in range(world):
        slots, counts = plan_dispatch(ids_all[r].cpu(), epr, world)
        assert torch.equal(tds[r][:T_rank].cpu(), slots)
        for d in range(world):
            got = bufs[d][lay.recv_counts:lay.recv_counts + world * 4].view(torch.int32)[r]
            assert int(got) == int(counts[d])
    # output: the oracle over all 256 experts
    got = torch.cat(outs).view(torch.int16).cpu().numpy().view(np.uint16)
    ids, w = orouting.route(act.routing_logits.numpy(), act.routing_bias.float().numpy(), RSF)
    w1, s1, w2, s2 = (x.cpu() for x in all_weights)
    W1 = {e: w1[e].view(torch.uint8).numpy() for e in range(256)}
    W2 = {e: w2[e].view(torch.uint8).numpy() for e in range(256)}
    ref = omoe.moe_reference(act.hidden_states.view(torch.uint8).numpy(),
                             act.hidden_states_scale.numpy(), W1, s1.numpy(), W2, s2.numpy(),
                             ids, w, 0)
    frac, err = omoe.allclose_report(got, ref, atol=1e-2, rtol=1e-2)
    assert frac == 1.0, (frac, err)


def test_emulated_ranks_are_deterministic(all_weights):
    act = wl.make_activations(2 * 160, 71, hidden=H)
    a, *_ = _emulate(2, act, 160, all_weights, 160)
    a = [x.clone() for x in a]
    b, *_ = _emulate(2, act, 160, all_weights, 160)
    for x, y in zip(a, b):
        assert torch.equal(x.view(torch.int16), y.view(torch.int16))
