"""Input quantisation on the GPU (fmoe_quantize_activations through the C ABI) against the
numpy oracle and torch's own e4m3 conversion: bit-exact e4m3 bytes and fp32 scales."""
import ctypes

import numpy as np
import pytest
import torch

from flashinfer_b200 import _lib
from flashinfer_b200 import moe as fmoe
from flashinfer_b200 import workload as wl
from oracle import quant as oquant
from oracle.fp8 import e4m3_to_f32
from tests.test_oracle_pins import _quant_inputs


def test_quantize_rejects_bad_arguments_on_host():
    lib = _lib.load()
    f = lib.fmoe_quantize_activations
    assert f(None, 4, 100, None, None, None) == -2          # H not a multiple of 128
    assert f(None, -1, 128, None, None, None) == -2
    assert f(None, 0, 128, None, None, None) == 0            # nothing to do
    assert f(None, 4, 128, None, None, None) == -1           # NULL input
    assert f(ctypes.c_void_p(8), 4, 128, ctypes.c_void_p(4096), ctypes.c_void_p(8192),
             None) == -3                                     # misaligned input


@pytest.mark.gpu
@pytest.mark.parametrize("T,H", [(1, 7168), (5, 256), (64, 7168), (1000, 1024), (4096, 7168)])
def test_quantize_bit_exact(T, H):
    x = _quant_inputs(T, H, 11 + T)
    q, s = fmoe.quantize_activations(x.cuda())
    torch.cuda.synchronize()
    q_t, s_t = wl.quantize_activations(x)
    np.testing.assert_array_equal(q.view(torch.uint8).cpu().numpy(), q_t.view(torch.uint8).numpy())
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), s_t.numpy().view(np.uint32))
    q_o, s_o = oquant.quantize_activations(x.float().numpy())
    np.testing.assert_array_equal(e4m3_to_f32(q.view(torch.uint8).cpu().numpy()), q_o)
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), s_o.view(np.uint32))


@pytest.mark.gpu
def test_quantized_inputs_feed_the_operator():
    """GPU-quantised activations give the operator the same output as the host-quantised ones."""
    cfg = wl.CONFIGS["t16_s0"]
    act = cfg.activations()
    g = torch.Generator().manual_seed(100 + cfg.seed)
    xb = torch.randn(cfg.T, wl.HIDDEN, generator=g).to(torch.bfloat16)
    q_h, s_h = wl.quantize_activations(xb)
    q_d, s_d = fmoe.quantize_activations(xb.cuda())
    w = tuple(t.cuda() for t in wl.local_weights(32, 0))
    lg, b = act.routing_logits.cuda(), act.routing_bias.cuda()
    o_h = fmoe.run(lg, b, q_h.cuda(), s_h.cuda(), *w, 0, cfg.rsf)
    o_d = fmoe.run(lg, b, q_d, s_d, *w, 0, cfg.rsf)
    assert torch.equal(o_h.view(torch.int16), o_d.view(torch.int16))


@pytest.mark.gpu
def test_quantize_rounding_ties():
    """Blocks whose quotients land on or next to e4m3 rounding midpoints (ties to even), where
    a quotient off by one fp32 ulp would round the other way."""
    grid = np.unique(np.abs(e4m3_to_f32(np.arange(256, dtype=np.uint8))))
    grid = grid[np.isfinite(grid) & (grid > 0)]
    mids = (grid[:-1] + grid[1:]) / 2                     # every e4m3 rounding midpoint
    rows = []
    for c in (1.0, 3.0, 0.7, 1e-3, 2.0 ** -20, 5.0e3):
        for start in range(0, mids.size, 127):
            v = np.full(128, 0.0, dtype=np.float32)
            v[0] = 448.0 * c                                # the block maximum -> scale ~ c
            seg = mids[start:start + 127] * c
            v[1:1 + seg.size] = seg
            rows.append(v)
    x = torch.from_numpy(np.stack(rows)).to(torch.bfloat16)   # bf16-rounded: on or near ties
    x = x.reshape(-1, 256) if x.shape[0] % 2 == 0 else x[:-1].reshape(-1, 256)
    q, s = fmoe.quantize_activations(x.cuda())
    torch.cuda.synchronize()
    q_t, s_t = wl.quantize_activations(x)
    np.testing.assert_array_equal(q.view(torch.uint8).cpu().numpy(), q_t.view(torch.uint8).numpy())
    np.testing.assert_array_equal(s.cpu().numpy().view(np.uint32), s_t.numpy().view(np.uint32))
