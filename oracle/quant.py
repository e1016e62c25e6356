"""Input quantisation restated in numpy (bf16 activations -> e4m3 + per-128 scales).

Test infrastructure only: the GPU quantiser (fmoe_quant.cu) is checked against this.

The reference receives ``hidden_states`` already quantised: e4m3 [T, H] with one fp32 scale
per token and 128 columns, stored transposed as ``hidden_states_scale[kb, token]``
(solution/triton/kernel.py:601-602, indexed that way at :169). The rule restated here is the
DeepSeek-V3 convention the benchmark inputs follow: scale = max(amax, 1e-30) / 448 and
q = e4m3(x / scale), each fp32 operation rounded to nearest and the e4m3 rounding to nearest
even (``round_e4m3``). Parity: pinned against torch's own ``float8_e4m3fn`` conversion on
seeded inputs (tests/test_oracle_pins.py).
"""
import numpy as np

from .fp8 import round_e4m3

BLOCK = 128
E4M3_MAX = np.float32(448.0)


def quantize_activations(x: np.ndarray):
    """x: float32 [T, H] (values exactly representable in bf16). Returns (q float32 [T, H],
    e4m3-representable values; scale float32 [H/128, T])."""
    x = np.asarray(x, dtype=np.float32)
    t, h = x.shape
    xb = x.reshape(t, h // BLOCK, BLOCK)
    amax = np.abs(xb).max(axis=2).astype(np.float32)
    scale = (np.maximum(amax, np.float32(1e-30)) / E4M3_MAX).astype(np.float32)
    q = round_e4m3((xb / scale[:, :, None]).astype(np.float32))
    return q.reshape(t, h), np.ascontiguousarray(scale.T)
