"""Expert compute of the fused MoE in numpy fp32. Test infrastructure only.

``moe_reference`` restates the definition's expert loop
(``flashinfer/trace/templates/moe.py:28-100``; the reference kernel's phases
``solution/triton/kernel.py:699-823`` compute the same function):

    A   = e4m3(hidden) * scale[kb, t]              (moe.py:56-62)
    W13 = e4m3(W1[e]) * S1[e, n/128, k/128]        (moe.py:64-68)
    W2  = e4m3(W2[e]) * S2[e, n/128, k/128]        (moe.py:70-74)
    for each local expert e (ascending):           (moe.py:79)
        tokens t selecting e, ascending            (moe.py:87)
        G1 = A_t @ W13^T ; X1, X2 = G1[:, :I], G1[:, I:]
        h  = X2 / (1 + exp(-X2)) * X1              (moe.py:90-92)
        O  = h @ W2^T
        out[t] += w[t, e] * O                      (moe.py:94-98)
    return bf16(out)                               (moe.py:100)

``moe_device_numerics`` mirrors the arithmetic the CUDA path performs (fp32
promotion of each 128-wide K block, the two-term e4m3 intermediate, bf16 Y
rows), for design studies and tighter intermediate checks.
"""
from __future__ import annotations

import numpy as np

from .fp8 import e4m3_to_f32, round_e4m3, bf16_round, bf16_to_f32

F32 = np.float32
BLOCK = 128


def _expand_block_scale(s: np.ndarray, rows: int, cols: int) -> np.ndarray:
    return np.repeat(np.repeat(s, BLOCK, axis=0), BLOCK, axis=1)[:rows, :cols]


def dequant_activations(hs_raw: np.ndarray, hs_scale: np.ndarray) -> np.ndarray:
    """hs_raw uint8 [T, H]; hs_scale fp32 [H/128, T] -> fp32 [T, H]."""
    a = e4m3_to_f32(hs_raw)
    return (a * np.repeat(hs_scale.T, BLOCK, axis=1)).astype(F32)


def dequant_weight(w_raw: np.ndarray, s: np.ndarray) -> np.ndarray:
    w = e4m3_to_f32(w_raw)
    return (w * _expand_block_scale(s, *w.shape)).astype(F32)


def expert_pairs(ids: np.ndarray, weights: np.ndarray, local_start: int, e_local: int):
    """For each local expert: (ascending token ids, their routing weights)."""
    out = []
    for le in range(e_local):
        ge = local_start + le
        match = ids == ge
        tok = np.nonzero(match.any(axis=1))[0]
        w = (weights * match).sum(axis=1)[tok].astype(F32)
        out.append((tok, w))
    return out


def moe_reference(hs_raw, hs_scale, w1_raw, s1, w2_raw, s2, ids, weights,
                  local_start: int, return_f32: bool = False):
    """fp32 restatement of the definition reference. Weights are indexed by local expert.

    ``w1_raw``/``w2_raw`` may be dicts {local_expert: uint8 array} holding only the
    experts that are selected, so small checks avoid dequantising all 32.
    Returns bf16 bit patterns uint16 [T, H] (or fp32 if ``return_f32``).
    """
    T, H = hs_raw.shape
    A = dequant_activations(hs_raw, hs_scale)
    e_local = len(s1)
    out = np.zeros((T, H), dtype=F32)
    for le, (tok, w) in enumerate(expert_pairs(ids, weights, local_start, e_local)):
        if tok.size == 0:
            continue
        W13 = dequant_weight(w1_raw[le], s1[le])
        I = W13.shape[0] // 2
        G1 = A[tok] @ W13.T
        X1, X2 = G1[:, :I], G1[:, I:]
        h = (X2 / (F32(1.0) + np.exp(-X2)) * X1).astype(F32)
        W2 = dequant_weight(w2_raw[le], s2[le])
        O = h @ W2.T
        np.add.at(out, tok, O * w[:, None])
    return out if return_f32 else bf16_round(out)


def _blockwise_gemm(a_raw_f32, a_scale, w_raw_f32, w_scale):
    """sum_kb (A[:, kb] @ W[:, kb]^T) * a_scale[:, kb] * w_scale[n/128, kb] in fp32."""
    M, K = a_raw_f32.shape
    N = w_raw_f32.shape[0]
    acc = np.zeros((M, N), dtype=F32)
    for kb in range(K // BLOCK):
        ks = slice(kb * BLOCK, (kb + 1) * BLOCK)
        part = (a_raw_f32[:, ks] @ w_raw_f32[:, ks].T).astype(F32)
        f = (a_scale[:, kb:kb + 1] * np.repeat(w_scale[:, kb], BLOCK)[None, :N]).astype(F32)
        acc = (acc + part * f).astype(F32)
    return acc


def quantize_intermediate(h: np.ndarray):
    """Two-term e4m3 encoding of the SwiGLU output with one scale per row per 128 columns.

    scale = amax/448; hi = e4m3(h/scale); lo = e4m3(h/scale - hi); h ~= (hi + lo) * scale.
    """
    M, N = h.shape
    hb = h.reshape(M, N // BLOCK, BLOCK)
    amax = np.abs(hb).max(axis=2)
    inv = np.where(amax > 0, F32(448.0) / np.maximum(amax, F32(1e-30)), F32(0.0)).astype(F32)
    scale = np.where(amax > 0, amax / F32(448.0), F32(0.0)).astype(F32)
    x = (hb * inv[:, :, None]).astype(F32)
    hi = round_e4m3(x)
    lo = round_e4m3((x - hi).astype(F32))
    return hi.reshape(M, N), lo.reshape(M, N), scale


def f16_pow2_tiles(y: np.ndarray, tile: int = 256) -> np.ndarray:
    """fp16 storage of GEMM2 rows with one power-of-two scale per row per 256 columns.

    scale = 2^ceil(log2(amax / 16384)) keeps |y / scale| <= 16384 (fp16 max is 65504).
    """
    M, N = y.shape
    yt = y.reshape(M, N // tile, tile).astype(np.float32)
    amax = np.abs(yt).max(axis=2)
    e = np.where(amax > 0, np.ceil(np.log2(np.maximum(amax, 1e-30) / 16384.0)), 0).astype(np.int32)
    scale = np.ldexp(np.float32(1.0), e).astype(np.float32)
    q = (yt / scale[:, :, None]).astype(np.float16).astype(np.float32)
    return (q * scale[:, :, None]).reshape(M, N).astype(np.float32)


def moe_device_numerics(hs_raw, hs_scale, w1_raw, s1, w2_raw, s2, ids, weights,
                        local_start: int, y_bf16: bool = True, two_term: bool = True,
                        y_format: str = ""):
    """Emulates the CUDA path's arithmetic; returns bf16 bit patterns [T, H]."""
    T, H = hs_raw.shape
    a_all = e4m3_to_f32(hs_raw)
    e_local = len(s1)
    out = np.zeros((T, H), dtype=F32)
    for le, (tok, w) in enumerate(expert_pairs(ids, weights, local_start, e_local)):
        if tok.size == 0:
            continue
        w1 = e4m3_to_f32(w1_raw[le])
        I = w1.shape[0] // 2
        g1 = _blockwise_gemm(a_all[tok], hs_scale[:, tok].T, w1, s1[le])
        gate, up = g1[:, :I], g1[:, I:]
        h = (up / (F32(1.0) + np.exp(-up)) * gate).astype(F32)
        hi, lo, hsc = quantize_intermediate(h)
        w2 = e4m3_to_f32(w2_raw[le])
        if two_term:
            y = _blockwise_gemm((hi + lo).astype(F32), hsc, w2, s2[le])
        else:
            y = _blockwise_gemm(hi, hsc, w2, s2[le])
        if y_format == "f16s":
            y = f16_pow2_tiles(y)
        elif y_bf16:
            y = bf16_to_f32(bf16_round(y))
        np.add.at(out, tok, y * w[:, None])
    return bf16_round(out)


def allclose_report(got_bits: np.ndarray, ref_bits: np.ndarray, atol=1e-2, rtol=1e-2):
    """Fraction of elements within atol + rtol*|ref| and the max abs error."""
    g = bf16_to_f32(got_bits).astype(np.float64)
    r = bf16_to_f32(ref_bits).astype(np.float64)
    err = np.abs(g - r)
    ok = err <= atol + rtol * np.abs(r)
    return float(ok.mean()), float(err.max() if err.size else 0.0)
