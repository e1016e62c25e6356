"""DeepSeek-V3 grouped routing and the canonical local permutation (numpy). Test infrastructure only.

Restates the reference's routing:

* ``solution/triton/kernel.py:400-404``  s = sigmoid(logits), s_with_bias = s + bias
* ``kernel.py:406-416``                  group score = sum of the top-2 biased scores in each
                                         group of 32 experts
* ``kernel.py:418-426``                  keep the 4 best of 8 groups
* ``kernel.py:428-438``                  top-8 biased scores over the kept groups; ties go to the
                                         lowest index (``tl.argmax``)
* ``kernel.py:440-452`` / definition ``moe.py:165-168``
                                         weights from the un-biased s, normalised by their sum
                                         (+1e-20) and scaled by routed_scaling_factor; experts
                                         outside [local_start, local_start + E_local) are non-local

Arithmetic contract (the device kernel performs the identical sequence, so the
two agree bit for bit):

* ``exp(-x)`` correctly rounded to fp32 (evaluated in float64, then rounded),
  then ``1 + e`` and ``1 / (1 + e)`` as IEEE fp32 operations -- the same three
  steps as the definition's ``1.0 / (1.0 + torch.exp(-logits))`` (``moe.py:143``);
* the normalising sum adds the 8 selected s values in selection order
  (descending biased score) in fp32, and the weight is
  ``(s_k / (sum + 1e-20)) * rsf`` in fp32 (``moe.py:167-168``).
"""
from __future__ import annotations

import numpy as np

F32 = np.float32


def sigmoid_f32(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=F32)
    e = np.exp(-x.astype(np.float64)).astype(F32)
    return (F32(1.0) / (F32(1.0) + e)).astype(F32)


def route(logits: np.ndarray, bias: np.ndarray, rsf: float, top_k: int = 8,
          n_group: int = 8, topk_group: int = 4):
    """Global top-k routing for every token.

    Returns ``ids`` int32 ``[T, top_k]`` (selection order: descending biased
    score, lowest index first on ties) and ``weights`` fp32 ``[T, top_k]``.
    """
    logits = np.asarray(logits, dtype=F32)
    T, E = logits.shape
    bias = np.asarray(bias, dtype=F32).reshape(1, E)
    s = sigmoid_f32(logits)
    sb = (s + bias).astype(F32)
    gsize = E // n_group
    grouped = sb.reshape(T, n_group, gsize)
    srt = -np.sort(-grouped, axis=2)                     # descending within each group
    gscore = (srt[:, :, 0] + srt[:, :, 1]).astype(F32)    # top-2 sum (kernel.py:413-415)
    gorder = np.argsort(-gscore, axis=1, kind="stable")   # ties -> lower group index
    keep = np.zeros((T, n_group), dtype=bool)
    np.put_along_axis(keep, gorder[:, :topk_group], True, axis=1)
    pruned = np.where(np.repeat(keep, gsize, axis=1), sb, -np.inf).astype(F32)
    eorder = np.argsort(-pruned, axis=1, kind="stable")   # ties -> lower expert index
    ids = eorder[:, :top_k].astype(np.int32)
    s_sel = np.take_along_axis(s, ids, axis=1)
    denom = np.zeros(T, dtype=F32)
    for k in range(top_k):                                 # fixed, sequential order
        denom = (denom + s_sel[:, k]).astype(F32)
    denom = (denom + F32(1e-20)).astype(F32)
    w = ((s_sel / denom[:, None]).astype(F32) * F32(rsf)).astype(F32)
    return ids, w


def local_view(ids: np.ndarray, weights: np.ndarray, local_start: int, e_local: int):
    """Reference ``kernel.py:442-452``: local expert id per pick (-1 if non-local)."""
    loc = ids.astype(np.int64) - int(local_start)
    is_local = (loc >= 0) & (loc < e_local)
    local_ids = np.where(is_local, loc, -1).astype(np.int32)
    local_w = np.where(is_local, weights, 0.0).astype(F32)
    return local_ids, local_w


def permute(local_ids: np.ndarray, local_w: np.ndarray, e_local: int):
    """Canonical permutation: experts ascending, tokens ascending within each.

    The reference fills slots with atomics (``kernel.py:480-505``), so its order
    within an expert is not fixed; the definition visits tokens in ascending
    order per expert (``moe.py:87``), which is the order used here and by the
    device kernel. Returns (counts [E], offsets [E+1], sorted_token_ids [P],
    sorted_weights [P]).
    """
    T, K = local_ids.shape
    counts = np.zeros(e_local, dtype=np.int64)
    toks, ws = [], []
    for e in range(e_local):
        hit = local_ids == e
        tok = np.nonzero(hit.any(axis=1))[0]
        counts[e] = tok.size
        toks.append(tok)
        ws.append((local_w * hit).sum(axis=1)[tok])
    offsets = np.zeros(e_local + 1, dtype=np.int64)
    offsets[1:] = np.cumsum(counts)
    sorted_ids = np.concatenate(toks).astype(np.int32) if toks else np.zeros(0, np.int32)
    sorted_w = np.concatenate(ws).astype(F32) if ws else np.zeros(0, F32)
    return counts.astype(np.int32), offsets.astype(np.int32), sorted_ids, sorted_w


def sorted_id_sets(ids: np.ndarray) -> np.ndarray:
    """Per-token ascending id sets (the torch reference's top-k order is unspecified)."""
    return np.sort(np.asarray(ids), axis=1)


# The definition family's other routing methods (flashinfer/trace/templates/moe.py; the
# numbers are FMOE_ROUTING_* of include/fmoe.h). Each starts from z = logits + bias in fp32.
DEFAULT, RENORMALIZE, LLAMA4, RENORMALIZE_NAIVE, TOPK = 1, 2, 3, 4, 5


def _softmax_f32(z: np.ndarray) -> np.ndarray:
    m = z.max(axis=-1, keepdims=True)
    e = np.exp((z - m).astype(F32)).astype(F32)
    return (e / e.sum(axis=-1, keepdims=True, dtype=F32)).astype(F32)


def route_method(logits: np.ndarray, bias: np.ndarray, rsf: float, method: int, top_k: int):
    """Routing by ``method`` with ``top_k`` picks per token.

    * DEFAULT (moe.py:205-209): s = softmax(z); the top_k of s; weight = s * rsf
    * RENORMALIZE (moe.py:245-249): the top_k of z; weight = softmax over the picked z * rsf
    * LLAMA4 (moe.py:285-288): argmax of z; weight = 1 / (1 + exp(-z)) * rsf (top_k = 1)
    * RENORMALIZE_NAIVE (moe.py:321-326): s = softmax(z); the top_k of s;
      weight = s / (their sum + 1e-20) * rsf
    * TOPK (moe.py:370-378): the top_k of z; every weight rsf / top_k

    Returns ``ids`` int32 ``[T, 8]`` in descending order of the selected value (ties to the
    lowest index), -1 after ``top_k``, and ``weights`` fp32 ``[T, 8]`` (0 after ``top_k``).
    """
    z = (np.asarray(logits, dtype=F32) + np.asarray(bias, dtype=F32)[None, :]).astype(F32)
    T = z.shape[0]
    softmax_first = method in (DEFAULT, RENORMALIZE_NAIVE)
    sel = _softmax_f32(z) if softmax_first else z
    order = np.argsort(-sel, axis=1, kind="stable")[:, :top_k]
    pv = np.take_along_axis(sel, order, axis=1).astype(F32)
    pz = np.take_along_axis(z, order, axis=1).astype(F32)
    if method == DEFAULT:
        w = (pv * F32(rsf)).astype(F32)
    elif method == RENORMALIZE_NAIVE:
        w = (pv / (pv.sum(axis=1, keepdims=True, dtype=F32) + F32(1e-20)) * F32(rsf)).astype(F32)
    elif method == RENORMALIZE:
        w = (_softmax_f32(pz) * F32(rsf)).astype(F32)
    elif method == LLAMA4:
        w = (F32(1.0) / (F32(1.0) + np.exp(-pz).astype(F32)) * F32(rsf)).astype(F32)
    elif method == TOPK:
        w = np.full((T, top_k), F32(rsf) / F32(top_k), dtype=F32)
    else:
        raise ValueError(method)
    ids = np.full((T, 8), -1, dtype=np.int32)
    wts = np.zeros((T, 8), dtype=F32)
    ids[:, :top_k] = order
    wts[:, :top_k] = w
    return ids, wts
