"""CPU oracle for packed single-token decode attention.

TEST INFRASTRUCTURE ONLY (checker and timed CPU baseline; never the product path).

The reference computes decode attention by dequantising every page to fp16 and
calling ``F.scaled_dot_product_attention`` with the KV heads repeated for GQA
(``src/anchorkv/packed_decode.py:197-203``, ``dense_attention``), or, with
visibility and eviction, by materialising only the resident visible blocks
(``src/anchorkv/backend.py:549-591``) and attending over those.  Its GPU kernel
(``src/anchorkv/triton_decode.py:35-82``) computes the same quantity as a split-K
online softmax whose splits are merged by their log-sum-exp.

This module restates those computations:

* :func:`attention_f64` is the exact answer (float64) over fp16 K/V/q values;
  the CUDA kernel and the reference's SDPA output are both compared to it.
* :func:`split_merge_f64` restates the split-K + merge algorithm of
  triton_decode.py:35-82 (page-strided splits, ``w = exp(m_s - max m)``, empty
  splits weighted 0) so the merge semantics can be checked on their own.
* :func:`dense_attention_torch` restates the reference's CPU path with torch ops
  (dequantised pages, ``repeat_interleave``, SDPA); it is the CPU baseline timed
  beside the GPU numbers.
"""

from __future__ import annotations

import math

import numpy as np


def kv_head_for(q_head: int, q_heads: int, kv_heads: int) -> int:
    """GQA mapping ``q // (Hq / Hkv)`` (heads.py:112-126, triton_decode.py:41)."""
    if q_heads % kv_heads:
        raise ValueError("query heads must be divisible by KV heads")
    return q_head // (q_heads // kv_heads)


def attention_f64(q, k, v, scale: float) -> np.ndarray:
    """Single-query GQA attention in float64.

    ``q``: ``[Hq, D]``; ``k``, ``v``: ``[Hkv, T, D]`` (already dequantised fp16
    values, as ``layer.dense()`` returns them).  Returns ``[Hq, D]`` float64.
    ``T == 0`` returns zeros (an all-masked context has nothing to attend to).
    """
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    hq, d = q.shape
    hkv, t, _ = k.shape
    g = hq // hkv
    out = np.zeros((hq, d), np.float64)
    if t == 0:
        return out
    for h in range(hq):
        kh = h // g
        s = k[kh] @ q[h] * scale
        s = s - s.max()
        p = np.exp(s)
        out[h] = (p[:, None] * v[kh]).sum(0) / p.sum()
    return out


def split_merge_f64(q, k, v, scale: float, splits: int, block: int = 16) -> np.ndarray:
    """Split-K decode with an LSE merge, as triton_decode.py:35-82 computes it.

    Pages (``block`` tokens) are assigned to splits ``split, split+S, ...``
    (triton_decode.py:48); each split keeps ``(num[D], max, den)``; the merge
    weights each split by ``exp(m_s - max_s m_s)`` and an empty split (max
    ``-inf``) gets weight 0 (triton_decode.py:76-82).
    """
    q = np.asarray(q, np.float64)
    k = np.asarray(k, np.float64)
    v = np.asarray(v, np.float64)
    hq, d = q.shape
    hkv, t, _ = k.shape
    g = hq // hkv
    pages = -(-t // block)
    out = np.zeros((hq, d), np.float64)
    for h in range(hq):
        kh = h // g
        parts = []
        for sp in range(splits):
            num = np.zeros(d)
            mx = -np.inf
            den = 0.0
            for page in range(sp, pages, splits):
                lo, hi = page * block, min((page + 1) * block, t)
                s = k[kh, lo:hi] @ q[h] * scale
                new = max(mx, s.max())
                r = math.exp(mx - new) if mx != -np.inf else 0.0
                p = np.exp(s - new)
                num = num * r + (p[:, None] * v[kh, lo:hi]).sum(0)
                den = den * r + p.sum()
                mx = new
            parts.append((num, mx, den))
        top = max(m for _, m, _ in parts)
        w = [math.exp(m - top) if m != -np.inf else 0.0 for _, m, _ in parts]
        den = sum(wi * dn for wi, (_, _, dn) in zip(w, parts))
        out[h] = sum(wi * nm for wi, (nm, _, _) in zip(w, parts)) / den
    return out


def lse_merge_f64(states) -> np.ndarray:
    """Merge ``(acc[D], m, l)`` partial states by log-sum-exp.

    ``m`` is the natural-log running max; ``acc`` and ``l`` are relative to it.
    Returns the normalised output (zeros when every state is empty).
    """
    ms = [m for _, m, _ in states]
    top = max(ms)
    if top == -np.inf:
        return np.zeros_like(np.asarray(states[0][0], np.float64))
    w = [math.exp(m - top) if m != -np.inf else 0.0 for m in ms]
    den = sum(wi * l for wi, (_, _, l) in zip(w, states))
    num = sum(wi * np.asarray(a, np.float64) for wi, (a, _, _) in zip(w, states))
    return num / den


def dense_attention_torch(q, k, v, scale: float):
    """The reference's CPU path (packed_decode.py:197-203) restated with torch.

    ``q``: ``[B, Hq, 1, D]`` fp16 torch tensor; ``k``, ``v``: ``[B, Hkv, T, D]``
    fp16.  Returns SDPA's fp16 output.
    """
    import torch.nn.functional as F

    repeats = q.shape[1] // k.shape[1]
    return F.scaled_dot_product_attention(
        q, k.repeat_interleave(repeats, 1), v.repeat_interleave(repeats, 1),
        is_causal=False, scale=scale,
    )
