"""Timed CPU baseline for decode: the reference's PyTorch CPU path, restated.

TEST/MEASUREMENT INFRASTRUCTURE ONLY: ``bench.py`` times this on the host
cores beside the GPU numbers (its ``cpu_baseline`` leg and ``--impl
reference`` arm).  It is never the product path.

Per decode call the reference dequantises every resident page to fp16
(``QuantizedPage.dense``, packed_decode.py:34-45: ``(int * float(scale)).half()``
with nibbles sign-extended for INT4), concatenates them
(``PagedLayer.dense``, packed_decode.py:189-194), repeats KV heads for GQA
and calls ``F.scaled_dot_product_attention`` (``dense_attention``,
packed_decode.py:197-203).  :func:`decode_cpu` does the same work with the
same torch ops; evicted/invisible blocks are dropped first, as
``materialize_segments`` does (backend.py:557-591).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch
import torch.nn.functional as F

from . import codec as OC


@dataclass
class CpuPage:
    bits: int
    k: torch.Tensor
    v: torch.Tensor
    ks: torch.Tensor | None
    vs: torch.Tensor | None
    shape: tuple
    group: int

    @property
    def nbytes(self) -> int:
        n = self.k.numel() * self.k.element_size() + self.v.numel() * self.v.element_size()
        if self.ks is not None:
            n += 2 * (self.ks.numel() * self.ks.element_size())
        return n


def _dense(payload: torch.Tensor, scales, bits: int, shape, group: int) -> torch.Tensor:
    """QuantizedPage.dense (packed_decode.py:34-45) on CPU tensors."""
    if bits == 16:
        return payload
    if bits == 8:
        ints = payload.float()
    else:
        lo = payload & 15
        hi = payload >> 4
        vals = torch.stack((lo, hi), -1).reshape(shape).short()
        ints = torch.where(vals >= 8, vals - 16, vals).float()
    groups = ints.reshape(-1, group)
    return (groups * scales.float().reshape(-1, 1)).reshape(shape).half()


def build_sequence(seed: int, heads: int, dim: int, blocks: int, bits_per_block, group: int):
    """Pages of one sequence: fp16 N(0,1) K/V quantized per (block, head) slab with
    quantize_tensor semantics at ``group`` (one scale per slab when group = 16*dim)."""
    g = torch.Generator().manual_seed(seed)
    pages = []
    shape = (heads, 16, dim)
    for j in range(blocks):
        bits = int(bits_per_block[j])
        if bits == 0:
            pages.append(None)
            continue
        kv = [torch.randn(shape, generator=g).half() for _ in range(2)]
        if bits == 16:
            pages.append(CpuPage(16, kv[0], kv[1], None, None, shape, group))
            continue
        packed = [OC.quantize_tensor(t.numpy(), bits, group) for t in kv]
        pages.append(CpuPage(bits, torch.from_numpy(packed[0][0]), torch.from_numpy(packed[1][0]),
                             torch.from_numpy(packed[0][1]), torch.from_numpy(packed[1][1]), shape, group))
    return pages


def decode_cpu(pages, query: torch.Tensor, scale: float) -> torch.Tensor:
    """One decode call of the reference path on the host: ``query`` [1, Hq, 1, D] fp16."""
    keys, values = [], []
    for p in pages:
        if p is None:
            continue
        keys.append(_dense(p.k, p.ks, p.bits, p.shape, p.group))
        values.append(_dense(p.v, p.vs, p.bits, p.shape, p.group))
    k = torch.cat(keys, dim=1).unsqueeze(0)
    v = torch.cat(values, dim=1).unsqueeze(0)
    rep = query.shape[1] // k.shape[1]
    return F.scaled_dot_product_attention(query, k.repeat_interleave(rep, 1), v.repeat_interleave(rep, 1),
                                          is_causal=False, scale=scale)


def resident_bytes(pages) -> int:
    return sum(p.nbytes for p in pages if p is not None)


def random_bits(seed: int, count: int, mix) -> np.ndarray:
    """Per-block precision draws: ``mix`` maps bits (16/8/4/0) -> probability."""
    rng = np.random.default_rng(seed)
    keys = list(mix)
    return rng.choice(np.array(keys), size=count, p=np.array([mix[k] for k in keys]))
