"""Oracle expectations for paged stores (test infrastructure).

Builds, with the CPU oracle, what the reference computes for a batch of
sequences stored as 16-token blocks of mixed precision: the dense fp16 values
the reference would attend over (per-block ``quantize_tensor`` or
``pack_page``, evicted/hidden blocks dropped, backend.py:557-591) and the
float64 attention output, plus the exact bytes of a page record.
"""

from __future__ import annotations

import math

import numpy as np

from oracle import attention as OA
from oracle import codec as OC

BLOCK = 16


def block_values(slab: np.ndarray, bits: int, group: int, semantics: str) -> np.ndarray:
    """fp16 values the reference holds for one [heads?, 16, D] slab after quantization."""
    slab = np.asarray(slab, np.float16)
    if bits == 16:
        return slab
    if semantics == "tensor":
        payload, scales = OC.quantize_tensor(slab, bits, group)
        return OC.dequantize_tensor(payload, scales, bits, group, slab.size).astype(np.float16).reshape(slab.shape)
    s3 = slab.reshape(-1, slab.shape[-2], slab.shape[-1])
    payload, scales = OC.pack_page(s3, bits, group)
    return OC.page_dense(payload, scales, bits, group, s3.shape).reshape(slab.shape)


def slab_payload(slab: np.ndarray, bits: int, group: int, semantics: str):
    """(payload bytes, scale bytes) of one [16, D] slab, reference layout."""
    slab = np.asarray(slab, np.float16)
    if bits == 16:
        return slab.tobytes(), b""
    if semantics == "tensor":
        payload, scales = OC.quantize_tensor(slab, bits, group)
    else:
        payload, scales = OC.pack_page(slab[None], bits, group)
    return np.asarray(payload).tobytes(), np.asarray(scales, np.float16).tobytes()


def v_stored(payload: bytes, dim: int, bits: int) -> bytes:
    """A row-major V payload in the pool's stored order: the 16-byte unit u of
    the 128-byte line that holds token row r is stored at unit u ^ key(r),
    key chosen per row width so the decode's V fragment loads are free of
    bank conflicts."""
    row = dim * bits // 8
    src = np.frombuffer(payload, np.uint8).reshape(-1, 16)  # 16-byte units
    out = np.empty_like(src)
    for u in range(src.shape[0]):
        r = 16 * u // row
        if row == 256:
            t = (r >> 1) & 3
            key = (t & 1) | ((t & 2) << 1)
        elif row in (128, 64):
            key = r & 6
        else:
            key = (r >> 1) & 2
        line, unit = divmod(u, 8)
        out[8 * line + (unit ^ key)] = src[u]
    return out.tobytes()


def record_bytes_expected(kslab, vslab, bits, group, semantics, record_size) -> bytes:
    kp, ks = slab_payload(kslab, bits, group, semantics)
    vp, vs = slab_payload(vslab, bits, group, semantics)
    vp = v_stored(vp, np.asarray(vslab).shape[-1], bits)
    rec = kp + vp + ks + vs
    return rec + b"\0" * (record_size - len(rec))


def paged_decode_f64(q, k, v, bits, scale, *, group=64, semantics="tensor", visible=None, lengths=None):
    """Expected decode output [B, Hq, D] (float64).

    q: [B, Hq, D] fp16; k, v: [B, Hkv, T, D] fp16; bits: [B, nblk] in {16, 8, 4, 0}.
    The per-block quantization is applied per (sequence, KV head) slab."""
    q = np.asarray(q, np.float16)
    k = np.asarray(k, np.float16)
    v = np.asarray(v, np.float16)
    batch, hkv, tokens, dim = k.shape
    nblk = -(-tokens // BLOCK)
    bits = np.asarray(bits).reshape(batch, nblk)
    lengths = np.full(batch, tokens) if lengths is None else np.asarray(lengths)
    out = np.zeros((batch, q.shape[1], dim))
    for b in range(batch):
        ks, vs = [], []
        for j in range(nblk):
            lo = j * BLOCK
            if lo >= lengths[b] or bits[b, j] == 0:
                continue
            if visible is not None and not visible[b][j]:
                continue
            n = min(BLOCK, lengths[b] - lo)
            kslab = np.zeros((hkv, BLOCK, dim), np.float16)
            vslab = np.zeros_like(kslab)
            avail = min(BLOCK, tokens - lo)
            kslab[:, :avail] = k[b, :, lo:lo + avail]
            vslab[:, :avail] = v[b, :, lo:lo + avail]
            kd = np.stack([block_values(kslab[h], int(bits[b, j]), group, semantics) for h in range(hkv)])
            vd = np.stack([block_values(vslab[h], int(bits[b, j]), group, semantics) for h in range(hkv)])
            ks.append(kd[:, :n])
            vs.append(vd[:, :n])
        if ks:
            out[b] = OA.attention_f64(q[b], np.concatenate(ks, 1), np.concatenate(vs, 1), scale)
    return out


def default_scale(dim: int) -> float:
    return 1.0 / math.sqrt(dim)
