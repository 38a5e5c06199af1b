"""Packed decode at the benchmark sizes, checked on the GPU (the CPU oracle would take hours there).

Two size-independent checks:

* a float32 torch attention over the dequantised pages (``akv_unpack_pages``, which is bit-exact with
  the oracle on small cases), skipped pages masked out, agrees with ``packed_attention`` within the
  decode's tolerance against the reference (max-abs 2e-3, rel 1e-2);
* the log-sum-exp merge identity (triton_decode.py:70-82 algebra): the decode of a store equals the
  merge of the decodes of its two page halves, within fp32 rounding;
* the pack kernel over one layer of the pack workload gives, bit for bit, the values of a torch
  restatement of quantize_tensor + dequantize (the reference's own function, run on CPU over sampled
  blocks, agrees with both).

Geometries: one layer of the batched workload (64 sequences x 8192 tokens, 16 query / 8 KV heads,
head_dim 128, pages 15/35/40/10 % FP16/INT8/INT4/evicted), one 1,048,576-token sequence (32 query
/ 8 KV heads, 5/25/70 % FP16/INT8/INT4) and one layer of the large-batch workload (128 sequences x
32,768 tokens, 32 query / 8 KV heads, 5 % evicted, the rest 10/20/70 % FP16/INT8/INT4), one fp16 scale
per (page, KV head) as in the benchmark, K and V N(0, 1) with 4 outlier channels per (sequence, head)
scaled by 8."""

import math

import numpy as np
import pytest
import torch

import anchorkv_b200 as akv
from anchorkv_b200 import _lib
from anchorkv_b200 import pool as P

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-3, 1e-2
D = 128
BATCHED = dict(batch=64, kv_heads=8, q_heads=16, tokens=8192, mix={16: .15, 8: .35, 4: .40, 0: .10})
LONG = dict(batch=1, kv_heads=8, q_heads=32, tokens=1 << 20, mix={16: .05, 8: .25, 4: .70})
# One layer of the large-batch workload: GQA 4, 128 sequences x 32,768 tokens, 5 % of pages evicted
# and the rest 10/20/70 % FP16/INT8/INT4.
LARGE = dict(batch=128, kv_heads=8, q_heads=32, tokens=32768, mix={16: .095, 8: .19, 4: .665, 0: .05})


def _kv(gen, shape, device):
    x = torch.randn(shape, generator=gen, device=device)
    channels = torch.randint(0, shape[-1], shape[:2] + (4,), generator=gen, device=device)
    boost = torch.ones(shape[:2] + (shape[-1],), device=device).scatter_(2, channels, 8.0)
    return (x * boost[:, :, None, :]).half()


def _store(cuda, seed, batch, kv_heads, tokens, mix, **_):
    gen = torch.Generator(device=cuda).manual_seed(seed)
    k = _kv(gen, (batch, kv_heads, tokens, D), cuda)
    v = _kv(gen, (batch, kv_heads, tokens, D), cuda)
    rng = np.random.default_rng(seed)
    keys = list(mix)
    bits = rng.choice(np.array(keys), size=(batch, tokens // 16), p=[mix[x] for x in keys])
    pool = P.PagePool(kv_heads, D, group=16 * D, pages={b: int((bits == b).sum()) for b in (16, 8, 4)},
                      device=cuda, shuffle_seed=seed, zero=False)
    store = P.pack_dense(pool, k, v, bits, semantics="tensor")
    del k, v
    return store


def _dense(store, b0, b1):
    """fp16 K and V ``[sequence, head, token, D]`` of sequences b0..b1 read back from their records
    (skipped pages as zeros), and the mask of tokens on resident pages."""
    desc = store.table[b0:b1].contiguous().view(-1)
    n, heads, dev = desc.numel(), store.heads, desc.device
    k = torch.empty((heads, n * 16, D), dtype=torch.float16, device=dev)
    v = torch.empty_like(k)
    _lib.call("akv_unpack_pages", desc.data_ptr(), n, store.pool.arena.data_ptr(), store.pool.nbytes, heads, D,
              store.group, k.data_ptr(), v.data_ptr(), _lib.DTYPE_F16, _lib.status_word(dev).data_ptr(),
              _lib.stream_of(dev))
    keep = ((desc & 3) != 0).view(b1 - b0, -1).repeat_interleave(16, dim=1)
    return k.view(heads, b1 - b0, -1, D).transpose(0, 1), v.view(heads, b1 - b0, -1, D).transpose(0, 1), keep


def _reference(store, q, scale, chunk):
    """float32 softmax(q K^T * scale) V over the resident tokens, GQA by grouping query heads."""
    batch, q_heads = q.shape[0], q.shape[1]
    g = q_heads // store.heads
    out = []
    for b0 in range(0, batch, chunk):
        b1 = min(batch, b0 + chunk)
        k, v, keep = _dense(store, b0, b1)
        qq = q[b0:b1, :, 0].float().view(b1 - b0, store.heads, g, D)
        s = torch.einsum("bhgd,bhtd->bhgt", qq, k.float()) * scale
        s.masked_fill_(~keep[:, None, None, :], float("-inf"))
        o = torch.einsum("bhgt,bhtd->bhgd", torch.softmax(s, dim=-1), v.float())
        out.append(o.reshape(b1 - b0, q_heads, 1, D))
        del k, v, s
    return torch.cat(out)


@pytest.mark.parametrize("geometry,splits,chunk", [(BATCHED, 8, 16), (LONG, 0, 1), (LARGE, 8, 4)],
                         ids=["batched", "long", "large"])
def test_full_size_decode_against_float32_attention(cuda, geometry, splits, chunk):
    store = _store(cuda, 90 + splits, **geometry)
    gen = torch.Generator(device=cuda).manual_seed(7)
    q = torch.randn((geometry["batch"], geometry["q_heads"], 1, D), generator=gen, device=cuda).half()
    scale = 1 / math.sqrt(D)
    out = akv.packed_attention(q, store, scale, splits=splits)
    ref = _reference(store, q, scale, chunk)
    assert akv.take_device_status(cuda) == 0
    torch.testing.assert_close(out.float(), ref, atol=ATOL, rtol=RTOL)


def test_full_size_long_sequence_equals_merge_of_its_halves(cuda):
    store = _store(cuda, 77, **LONG)
    gen = torch.Generator(device=cuda).manual_seed(8)
    q = torch.randn((1, LONG["q_heads"], 1, D), generator=gen, device=cuda).half()
    scale = 1 / math.sqrt(D)
    full = akv.packed_attention(q, store, scale, splits=0)
    half = store.max_blocks // 2
    states = []
    for lo, hi in ((0, half), (half, store.max_blocks)):
        shard = P.PagedBatch(store.pool, 1, hi - lo)
        shard.table.copy_(store.table[:, lo:hi])
        states.append(akv.decode_partial_states(q, shard, scale, splits=0))
    merged = akv.merge_states(torch.stack(states))
    assert akv.take_device_status(cuda) == 0
    torch.testing.assert_close(merged.float(), full.float(), atol=1e-3, rtol=1e-3)


def _quantized_values(x, bits):
    """What the reference attends over for blocks ``[n, 2048]`` (one per page and KV head):
    quantize_tensor (backend.py:210-219: fp32 absmax / qmax, 1 for an all-zero group, round half to
    even of x / scale, clamp, int8, fp16 scale after the division) then fp16(int * float(scale))."""
    xf = x.float()
    qmax = 127.0 if bits == 8 else 7.0
    amax = xf.abs().amax(dim=1, keepdim=True)
    # A tensor divisor: torch on CUDA turns division by a Python scalar into a multiply by its
    # reciprocal, which is not the correctly rounded quotient of the reference's division.
    scale = torch.where(amax == 0, torch.ones_like(amax), amax / torch.full_like(amax, qmax))
    # Through int8 as in the reference: a value that rounds to zero dequantises to +0, never -0.
    q = torch.round(xf / scale).clamp(-qmax, qmax).to(torch.int8).float()
    return (q * scale.half().float()).half()


def test_full_size_pack_matches_quantize_tensor_bit_for_bit(cuda):
    """One layer of the pack workload (32 sequences x 8 KV heads x 4096 tokens, 20/30/50 %
    FP16/INT8/INT4 pages, one scale per (page, KV head)): the values read back from the records are
    those of quantize_tensor then dequantize, bit for bit."""
    batch, heads, tokens = 32, 8, 4096
    gen = torch.Generator(device=cuda).manual_seed(11)
    k = _kv(gen, (batch, heads, tokens, D), cuda)
    v = _kv(gen, (batch, heads, tokens, D), cuda)
    bits = np.random.default_rng(11).choice(np.array([16, 8, 4]), size=(batch, tokens // 16), p=[.2, .3, .5])
    pool = P.PagePool(heads, D, group=16 * D, pages={b: int((bits == b).sum()) for b in (16, 8, 4)}, device=cuda)
    store = P.pack_dense(pool, k, v, bits, semantics="tensor")
    dk, dv, _ = _dense(store, 0, batch)
    assert akv.take_device_status(cuda) == 0
    mode = torch.from_numpy(bits).to(cuda)[:, None, :].expand(batch, heads, -1).reshape(-1)
    for name, src, got in (("K", k, dk), ("V", v, dv)):
        blocks = src.reshape(batch, heads, tokens // 16, 16 * D).reshape(-1, 16 * D)
        read = got.reshape(batch, heads, tokens // 16, 16 * D).reshape(-1, 16 * D)
        for b in (16, 8, 4):
            sel = mode == b
            want = blocks[sel] if b == 16 else _quantized_values(blocks[sel], b)
            bad = int((read[sel].view(torch.int16) != want.view(torch.int16)).sum())
            assert bad == 0, f"{name}: {bad} values of the {b}-bit pages differ"
