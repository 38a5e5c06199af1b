"""Packed decode attention on the GPU against the reference fixtures and the oracle.

Tolerance: max-abs 2e-3 and relative 1e-2 against the float64 oracle and the
reference's fp16 SDPA output (fp16 inputs, fp32 accumulation)."""

import json
import math
from pathlib import Path

import numpy as np
import pytest
import torch

import anchorkv_b200 as akv
import workloads as W
from anchorkv_b200 import _lib
from anchorkv_b200 import pool as P
from paged_reference import paged_decode_f64

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-2
GOLDEN = Path(__file__).resolve().parent / "golden"
ATTN = np.load(GOLDEN / "attention.npz")
META = json.loads((GOLDEN / "attention.json").read_text())
BITS = {"fp16": 16, "int8": 8, "int4": 4, "evicted": 0}


def _close(actual: torch.Tensor, expected, atol=ATOL, rtol=RTOL):
    a = actual.detach().float().cpu().numpy().reshape(-1)
    e = np.asarray(expected, np.float64).reshape(-1)
    np.testing.assert_allclose(a, e, atol=atol, rtol=rtol)


@pytest.mark.parametrize("meta", META["gate"], ids=lambda m: m["key"])
def test_kernel_gate_against_reference(cuda, meta):
    """The reference's GPU acceptance gate (colab_experiment.py:271-291) on the
    same inputs: page lifecycle, dense values and packed output."""
    q, k, v = (t.to(cuda) for t in W.gate_workload(meta["dim"], meta["length"], meta["seed"]))
    layer = akv.PagedLayer(2, meta["dim"], 128, archive_bits=meta["bits"], protected=(0,),
                           recent_pages=1, device=cuda)
    for begin in range(0, meta["length"], 7):
        layer.append(k[:, :, begin:begin + 7], v[:, :, begin:begin + 7])
    assert [pair[0].bits for pair in layer.pages] == meta["page_bits"]
    assert layer.demotions == meta["demotions"]
    assert layer.payload_bytes == meta["payload_bytes"]
    dk, dv = layer.dense()
    assert W.sha256(dk, dv) == meta["dense_sha"]
    out = akv.packed_attention(q, layer, meta["dim"] ** -0.5)
    assert out.shape == q.shape and out.dtype == torch.float16
    golden = ATTN[meta["key"]]
    _close(out, golden.astype(np.float64))
    ref = akv.dense_attention(q, layer, meta["dim"] ** -0.5)
    _close(out, ref.float().cpu().numpy())
    assert akv.take_device_status(cuda) == 0


@pytest.mark.parametrize("meta", META["parity"], ids=lambda m: m["key"])
@pytest.mark.parametrize("splits", [1, 4, 7])
def test_parity_workload_against_reference(cuda, meta, splits):
    """16 query / 8 KV heads, 512 tokens, per-block-per-head scales, FP16/INT8/INT4
    blocks, evicted blocks and focus/local visibility (backend.py:530-591)."""
    q, k, v, _ = W.parity_workload(meta["seed"])
    bits = np.array([BITS[m] for m in meta["modes"]])[None]
    visible = np.array([[i in set(meta["visible"]) for i in range(bits.shape[1])]])
    counts = {b: int((bits == b).sum()) for b in (16, 8, 4)}
    pool = P.PagePool(8, 128, group=2048, pages=counts, device=cuda, shuffle_seed=1)
    store = P.pack_dense(pool, k.to(cuda), v.to(cuda), bits, visible=visible, semantics="tensor")
    out = akv.packed_attention(q.to(cuda), store, 1 / math.sqrt(128), splits=splits)
    _close(out, ATTN[meta["key"]].astype(np.float64))
    oracle = paged_decode_f64(q[:, :, 0].numpy(), k.numpy(), v.numpy(), bits, 1 / math.sqrt(128),
                              group=2048, visible=visible)
    _close(out, oracle)
    assert akv.take_device_status(cuda) == 0


CASES = [
    # dim, q_heads, kv_heads, group, semantics, splits, lengths
    (128, 16, 8, 2048, "tensor", 4, [512, 333, 17]),
    (128, 32, 8, 2048, "tensor", 8, [200, 16, 1]),
    (128, 8, 8, 64, "page", 3, [97, 65]),
    (128, 64, 8, 64, "page", 2, [129]),
    (128, 4, 1, 128, "page", 64, [300]),
    (64, 4, 2, 64, "page", 4, [97, 33, 15]),
    (64, 8, 1, 1024, "tensor", 5, [250, 64]),
    (64, 16, 16, 32, "page", 1, [40]),
    (128, 32, 2, 2048, "tensor", 3, [100, 50]),
]


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"d{c[0]}_q{c[1]}_kv{c[2]}_g{c[3]}_s{c[5]}")
def test_random_batches_against_oracle(cuda, case):
    dim, hq, hkv, group, semantics, splits, lengths = case
    batch, tokens = len(lengths), max(lengths)
    nblk = -(-tokens // 16)
    seed = dim + hq * 3 + group + splits
    k = W.outlier_kv(seed, (batch, hkv, tokens, dim))
    v = W.outlier_kv(seed + 1, (batch, hkv, tokens, dim))
    q = W.normal(seed + 2, (batch, hq, 1, dim))
    bits = np.array(W.draw_modes(seed + 3, batch * nblk, {16: .2, 8: .3, 4: .4, 0: .1})).reshape(batch, nblk)
    visible = np.array(W.draw_modes(seed + 4, batch * nblk, {16: .9, 0: .1})).reshape(batch, nblk) > 0
    counts = {b: int((bits == b).sum()) for b in (16, 8, 4)}
    pool = P.PagePool(hkv, dim, group=group, pages=counts, device=cuda, shuffle_seed=seed)
    store = P.pack_dense(pool, k.to(cuda), v.to(cuda), bits, visible=visible, semantics=semantics,
                         lengths=lengths)
    scale = 1 / math.sqrt(dim)
    out = akv.packed_attention(q.to(cuda), store, scale, splits=splits)
    oracle = paged_decode_f64(q[:, :, 0].numpy(), k.numpy(), v.numpy(), bits, scale, group=group,
                              semantics=semantics, visible=visible, lengths=lengths)
    _close(out, oracle)
    assert akv.take_device_status(cuda) == 0


@pytest.mark.parametrize("scale_sign,v_big", [(-1, None), (1, "all"), (1, "some")],
                         ids=["negative_scale", "large_v_scales", "mixed_v_scales"])
def test_scale_edge_cases_against_oracle(cuda, scale_sign, v_big):
    """A negative softmax scale (the page max must be taken after scaling), and
    V values beyond +-1785 whose INT4/INT8 scales exceed 255: P times such a
    scale stays finite only under an exact running max (P <= 1)."""
    batch, hq, hkv, dim, tokens = 3, 16, 8, 128, 16 * 37 + 5
    nblk = -(-tokens // 16)
    k = W.outlier_kv(31, (batch, hkv, tokens, dim))
    v = W.outlier_kv(32, (batch, hkv, tokens, dim))
    if v_big == "all":
        v = (v * 400).clamp(-60000, 60000)
    elif v_big == "some":
        v[:, :, 16 * 5:16 * 9] *= 400  # pages 5-8 of every sequence
        v = v.clamp(-60000, 60000)
    q = W.normal(33, (batch, hq, 1, dim))
    bits = np.array(W.draw_modes(34, batch * nblk, {16: .1, 8: .4, 4: .5})).reshape(batch, nblk)
    counts = {b: int((bits == b).sum()) for b in (16, 8, 4)}
    pool = P.PagePool(hkv, dim, group=16 * dim, pages=counts, device=cuda, shuffle_seed=5)
    store = P.pack_dense(pool, k.to(cuda), v.to(cuda), bits)
    scale = scale_sign / math.sqrt(dim)
    out = akv.packed_attention(q.to(cuda), store, scale, splits=4)
    oracle = paged_decode_f64(q[:, :, 0].numpy(), k.numpy(), v.numpy(), bits, scale, group=16 * dim,
                              semantics="tensor")
    assert torch.isfinite(out).all()
    norm = 400.0 if v_big else 1.0  # same tolerance relative to the V magnitude
    _close(out.float() / norm, oracle / norm)
    assert akv.take_device_status(cuda) == 0


def test_fully_masked_sequence_outputs_zeros(cuda):
    k = W.outlier_kv(1, (2, 2, 64, 128))
    q = W.normal(2, (2, 4, 1, 128)).to(cuda)
    bits = np.array([[16, 8, 4, 4], [0, 0, 0, 0]])
    pool = P.PagePool(2, 128, group=64, pages={16: 1, 8: 1, 4: 2}, device=cuda)
    store = P.pack_dense(pool, k.to(cuda), k.to(cuda), bits, semantics="page")
    out = akv.packed_attention(q, store, 0.1, splits=3)
    assert torch.isfinite(out).all()
    assert (out[1] == 0).all()


def test_sharded_states_merge_to_full_result(cuda):
    """Contiguous sequence shards merged by LSE state equal the unsharded decode
    (the long-context multi-GPU algebra, emulated on one GPU)."""
    tokens, dim = 16 * 40, 128
    k = W.outlier_kv(21, (1, 8, tokens, dim))
    v = W.outlier_kv(22, (1, 8, tokens, dim))
    q = W.normal(23, (1, 32, 1, dim)).to(cuda)
    bits = np.array(W.draw_modes(24, 40, {16: .05, 8: .25, 4: .7}))[None]
    counts = {b: int((bits == b).sum()) for b in (16, 8, 4)}
    pool = P.PagePool(8, dim, group=2048, pages=counts, device=cuda)
    full = P.pack_dense(pool, k.to(cuda), v.to(cuda), bits)
    ref = akv.packed_attention(q, full, 0.088, splits=5)
    states = []
    for lo, hi in ((0, 13), (13, 27), (27, 40)):
        shard = P.PagedBatch(pool, 1, hi - lo)
        shard.table.copy_(full.table[:, lo:hi])
        states.append(akv.decode_partial_states(q, shard, 0.088, splits=3))
    out = akv.merge_states(torch.stack(states))
    oracle = paged_decode_f64(q[:, :, 0].cpu().numpy(), k.numpy(), v.numpy(), bits, 0.088, group=2048)
    _close(ref, oracle)
    _close(out, oracle)
    _close(out, ref.float().cpu().numpy())


def test_out_of_arena_descriptor_is_skipped_and_reported(cuda):
    k = W.outlier_kv(31, (1, 2, 48, 64))
    q = W.normal(32, (1, 2, 1, 64)).to(cuda)
    pool = P.PagePool(2, 64, group=64, pages={16: 3}, device=cuda)
    store = P.pack_dense(pool, k.to(cuda), k.to(cuda), [[16, 16, 16]], semantics="page")
    good = akv.packed_attention(q, store, 0.125)
    ref_two = P.PagedBatch(pool, 1, 2)
    ref_two.table.copy_(store.table[:, :2])
    expect = akv.packed_attention(q, ref_two, 0.125)
    assert akv.take_device_status(cuda) == 0
    store.table[0, 2] = P.encode(16, 16, pool.nbytes + 4096)  # beyond the arena: bounds check skips it
    bad = akv.packed_attention(q, store, 0.125)
    torch.cuda.synchronize(cuda)  # the kernel has finished: its report is visible to the host
    with pytest.raises(akv.KernelError, match="outside the arena"):
        akv.packed_attention(q, store, 0.125)  # the next call raises before it launches
    assert akv.take_device_status(cuda) == 0  # raising cleared the word
    torch.testing.assert_close(bad, expect)
    assert not torch.equal(good, expect)
    bad_again = akv.packed_attention(q, store, 0.125)
    assert akv.take_device_status(cuda) & 1  # the synchronising read reports it as well
    torch.testing.assert_close(bad_again, expect)


def _batch_store(cuda, batch, tokens, hq=16, hkv=8, dim=128, seed=41):
    nblk = -(-tokens // 16)
    k = W.outlier_kv(seed, (batch, hkv, tokens, dim))
    v = W.outlier_kv(seed + 1, (batch, hkv, tokens, dim))
    q = W.normal(seed + 2, (batch, hq, 1, dim))
    bits = np.array(W.draw_modes(seed + 3, batch * nblk, {16: .15, 8: .35, 4: .4, 0: .1})).reshape(batch, nblk)
    counts = {b: int((bits == b).sum()) for b in (16, 8, 4)}
    pool = P.PagePool(hkv, dim, group=16 * dim, pages=counts, device=cuda, shuffle_seed=seed)
    store = P.pack_dense(pool, k.to(cuda), v.to(cuda), bits)
    return store, q, k, v, bits


def _c_attention(store, q, scale, splits, ws, out, status):
    """akv_packed_attention through the C ABI with a caller-owned workspace."""
    lib = _lib.load()
    stream = torch.cuda.current_stream(q.device).cuda_stream
    B, Hq, _, D = q.shape
    return lib.akv_packed_attention(store.pool.arena.data_ptr(), store.pool.nbytes, store.table.data_ptr(),
                                    store.table.stride(0), store.seq_blocks.data_ptr(), store.max_blocks,
                                    q.data_ptr(), q.stride(0), q.stride(1), B, Hq, store.heads, D, store.group,
                                    scale, splits, out.data_ptr(), out.stride(0), out.stride(1), ws.data_ptr(),
                                    ws.numel(), status.data_ptr(), stream)


@pytest.mark.parametrize("batch,tokens,splits", [(24, 16 * 64, 8), (20, 16 * 200 + 7, 4), (64, 16 * 32, 0)])
def test_row_merge_outputs_and_states_against_oracle(cuda, batch, tokens, splits):
    """Many (sequence, query head) rows: the one-warp-per-row merge, into the
    output and into LSE states (whose own merge gives the same output)."""
    store, q, k, v, bits = _batch_store(cuda, batch, tokens)
    qd = q.to(cuda)
    assert batch * q.shape[1] >= 2 * 148  # the row merge
    out = akv.packed_attention(qd, store, 0.088, splits=splits)
    oracle = paged_decode_f64(q[:, :, 0].numpy(), k.numpy(), v.numpy(), bits, 0.088, group=16 * 128)
    _close(out, oracle)
    states = akv.decode_partial_states(qd, store, 0.088, splits=splits)
    torch.testing.assert_close(akv.merge_states(states[None]), out, atol=1e-3, rtol=1e-3)
    assert akv.take_device_status(cuda) == 0


def test_long_sequence_wide_merge_against_oracle(cuda):
    """Hundreds of warps per (sequence, KV head): a CTA of 32 warps per row."""
    store, q, k, v, bits = _batch_store(cuda, 1, 16 * 3000, hq=32, seed=51)
    out = akv.packed_attention(q.to(cuda), store, 0.088, splits=0)
    oracle = paged_decode_f64(q[:, :, 0].numpy(), k.numpy(), v.numpy(), bits, 0.088, group=2048)
    _close(out, oracle)
    assert akv.take_device_status(cuda) == 0


def test_workspace_needs_no_initialisation_and_survives_geometry_changes(cuda):
    """Any bytes in the workspace, and partials of other geometries left in it,
    do not change a result: each decode rewrites the header and every partial
    the merge reads."""
    lib = _lib.load()
    status = _lib.status_word(cuda)
    small, q_s, *_ = _batch_store(cuda, 2, 16 * 40, seed=61)
    big, q_b, *_ = _batch_store(cuda, 24, 16 * 40, seed=71)
    qs, qb = q_s.to(cuda), q_b.to(cuda)
    nbytes = max(lib.akv_workspace_bytes(24, 16, 8, 128, big.max_blocks, 8),
                 lib.akv_workspace_bytes(2, 16, 8, 128, small.max_blocks, 8))
    clean = torch.zeros(nbytes, dtype=torch.uint8, device=cuda)
    ref_s, ref_b = torch.empty_like(qs), torch.empty_like(qb)
    assert _c_attention(small, qs, 0.088, 8, clean, ref_s, status) == 0
    assert _c_attention(big, qb, 0.088, 8, clean, ref_b, status) == 0
    gen = torch.Generator(device=cuda).manual_seed(3)
    for fill in ("ones", "random"):
        ws = (torch.full((nbytes,), 255, dtype=torch.uint8, device=cuda) if fill == "ones" else
              torch.randint(0, 256, (nbytes,), generator=gen, dtype=torch.uint8, device=cuda))
        for store, qq, ref in ((small, qs, ref_s), (big, qb, ref_b), (small, qs, ref_s)):
            out = torch.empty_like(qq)
            assert _c_attention(store, qq, 0.088, 8, ws, out, status) == 0
            assert torch.equal(out, ref)
    assert akv.take_device_status(cuda) == 0


def _sdpa_over_pages(store, q, scale):
    """The reference's dense path on the GPU (packed_decode.py:197-203): fp16 SDPA
    over the dequantised pages (akv_unpack_pages, bit-exact with
    QuantizedPage.dense), skipped pages masked out, GQA by repetition."""
    desc = store.table.reshape(-1).contiguous()
    n, heads, dim, batch = desc.numel(), store.heads, q.shape[-1], q.shape[0]
    k = torch.empty((heads, n * 16, dim), dtype=torch.float16, device=q.device)
    v = torch.empty_like(k)
    _lib.call("akv_unpack_pages", desc.data_ptr(), n, store.pool.arena.data_ptr(), store.pool.nbytes, heads, dim,
              store.group, k.data_ptr(), v.data_ptr(), _lib.DTYPE_F16, _lib.status_word(q.device).data_ptr(),
              _lib.stream_of(q.device))
    k, v = (t.view(heads, batch, -1, dim).transpose(0, 1) for t in (k, v))
    keep = ((desc & 3) != 0).view(batch, -1).repeat_interleave(16, 1)
    mask = torch.zeros(keep.shape, dtype=torch.float16, device=q.device).masked_fill(~keep, float("-inf"))
    g = q.shape[1] // heads
    out = torch.nn.functional.scaled_dot_product_attention(q, k.repeat_interleave(g, 1), v.repeat_interleave(g, 1),
                                                           attn_mask=mask[:, None, None, :], scale=scale)
    return torch.nan_to_num(out, nan=0.0)  # a sequence with every page skipped: zeros, as the kernel gives


@pytest.mark.parametrize("batch,hq,tokens", [(2048, 64, 16), (512, 16, 32)], ids=["one_page", "two_pages"])
def test_many_short_sequences_against_the_reference_path(cuda, batch, hq, tokens):
    """Thousands of one- and two-page sequences (a warp's range spans several
    items; 16.7 M and 1 M outputs) with outlier channels: against the
    reference's own dense path on the GPU (fp16 SDPA over the same dequantised
    pages) within 2e-3 / 1e-2 everywhere, and no further from the float64
    oracle than that path is.  At this many outputs the float64 oracle itself
    is beyond 2e-3 of the fp16 path in a few places (P rounded to fp16 in the
    P.V product, in both)."""
    store, q, k, v, bits = _batch_store(cuda, batch, tokens, hq=hq, seed=57)
    qd = q.to(cuda)
    out = akv.packed_attention(qd, store, 0.088, splits=4)
    ref = _sdpa_over_pages(store, qd, 0.088)
    torch.testing.assert_close(out.float(), ref.float(), atol=ATOL, rtol=RTOL)
    oracle = paged_decode_f64(q[:, :, 0].numpy(), k.numpy(), v.numpy(), bits, 0.088, group=16 * 128).reshape(-1)
    ours = np.abs(out.float().cpu().numpy().reshape(-1) - oracle).max()
    theirs = np.abs(ref.float().cpu().numpy().reshape(-1) - oracle).max()
    assert ours <= 1.25 * theirs + 1e-4, (ours, theirs)
    assert akv.take_device_status(cuda) == 0
