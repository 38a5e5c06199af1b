"""The declarative block store on the page pool, against the reference.

Fixtures (tests/golden/declarative.*, attention.*) were written by running the
reference's DeclarativeKVCache on the same seeded inputs.  Per recorded state
this checks, through this package on CUDA: the visible segments, positions and
block ids, the storage report, the dense K/V it materialises bit for bit (as
fp16, fp32 and bf16, through akv_unpack_pages), and the decode of every layer
through packed_attention over the store's page table (visibility compiled into
skip descriptors) against the reference's SDPA over its materialised K/V, at
max-abs 2e-3 / relative 1e-2."""

import json
import math
from pathlib import Path

import numpy as np
import pytest
import torch

import anchorkv_b200 as akv
import workloads as W
from anchorkv_b200 import CacheMode, SegmentRole

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-2
GOLDEN = Path(__file__).resolve().parent / "golden"
DECL = {r["name"]: r for r in json.loads((GOLDEN / "declarative.json").read_text())}
DECL_OUT = np.load(GOLDEN / "declarative.npz")
ATTN = np.load(GOLDEN / "attention.npz")
PARITY = json.loads((GOLDEN / "attention.json").read_text())["parity"]


def _close(actual, expected):
    np.testing.assert_allclose(actual.float().cpu().numpy().reshape(-1),
                               np.asarray(expected).reshape(-1).astype(np.float32), atol=ATOL, rtol=RTOL)


def _build(spec, cuda):
    kv, queries = W.declarative_inputs(spec)
    cache = akv.DeclarativeKVCache(block_size=16, group_size=spec["group"])
    for sid, start, _, role in spec["segments"]:
        cache.add_segment(sid, kv[sid][0].to(cuda), kv[sid][1].to(cuda), token_start=start, role=SegmentRole(role))
    for step in spec["steps"]:
        if step[0] == "feed":
            cache.feed_declarations(step[1])
        else:
            cache.requantize_segment(step[1], CacheMode(step[2]))
    return cache, kv, queries


@pytest.mark.parametrize("spec", W.DECLARATIVE, ids=lambda s: s["name"])
def test_declarative_store_matches_the_reference(cuda, spec):
    rec = DECL[spec["name"]]
    cache, kv, queries = _build(spec, cuda)
    assert W.sha256(*[t for sid in sorted(kv) for t in kv[sid]], *queries) == rec["inputs_sha"]
    scale = 1.0 / math.sqrt(spec["dim"])
    for view in rec["views"]:
        cache.feed_declarations(view["directive"])
        assert list(cache.visible_segment_ids()) == view["visible"]
        mat = cache.materialize_visible()
        assert list(mat.key.shape) == view["shape"] and mat.key.dtype == torch.float16
        assert mat.positions.tolist() == view["positions"]
        assert list(mat.block_ids) == view["block_ids"] and list(mat.segment_ids) == view["segment_ids"]
        assert W.sha256(mat.key, mat.value) == view["dense_sha_f16"]
        f32 = cache.materialize_visible(dtype=torch.float32)
        assert W.sha256(f32.key, f32.value) == view["dense_sha_f32"]
        b16 = cache.materialize_visible(dtype=torch.bfloat16)
        assert W.sha256(b16.key, b16.value) == view["dense_sha_bf16"]
        assert cache.storage_report() == view["report"]
        want = DECL_OUT[view["out"]]
        if spec["name"] == "mixed" and 1 in view["visible"]:  # a visible segment the decode kernel cannot read
            with pytest.raises(ValueError, match="decode page format"):
                cache.decode_view(0)
            continue
        for layer, q in enumerate(queries):
            _close(akv.packed_attention(q.to(cuda), cache.decode_view(layer), scale), want[layer])
        if cache.layers == 1:  # a one-layer store is accepted as is
            _close(akv.packed_attention(queries[0].to(cuda), cache, scale), want[0])
    assert akv.take_device_status(cuda) == 0


@pytest.mark.parametrize("meta", PARITY, ids=lambda m: m["key"])
def test_parity_variants_through_the_declarative_store(cuda, meta):
    """The reference's parity workload as the reference built it (one
    16-token segment per block, per-block-per-head scales, roles, directives):
    the store's digest of the dense K/V, its resident bytes, its visibility,
    and packed_attention over the store against the reference's output."""
    q, k, v, _ = W.parity_workload(meta["seed"])
    assert W.sha256(q, k, v) == meta["inputs_sha"]
    p = W.PARITY
    cache = akv.DeclarativeKVCache(block_size=16, group_size=p["group"])
    for i, role in enumerate(meta["roles"]):
        sl = slice(16 * i, 16 * (i + 1))
        cache.add_segment(i, k[:, :, sl].to(cuda), v[:, :, sl].to(cuda), token_start=16 * i, role=SegmentRole(role))
    for i, mode in enumerate(meta["modes"]):
        cache.requantize_segment(i, CacheMode(mode))
    if meta["directive"]:
        cache.feed_declarations(meta["directive"])
    assert list(cache.visible_segment_ids()) == meta["visible"]
    assert cache.resident_bytes == meta["resident_bytes"]
    mat = cache.materialize_visible(dtype=torch.float16)
    assert W.sha256(mat.key, mat.value) == meta["dense_sha"] and mat.key.shape[-2] == meta["tokens"]
    _close(akv.packed_attention(q.to(cuda), cache, 1.0 / math.sqrt(p["dim"]), splits=4), ATTN[meta["key"]])
    assert akv.take_device_status(cuda) == 0


def test_requantize_is_one_repack_and_frees_pages(cuda):
    """Demoting a paged segment moves all of its pages at once (the pool's FP16
    slots come back), eviction frees them, and the decode table follows each
    change without a rebuild by the caller."""
    spec = W.DECLARATIVE[0]
    cache, _, queries = _build(dict(spec, steps=[]), cuda)
    q = queries[0].to(cuda)
    pool = cache.decode_view(0).pool
    free16 = pool.free_slots(16)
    cache.requantize_segment(4, CacheMode.INT4)  # 5 blocks x 1 row
    assert pool.free_slots(16) == free16 + 5
    before = akv.packed_attention(q, cache, 0.088)
    cache.requantize_segment(4, CacheMode.EVICTED)
    assert pool.free_slots(4) >= 5
    after = akv.packed_attention(q, cache, 0.088)
    assert not torch.equal(before, after)
    cache.feed_declarations("<local>")  # sink, scaffold and response only
    local = akv.packed_attention(q, cache, 0.088)
    mat = cache.materialize_visible()
    g = spec["q_heads"] // mat.key.shape[1]
    want = torch.nn.functional.scaled_dot_product_attention(
        q, mat.key.repeat_interleave(g, 1), mat.value.repeat_interleave(g, 1), scale=0.088)
    torch.testing.assert_close(local, want, atol=ATOL, rtol=RTOL)
    for sid in (0, 1, 5):  # the sink, scaffold and response segments <local> keeps visible
        cache.requantize_segment(sid, CacheMode.EVICTED)
    with pytest.raises(RuntimeError, match="no resident"):  # every visible block is evicted
        cache.decode_view(0)
    assert akv.take_device_status(cuda) == 0
