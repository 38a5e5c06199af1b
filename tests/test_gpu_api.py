"""The reference's own unit tests (tests/test_backend.py, tests/test_packed_decode.py)
run against this package on CUDA tensors, plus the requantize-demo known answers."""

import json
from pathlib import Path

import pytest
import torch

import anchorkv_b200 as akv
from anchorkv_b200 import CacheMode, CachePlan, PlannedSegment, SegmentRole

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture
def tensor(cuda):
    torch.manual_seed(7)
    return torch.randn(1, 2, 10, 8, dtype=torch.float32).to(cuda)


def test_int8_round_trip_uses_real_quantized_storage(tensor):
    packed = akv.quantize_tensor(tensor, CacheMode.INT8, group_size=16)
    restored = packed.dequantize()
    assert packed.payload.dtype == torch.int8 and packed.scales.dtype == torch.float16
    assert restored.shape == tensor.shape
    assert float((restored - tensor).abs().max()) < 0.02
    assert packed.stored_bytes < tensor.numel() * 2


def test_int4_is_nibble_packed_and_reconstructs_shape(tensor):
    int8 = akv.quantize_tensor(tensor, CacheMode.INT8, group_size=16)
    int4 = akv.quantize_tensor(tensor, CacheMode.INT4, group_size=16)
    restored = int4.dequantize()
    assert int4.payload.dtype == torch.uint8 and int4.payload.numel() == 80
    assert restored.shape == tensor.shape
    assert float((restored - tensor).abs().max()) < 0.3
    assert int4.stored_bytes < int8.stored_bytes


def test_zero_groups_round_trip_exactly(cuda):
    zeros = torch.zeros(1, 1, 4, 8, device=cuda)
    torch.testing.assert_close(akv.quantize_tensor(zeros, CacheMode.INT4, group_size=16).dequantize(), zeros)


def test_evicted_tensor_cannot_be_materialized(tensor):
    packed = akv.quantize_tensor(tensor, CacheMode.EVICTED)
    assert packed.stored_bytes == 0
    with pytest.raises(RuntimeError, match="evicted"):
        packed.dequantize()


class _Store:
    """The reference test's cache plus the tensors it was built from."""

    def __init__(self, cache, tensors):
        self.cache, self.tensors = cache, tensors

    def __getattr__(self, name):
        return getattr(self.cache, name)


@pytest.fixture
def cache(cuda):
    torch.manual_seed(11)
    c = akv.DeclarativeKVCache(block_size=4, group_size=16)
    tensors = {}
    for sid, start, count, role in [(0, 0, 4, SegmentRole.SINK), (1, 4, 6, SegmentRole.CONTEXT),
                                    (2, 10, 6, SegmentRole.CONTEXT), (3, 16, 4, SegmentRole.RESPONSE)]:
        key = torch.randn(1, 2, count, 8).to(cuda)
        value = torch.randn(1, 2, count, 8).to(cuda)
        tensors[sid] = (key, value)
        c.add_segment(sid, key, value, token_start=start, role=role)
    return _Store(c, tensors)


def test_archive_reduces_physical_storage(cache):
    before = cache.resident_bytes
    cache.requantize_segment(1, CacheMode.INT4)
    assert cache.segment_mode(1) == CacheMode.INT4
    assert cache.resident_bytes < before
    assert cache.compression_ratio > 1.0


def test_precision_loss_is_not_reported_as_reversible(cache):
    cache.requantize_segment(1, CacheMode.INT4)
    with pytest.raises(akv.LossyPromotionError):
        cache.requantize_segment(1, CacheMode.FP16)
    with pytest.raises(akv.LossyPromotionError):
        cache.protect_segment(1)


def test_protected_anchor_cannot_be_archived(cache):
    cache.feed_declarations('<anchor segments="2">')
    with pytest.raises(ValueError, match="protected"):
        cache.feed_declarations('<archive segments="2">')


def test_focus_and_local_modes_control_visible_blocks(cache):
    cache.requantize_segment(1, CacheMode.INT4)
    cache.feed_declarations('<focus segments="1">')
    focused = cache.materialize_visible(dtype=torch.float32)
    assert cache.visible_segment_ids() == (0, 1, 3)
    assert focused.key.shape[-2] == 14
    assert focused.positions.tolist() == list(range(0, 10)) + list(range(16, 20))
    assert float((focused.key[..., 4:10, :] - cache.tensors[1][0]).abs().max()) < 0.4
    cache.feed_declarations("</focus><local>")
    assert cache.visible_segment_ids() == (0, 3)


def test_evict_removes_segment_from_materialization(cache):
    cache.requantize_segment(1, CacheMode.EVICTED)
    cache.feed_declarations('<focus segments="1">')
    assert cache.visible_segment_ids() == (0, 3)


def test_stacked_layers_convert_to_legacy_hugging_face_cache(cuda):
    c = akv.DeclarativeKVCache(block_size=4, group_size=16)
    key = torch.randn(3, 1, 2, 6, 8).to(cuda)
    c.add_segment(0, key, torch.randn(3, 1, 2, 6, 8).to(cuda), token_start=0)
    c.requantize_segment(0, CacheMode.INT8)
    materialized = c.materialize_visible(dtype=torch.float32)
    legacy = materialized.to_legacy_cache()
    assert len(legacy) == 3 and legacy[0][0].shape == (1, 2, 6, 8)
    assert float((materialized.key - key).abs().max()) < 0.03


def test_applies_cache_plan_to_physical_blocks(cache):
    modes = [CacheMode.FP16, CacheMode.INT4, CacheMode.INT8, CacheMode.FP16]
    plan = CachePlan(tuple(PlannedSegment(i, m, 0, 0.0, "test") for i, m in enumerate(modes)),
                     budget_bytes=1, used_bytes=0, full_cache_bytes=0)
    cache.apply_plan(plan)
    assert [cache.segment_mode(i) for i in range(4)] == modes


def test_requantize_demo_known_answers(cuda):
    """cli.run_requantization_demo (cli.py:232-298) through this package on the GPU
    reproduces the reference's storage and error figures exactly."""
    demo = json.loads((GOLDEN / "demo.json").read_text())
    for archive in (CacheMode.INT4, CacheMode.INT8):
        torch.manual_seed(7)
        c = akv.DeclarativeKVCache(block_size=16, group_size=64, archive_mode=archive)
        originals, start = {}, 0
        for sid, count, role in ((0, 16, SegmentRole.SINK), (1, 16, SegmentRole.SCAFFOLD),
                                 (2, 64, SegmentRole.CONTEXT), (3, 64, SegmentRole.CONTEXT),
                                 (4, 32, SegmentRole.RESPONSE)):
            key = torch.randn(1, 2, count, 8, dtype=torch.float32)
            value = torch.randn(1, 2, count, 8, dtype=torch.float32)
            originals[sid] = (key, value)
            c.add_segment(sid, key.to(cuda), value.to(cuda), token_start=start, role=role)
            start += count
        c.feed_declarations('<anchor segments="4"><archive segments="2,3"><focus segments="3">')
        restored = c.materialize_segments([3], dtype=torch.float32)
        errors = torch.cat(((restored.key.cpu() - originals[3][0]).reshape(-1),
                            (restored.value.cpu() - originals[3][1]).reshape(-1))).abs()
        report = c.storage_report()
        want = demo[archive.value]
        for field in ("full_precision_bytes", "resident_bytes", "compression_ratio", "attention_mode",
                      "focus_segment_ids", "visible_segment_ids", "segments"):
            assert report[field] == want[field], field
        assert float(errors.max()) == want["max_abs_error"]
        assert float(errors.mean()) == want["mean_abs_error"]
        assert int(c.materialize_visible().key.shape[-2]) == want["materialized_focus_tokens"]


def test_page_quantization_counts_storage_and_handles_tiny_values(cuda):
    torch.manual_seed(11)
    source = torch.randn(2, 16, 128).half().to(cuda)
    sizes = []
    for bits in (4, 8, 16):
        packed = akv.pack_page(source, bits)
        sizes.append(packed.nbytes)
        assert packed.dense().shape == source.shape
        assert torch.isfinite(packed.dense()).all()
        expected = source.numel() * bits // 8 + (0 if bits == 16 else source.numel() // 64 * 2)
        assert packed.nbytes == expected
        if bits == 16:
            assert source.data_ptr() != packed.data.data_ptr()
            torch.testing.assert_close(packed.dense(), source, atol=0, rtol=0)
    assert sizes[0] < sizes[1] < sizes[2]
    assert torch.isfinite(akv.pack_page(torch.full_like(source, 1e-7), 4).dense()).all()


def test_append_demotion_protection_and_partial_page(cuda):
    layer = akv.PagedLayer(2, 128, 128, protected=(0,), recent_pages=1, device=cuda)
    source = torch.randn(1, 2, 83, 128).half().to(cuda)
    for start in range(0, 83, 7):
        layer.append(source[:, :, start:start + 7], source[:, :, start:start + 7])
    assert layer.length == 83
    assert [pair[0].bits for pair in layer.pages] == [16, 4, 4, 4, 16, 16]
    assert layer.demotions == 3
    k, v = layer.dense()
    assert k.shape == source.shape
    torch.testing.assert_close(k[:, :, :16], source[:, :, :16], atol=0, rtol=0)
    torch.testing.assert_close(k[:, :, 64:], source[:, :, 64:], atol=0, rtol=0)
    torch.testing.assert_close(k, v)
    with pytest.raises(ValueError):
        layer.protect(1)
    with pytest.raises(ValueError):
        layer.demote(0, 4)
    with pytest.raises(ValueError):
        layer.demote(1, 16)


@pytest.mark.parametrize("dim", [64, 128])
@pytest.mark.parametrize("bits", [4, 8, 16])
def test_pooled_page_views_hold_pack_page_payloads(cuda, dim, bits):
    """PagedLayer's page views over the pool (K row-major, V stored in the
    decode's bank-swizzled byte order behind a byte map) present the payload,
    scales and values pack_page gives the same 16 tokens (packed_decode.py:48-67);
    appended rows, a partial page included, read back as written."""
    torch.manual_seed(dim + bits)
    tokens = 45
    layer = akv.PagedLayer(2, dim, 64, archive_bits=bits, recent_pages=0, device=cuda)
    k = torch.randn(1, 2, tokens, dim).half().to(cuda)
    v = torch.randn_like(k)
    for start in range(0, tokens, 9):
        layer.append(k[:, :, start:start + 9], v[:, :, start:start + 9])
    assert [pair[0].bits for pair in layer.pages] == [bits, bits, 16]
    for p, (kp, vp) in enumerate(layer.pages):
        n = min(16, tokens - 16 * p)
        for page, src in ((kp, k), (vp, v)):
            slab = src[0, :, 16 * p:16 * p + n]
            if page.bits == 16:
                assert torch.equal(page.data[:, :n], slab)
                assert not page.data[:, n:].any()
                continue
            want = akv.pack_page(slab, page.bits, 64)
            assert torch.equal(page.data.view(torch.uint8), want.data.view(torch.uint8))
            assert torch.equal(page.scales, want.scales)
            assert torch.equal(page.dense(), want.dense())
    assert akv.take_device_status(cuda) == 0


def test_fp16_attention_matches_original_tensors_with_gqa(cuda):
    torch.manual_seed(2)
    key = torch.randn(1, 2, 37, 64).half().to(cuda)
    value = torch.randn_like(key)
    query = torch.randn(1, 4, 1, 64).half().to(cuda)
    layer = akv.PagedLayer(2, 64, 64, archive_bits=16, device=cuda)
    layer.append(key, value)
    expected = torch.nn.functional.scaled_dot_product_attention(
        query, key.repeat_interleave(2, 1), value.repeat_interleave(2, 1), scale=0.125)
    torch.testing.assert_close(akv.dense_attention(query, layer, 0.125), expected)
    torch.testing.assert_close(akv.packed_attention(query, layer, 0.125), expected, atol=2e-3, rtol=1e-2)


def test_online_anchor_prevents_later_demotion(cuda):
    layer = akv.PagedLayer(1, 64, 96, recent_pages=1, device=cuda)
    values = torch.ones(1, 1, 16, 64).half().to(cuda)
    layer.append(values, values)
    layer.protect(0)
    for _ in range(4):
        layer.append(values, values)
    assert layer.pages[0][0].bits == 16 and layer.pages[1][0].bits == 4


def test_packed_attention_validates_like_the_reference(cuda):
    layer = akv.PagedLayer(2, 64, 64, device=cuda)
    q = torch.zeros(1, 4, 1, 64, dtype=torch.float16, device=cuda)
    with pytest.raises(ValueError, match="nonempty"):
        akv.packed_attention(q, layer, 0.1)
    layer.append(torch.ones(1, 2, 5, 64, device=cuda).half(), torch.ones(1, 2, 5, 64, device=cuda).half())
    with pytest.raises(ValueError, match="batch=1"):
        akv.packed_attention(torch.zeros(2, 4, 1, 64, dtype=torch.float16, device=cuda), layer, 0.1)
    with pytest.raises(ValueError, match="divisible"):
        akv.packed_attention(torch.zeros(1, 3, 1, 64, dtype=torch.float16, device=cuda), layer, 0.1)
    with pytest.raises(ValueError, match="FP16"):
        akv.packed_attention(q.float(), layer, 0.1)
