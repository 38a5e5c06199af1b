"""The reference's small functions and error paths, side by side on CPU.

Everything here needs no kernel: argument checks (which run before any
device work), FP16 and EVICTED storage, attention and KL helpers over given
tensors, and the Hugging Face cache stacking.  Each case runs on the
reference installed unmodified in baseline/_ref and on this package; results
must be equal bit for bit, errors equal in type name and message.  INT8/INT4
values are compared with the reference on the GPU (tests/test_gpu_codec.py).
"""

import pytest
import torch

import anchorkv_b200 as akv



@pytest.fixture(scope="module")
def ref(reference_install):
    from anchorkv import backend, packed_decode, policy

    return backend, packed_decode, policy


def _outcome(fn):
    try:
        return ("ok", fn())
    except Exception as error:
        return ("error", type(error).__name__, str(error))


def _same(a, b):
    if isinstance(a, torch.Tensor):
        return (isinstance(b, torch.Tensor) and a.dtype == b.dtype and a.shape == b.shape
                and torch.equal(a.view(torch.uint8) if a.is_floating_point() else a,
                                b.view(torch.uint8) if b.is_floating_point() else b))
    if isinstance(a, (tuple, list)):
        return isinstance(b, (tuple, list)) and len(a) == len(b) and all(_same(x, y) for x, y in zip(a, b))
    return a == b


def _both(ref_fn, our_fn):
    a, b = _outcome(ref_fn), _outcome(our_fn)
    assert a[0] == b[0], (a, b)
    if a[0] == "error":
        assert a == b
    else:
        assert _same(a[1], b[1]), (a, b)
    return a


def test_quantize_tensor_checks_and_lossless_modes(ref):
    RB, _, RPol = ref
    g = torch.Generator().manual_seed(3)
    x = torch.randn(3, 5, generator=g)
    cases = [
        (torch.arange(6), "int8", 16),            # not floating point
        ([1.0, 2.0], "int8", 16),                 # not a tensor
        (x, "int8", 0), (x, "int4", -2),          # group sizes
        (x, "int4", 7),                           # odd INT4 group
        (torch.zeros(0), "int8", 16),             # empty
    ]
    for t, mode, group in cases:
        _both(lambda: RB.quantize_tensor(t, RPol.CacheMode(mode), group_size=group),
              lambda: akv.quantize_tensor(t, akv.CacheMode(mode), group_size=group))
    for dtype in (torch.float32, torch.float16, torch.bfloat16):
        t = x.to(dtype)
        for mode in ("fp16", "evicted"):
            r = RB.quantize_tensor(t, RPol.CacheMode(mode), group_size=4)
            o = akv.quantize_tensor(t, akv.CacheMode(mode), group_size=4)
            assert (r.shape, r.original_dtype, r.group_size, r.original_numel, r.stored_bytes) == \
                (o.shape, o.original_dtype, o.group_size, o.original_numel, o.stored_bytes)
            assert _same(r.payload, o.payload) if r.payload is not None else o.payload is None
            for kwargs in ({}, {"dtype": torch.float32}, {"dtype": torch.bfloat16}):
                _both(lambda: r.dequantize(**kwargs), lambda: o.dequantize(**kwargs))


def test_pack_page_checks_and_fp16_pages(ref):
    _, RP, _ = ref
    g = torch.Generator().manual_seed(4)
    page = torch.randn(2, 16, 64, generator=g)
    for t, bits, group in [(page, 3, 64), (page, 32, 64), (page[0], 4, 64), (page, 4, 48), (page, 8, 7),
                           (page.unsqueeze(0), 8, 64)]:
        _both(lambda: RP.pack_page(t, bits, group), lambda: akv.pack_page(t, bits, group))
    r, o = RP.pack_page(page, 16, 32), akv.pack_page(page, 16, 32)
    assert (r.bits, r.shape, r.group, r.nbytes) == (o.bits, o.shape, o.group, o.nbytes)
    assert _same(r.data, o.data) and _same(r.dense(), o.dense()) and r.scales is None and o.scales is None
    assert RP.tensor_bytes(page) == akv.tensor_bytes(page)


def test_attention_and_kl_helpers(ref):
    _, RP, _ = ref
    g = torch.Generator().manual_seed(5)
    for hq, hkv, tokens, dtype in [(8, 2, 40, torch.float32), (4, 4, 17, torch.float16), (16, 8, 64, torch.float32)]:
        key = torch.randn(1, hkv, tokens, 64, generator=g).to(dtype)
        value = torch.randn(1, hkv, tokens, 64, generator=g).to(dtype)
        q = torch.randn(1, hq, 1, 64, generator=g).to(dtype)

        class Layer:  # both implementations read K/V through layer.dense()
            @staticmethod
            def dense():
                return key, value

        _both(lambda: RP.dense_attention(q, Layer, 0.125), lambda: akv.dense_attention(q, Layer, 0.125))
    for shape in [(3, 11), (2, 4, 50)]:
        a, b = torch.randn(shape, generator=g), torch.randn(shape, generator=g)
        _both(lambda: RP.kl_divergence(a, b), lambda: akv.kl_divergence(a, b))
        _both(lambda: RP.kl_divergence(a, a), lambda: akv.kl_divergence(a, a))
        _both(lambda: RP.kl_divergence(a.half(), b), lambda: akv.kl_divergence(a.half(), b))


def test_stack_legacy_cache(ref):
    RB, _, _ = ref
    g = torch.Generator().manual_seed(6)
    kv = [(torch.randn(1, 2, 5, 8, generator=g), torch.randn(1, 2, 5, 8, generator=g)) for _ in range(3)]

    class Cache:  # a cache object with the Hugging Face conversion method
        @staticmethod
        def to_legacy_cache():
            return tuple(kv)

    for source in [tuple(kv), Cache, (), ((kv[0][0],),), (kv[0], (kv[1][0][..., :4, :], kv[1][1]))]:
        _both(lambda: RB.stack_legacy_cache(source), lambda: akv.stack_legacy_cache(source))


def test_packed_attention_argument_errors(ref):
    """The checks triton_decode.py:86-94 makes before any launch, on empty CPU layers of
    both implementations (the kernels are never reached)."""
    from anchorkv import triton_decode

    _, RP, _ = ref
    ref_layer = RP.PagedLayer(2, 64, 64, device="cpu")
    our_layer = akv.PagedLayer(2, 64, 64, device="cpu")
    g = torch.Generator().manual_seed(7)
    queries = [torch.randn(2, 4, 1, 64, generator=g).half(),   # batch 2
               torch.randn(1, 4, 3, 64, generator=g).half(),   # three query tokens
               torch.randn(1, 4, 1, 32, generator=g).half(),   # head_dim mismatch
               torch.randn(1, 4, 1, 64, generator=g).half(),   # a CPU query (and an empty cache)
               torch.randn(1, 4, 1, 64, generator=g)]          # fp32
    for q in queries:
        _both(lambda: triton_decode.packed_attention(q, ref_layer, 0.125),
              lambda: akv.packed_attention(q, our_layer, 0.125))


def test_gqa_head_map(ref):
    """query_head_to_kv_head (heads.py:112-126), the map the decode kernel serves query heads by."""
    from anchorkv import heads

    for hq in (0, 1, 4, 8, 12, 16, 32, -8):
        for hkv in (0, 1, 2, 3, 4, 8, -1):
            for q in (-1, 0, 1, 3, 7, 15, 31, 32):
                _both(lambda: heads.query_head_to_kv_head(q, num_query_heads=hq, num_kv_heads=hkv),
                      lambda: akv.query_head_to_kv_head(q, num_query_heads=hq, num_kv_heads=hkv))
