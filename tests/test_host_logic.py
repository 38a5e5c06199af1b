"""Host-side logic that needs no GPU: descriptors, pool bookkeeping, the
declarative parser and the block-store lifecycle (data plane replaced by the
oracle in this test only)."""

import numpy as np
import pytest
import torch

import anchorkv_b200 as akv
from anchorkv_b200 import pool as P
from anchorkv_b200.policy import CacheMode
from host_codec import use_oracle_codec


def test_descriptor_round_trip():
    for bits in (4, 8, 16):
        for ntok in (1, 7, 16):
            for off in (0, 16, 4096 * 123, (1 << 40) + 48):
                assert P.decode(P.encode(bits, ntok, off)) == (bits, ntok, off)
    assert P.encode(None, 5, 0) == 0 and P.decode(0)[0] is None
    with pytest.raises(ValueError):
        P.encode(4, 0, 0)
    with pytest.raises(ValueError):
        P.encode(4, 3, 8)
    codes = np.array([1, 2, 3, 0])
    arr = P.encode_array(codes, np.array([16, 3, 1, 9]), np.array([32, 64, 0, 16]))
    assert list(arr) == [P.encode(4, 16, 32), P.encode(8, 3, 64), P.encode(16, 1, 0), 0]


def test_record_sizes_are_reference_bytes_plus_pad():
    # QuantizedPage.nbytes per head: payload + scales (packed_decode.py:28-32)
    assert P.algorithmic_record_bytes(128, 2048, 4) == 2 * 1024 + 4
    assert P.record_bytes(128, 2048, 4) == 2064
    assert P.algorithmic_record_bytes(128, 64, 8) == P.record_bytes(128, 64, 8) == 4096 + 128
    assert P.record_bytes(128, 64, 16) == 8192


def _bank_ways(addrs, width):
    """Worst bank conflict of one shared-memory load: lanes are served in
    phases of 128 / width lanes; equal addresses broadcast."""
    per, worst = 128 // width, 1
    for ph in range(32 // per):
        banks = {}
        for x in set(addrs[ph * per:(ph + 1) * per]):
            for w in range(width // 4):
                banks.setdefault((x // 4 + w) % 32, set()).add(x // 128)
        worst = max(worst, max(len(v) for v in banks.values()))
    return worst


@pytest.mark.parametrize("dim", [64, 128])
@pytest.mark.parametrize("bits", [4, 8, 16])
def test_v_payload_order_is_line_local_involution_without_bank_conflicts(dim, bits):
    from paged_reference import v_stored
    n = 16 * dim * bits // 8
    o = np.arange(n)
    s = P.v_swizzle(dim, bits, o)
    assert (np.sort(s) == o).all() and (s // 128 == o // 128).all()
    assert (P.v_swizzle(dim, bits, s) == o).all()
    logical = (np.arange(n) * 7 % 251).astype(np.uint8)
    assert v_stored(logical.tobytes(), dim, bits) == logical[s].tobytes()
    # The decode's V fragment loads: lane (g, t) reads token rows 2t, 2t+1,
    # 2t+8, 2t+9 at its dim slice g (dim / 8 dims; 32-byte slices in halves).
    row, slice_bytes = dim * bits // 8, dim // 8 * bits // 8
    width = min(slice_bytes, 16)
    linear, stored = [], []
    for half in range(slice_bytes // width):
        for dr in (0, 1, 8, 9):
            a = [(2 * (ln & 3) + dr) * row + (ln >> 2) * slice_bytes + width * half for ln in range(32)]
            linear.append(_bank_ways(a, width))
            stored.append(_bank_ways(list(P.v_swizzle(dim, bits, a)), width))
    assert max(linear) >= 2 and max(stored) == 1


def test_pooled_v_page_rows_round_trip_through_the_stored_order():
    from anchorkv_b200.packed_decode import QuantizedPage
    from paged_reference import v_stored
    heads, dim = 2, 128
    rec = torch.zeros(heads, 16 * dim * 2 + 48, dtype=torch.uint8)  # strided like a pool record view
    view = rec[:, :16 * dim * 2].view(torch.float16).view(heads, 16, dim)
    page = QuantizedPage(16, view, None, (heads, 16, dim), 64, order=P.v_order(dim, 16, "cpu"))
    rows = torch.randn(heads, 5, dim).half()
    page.write_rows(3, rows)
    page.write_rows(8, rows[:, :2])
    want = torch.zeros(heads, 16, dim, dtype=torch.float16)
    want[:, 3:8], want[:, 8:10] = rows, rows[:, :2]
    assert torch.equal(page.data, want)
    for h in range(heads):
        assert rec[h, :16 * dim * 2].numpy().tobytes() == v_stored(want[h].numpy().tobytes(), dim, 16)
    assert (rec[:, 16 * dim * 2:] == 0).all()


def test_parser_matches_reference_behaviour():
    parser = akv.DeclarativeAttentionParser()
    assert parser.feed("reason <fo") == ()
    focus = parser.feed('cus magic_chunks="2, 3">inspect')
    closing = parser.feed("</focus><local>")
    anchor = parser.feed("<anchor segments='4, 4'>")
    assert focus[0].mode == akv.AttentionMode.FOCUS and focus[0].segment_ids == (2, 3)
    assert closing[0].mode == akv.AttentionMode.GLOBAL and closing[1].mode == akv.AttentionMode.LOCAL
    assert anchor[0].kind == akv.DirectiveKind.ANCHOR and anchor[0].segment_ids == (4,)
    assert parser.state.mode == akv.AttentionMode.LOCAL
    with pytest.raises(ValueError, match="missing a segment list"):
        akv.DeclarativeAttentionParser().feed("<focus>")
    p2 = akv.DeclarativeAttentionParser()
    with pytest.raises(ValueError):
        p2.feed("<archive>")
    assert p2.feed("<global>")[0].mode == akv.AttentionMode.GLOBAL  # bad tag was consumed


@pytest.fixture
def cpu_cache(monkeypatch):
    use_oracle_codec(monkeypatch)
    torch.manual_seed(11)
    cache = akv.DeclarativeKVCache(block_size=4, group_size=16)
    for sid, start, count, role in [(0, 0, 4, akv.SegmentRole.SINK), (1, 4, 6, akv.SegmentRole.CONTEXT),
                                    (2, 10, 6, akv.SegmentRole.CONTEXT), (3, 16, 4, akv.SegmentRole.RESPONSE)]:
        cache.add_segment(sid, torch.randn(1, 2, count, 8), torch.randn(1, 2, count, 8),
                          token_start=start, role=role)
    return cache


def test_block_store_lifecycle_rules(cpu_cache):
    c = cpu_cache
    assert [s["blocks"] for s in c.storage_report()["segments"]] == [1, 2, 2, 1]
    with pytest.raises(ValueError, match="overlap"):
        c.add_segment(9, torch.randn(1, 2, 3, 8), torch.randn(1, 2, 3, 8), token_start=2)
    with pytest.raises(ValueError, match="already registered"):
        c.add_segment(0, torch.randn(1, 2, 3, 8), torch.randn(1, 2, 3, 8), token_start=40)
    before = c.resident_bytes
    c.requantize_segment(1, CacheMode.INT8)
    c.requantize_segment(1, CacheMode.INT4)
    assert c.resident_bytes < before
    with pytest.raises(akv.LossyPromotionError):
        c.requantize_segment(1, CacheMode.INT8)
    c.protect_segment(2)
    with pytest.raises(ValueError, match="protected"):
        c.requantize_segment(2, CacheMode.INT4)
    c.requantize_segment(1, CacheMode.EVICTED)
    assert c.visible_segment_ids() == (0, 2, 3)
    with pytest.raises(RuntimeError, match="no resident"):
        c.materialize_segments([1])
    c.feed_declarations('<focus segments="2">')
    mat = c.materialize_visible(dtype=torch.float32)
    assert mat.positions.tolist() == list(range(0, 4)) + list(range(10, 20))
    report = c.storage_report()
    assert report["attention_mode"] == "focus" and report["visible_segment_ids"] == [0, 2, 3]
    assert [s["mode"] for s in report["segments"]] == ["fp16", "evicted", "fp16", "fp16"]


def test_apply_plan_validates_before_changing_anything(cpu_cache):
    c = cpu_cache
    c.protect_segment(0)
    plan = akv.CachePlan(tuple(akv.PlannedSegment(i, m, 0, 0.0, "t") for i, m in
                               enumerate([CacheMode.INT4, CacheMode.INT4, CacheMode.INT8, CacheMode.FP16])),
                         1, 0, 0)
    with pytest.raises(ValueError, match="protected"):
        c.apply_plan(plan)
    assert [c.segment_mode(i) for i in range(4)] == [CacheMode.FP16] * 4


def test_cpu_tensors_are_refused_by_the_kernels():
    with pytest.raises(ValueError, match="CUDA"):
        akv.quantize_tensor(torch.randn(4, 8), CacheMode.INT8, group_size=16)
    with pytest.raises(ValueError, match="CUDA"):
        akv.pack_page(torch.randn(2, 16, 64), 4)


def test_demotion_into_a_full_pool_changes_nothing(monkeypatch):
    """A PagedLayer over a shared pool with too few archive slots refuses a demotion of
    several pages as a whole: MemoryError before any slot, view or count changes."""
    from anchorkv_b200 import _lib

    monkeypatch.setattr(_lib, "status_ptr", lambda device: 0)  # host stand-ins: no kernel runs here
    monkeypatch.setattr(_lib, "stream_of", lambda device: 0)
    pool = P.PagePool(2, 64, group=64, pages={16: 3, 8: 0, 4: 1}, device="cpu")
    layer = akv.PagedLayer(2, 64, 48, group=64, pool=pool, device="cpu")
    layer._slots = [(16, pool.alloc(16)) for _ in range(3)]  # three complete FP16 pages
    layer.pages = [layer._views(16, off) for _, off in layer._slots]
    layer.length = 48
    slots, free4 = list(layer._slots), pool.free_slots(4)
    with pytest.raises(MemoryError, match="1 free 4-bit slots, 2 requested"):
        layer._demote_many([0, 1], 4)
    assert layer._slots == slots and pool.free_slots(4) == free4 and layer.demotions == 0
    assert all(k.bits == 16 for k, _ in layer.pages)


class _Query:
    """Shape, dtype and device of a query, without a tensor (the checks run before any launch)."""

    def __init__(self, shape, dtype=torch.float16, is_cuda=True):
        self.shape, self.dtype, self.is_cuda = torch.Size(shape), dtype, is_cuda

    def dim(self):
        return len(self.shape)


def test_decode_arguments_are_checked_before_any_launch():
    """decode_partial_states, merge_states and packed_attention refuse what the kernels would
    misread (a query that is not CUDA fp16, states that are not float32), with the reference's
    messages (triton_decode.py:86-94); only the partial-state decode admits a table with no pages."""
    from anchorkv_b200.decode import _check_query

    pool = P.PagePool(2, 64, group=1024, pages={16: 4, 8: 0, 4: 0}, device="cpu")
    table, empty = P.PagedBatch(pool, 2, 3), P.PagedBatch(pool, 2, 0)
    for bad in (torch.zeros(2, 4, 1, 64, dtype=torch.float16), torch.zeros(2, 4, 1, 64)):
        with pytest.raises(ValueError, match="CUDA FP16"):
            akv.decode_partial_states(bad, table, 0.1)
        with pytest.raises(ValueError, match="CUDA FP16"):
            akv.packed_attention(bad, table, 0.1)
    with pytest.raises(ValueError, match="CUDA float32"):
        akv.merge_states(torch.zeros(2, 2, 4, 66))  # a CPU tensor
    with pytest.raises(ValueError, match="CUDA float32"):
        akv.merge_states(torch.zeros(2, 4, 66))  # not [n, batch, heads, D + 2]

    assert _check_query(_Query((2, 4, 1, 64)), table, 0, empty_ok=False) == 2
    assert _check_query(_Query((2, 4, 1, 64)), empty, 0, empty_ok=True) == 2
    with pytest.raises(ValueError, match="nonempty CUDA FP16 cache"):
        _check_query(_Query((2, 4, 1, 64)), empty, 0, empty_ok=False)
    with pytest.raises(ValueError, match="nonempty CUDA FP16 cache"):
        _check_query(_Query((2, 4, 1, 64), dtype=torch.float32), empty, 0, empty_ok=True)
    with pytest.raises(ValueError, match=r"\[batch, heads, 1, head_dim\]"):
        _check_query(_Query((2, 4, 64)), table, 0, empty_ok=True)
    with pytest.raises(ValueError, match=r"\[batch, heads, 1, head_dim\]"):
        _check_query(_Query((1, 4, 1, 64)), table, 0, empty_ok=True)
    with pytest.raises(ValueError, match="divisible by KV heads"):
        _check_query(_Query((2, 3, 1, 64)), table, 0, empty_ok=True)
    with pytest.raises(ValueError, match="non-negative"):
        _check_query(_Query((2, 4, 1, 64)), table, -1, empty_ok=True)


class _HostWord:
    """A status word in plain host memory standing in for the mapped pinned one."""

    def __init__(self, index):
        import ctypes

        self.index = index
        self._buf = ctypes.c_int32(0)

    def data_ptr(self):
        import ctypes

        return ctypes.addressof(self._buf)

    @property
    def value(self):
        return self._buf.value

    def clear(self):
        self._buf.value = 0

    def set(self, bits):
        self._buf.value |= bits


def test_reported_device_errors_raise_on_the_next_call(monkeypatch):
    from anchorkv_b200 import _lib

    word = _HostWord(5)
    monkeypatch.setitem(_lib._status, "fake-device", word)
    assert _lib.status_ptr("fake-device") == word.data_ptr()  # clean: no raise
    word.set(_lib.DEV_BAD_DESCRIPTOR)  # a kernel skipped a bad page
    with pytest.raises(akv.KernelError, match="cuda:5 reported: a page descriptor outside the arena"):
        _lib.status_ptr("fake-device")
    assert word.value == 0  # raising cleared it: the call after runs
    assert _lib.status_ptr("fake-device") == word.data_ptr()
    word.set(_lib.DEV_BAD_DESCRIPTOR | _lib.DEV_TIMEOUT)
    with pytest.raises(akv.KernelError, match="misaligned.*bounded wait"):
        _lib.raise_pending("fake-device")
    assert _lib.describe_status(8).startswith("unknown")


def test_peer_exchange_setup_failure_releases_its_buffers(monkeypatch):
    """A rank that cannot map a peer's exchange buffer unmaps what it mapped and frees
    its own buffer before raising (library and process group replaced by recorders)."""
    from anchorkv_b200 import _lib
    from anchorkv_b200 import sharded as S

    released = []

    class FakeLib:
        def akv_exchange_bytes(self, world, batch, q_heads, dim):
            return 4096

        def akv_ipc_close(self, ptr):
            released.append(("close", ptr.value))
            return 0

        def akv_ipc_free(self, ptr):
            released.append(("free", ptr.value))
            return 0

    opened = []

    def call(name, *args):
        if name == "akv_ipc_alloc":
            args[1]._obj.value = 0x1000  # this rank's buffer
        elif name == "akv_ipc_open":
            if len(opened) == 1:
                raise akv.KernelError("akv_ipc_open: CUDA launch error")
            opened.append(0x2000)
            args[1]._obj.value = 0x2000
        else:
            raise AssertionError(name)

    monkeypatch.setattr(_lib, "load", lambda *a: FakeLib())
    monkeypatch.setattr(_lib, "call", call)
    monkeypatch.setattr(S.dist, "get_world_size", lambda group=None: 3)
    monkeypatch.setattr(S.dist, "get_rank", lambda group=None: 0)
    monkeypatch.setattr(S.dist, "all_gather_object", lambda out, obj, group=None: out.__setitem__(
        slice(None), [obj, b"\1" * 64, b"\2" * 64]))
    monkeypatch.setattr(S.dist, "barrier", lambda group=None: pytest.fail("no barrier after a failed setup"))
    with pytest.raises(akv.KernelError, match="akv_ipc_open"):
        S.PeerExchange(1, 32, 128)
    assert released == [("close", 0x2000), ("free", 0x1000)]


def test_decode_workspaces_are_kept_for_a_bounded_number_of_streams():
    from anchorkv_b200 import decode as D

    cpu = torch.device("cpu")
    saved = dict(D._workspaces)
    D._workspaces.clear()
    try:
        first = D._workspace(cpu, 100, stream=1)
        assert D._workspace(cpu, 100, stream=1) is first  # reused on its stream
        for s in range(2, 2 + 3 * D._MAX_WORKSPACES):
            D._workspace(cpu, 100, stream=s)
        assert len(D._workspaces) == D._MAX_WORKSPACES
        assert (None, 1) not in D._workspaces and (None, 1 + 3 * D._MAX_WORKSPACES) in D._workspaces
        grown = D._workspace(cpu, 1 << 20, stream=1 + 3 * D._MAX_WORKSPACES)  # a larger request replaces it
        assert grown.numel() == 1 << 20 and len(D._workspaces) == D._MAX_WORKSPACES
    finally:
        D._workspaces.clear()
        D._workspaces.update(saved)
