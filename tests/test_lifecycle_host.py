"""Page lifecycle bookkeeping on the host, against the reference's own PagedLayer on CPU.

Which pages a store demotes, when, and to what precision is host logic: the
kernels only move the bytes.  These tests replay random append patterns
(chunk sizes, recent windows, protected pages, archive precisions) through
the reference's ``PagedLayer`` (packed_decode.py:108-194, installed unmodified
in baseline/_ref, run on CPU) and through this package's ``PagedLayer`` and
batched ``live.PagedKVStore`` with their kernel calls recorded instead of
launched, and compare every page's precision, the demotion count, the length
and the payload bytes.  The bytes themselves are checked against the
reference on the GPU (tests/test_gpu_api.py, tests/test_live_route.py).
"""

import numpy as np
import pytest
import torch

import anchorkv_b200 as akv
from anchorkv_b200 import _lib, live
from anchorkv_b200 import packed_decode as PD
from anchorkv_b200 import pool as P

HEADS, DIM, GROUP = 2, 64, 64


@pytest.fixture
def reference(reference_install):
    from anchorkv import packed_decode

    return packed_decode


@pytest.fixture
def launches(monkeypatch):
    """Record C-ABI calls instead of launching them; keep descriptor arrays on the host."""
    calls = []
    monkeypatch.setattr(_lib, "call", lambda name, *args: calls.append(name))
    monkeypatch.setattr(_lib, "require_cuda", lambda *a, **k: None)
    monkeypatch.setattr(_lib, "status_ptr", lambda device: 0)
    monkeypatch.setattr(_lib, "stream_of", lambda device: 0)

    def host(array, device):
        return torch.from_numpy(np.ascontiguousarray(array, np.int64)).to(device)

    monkeypatch.setattr(P, "to_device", host)
    monkeypatch.setattr(PD, "to_device", host)
    return calls


def _kv(gen, tokens, batch=1):
    shape = (batch, HEADS, tokens, DIM)
    return torch.randn(shape, generator=gen).half(), torch.randn(shape, generator=gen).half()


def _cases(n):
    rng = np.random.default_rng(11)
    for _ in range(n):
        pages = int(rng.integers(3, 12))
        protected = tuple(int(p) for p in rng.choice(pages, size=int(rng.integers(0, 3)), replace=False))
        yield (int(rng.choice([4, 8, 16])), int(rng.integers(0, 4)), protected, pages,
               [int(c) for c in rng.integers(1, 40, size=8)])


@pytest.mark.parametrize("archive_bits,recent,protected,pages,chunks", list(_cases(12)))
def test_paged_layer_demotes_what_the_reference_demotes(reference, launches, archive_bits, recent,
                                                        protected, pages, chunks):
    gen = torch.Generator().manual_seed(pages * 31 + recent)
    max_tokens = 16 * pages
    kw = dict(group=GROUP, archive_bits=archive_bits, protected=protected, recent_pages=recent, device="cpu")
    ref = reference.PagedLayer(HEADS, DIM, max_tokens, **kw)
    ours = akv.PagedLayer(HEADS, DIM, max_tokens, **kw)
    pieces = 0  # one append launch per page a chunk writes into
    for take in chunks:
        take = min(take, max_tokens - ref.length)
        if take == 0:
            break
        pieces += (ref.length + take - 1) // 16 - ref.length // 16 + 1
        k, v = _kv(gen, take)
        ref.append(k, v)
        ours.append(k, v)
        assert ours.length == ref.length
        assert [kp.bits for kp, _ in ours.pages] == [kp.bits for kp, _ in ref.pages]
        assert ours.demotions == ref.demotions
        assert ours.payload_bytes == ref.payload_bytes
    assert launches.count("akv_append_rows") == pieces
    # demotions travel in batches: at most one repack launch per demoted page, none without one
    assert (launches.count("akv_repack_pages") > 0) == (ours.demotions > 0)
    assert launches.count("akv_repack_pages") <= ours.demotions
    # explicit demotion to a precision the layer does not archive to (its own pool grows for it;
    # every page view then reads the new arena) and the lifecycle errors, as the reference raises them
    full = [p for p in range(ref.length // 16) if p not in protected and ref.pages[p][0].bits == 16]
    if full:
        page = full[0]
        ref.demote(page, 8)
        ours.demote(page, 8)
        assert [kp.bits for kp, _ in ours.pages] == [kp.bits for kp, _ in ref.pages]
        arena = ours.pool.arena.untyped_storage().data_ptr()
        assert all(kp.stored.untyped_storage().data_ptr() == arena for kp, _ in ours.pages)
        with pytest.raises(ValueError, match="lossy promotion"):
            ours.demote(page, 16)
        for layer in (ref, ours):
            with pytest.raises(ValueError, match="bits must be 4, 8, or 16"):
                layer.demote(page, 2)
    for page in protected:
        if page < len(ours.pages):
            with pytest.raises(ValueError, match="protected"):
                ours.demote(page, 4)


@pytest.mark.parametrize("archive_bits,recent,protected,prefix,steps",
                         [(4, 2, (), 37, 40), (8, 1, (1,), 64, 20), (4, 0, (0, 2), 5, 50), (16, 2, (), 48, 17)])
def test_batched_store_pages_follow_the_reference_per_sequence(reference, launches, archive_bits, recent,
                                                               protected, prefix, steps):
    """PagedKVStore (prefill packs old pages straight to the archive precision, then one append per
    step) leaves every sequence's pages where the reference's append-then-demote leaves them."""
    batch, layers = 3, 2
    gen = torch.Generator().manual_seed(prefix + steps)
    max_tokens = prefix + steps + 3
    store = live.PagedKVStore(layers, batch, HEADS, DIM, max_tokens, group=GROUP, archive_bits=archive_bits,
                              recent_pages=recent, protected=protected, device="cpu")
    refs = [[reference.PagedLayer(HEADS, DIM, max_tokens, group=GROUP, archive_bits=archive_bits,
                                  protected=protected, recent_pages=recent, device="cpu")
             for _ in range(batch)] for _ in range(layers)]
    for layer in range(layers):
        k, v = _kv(gen, prefix, batch)
        store.prefill(layer, k, v)
        for b in range(batch):
            refs[layer][b].append(k[b:b + 1], v[b:b + 1])
    for _ in range(steps):
        for layer in range(layers):
            k, v = _kv(gen, 1, batch)
            store.append(layer, k, v)
            for b in range(batch):
                refs[layer][b].append(k[b:b + 1], v[b:b + 1])
    for layer in range(layers):
        expected = np.array([[kp.bits for kp, _ in r.pages] for r in refs[layer]])
        np.testing.assert_array_equal(store.bits(layer), expected)
        assert store.lengths[layer] == refs[layer][0].length
    assert store.demotions == sum(r.demotions for rs in refs for r in rs)
    assert store.payload_bytes == sum(r.payload_bytes for rs in refs for r in rs)
    assert launches.count("akv_pack_pages") == layers
    assert launches.count("akv_append_rows") == layers * steps


@pytest.fixture
def pending(launches, monkeypatch):
    """After ``pending.set()``, the status word reports an earlier kernel's error, as
    ``_lib.status_ptr`` does when a finished kernel left a bit."""

    class Pending:
        on = False

        def set(self):
            self.on = True

    flag = Pending()

    def status_ptr(device):
        if flag.on:
            raise akv.KernelError("an earlier kernel on cuda:0 reported: a page descriptor outside the arena")
        return 0

    monkeypatch.setattr(_lib, "status_ptr", status_ptr)
    return flag


def _pool_state(pool):
    return {b: pool.free_slots(b) for b in (16, 8, 4)}, pool.nbytes


def test_a_reported_device_error_leaves_every_store_unchanged(pending):
    """The error an earlier kernel reported is raised before a store changes anything:
    no slot is taken, no page or descriptor moves, no count advances."""
    gen = torch.Generator().manual_seed(2)
    layer = akv.PagedLayer(HEADS, DIM, 160, group=GROUP, archive_bits=4, recent_pages=1, device="cpu")
    layer.append(*_kv(gen, 48))  # whole pages: the next append takes a fresh slot
    before = (layer.length, list(layer._slots), [k.bits for k, _ in layer.pages], layer.demotions,
              _pool_state(layer.pool), layer.table.clone())
    pending.set()
    assert [k.bits for k, _ in layer.pages] == [4, 4, 16]  # pages 0-1 archived, page 2 recent
    for step in (lambda: layer.append(*_kv(gen, 30)), lambda: layer.demote(2, 8),
                 lambda: layer._demote_many([2], 4)):
        with pytest.raises(akv.KernelError, match="reported"):
            step()
        after = (layer.length, list(layer._slots), [k.bits for k, _ in layer.pages], layer.demotions,
                 _pool_state(layer.pool), layer.table.clone())
        assert after[:5] == before[:5] and torch.equal(after[5], before[5])

    pending.on = False
    store = live.PagedKVStore(2, 3, HEADS, DIM, 96, group=GROUP, archive_bits=4, recent_pages=1, device="cpu")
    store.prefill(0, *_kv(gen, 50, batch=3))
    snap = (list(store.lengths), store._desc.copy(), list(store._archived), store.demotions, _pool_state(store.pool))
    pending.set()
    for step in (lambda: store.append(0, *_kv(gen, 1, batch=3)), lambda: store.prefill(1, *_kv(gen, 20, batch=3))):
        with pytest.raises(akv.KernelError, match="reported"):
            step()
        assert (store.lengths, store._archived, store.demotions, _pool_state(store.pool)) == \
            (snap[0], snap[2], snap[3], snap[4])
        np.testing.assert_array_equal(store._desc, snap[1])
    store.lengths[0] += 16  # a page became eligible for the archive: the archive step raises first too
    with pytest.raises(akv.KernelError, match="reported"):
        store._archive(0)
    assert store._archived == snap[2] and _pool_state(store.pool) == snap[4]

    pool = P.PagePool(HEADS, DIM, group=GROUP, pages={16: 4, 8: 4, 4: 4}, device="cpu")
    with pytest.raises(akv.KernelError, match="reported"):
        P.pack_dense(pool, *_kv(gen, 32, batch=2), [[16, 8], [4, 0]], semantics="page")
    assert _pool_state(pool) == ({16: 4, 8: 4, 4: 4}, pool.nbytes)
    pending.on = False
    with pytest.raises(MemoryError, match="2 free 16-bit slots, 3 requested"):
        P.pack_dense(P.PagePool(HEADS, DIM, group=GROUP, pages={16: 2, 8: 4, 4: 0}, device="cpu"),
                     *_kv(gen, 32, batch=2), [[16, 8], [16, 16]], semantics="page")
