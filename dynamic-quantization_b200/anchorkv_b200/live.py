"""Batched Hugging Face decode over the packed store.

The reference decodes one sequence at a time: its ``LiveCache`` holds one
``PagedLayer`` per layer and its attention route calls the packed kernel per
layer (``src/anchorkv/colab_experiment.py:92-148``).  That route runs
unchanged on this package: its ``PagedLayer``, ``dense_attention`` and
``packed_attention`` are drop-ins (see the integration notes), and the tests
run the reference's own route, model gate and controlled-decode harness
(``src/anchorkv/benchmark_suite.py:155-264``) with them substituted.

What is new here is a batch: :class:`PagedKVStore` keeps the pages of
``batch`` sequences for every layer in one shared :class:`PagePool`, one page
table per layer that :func:`packed_attention` reads as a ``PagedBatch``:

* prefill packs every layer's prefix in one ``akv_pack_pages`` launch, pages
  older than the recent window straight to the archive precision (pack_page
  rounding, the same bytes the reference's append-then-demote gives);
* a decode step appends each layer's new K/V rows for all sequences in one
  ``akv_append_rows`` launch, which also advances the pages' valid-token
  counts on the device; a fresh page's descriptors reach the table through
  the same launch (one pinned, non-blocking copy of ``batch`` descriptors);
* when a page leaves the recent window it is demoted for all sequences at
  once (``akv_repack_pages``) and its FP16 slots return to the pool.

:func:`batched_live_cache` wraps the store as a transformers ``DynamicCache``
and :func:`paged_route` registers an attention function that decodes through
it, so a batched ``model(...)`` step runs two kernel launches per layer for
attention (decode, merge) plus one append.

Model code (``transformers``) is imported lazily: it is needed only when a
model runs.
"""

from __future__ import annotations

from contextlib import contextmanager

import numpy as np
import torch

from . import _lib
from . import pool as P
from .decode import packed_attention

# Name the batched attention function is registered under.
ROUTE = "anchorkv_b200_batched"


class PagedKVStore:
    """Pages of ``batch`` sequences for ``layers`` layers over one shared pool.

    Sequences of a batch advance together (one decode token each per step).
    Pages start FP16; a complete page older than the ``recent_pages`` most
    recent ones is demoted to ``archive_bits`` unless its index is in
    ``protected`` (the lifecycle of the reference's PagedLayer,
    packed_decode.py:135-179, for every sequence at once)."""

    def __init__(self, layers: int, batch: int, heads: int, dim: int, max_tokens: int, *, group: int = 64,
                 archive_bits: int = 4, recent_pages: int = 2, protected=(), device="cuda"):
        if archive_bits not in (4, 8, 16):
            raise ValueError("archive_bits must be 4, 8 or 16")
        if dim not in (64, 128) or not P.group_ok(dim, group) or group > dim:
            raise ValueError("supported geometry: head dim 64/128, group 32/64/128 dividing it")
        self.layers, self.batch, self.heads, self.dim, self.group = layers, batch, heads, dim, group
        self.archive_bits, self.recent_pages = archive_bits, recent_pages
        self.protected = frozenset(int(p) for p in protected)
        self.device = torch.device(device)
        self.capacity = -(-max_tokens // P.BLOCK)
        hot = self.capacity if archive_bits == 16 else min(self.capacity, recent_pages + 2 + len(self.protected))
        sizes = {16: layers * batch * hot}
        if archive_bits != 16:
            sizes[archive_bits] = layers * batch * self.capacity
        self.pool = P.PagePool(heads, dim, group=group, pages=sizes, device=self.device, zero=False)
        self.tables = torch.zeros((layers, batch, self.capacity), dtype=torch.int64, device=self.device)
        self._desc = np.zeros((layers, batch, self.capacity), np.int64)  # host mirror of the tables
        self.lengths = [0] * layers
        self._archived = [-1] * layers
        self.demotions = 0

    # ------------------------------------------------------------- writes
    def prefill(self, layer: int, key: torch.Tensor, value: torch.Tensor) -> None:
        """Store a prefix ``[batch, heads, tokens, dim]`` of an empty layer."""
        if self.lengths[layer]:
            raise ValueError("prefill needs an empty layer; decode steps go through append")
        batch, heads, tokens, dim = key.shape
        if (batch, heads, dim) != (self.batch, self.heads, self.dim) or value.shape != key.shape:
            raise ValueError("key/value geometry does not match the store")
        if tokens > self.capacity * P.BLOCK:
            raise ValueError("cache geometry or capacity exceeded")
        _lib.require_cuda(key, "key")
        status, stream = _lib.status_ptr(self.device), _lib.stream_of(self.device)  # raises before any change
        n = -(-tokens // P.BLOCK)
        eligible = tokens // P.BLOCK - self.recent_pages  # complete pages older than the recent window
        bits = np.full(n, 16)
        if self.archive_bits != 16:
            old = np.arange(n) < eligible
            old[list(p for p in self.protected if p < n)] = False
            bits[old] = self.archive_bits
        ntok = np.minimum(P.BLOCK, tokens - P.BLOCK * np.arange(n))
        desc = np.zeros((batch, n), np.int64)
        for b_ in (16, 8, 4):
            cols = np.nonzero(bits == b_)[0]
            if cols.size:
                self.pool.reserve(b_, batch * cols.size)
                offs = self.pool.alloc_many(b_, batch * cols.size).reshape(batch, cols.size)
                desc[:, cols] = P.encode_array(np.full(offs.shape, P.BITS_TO_MODE[b_]),
                                               np.broadcast_to(ntok[cols], offs.shape), offs)
        pad = n * P.BLOCK - tokens
        k = torch.nn.functional.pad(key.half(), (0, 0, 0, pad)).contiguous()
        v = torch.nn.functional.pad(value.half(), (0, 0, 0, pad)).contiguous()
        d = P.to_device(desc.reshape(-1), self.device)
        _lib.call("akv_pack_pages", k.data_ptr(), v.data_ptr(), heads * n * P.BLOCK * dim, n * P.BLOCK * dim, n,
                  batch * n, d.data_ptr(), self.pool.arena.data_ptr(), self.pool.nbytes, heads, dim, self.group,
                  _lib.SEM_PAGE, status, stream)
        self.tables[layer, :, :n].copy_(d.view(batch, n))
        self.demotions += batch * int((bits != 16).sum())  # the reference appends, then demotes, these pages
        self._desc[layer, :, :n] = desc
        self.lengths[layer] = tokens
        self._archived[layer] = max(eligible - 1, -1)

    def append(self, layer: int, key: torch.Tensor, value: torch.Tensor) -> None:
        """Append ``[batch, heads, rows, dim]`` decode-step K/V to every sequence."""
        if key.shape != value.shape or key.shape[0] != self.batch or key.shape[1] != self.heads \
                or key.shape[-1] != self.dim:
            raise ValueError("key/value geometry does not match the store")
        rows = key.shape[2]
        if self.lengths[layer] + rows > self.capacity * P.BLOCK:
            raise ValueError("cache geometry or capacity exceeded")
        key, value = P.as_fp16_rows(key), P.as_fp16_rows(value)
        status, stream = _lib.status_ptr(self.device), _lib.stream_of(self.device)
        done = 0
        while done < rows:
            page, row = divmod(self.lengths[layer], P.BLOCK)
            take = min(P.BLOCK - row, rows - done)
            fresh = None
            if row == 0:  # a new FP16 page for every sequence
                self.pool.reserve(16, self.batch)
                offs = self.pool.alloc_many(16, self.batch)
                new = P.encode_array(np.full(self.batch, _lib.MODE_FP16), np.full(self.batch, take), offs)
                fresh = P.to_device(new, self.device)
                self._desc[layer, :, page] = new
            else:
                self._desc[layer, :, page] = (self._desc[layer, :, page] & ~np.int64(15 << 2)) | ((row + take - 1) << 2)
            k, v = key[:, :, done:done + take], value[:, :, done:done + take]
            tbl = self.tables[layer]
            _lib.call("akv_append_rows", k.data_ptr(), v.data_ptr(), k.stride(0), k.stride(1), k.stride(2),
                      self.batch, take, row, tbl.data_ptr(), tbl.stride(0), page,
                      None if fresh is None else fresh.data_ptr(), self.pool.arena.data_ptr(), self.pool.nbytes,
                      self.heads, self.dim, status, stream)
            self.lengths[layer] += take
            done += take
            self._archive(layer)

    def _archive(self, layer: int) -> None:
        last = self.lengths[layer] // P.BLOCK - self.recent_pages - 1
        pages = [p for p in range(self._archived[layer] + 1, last + 1) if p not in self.protected]
        if self.archive_bits == 16 or not pages:
            self._archived[layer] = max(self._archived[layer], last)
            return
        status, stream = _lib.status_ptr(self.device), _lib.stream_of(self.device)  # raises before any change
        self._archived[layer] = max(self._archived[layer], last)
        src = self._desc[layer][:, pages]  # [batch, n]
        self.pool.reserve(self.archive_bits, src.size)
        offs = self.pool.alloc_many(self.archive_bits, src.size)
        dst = P.encode_array(np.full(src.shape, P.BITS_TO_MODE[self.archive_bits]), ((src >> 2) & 15) + 1,
                             offs.reshape(src.shape))
        s_dev, d_dev = P.to_device(src.reshape(-1), self.device), P.to_device(dst.reshape(-1), self.device)
        _lib.call("akv_repack_pages", s_dev.data_ptr(), d_dev.data_ptr(), src.size, self.pool.arena.data_ptr(),
                  self.pool.nbytes, self.heads, self.dim, self.group, _lib.SEM_PAGE, status, stream)
        self.tables[layer].index_copy_(1, P.to_device(pages, self.device), d_dev.view(src.shape))
        self._desc[layer][:, pages] = dst
        self.pool.free_many(16, src >> 8)  # stream order: later writes to these slots follow the repack
        self.demotions += src.size

    # -------------------------------------------------------------- reads
    def pages(self, layer: int = 0) -> int:
        return -(-self.lengths[layer] // P.BLOCK)

    def batch_view(self, layer: int) -> P.PagedBatch:
        """Layer ``layer``'s page table for :func:`packed_attention` (query ``[batch, Hq, 1, D]``)."""
        return P.PagedBatch.over(self.pool, self.tables[layer, :, :self.pages(layer)])

    def bits(self, layer: int = 0) -> np.ndarray:
        """Precision of every page, ``[batch, pages]``."""
        modes = self._desc[layer, :, :self.pages(layer)] & 3
        return np.vectorize(P.MODE_TO_BITS.get)(modes)

    @property
    def payload_bytes(self) -> int:
        """Payload + scale bytes of every page (QuantizedPage.nbytes of K and V, packed_decode.py:28-32)."""
        total = 0
        for layer in range(self.layers):
            bits = self.bits(layer)
            for b_ in (16, 8, 4):
                per_page = self.heads * (2 * P.BLOCK * self.dim * b_ // 8 +
                                         (0 if b_ == 16 else 4 * P.BLOCK * self.dim // self.group))
                total += int((bits == b_).sum()) * per_page
        return total

    @property
    def resident_bytes(self) -> int:
        """Payload + scales + the page tables (8 bytes per page slot)."""
        return self.payload_bytes + self.tables.numel() * 8

    def dense(self, layer: int) -> tuple[torch.Tensor, torch.Tensor]:
        """fp16 K, V ``[batch, heads, tokens, dim]`` as the pages hold them."""
        n = self.pages(layer)
        desc = self.tables[layer, :, :n].contiguous()
        k = torch.empty((self.heads, self.batch * n * P.BLOCK, self.dim), dtype=torch.float16, device=self.device)
        v = torch.empty_like(k)
        _lib.call("akv_unpack_pages", desc.data_ptr(), self.batch * n, self.pool.arena.data_ptr(), self.pool.nbytes,
                  self.heads, self.dim, self.group, k.data_ptr(), v.data_ptr(), _lib.DTYPE_F16,
                  _lib.status_ptr(self.device), _lib.stream_of(self.device))
        shape = (self.heads, self.batch, n * P.BLOCK, self.dim)
        length = self.lengths[layer]
        return (k.view(shape).transpose(0, 1)[:, :, :length], v.view(shape).transpose(0, 1)[:, :, :length])

    def report(self) -> dict:
        return {"resident_bytes": self.resident_bytes, "payload_bytes": self.payload_bytes,
                "demotions": self.demotions, "tokens": self.lengths[0], "batch": self.batch}


_CACHE_CLASS = None


def batched_live_cache(source, *, max_tokens: int, group: int = 64, archive_bits: int = 4, recent_pages: int = 2,
                       protected=(), device="cuda"):
    """A transformers ``DynamicCache`` over a :class:`PagedKVStore`, prefilled
    from ``source`` = [(key, value)] per layer, each ``[batch, heads, tokens,
    dim]`` (e.g. a stock cache's layers after a batched prefill).  ``update``
    appends the step's keys/values to the store and hands them back unchanged;
    the routed attention (:func:`paged_route`) reads the store."""
    global _CACHE_CLASS
    if _CACHE_CLASS is None:
        from transformers import DynamicCache

        class BatchedLiveCache(DynamicCache):
            def __init__(self, store: PagedKVStore):
                super().__init__()
                self.store = store

            def get_seq_length(self, layer_idx=0):
                return self.store.lengths[layer_idx]

            def update(self, key_states, value_states, layer_idx, cache_kwargs=None):
                self.store.append(layer_idx, key_states, value_states)
                return key_states, value_states

            def report(self):
                return self.store.report()

        _CACHE_CLASS = BatchedLiveCache
    key0 = source[0][0]
    store = PagedKVStore(len(source), key0.shape[0], key0.shape[1], key0.shape[-1], max_tokens, group=group,
                         archive_bits=archive_bits, recent_pages=recent_pages, protected=protected, device=device)
    for layer, (key, value) in enumerate(source):
        store.prefill(layer, key.to(device), value.to(device))
    return _CACHE_CLASS(store)


@contextmanager
def paged_route(model, cache, backend: str = "packed"):
    """Route ``model``'s attention over ``cache``'s pages (one query token per
    sequence) for the duration of the block: ``backend="packed"`` decodes with
    :func:`packed_attention`, ``"dense"`` dequantises the pages and runs SDPA
    (the reference route's two backends, colab_experiment.py:123-148).  On exit
    the model's attention implementation is restored and the registry entry
    points back at SDPA, so it keeps no reference to the cache."""
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS

    if backend not in ("packed", "dense"):
        raise ValueError("backend must be 'packed' or 'dense'")
    sdpa = ALL_ATTENTION_FUNCTIONS["sdpa"]
    store = cache.store

    def attention(module, query, key, value, attention_mask, scaling, **kwargs):
        if query.shape[2] != 1:
            raise ValueError("the paged route decodes one token per sequence; prefill with the stock model")
        if backend == "packed":
            out = packed_attention(query, store.batch_view(module.layer_idx), scaling)
        else:
            k, v = store.dense(module.layer_idx)
            g = query.shape[1] // k.shape[1]
            out = torch.nn.functional.scaled_dot_product_attention(
                query, k.repeat_interleave(g, 1), v.repeat_interleave(g, 1), scale=scaling)
        return out.transpose(1, 2), None

    previous = model.config._attn_implementation
    ALL_ATTENTION_FUNCTIONS.register(ROUTE, attention)
    model.config._attn_implementation = ROUTE
    try:
        yield
    finally:
        model.config._attn_implementation = previous
        ALL_ATTENTION_FUNCTIONS.register(ROUTE, sdpa)


def decode_step(model, cache, tokens: torch.Tensor):
    """One batched decode step: ``tokens`` ``[batch]`` -> last-position logits ``[batch, vocab]``."""
    position = cache.get_seq_length()
    out = model(input_ids=tokens.view(-1, 1), past_key_values=cache,
                cache_position=torch.tensor([position], device=tokens.device),
                attention_mask={"full_attention": None}, use_cache=True, logits_to_keep=1)
    return out.logits[:, -1]
