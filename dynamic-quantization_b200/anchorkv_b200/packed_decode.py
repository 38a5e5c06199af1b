"""Append-only paged KV layer and the page codec, on the GPU.

Drop-in for ``src/anchorkv/packed_decode.py`` (QuantizedPage, pack_page,
PagedLayer, dense_attention): same names, arguments, errors and byte
accounting.  Differences in the physical plane:

* pages live in a :class:`~anchorkv_b200.pool.PagePool` arena (16-byte aligned
  head records) instead of one allocation per page, and the page table holds
  one int64 descriptor per page instead of five host-built pointers, so
  publishing a page is a device-side write with no host->device copy
  (packed_decode.py:126-133 copies five pointers per publish);
* demotion requantizes in a kernel (akv_repack_pages) straight from the old
  record to a new slot; the FP16 slot returns to the pool;
* pages are 16 tokens (the reference allows other sizes for its dense path
  only; its packed kernel also requires 16, triton_decode.py:90).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from . import _lib
from .pool import BLOCK, PagePool, as_fp16_rows, encode, group_ok, record_bytes, to_device, v_order


def tensor_bytes(tensor) -> int:
    return tensor.numel() * tensor.element_size()


class QuantizedPage:
    """One page of K or V: ``[KV heads, 16, head dim]`` as fp16, int8 or packed int4.

    ``data`` is the row-major payload and ``scales`` the fp16 scales, as the
    reference holds them; either may be a view into a page pool (strided
    across heads).  A V page of a pool record stores its payload bytes in the
    decode kernel's swizzled order (:func:`~anchorkv_b200.pool.v_swizzle`):
    ``order`` is then the byte map, ``stored`` the record view, and ``data``
    a row-major copy.  ``nbytes`` counts payload + scales
    (packed_decode.py:28-32)."""

    def __init__(self, bits: int, data: torch.Tensor, scales: torch.Tensor | None, shape: tuple, group: int,
                 *, order: torch.Tensor | None = None):
        self.bits = bits
        self.stored = data
        self.scales = scales
        self.shape = shape
        self.group = group
        self.order = order

    @property
    def data(self) -> torch.Tensor:
        if self.order is None:
            return self.stored
        heads = self.stored.shape[0]
        flat = self.stored.reshape(heads, -1).view(torch.uint8)
        return flat[:, self.order].view(self.stored.dtype).view(self.stored.shape)

    @property
    def nbytes(self) -> int:
        return tensor_bytes(self.stored) + (tensor_bytes(self.scales) if self.scales is not None else 0)

    def write_rows(self, start: int, rows: torch.Tensor) -> None:
        """Store token rows ``[heads, n, dim]`` (fp16 pages) from ``start``."""
        n = rows.shape[1]
        if self.order is None:
            self.stored[:, start:start + n].copy_(rows)
            return
        if self.bits != 16:
            raise ValueError('token rows are written into FP16 pages only')
        rb = self.shape[-1] * 2  # the swizzle keeps every fp16 row inside its own bytes
        src = rows.to(torch.float16).contiguous().view(torch.uint8).reshape(rows.shape[0], n * rb)
        idx = self.order[start * rb:(start + n) * rb] - start * rb
        dst = self.stored.view(torch.uint8).view(self.stored.shape[0], -1)  # a view: writes reach the pool
        dst[:, start * rb:(start + n) * rb] = src[:, idx]

    def dense(self) -> torch.Tensor:
        """fp16 values: ``fp16(int * float(scale))`` (packed_decode.py:34-45)."""
        if self.bits == 16:
            return self.data
        _lib.require_cuda(self.stored, "page payload")
        payload = self.data.contiguous()
        scales = self.scales.contiguous()
        out = torch.empty(self.shape, dtype=torch.float16, device=payload.device)
        _lib.call("akv_dequantize", payload.data_ptr(), scales.data_ptr(), out.numel(), self.group,
                  self.bits, out.data_ptr(), _lib.DTYPE_F16, _lib.stream_of(out.device))
        return out


def pack_page(tensor: torch.Tensor, bits: int = 4, group: int = 64) -> QuantizedPage:
    """Quantize ``[KV heads, page tokens, head dim]`` (packed_decode.py:48-67).

    The source is rounded to fp16, groups run along the last dimension, scales
    are ``fp16(max(amax/qmax, 2^-14))`` and values are divided by that fp16
    scale; bit-exact with the reference (kernel: akv_quantize, page semantics).
    """
    if bits not in (4, 8, 16):
        raise ValueError('bits must be 4, 8, or 16')
    if tensor.ndim != 3 or tensor.shape[-1] % group or group % 2:
        raise ValueError('expected [KV heads, page tokens, head dim], with even groups')
    source = tensor.detach().half().contiguous()
    if bits == 16:
        return QuantizedPage(bits, source.clone(), None, tuple(source.shape), group)
    _lib.require_cuda(source, "page")
    n = source.numel()
    h, t, d = source.shape
    payload = torch.empty(n if bits == 8 else n // 2, dtype=torch.int8 if bits == 8 else torch.uint8,
                          device=source.device)
    scales = torch.empty(n // group, dtype=torch.float16, device=source.device)
    _lib.call("akv_quantize", source.data_ptr(), _lib.DTYPE_F16, n, group, bits, _lib.SEM_PAGE,
              payload.data_ptr(), scales.data_ptr(), _lib.stream_of(source.device))
    data = payload.view(h, t, d if bits == 8 else d // 2)
    return QuantizedPage(bits, data, scales.view(h, t, d // group), tuple(source.shape), group)


class PagedLayer:
    """Append-only, batch-one KV pages of one layer (packed_decode.py:108-194).

    Pages start FP16; complete pages older than ``recent_pages`` are demoted to
    ``archive_bits`` unless protected.  ``table`` is a device int64 descriptor
    per page slot, read directly by :func:`anchorkv_b200.packed_attention`.
    """

    def __init__(self, heads, dim, max_tokens, *, block=16, group=64, archive_bits=4,
                 protected=(), recent_pages=2, device='cuda', pool: PagePool | None = None):
        if dim % group or archive_bits not in (4, 8, 16):
            raise ValueError('invalid quantization geometry')
        if block != BLOCK:
            raise ValueError('anchorkv_b200 pages hold 16 tokens (block=16)')
        if dim not in (64, 128) or not group_ok(dim, group):
            raise ValueError('supported geometry: head dim 64/128, group 32/64/128')
        self.heads, self.dim, self.block, self.group = heads, dim, block, group
        self.archive_bits = archive_bits
        self.protected = frozenset(protected)
        self.recent_pages = recent_pages
        self.capacity = math.ceil(max_tokens / block)
        self.device = torch.device(device)
        self._own_pool = pool is None  # a pool of its own may grow; a shared one is the caller's to size
        if pool is None:
            sizes = {16: self.capacity}
            if archive_bits != 16:
                sizes[archive_bits] = self.capacity
            pool = PagePool(heads, dim, group=group, pages=sizes, device=self.device)
        elif (pool.heads, pool.dim, pool.group) != (heads, dim, group):
            raise ValueError('page pool geometry does not match the layer')
        self.pool = pool
        self.pages = []
        self.length = 0
        self.demotions = 0
        self.table = torch.zeros(self.capacity, dtype=torch.int64, device=self.device)
        self.archived_through = -1
        self._slots = []  # (bits, byte offset) per page

    # -------------------------------------------------------------- internals
    def _views(self, bits: int, offset: int):
        """QuantizedPage views (K, V) of the page record at ``offset``."""
        rec = self.pool.page_view(offset, bits)
        pb = BLOCK * self.dim * bits // 8
        shape = (self.heads, BLOCK, self.dim)
        out = []
        for kv in range(2):
            raw = rec[:, kv * pb:(kv + 1) * pb]
            if bits == 16:
                data = raw.view(torch.float16).view(self.heads, BLOCK, self.dim)
                scales = None
            else:
                dtype = torch.int8 if bits == 8 else torch.uint8
                data = raw.view(dtype).view(self.heads, BLOCK, self.dim * bits // 8)
                ns = BLOCK * self.dim // self.group
                sraw = rec[:, 2 * pb + kv * 2 * ns:2 * pb + (kv + 1) * 2 * ns]
                scales = sraw.view(torch.float16).view(self.heads, BLOCK, self.dim // self.group)
            order = v_order(self.dim, bits, data.device) if kv == 1 else None
            out.append(QuantizedPage(bits, data, scales, shape, self.group, order=order))
        return tuple(out)

    # ------------------------------------------------------------------ API
    def append(self, key, value):
        if key.shape != value.shape or key.ndim != 4 or key.shape[:2] != (1, self.heads):
            raise ValueError('only batch-one matching K/V tensors are supported')
        if key.shape[-1] != self.dim or self.length + key.shape[-2] > self.capacity * self.block:
            raise ValueError('cache geometry or capacity exceeded')
        _lib.require_cuda(key, "key")
        key, value = as_fp16_rows(key), as_fp16_rows(value)
        dev = self.device
        # an error an earlier kernel reported is raised here, before any page changes
        status, stream = _lib.status_ptr(dev), _lib.stream_of(dev)
        offset = 0
        while offset < key.shape[-2]:
            page, position = divmod(self.length, self.block)
            take = min(self.block - position, key.shape[-2] - offset)
            fresh = None
            if position == 0:  # a new FP16 page: its descriptor reaches the table in the append launch
                slot = self.pool.alloc(16)
                self._slots.append((16, slot))
                self.pages.append(self._views(16, slot))
                fresh = to_device([encode(16, take, slot)], dev)
            k, v = key[:, :, offset:offset + take], value[:, :, offset:offset + take]
            # one launch writes the rows (V in the stored byte order), zeroes the
            # rest of a fresh page and moves the page's valid-token count
            _lib.call("akv_append_rows", k.data_ptr(), v.data_ptr(), k.stride(0), k.stride(1), k.stride(2), 1,
                      take, position, self.table.data_ptr(), self.capacity, page,
                      None if fresh is None else fresh.data_ptr(), self.pool.arena.data_ptr(), self.pool.nbytes,
                      self.heads, self.dim, status, stream)
            self.length += take
            offset += take
            self._archive_old_pages()

    def _archive_old_pages(self):
        # Complete pages only; the partial append page always stays FP16.
        last_eligible = self.length // self.block - self.recent_pages - 1
        todo = [page for page in range(self.archived_through + 1, last_eligible + 1)
                if page not in self.protected and self.archive_bits != 16]
        self._demote_many(todo, self.archive_bits)
        self.archived_through = max(self.archived_through, last_eligible)

    def demote(self, page, bits):
        key, _ = self.pages[page]
        if bits > key.bits:
            raise ValueError('lossy promotion cannot restore FP16 values')
        if page in self.protected and bits != 16:
            raise ValueError('cannot demote a protected page')
        if bits not in (4, 8, 16):
            raise ValueError('bits must be 4, 8, or 16')
        if bits != key.bits:
            self._demote_many([page], bits)

    def _demote_many(self, pages, bits):
        pages = [p for p in pages if self._slots[p][0] != bits]
        if not pages:
            return
        dev = self.device
        status, stream = _lib.status_ptr(dev), _lib.stream_of(dev)  # an earlier kernel's error, before any change
        if self._own_pool and self.pool.free_slots(bits) < len(pages):
            # a precision this layer's pool has too few slots of (a manual demotion
            # to a class other than archive_bits): grow it, which moves the arena,
            # so every page view is rebuilt
            self.pool.reserve(bits, len(pages))
            self.pages = [self._views(*slot) for slot in self._slots]
        self.pool.check_free(bits, len(pages))  # a shared pool can run out: raises before any page changes
        src, dst = [], []
        for page, new in zip(pages, self.pool.alloc_many(bits, len(pages))):
            old_bits, old = self._slots[page]
            new = int(new)
            ntok = min(BLOCK, self.length - page * BLOCK)
            src.append(encode(old_bits, ntok, old))
            dst.append(encode(bits, ntok, new))
            self._slots[page] = (bits, new)
        src_t, dst_t = to_device(src, dev), to_device(dst, dev)  # pinned, non-blocking: no host stall
        _lib.call("akv_repack_pages", src_t.data_ptr(), dst_t.data_ptr(), len(pages),
                  self.pool.arena.data_ptr(), self.pool.nbytes, self.heads, self.dim, self.group,
                  _lib.SEM_PAGE, status, stream)
        for page, d in zip(pages, src):
            old_bits = {1: 4, 2: 8, 3: 16}[d & 3]
            self.pool.free(old_bits, d >> 8)  # stream order: later writes follow the repack
            self.pages[page] = self._views(*self._slots[page])
            self.demotions += 1
        # the new descriptors, written on the device after the repack (no host-built index)
        self.table.index_copy_(0, to_device(pages, dev), dst_t)

    def protect(self, page):
        if page < len(self.pages) and self.pages[page][0].bits != 16:
            raise ValueError('anchor must be declared before demotion')
        self.protected = self.protected | {page}

    @property
    def payload_bytes(self):
        return sum(k.nbytes + v.nbytes for k, v in self.pages)

    @property
    def resident_bytes(self):
        """Payload + scales + this layer's page table (8 bytes per page slot)."""
        return self.payload_bytes + tensor_bytes(self.table)

    def dense(self):
        if not self.pages:
            raise ValueError('cache is empty')
        n = len(self.pages)
        desc = self.table[:n].contiguous()
        k = torch.empty((self.heads, n * BLOCK, self.dim), dtype=torch.float16, device=self.device)
        v = torch.empty_like(k)
        _lib.call("akv_unpack_pages", desc.data_ptr(), n, self.pool.arena.data_ptr(), self.pool.nbytes,
                  self.heads, self.dim, self.group, k.data_ptr(), v.data_ptr(), _lib.DTYPE_F16,
                  _lib.status_ptr(self.device), _lib.stream_of(self.device))
        return k[:, :self.length].unsqueeze(0), v[:, :self.length].unsqueeze(0)


def dense_attention(query, layer, scale):
    """Dequantise every page, then SDPA with GQA by repetition (packed_decode.py:197-203)."""
    key, value = layer.dense()
    repeats = query.shape[1] // key.shape[1]
    return F.scaled_dot_product_attention(
        query, key.repeat_interleave(repeats, 1), value.repeat_interleave(repeats, 1),
        is_causal=False, scale=scale,
    )


def kl_divergence(reference, candidate):
    """Per-row KL(reference || candidate) of logits (packed_decode.py:206-209)."""
    p = reference.float().log_softmax(-1)
    q = candidate.float().log_softmax(-1)
    return (p.exp() * (p - q)).sum(-1).clamp_min(0)
