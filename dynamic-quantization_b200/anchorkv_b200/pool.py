"""Physical page storage: one HBM arena, three record size classes, page tables.

A page is 16 tokens of K and V for every KV head of one (sequence, layer).  It
is stored as ``heads`` head records back to back; a head record is
``[K payload][V payload][K scales][V scales][pad to 16 B]`` with the reference
byte layout for the payload (fp16, int8, or two's-complement nibbles with the
even element low, as ``packed_decode.pack_page`` writes them,
packed_decode.py:48-67) and fp16 scales.  K payloads are row-major; V payloads
hold the same bytes with 16-byte units permuted inside each 128-byte line
(:func:`v_swizzle`), the order the decode kernel reads without shared-memory
bank conflicts.  Pages live at 16-byte aligned offsets so one bulk copy moves a
head record from HBM into shared memory.

A page table entry (descriptor) is an int64: mode in bits 0-1 (0 = skip:
evicted or not visible, 1 = INT4, 2 = INT8, 3 = FP16), valid tokens - 1 in
bits 2-5, byte offset in bits 8-63.

:class:`PagePool` owns the arena and hands out page slots per size class.
Allocation is host bookkeeping (a free-list per class); only descriptors and
payloads live on the device.  :class:`PagedBatch` is the page table of a batch
of sequences of one layer over a shared pool, the batched counterpart of the
reference's batch-one ``PagedLayer`` table (packed_decode.py:122-133).
"""

from __future__ import annotations

import numpy as np
import torch

from . import _lib

BLOCK = 16
BITS_TO_MODE = {4: _lib.MODE_INT4, 8: _lib.MODE_INT8, 16: _lib.MODE_FP16}
MODE_TO_BITS = {v: k for k, v in BITS_TO_MODE.items()}


def record_bytes(dim: int, group: int, bits: int) -> int:
    """Bytes of one (page, KV head) record; mirrors akv_record_bytes."""
    payload = BLOCK * dim * bits // 8
    scales = 0 if bits == 16 else BLOCK * dim // group
    return (2 * payload + 4 * scales + 15) // 16 * 16


def v_swizzle(dim: int, bits: int, offsets) -> np.ndarray:
    """Stored byte offset of each row-major byte offset of a V payload, and
    back (the map is an involution); mirrors ``v_swizzle`` in akv_common.cuh.

    The 16-byte units of a V payload are permuted inside each 128-byte line by
    an XOR keyed on the line's token row, so the decode kernel's V fragment
    loads hit distinct shared-memory banks.  K payloads and scales are
    row-major."""
    o = np.asarray(offsets, np.int64)
    row = dim * bits // 8
    if row == 256:
        key = ((o >> 9) & 1) | (((o >> 10) & 1) << 2)
    elif row == 128:
        key = (o >> 7) & 6
    elif row == 64:
        key = (o >> 6) & 6
    elif row == 32:
        key = (o >> 6) & 2
    else:
        raise ValueError(f"no V payload layout for head_dim {dim} at {bits} bits")
    return o ^ (key << 4)


_V_ORDER: dict = {}


def v_order(dim: int, bits: int, device) -> torch.Tensor:
    """int64 index over one V payload's bytes: ``stored[i] == row_major[order[i]]``
    (and ``row_major[i] == stored[order[i]]``)."""
    key = (dim, bits, str(device))
    if key not in _V_ORDER:
        n = BLOCK * dim * bits // 8
        _V_ORDER[key] = torch.from_numpy(v_swizzle(dim, bits, np.arange(n))).to(device)
    return _V_ORDER[key]


def encode(bits: int | None, ntok: int, offset: int) -> int:
    """Descriptor for a page; ``bits=None`` gives a skip entry."""
    if bits is None:
        return 0
    if not 1 <= ntok <= BLOCK or offset % 16:
        raise ValueError("descriptor needs 1..16 valid tokens and a 16-byte aligned offset")
    return (offset << 8) | ((ntok - 1) << 2) | BITS_TO_MODE[bits]


def encode_array(mode_codes: np.ndarray, ntok: np.ndarray, offsets: np.ndarray) -> np.ndarray:
    """Vectorised :func:`encode`; mode code 0 (skip) yields 0."""
    d = (offsets.astype(np.int64) << 8) | ((ntok.astype(np.int64) - 1) << 2) | mode_codes.astype(np.int64)
    return np.where(mode_codes == 0, 0, d)


def decode(desc: int) -> tuple[int | None, int, int]:
    """(bits or None for skip, valid tokens, byte offset)."""
    mode = desc & 3
    return (MODE_TO_BITS.get(mode), ((desc >> 2) & 15) + 1, desc >> 8)


def to_device(array, device) -> torch.Tensor:
    """An int64 host array on ``device`` through pinned memory, without blocking
    the host (torch keeps the pinned block until the copy has run)."""
    return torch.from_numpy(np.ascontiguousarray(array, np.int64)).pin_memory().to(device, non_blocking=True)


def as_fp16_rows(t: torch.Tensor) -> torch.Tensor:
    """``t`` as fp16 with head_dim contiguous, 8-byte aligned rows and strides in
    whole 4-element units (the layout akv_append_rows reads)."""
    t = t.to(torch.float16)
    if t.stride(-1) != 1 or t.data_ptr() % 8 or any(s % 4 for s in t.stride()[:-1]):
        t = t.contiguous()
    return t


def group_ok(dim: int, group: int) -> bool:
    return group in (32, 64, 128, BLOCK * dim)


class PagePool:
    """An arena of page slots in three size classes (FP16 / INT8 / INT4).

    ``pages`` maps bits -> number of slots.  Slots of a class are contiguous;
    ``alloc`` pops from a free list (optionally shuffled, which gives the
    random physical placement of a long-lived shared pool).
    """

    def __init__(self, heads: int, dim: int, *, group: int = 64, pages: dict | None = None,
                 device="cuda", shuffle_seed: int | None = None, zero: bool = True):
        if dim not in (64, 128):
            raise ValueError("supported geometry: head dim 64 or 128")
        if not group_ok(dim, group):
            raise ValueError(f"supported scale groups for head dim {dim}: 32, 64, 128, {BLOCK * dim}")
        self.heads, self.dim, self.group = heads, dim, group
        self.device = torch.device(device)
        pages = dict(pages or {})
        self.page_bytes = {b: heads * record_bytes(dim, group, b) for b in (4, 8, 16)}
        self.base, self.capacity, self._free = {}, {}, {}
        cursor = 0
        rng = np.random.default_rng(shuffle_seed) if shuffle_seed is not None else None
        for bits in (16, 8, 4):
            n = int(pages.get(bits, 0))
            self.base[bits] = cursor
            self.capacity[bits] = n
            slots = np.arange(n, dtype=np.int64)
            if rng is not None:
                rng.shuffle(slots)
            # pop() takes from the end: reverse so slot order is allocation order.
            self._free[bits] = list((cursor + slots * self.page_bytes[bits])[::-1])
            cursor += n * self.page_bytes[bits]
        self.nbytes = max(cursor, 16)
        alloc = torch.zeros if zero else torch.empty
        self.arena = alloc(self.nbytes, dtype=torch.uint8, device=self.device)

    def free_slots(self, bits: int) -> int:
        return len(self._free[bits])

    def alloc(self, bits: int) -> int:
        if not self._free[bits]:
            raise MemoryError(f"page pool has no free {bits}-bit page slots")
        return int(self._free[bits].pop())

    def check_free(self, bits: int, n: int) -> None:
        """Raise MemoryError unless ``n`` slots of ``bits`` are free (nothing changes)."""
        if n > len(self._free[bits]):
            raise MemoryError(f"page pool has {len(self._free[bits])} free {bits}-bit slots, {n} requested")

    def alloc_many(self, bits: int, n: int) -> np.ndarray:
        self.check_free(bits, n)
        if n == 0:
            return np.zeros(0, np.int64)
        out = np.array(self._free[bits][-n:][::-1], dtype=np.int64)
        del self._free[bits][-n:]
        return out

    def free(self, bits: int, offset: int) -> None:
        self._free[bits].append(int(offset))

    def free_many(self, bits: int, offsets) -> None:
        self._free[bits].extend(int(o) for o in np.asarray(offsets).reshape(-1))

    def reserve(self, bits: int, n: int) -> None:
        """Make at least ``n`` slots of ``bits`` free, growing the arena if needed.

        Growth appends a region of new slots (at least doubling the class) and
        copies the old arena into a larger one on the current stream: byte
        offsets, and so descriptors, stay valid, but tensors viewing the old
        arena (``page_view``) do not follow.  Owners that hand out page views
        (``PagedLayer``) never grow their pool."""
        short = n - len(self._free[bits])
        if short <= 0:
            return
        extra = max(short, self.capacity[bits], 64)
        start = self.nbytes
        old = self.arena
        self.nbytes = start + extra * self.page_bytes[bits]
        self.arena = torch.empty(self.nbytes, dtype=torch.uint8, device=self.device)
        self.arena[:start].copy_(old[:start])
        self.arena[start:].zero_()
        new = start + np.arange(extra, dtype=np.int64) * self.page_bytes[bits]
        self._free[bits] = list(new[::-1]) + self._free[bits]  # old free slots are taken first
        self.capacity[bits] += extra

    def page_view(self, offset: int, bits: int) -> torch.Tensor:
        """uint8 view ``[heads, record_bytes]`` of one page."""
        rec = self.page_bytes[bits] // self.heads
        return self.arena[offset:offset + self.page_bytes[bits]].view(self.heads, rec)


class PagedBatch:
    """Page tables of ``batch`` sequences for one layer over a shared pool.

    ``table[b, j]`` is the descriptor of page ``j`` of sequence ``b``;
    ``seq_blocks[b]`` the number of pages sequence ``b`` uses.  Skip entries
    (evicted or invisible pages) are never read by the decode kernel.
    """

    def __init__(self, pool: PagePool, batch: int, max_blocks: int):
        self.pool = pool
        self.batch, self.max_blocks = batch, max_blocks
        self.table = torch.zeros((batch, max_blocks), dtype=torch.int64, device=pool.device)
        self.seq_blocks = torch.full((batch,), max_blocks, dtype=torch.int32, device=pool.device)

    @classmethod
    def over(cls, pool: PagePool, table: torch.Tensor) -> "PagedBatch":
        """A batch over an existing ``[batch, max_blocks]`` descriptor table (a
        view, no allocation); every sequence uses all ``max_blocks`` entries."""
        view = cls.__new__(cls)
        view.pool, view.table, view.seq_blocks = pool, table, None
        view.batch, view.max_blocks = int(table.shape[0]), int(table.shape[1])
        return view

    heads = property(lambda self: self.pool.heads)
    dim = property(lambda self: self.pool.dim)
    group = property(lambda self: self.pool.group)
    block = BLOCK

    def resident_bytes(self) -> int:
        """Payload + scale bytes of the pages this table references (skips excluded)."""
        d = self.table.cpu().numpy().reshape(-1)
        modes = d & 3
        total = 0
        for bits, mode in BITS_TO_MODE.items():
            total += int((modes == mode).sum()) * self.pool.heads * algorithmic_record_bytes(
                self.pool.dim, self.pool.group, bits)
        return total


def algorithmic_record_bytes(dim: int, group: int, bits: int) -> int:
    """Payload + scale bytes of one (page, head) record, without alignment pad."""
    payload = BLOCK * dim * bits // 8
    scales = 0 if bits == 16 else BLOCK * dim // group
    return 2 * payload + 4 * scales


def pack_dense(pool: PagePool, key: torch.Tensor, value: torch.Tensor, block_bits, *,
               visible=None, semantics: str = "tensor", lengths=None) -> PagedBatch:
    """Pack dense fp16 K/V ``[batch, heads, tokens, head_dim]`` into ``pool``.

    ``block_bits[b][j]`` is the precision of block ``j`` of sequence ``b``:
    16, 8 or 4, or 0 for an evicted block (no storage, skipped by decode).
    ``visible`` (same shape, bool): False hides a resident block (kept in the
    pool, skipped by decode), as focus/local visibility does.  ``lengths[b]`` (tokens,
    default all) lets the last block of a sequence be partial.  ``semantics``
    selects the quantizer: ``"tensor"`` = backend.quantize_tensor with
    ``group`` elements per scale (backend.py:183-226), ``"page"`` =
    packed_decode.pack_page (packed_decode.py:48-67).  Returns the batch's
    page table; physical placement follows the pool's free-list order.
    """
    if key.shape != value.shape or key.ndim != 4:
        raise ValueError("key and value must share [batch, heads, tokens, head_dim]")
    batch, heads, tokens, dim = key.shape
    if (heads, dim) != (pool.heads, pool.dim):
        raise ValueError("key/value geometry does not match the page pool")
    _lib.require_cuda(key, "key")
    nblk = -(-tokens // BLOCK)
    bits = np.asarray(block_bits, dtype=np.int64).reshape(batch, nblk)
    if not np.isin(bits, (0, 4, 8, 16)).all():
        raise ValueError("block precision must be 16, 8, 4 or 0 (evicted)")
    lengths = np.full(batch, tokens, np.int64) if lengths is None else np.asarray(lengths, np.int64)
    if (lengths < 0).any() or (lengths > tokens).any():
        raise ValueError("lengths must lie in [0, tokens]")
    padded = nblk * BLOCK
    if padded != tokens or key.dtype != torch.float16 or not key.is_contiguous():
        pad = lambda t: torch.nn.functional.pad(t.half(), (0, 0, 0, padded - tokens)).contiguous()
        key, value = pad(key), pad(value)
    blocks_used = -(-lengths // BLOCK)
    j = np.arange(nblk)[None, :]
    bits = np.where(j < blocks_used[:, None], bits, 0)
    ntok = np.clip(lengths[:, None] - j * BLOCK, 1, BLOCK)
    offsets = np.zeros((batch, nblk), np.int64)
    codes = np.zeros((batch, nblk), np.int64)
    for b_ in BITS_TO_MODE:  # every class checked before any slot is taken
        pool.check_free(b_, int((bits == b_).sum()))
    dev = pool.device
    status, stream = _lib.status_ptr(dev), _lib.stream_of(dev)  # an earlier kernel's error, before any change
    for b_, mode in BITS_TO_MODE.items():
        where = bits == b_
        offsets[where] = pool.alloc_many(b_, int(where.sum()))
        codes[where] = mode
    desc = encode_array(codes, ntok, offsets)
    dst = torch.from_numpy(desc.reshape(-1)).to(dev)
    sem = _lib.SEM_TENSOR if semantics == "tensor" else _lib.SEM_PAGE
    _lib.call("akv_pack_pages", key.data_ptr(), value.data_ptr(), heads * padded * dim, padded * dim,
              nblk, batch * nblk, dst.data_ptr(), pool.arena.data_ptr(), pool.nbytes, heads, dim,
              pool.group, sem, status, stream)
    out = PagedBatch(pool, batch, nblk)
    if visible is not None:
        desc = np.where(np.asarray(visible, bool).reshape(batch, nblk), desc, 0)
    out.table.copy_(torch.from_numpy(desc))
    out.seq_blocks.copy_(torch.from_numpy(blocks_used.astype(np.int32)))
    out.lengths = lengths
    return out
