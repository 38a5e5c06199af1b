"""Declarative block store and the flat-tensor codec, with a GPU data plane.

Drop-in for ``src/anchorkv/backend.py``: the same classes, method names,
arguments, lifecycle rules, error types and messages, and byte accounting.
The physical plane is this package's own:

* **Paged segments.**  A segment whose blocks fit the decode kernel's page
  format (16-token blocks, head_dim 64 or 128, scale groups of 32/64/128
  elements or one per block and KV head, fp16 values on a CUDA device) keeps
  each block as one page per (layer, sequence) row in a :class:`PagePool`
  owned by the store.  ``requantize_segment`` is one ``akv_repack_pages``
  launch over all of the segment's pages (quantize_tensor rounding, bit-exact
  with the reference's dequantise-then-quantize loop, backend.py:470-483), and
  eviction returns the pages to the pool.
* **Visibility in the page table.**  The store keeps one int64 descriptor per
  (row, block); the focus/local/global state and eviction are compiled into a
  device page table in which hidden or evicted blocks are skip entries, so
  :func:`anchorkv_b200.packed_attention` attends the store directly
  (``store.decode_view(layer)``) without materialising anything.
  ``materialize_visible`` / ``materialize_segments`` remain the dense API and
  read the pages back in one ``akv_unpack_pages`` launch.
* **Other geometries** (block sizes other than 16, other head dims or groups,
  fp32/bf16 values, a partial block that a scale group would straddle) keep a
  segment's blocks as :class:`PackedTensor` chunks, several blocks stacked per
  chunk when no quantization group straddles two blocks, so a requantize is one
  dequantize and one quantize launch per chunk.  They are stored and
  materialised exactly, but the decode kernel cannot read them.

Quantization and dequantization of flat tensors run in CUDA kernels behind the
C ABI (akv_quantize / akv_dequantize), bit-exact with the reference's torch ops
(backend.py:154-226).  Tensors to quantize must live on a CUDA device; there is
no CPU compute path.
"""

from __future__ import annotations

import math
import re
from dataclasses import dataclass, field
from enum import Enum
from typing import Any, Iterable

import numpy as np
import torch

from . import _lib
from . import pool as P
from .policy import PRECISION_RANK, CacheMode, CachePlan, as_mode


class BackendUnavailableError(RuntimeError):
    """A dependency of the data plane (torch, the CUDA library or a device) is missing."""


class LossyPromotionError(RuntimeError):
    """A segment was asked to move to a higher precision than it holds: its
    quantized values cannot give back the bits they dropped."""


class SegmentRole(str, Enum):
    SINK = "sink"
    SCAFFOLD = "scaffold"
    CONTEXT = "context"
    RESPONSE = "response"


class AttentionMode(str, Enum):
    GLOBAL = "global"
    FOCUS = "focus"
    LOCAL = "local"


class DirectiveKind(str, Enum):
    MODE = "mode"
    ANCHOR = "anchor"
    ARCHIVE = "archive"


# Roles every attention mode keeps visible (backend.py:530-547).
ALWAYS_VISIBLE = frozenset({SegmentRole.SINK, SegmentRole.SCAFFOLD, SegmentRole.RESPONSE})


@dataclass(frozen=True, slots=True)
class CacheDirective:
    kind: DirectiveKind
    mode: AttentionMode | None = None
    segment_ids: tuple[int, ...] = ()


@dataclass(slots=True)
class DeclarativeState:
    mode: AttentionMode = AttentionMode.GLOBAL
    focus_segment_ids: tuple[int, ...] = ()


# ------------------------------------------------------------------ parser
_TAG = re.compile(r"<([^>]*)>")
_IDS = re.compile(r'(?:segments|magic_chunks)\s*=\s*["\']([0-9,\s]+)["\']', re.IGNORECASE)
# Tag name -> the attention mode it switches to (tags that take no segment list).
_MODE_TAGS = {"global": AttentionMode.GLOBAL, "/focus": AttentionMode.GLOBAL, "/local": AttentionMode.GLOBAL,
              "local": AttentionMode.LOCAL}
# Tag prefix -> directive kind (tags that carry a segment list).
_LIST_TAGS = (("focus", DirectiveKind.MODE), ("anchor", DirectiveKind.ANCHOR), ("archive", DirectiveKind.ARCHIVE))


def _id_list(tag: str) -> tuple[int, ...]:
    found = _IDS.search(tag)
    if found is None:
        raise ValueError(f"declarative tag is missing a segment list: <{tag}>")
    ids = tuple(dict.fromkeys(int(part) for part in found.group(1).split(",")))
    if not ids or min(ids) < 0:
        raise ValueError("segment IDs must be non-negative")
    return ids


@dataclass(slots=True)
class DeclarativeAttentionParser:
    """Streaming reader of ``<focus segments="...">``, ``<local>``, ``<global>``,
    ``</focus>``, ``<anchor ...>`` and ``<archive ...>`` tags (the grammar of
    backend.py:64-135).  Text arrives in arbitrary chunks: complete tags are
    matched in the buffered text, text outside tags is dropped, and an
    unfinished tag waits in the buffer for its ``>``.  Unknown tags are
    consumed silently."""

    state: DeclarativeState = field(default_factory=DeclarativeState)
    _pending: str = field(default="", init=False, repr=False)

    def feed(self, text: str) -> tuple[CacheDirective, ...]:
        buffered = self._pending + text
        out: list[CacheDirective] = []
        end = 0
        for match in _TAG.finditer(buffered):
            end = match.end()
            self._pending = buffered[end:]  # a tag that raises is consumed all the same
            directive = self._directive(match.group(1).strip())
            if directive is not None:
                out.append(directive)
        rest = buffered[end:]
        opened = rest.find("<")
        self._pending = rest[opened:] if opened >= 0 else ""
        return tuple(out)

    def _directive(self, tag: str) -> CacheDirective | None:
        name = tag.lower()
        if name in _MODE_TAGS:
            mode = _MODE_TAGS[name]
            self.state.mode, self.state.focus_segment_ids = mode, ()
            return CacheDirective(DirectiveKind.MODE, mode=mode)
        for prefix, kind in _LIST_TAGS:
            if name.startswith(prefix):
                ids = _id_list(tag)
                if kind is not DirectiveKind.MODE:
                    return CacheDirective(kind, segment_ids=ids)
                self.state.mode, self.state.focus_segment_ids = AttentionMode.FOCUS, ids
                return CacheDirective(kind, mode=AttentionMode.FOCUS, segment_ids=ids)
        return None


# ------------------------------------------------------------------- codec
_KERNEL_DTYPES = {torch.float32: _lib.DTYPE_F32, torch.float16: _lib.DTYPE_F16,
                  torch.bfloat16: _lib.DTYPE_BF16}


@dataclass(frozen=True, slots=True)
class PackedTensor:
    """One tensor in a cache representation: fp16 values, or int8 / two-per-byte
    int4 payload with one fp16 absmax scale per group of ``group_size``
    elements (EVICTED keeps no payload)."""

    mode: CacheMode
    shape: tuple[int, ...]
    original_dtype: Any
    payload: Any | None
    scales: Any | None
    group_size: int
    original_numel: int

    @property
    def stored_bytes(self) -> int:
        return _tensor_bytes(self.payload) + _tensor_bytes(self.scales)

    def dequantize(self, *, dtype: Any | None = None, device: Any | None = None) -> Any:
        """``int * float32(scale)`` cast to ``dtype`` (default: the original dtype)."""
        if self.mode is CacheMode.EVICTED or self.payload is None:
            raise RuntimeError("evicted tensors cannot be materialized")
        out_dtype = self.original_dtype if dtype is None else dtype
        payload = self.payload if device is None else self.payload.to(device)
        if self.mode is CacheMode.FP16:
            return payload.to(dtype=out_dtype).reshape(self.shape)
        if self.scales is None:
            raise RuntimeError("quantized tensor is missing scales")
        scales = self.scales if device is None else self.scales.to(device)
        _lib.require_cuda(payload, "payload")
        kernel_dtype = out_dtype if out_dtype in _KERNEL_DTYPES else torch.float32
        out = torch.empty(self.original_numel, dtype=kernel_dtype, device=payload.device)
        bits = 8 if self.mode is CacheMode.INT8 else 4
        _lib.call("akv_dequantize", payload.data_ptr(), scales.data_ptr(), self.original_numel,
                  self.group_size, bits, out.data_ptr(), _KERNEL_DTYPES[kernel_dtype],
                  _lib.stream_of(payload.device))
        return out.reshape(self.shape).to(out_dtype)


def quantize_tensor(tensor: Any, mode: CacheMode, *, group_size: int = 64) -> PackedTensor:
    """Store a floating tensor in a cache representation (backend.py:183-226)."""
    if not isinstance(tensor, torch.Tensor) or not tensor.is_floating_point():
        raise TypeError("tensor must be a floating-point torch.Tensor")
    mode = as_mode(mode)
    if group_size <= 0:
        raise ValueError("group_size must be positive")
    if mode is CacheMode.INT4 and group_size % 2:
        raise ValueError("INT4 group_size must be even")
    source = tensor.detach().contiguous()
    shape = tuple(int(v) for v in source.shape)
    numel = int(source.numel())
    if numel == 0:
        raise ValueError("tensor must not be empty")
    if mode is CacheMode.EVICTED:
        return PackedTensor(mode, shape, source.dtype, None, None, group_size, numel)
    if mode is CacheMode.FP16:
        payload = source.to(torch.float16).contiguous()
        return PackedTensor(mode, shape, source.dtype, payload, None, group_size, numel)
    _lib.require_cuda(source)
    src = source if source.dtype in _KERNEL_DTYPES else source.to(torch.float32)
    groups = -(-numel // group_size)
    padded = groups * group_size
    bits = 8 if mode is CacheMode.INT8 else 4
    payload = torch.empty(padded if bits == 8 else padded // 2,
                          dtype=torch.int8 if bits == 8 else torch.uint8, device=src.device)
    scales = torch.empty(groups, dtype=torch.float16, device=src.device)
    _lib.call("akv_quantize", src.data_ptr(), _KERNEL_DTYPES[src.dtype], numel, group_size, bits,
              _lib.SEM_TENSOR, payload.data_ptr(), scales.data_ptr(), _lib.stream_of(src.device))
    return PackedTensor(mode, shape, source.dtype, payload, scales, group_size, numel)


def stack_legacy_cache(past_key_values: Any) -> tuple[Any, Any]:
    """Layer-first ``(key, value)`` tensors ``[layers, batch, heads, tokens, head_dim]``
    from a Hugging Face cache or its legacy tuple of per-layer pairs."""
    if hasattr(past_key_values, "to_legacy_cache"):
        past_key_values = past_key_values.to_legacy_cache()
    pairs = list(past_key_values)
    if not pairs:
        raise ValueError("past_key_values must contain at least one layer")
    if any(len(pair) != 2 for pair in pairs):
        raise ValueError("each legacy cache layer must contain one key and one value tensor")
    shape = pairs[0][0].shape
    if any(t.shape != shape for pair in pairs for t in pair):
        raise ValueError("all legacy cache tensors must share one shape")
    keys, values = zip(*pairs)
    return torch.stack(keys), torch.stack(values)


# ------------------------------------------------------------- block store
@dataclass(frozen=True, slots=True)
class KVBlock:
    """One block's key and value as :class:`PackedTensor` (the reference's block
    record, backend.py:253-281); the paged store keeps its blocks as page
    records instead and does not build these."""

    block_id: int
    segment_id: int
    token_start: int
    token_end: int
    key: PackedTensor
    value: PackedTensor

    @property
    def mode(self) -> CacheMode:
        if self.key.mode is not self.value.mode:
            raise RuntimeError("key and value cache modes diverged")
        return self.key.mode

    @property
    def stored_bytes(self) -> int:
        return self.key.stored_bytes + self.value.stored_bytes

    def materialize(self, *, dtype: Any | None = None, device: Any | None = None) -> tuple[Any, Any]:
        return (self.key.dequantize(dtype=dtype, device=device),
                self.value.dequantize(dtype=dtype, device=device))


@dataclass(frozen=True, slots=True)
class SegmentRecord:
    segment_id: int
    role: SegmentRole
    token_start: int
    token_end: int
    protected: bool = False


@dataclass(frozen=True, slots=True)
class MaterializedCache:
    key: Any
    value: Any
    positions: Any
    block_ids: tuple[int, ...]
    segment_ids: tuple[int, ...]

    def to_legacy_cache(self) -> tuple[tuple[Any, Any], ...]:
        """Per-layer ``(key, value)`` pairs of ``[layers, batch, heads, tokens, head_dim]`` tensors."""
        if self.key.ndim != 5 or self.value.ndim != 5:
            raise ValueError(
                "legacy conversion requires [layers, batch, heads, tokens, head_dim] tensors")
        return tuple(zip(self.key.unbind(0), self.value.unbind(0)))


def _stored_bytes(numel: int, mode: CacheMode, group: int) -> int:
    """Bytes the reference stores for one K (or V) tensor of ``numel`` elements
    (PackedTensor.stored_bytes of quantize_tensor's output, backend.py:150-152)."""
    if mode is CacheMode.EVICTED:
        return 0
    if mode is CacheMode.FP16:
        return 2 * numel
    groups = -(-numel // group)
    payload = groups * group if mode is CacheMode.INT8 else groups * group // 2
    return payload + 2 * groups


_BITS = {CacheMode.FP16: 16, CacheMode.INT8: 8, CacheMode.INT4: 4}


@dataclass(slots=True)
class _Chunk:
    """Blocks ``first .. first + count - 1`` of a flat segment, stacked along a new
    leading dim when ``count > 1`` (no quantization group straddles two blocks)."""

    first: int
    count: int
    key: PackedTensor
    value: PackedTensor


@dataclass(slots=True)
class _Segment:
    record: SegmentRecord
    mode: CacheMode
    dtype: Any
    lead: tuple[int, ...]            # leading dims of the segment's tensors (..., heads)
    dim: int
    lengths: list[int]               # tokens per block
    block_ids: list[int]
    columns: list[int] | None = None  # paged: page-table column of each block
    chunks: list[_Chunk] | None = None  # flat: the blocks' PackedTensor chunks

    @property
    def paged(self) -> bool:
        return self.columns is not None

    def numel(self, block: int) -> int:
        return math.prod(self.lead) * self.lengths[block] * self.dim


class DeclarativeKVCache:
    """Quantized KV blocks under declarative visibility/precision state
    (backend.py:314-601).  Segments are split into ``block_size``-token blocks
    stored FP16 on insert; a segment moves down the lifecycle FP16 -> INT8 ->
    INT4 -> EVICTED, never back up.

    Segments in the decode kernel's page format live as pages of a store-owned
    :class:`PagePool` (see the module docstring); :meth:`decode_view` is the
    page table of one layer with the current visibility compiled in, which
    :func:`anchorkv_b200.packed_attention` accepts (the store itself when it
    has one layer)."""

    __slots__ = ("block_size", "group_size", "archive_mode", "parser", "_segments", "_next_block_id",
                 "_pool", "_table_geometry", "_descriptors", "_columns", "_table_version", "_device_table")

    def __init__(self, block_size: int = 16, group_size: int = 64, archive_mode: CacheMode = CacheMode.INT4,
                 parser: DeclarativeAttentionParser | None = None):
        if block_size <= 0 or group_size <= 0:
            raise ValueError("block_size and group_size must be positive")
        archive_mode = as_mode(archive_mode)
        if archive_mode not in (CacheMode.INT4, CacheMode.INT8):
            raise ValueError("archive_mode must be INT4 or INT8")
        self.block_size, self.group_size, self.archive_mode = block_size, group_size, archive_mode
        self.parser = parser if parser is not None else DeclarativeAttentionParser()
        self._segments: dict[int, _Segment] = {}
        self._next_block_id = 0
        self._pool: P.PagePool | None = None
        self._table_geometry: tuple | None = None  # (lead, dim, device) of the paged segments
        self._descriptors = np.zeros((0, 0), np.int64)  # [rows, columns] resident descriptors
        self._columns = 0
        self._table_version = 0
        self._device_table = None  # (key, device tensor [rows, columns]) of the last visible table

    # ------------------------------------------------------------ accounting
    @property
    def resident_bytes(self) -> int:
        return sum(self._segment_bytes(seg) for seg in self._segments.values())

    @property
    def full_precision_bytes(self) -> int:
        return sum(4 * seg.numel(b) for seg in self._segments.values() for b in range(len(seg.lengths)))

    @property
    def compression_ratio(self) -> float:
        return self.full_precision_bytes / max(self.resident_bytes, 1)

    def _segment_bytes(self, seg: _Segment) -> int:
        return sum(2 * _stored_bytes(seg.numel(b), seg.mode, self.group_size) for b in range(len(seg.lengths)))

    # --------------------------------------------------------------- writes
    def add_segment(self, segment_id: int, key: Any, value: Any, *, token_start: int,
                    role: SegmentRole = SegmentRole.CONTEXT, protected: bool = False) -> SegmentRecord:
        if segment_id in self._segments:
            raise ValueError(f"segment {segment_id} is already registered")
        if token_start < 0:
            raise ValueError("token_start must be non-negative")
        if not isinstance(key, torch.Tensor) or not isinstance(value, torch.Tensor):
            raise TypeError("key and value must be torch tensors")
        if key.shape != value.shape or key.ndim not in (4, 5):
            raise ValueError("key and value must share [batch, heads, tokens, head_dim] or "
                             "[layers, batch, heads, tokens, head_dim] shape")
        count = int(key.shape[-2])
        if count <= 0:
            raise ValueError("segments must contain at least one token")
        token_end = token_start + count
        for other in self._segments.values():
            if token_start < other.record.token_end and other.record.token_start < token_end:
                raise ValueError("segment token ranges must not overlap")
        record = SegmentRecord(segment_id, SegmentRole(role), token_start, token_end, protected)
        lengths = [min(self.block_size, count - lo) for lo in range(0, count, self.block_size)]
        seg = _Segment(record, CacheMode.FP16, key.dtype, tuple(int(d) for d in key.shape[:-2]),
                       int(key.shape[-1]), lengths,
                       list(range(self._next_block_id, self._next_block_id + len(lengths))))
        if self._pageable(seg, key):
            self._add_pages(seg, key.detach(), value.detach())
        else:
            self._add_flat(seg, key.detach(), value.detach())
        self._next_block_id += len(lengths)
        self._segments[segment_id] = seg
        return record

    def segment_mode(self, segment_id: int) -> CacheMode:
        return self._get(segment_id).mode

    def storage_report(self) -> dict[str, object]:
        """JSON-safe physical storage and state-machine statistics."""
        rows = []
        for seg in sorted(self._segments.values(), key=lambda s: s.record.token_start):
            rec = seg.record
            rows.append({"segment_id": rec.segment_id, "role": rec.role.value, "token_start": rec.token_start,
                         "token_end": rec.token_end, "tokens": rec.token_end - rec.token_start,
                         "blocks": len(seg.lengths), "mode": seg.mode.value, "protected": rec.protected,
                         "stored_bytes": self._segment_bytes(seg)})
        return {"full_precision_bytes": self.full_precision_bytes, "resident_bytes": self.resident_bytes,
                "compression_ratio": self.compression_ratio, "attention_mode": self.parser.state.mode.value,
                "focus_segment_ids": list(self.parser.state.focus_segment_ids),
                "visible_segment_ids": list(self.visible_segment_ids()), "segments": rows}

    def protect_segment(self, segment_id: int) -> None:
        seg = self._get(segment_id)
        if seg.mode is not CacheMode.FP16:
            raise LossyPromotionError("a quantized segment cannot be restored to lossless FP16; "
                                      "protect it before archiving")
        rec = seg.record
        seg.record = SegmentRecord(rec.segment_id, rec.role, rec.token_start, rec.token_end, True)

    def _check_transition(self, seg: _Segment, target: CacheMode, what: str) -> None:
        sid = seg.record.segment_id
        if seg.record.protected and target is not CacheMode.FP16:
            raise ValueError(f"segment {sid} is protected")
        if PRECISION_RANK[target] > PRECISION_RANK[seg.mode]:
            raise LossyPromotionError(f"{what} {seg.mode.value} segment {sid} to {target.value}")

    def requantize_segment(self, segment_id: int, mode: CacheMode) -> None:
        mode = as_mode(mode)
        seg = self._get(segment_id)
        self._check_transition(seg, mode, "cannot restore")
        if mode is seg.mode:
            return
        if seg.mode is CacheMode.EVICTED:
            raise RuntimeError("evicted segments cannot be requantized")
        if seg.paged:
            self._requantize_pages(seg, mode)
        else:
            self._requantize_flat(seg, mode)
        seg.mode = mode

    def apply_directive(self, directive: CacheDirective) -> None:
        if directive.kind is DirectiveKind.MODE:
            for sid in directive.segment_ids:  # the ids must exist; visibility follows the parser state
                self._get(sid)
        elif directive.kind is DirectiveKind.ANCHOR:
            for sid in directive.segment_ids:
                self.protect_segment(sid)
        elif directive.kind is DirectiveKind.ARCHIVE:
            for sid in directive.segment_ids:
                self.requantize_segment(sid, self.archive_mode)
        else:  # pragma: no cover - DirectiveKind is exhaustive
            raise AssertionError(f"unsupported directive: {directive.kind}")

    def apply_plan(self, plan: CachePlan) -> None:
        """Apply a plan to physical storage; every target is checked before any change."""
        targets = {seg.segment_id: as_mode(seg.mode) for seg in plan.segments}
        if targets.keys() != self._segments.keys():
            raise ValueError("cache plan and backend must contain the same segment IDs")
        for sid, target in targets.items():
            self._check_transition(self._segments[sid], target, "plan cannot restore")
        for sid, target in targets.items():
            self.requantize_segment(sid, target)

    def feed_declarations(self, text: str) -> tuple[CacheDirective, ...]:
        directives = self.parser.feed(text)
        for directive in directives:
            self.apply_directive(directive)
        return directives

    # ---------------------------------------------------------------- reads
    def visible_segment_ids(self) -> tuple[int, ...]:
        state = self.parser.state
        if state.mode is AttentionMode.FOCUS:
            for sid in state.focus_segment_ids:  # a focused id that is not a segment fails as in the reference
                if sid not in self._segments:
                    raise KeyError(sid)
        chosen = [seg for seg in self._segments.values()
                  if state.mode is AttentionMode.GLOBAL or seg.record.role in ALWAYS_VISIBLE
                  or (state.mode is AttentionMode.FOCUS and seg.record.segment_id in state.focus_segment_ids)]
        chosen.sort(key=lambda seg: seg.record.token_start)
        return tuple(seg.record.segment_id for seg in chosen if seg.mode is not CacheMode.EVICTED)

    def materialize_visible(self, *, dtype: Any | None = None, device: Any | None = None) -> MaterializedCache:
        return self.materialize_segments(self.visible_segment_ids(), dtype=dtype, device=device)

    def materialize_segments(self, segment_ids: Iterable[int], *, dtype: Any | None = None,
                             device: Any | None = None) -> MaterializedCache:
        segs = [self._get(sid) for sid in dict.fromkeys(int(s) for s in segment_ids)]
        segs = sorted((s for s in segs if s.mode is not CacheMode.EVICTED), key=lambda s: s.record.token_start)
        if not segs:
            raise RuntimeError("no resident KV blocks were selected")
        if all(s.paged for s in segs):
            keys, values = self._unpack(segs, dtype)
        else:
            parts = [self._unpack([s], dtype) if s.paged else self._dequantize_flat(s, dtype) for s in segs]
            keys, values = torch.cat([p[0] for p in parts], -2), torch.cat([p[1] for p in parts], -2)
        if device is not None:
            keys, values = keys.to(device), values.to(device)
        positions = torch.cat([torch.arange(s.record.token_start, s.record.token_end, device=keys.device)
                               for s in segs])
        block_ids = tuple(b for s in segs for b in s.block_ids)
        owners = tuple(s.record.segment_id for s in segs for _ in s.block_ids)
        return MaterializedCache(keys, values, positions, block_ids, owners)

    # ------------------------------------------------------ decode page table
    @property
    def layers(self) -> int:
        """Layers of the paged segments (1 for ``[batch, heads, tokens, head_dim]`` segments)."""
        if self._table_geometry is None:
            return 0
        lead = self._table_geometry[0]
        return lead[0] if len(lead) == 3 else 1

    def decode_view(self, layer: int = 0) -> P.PagedBatch:
        """The page table of ``layer`` for :func:`anchorkv_b200.packed_attention`:
        one row per sequence, one descriptor per block of every paged segment,
        blocks of evicted or currently invisible segments as skip entries.  It
        is rebuilt on the device (one small copy) only when a segment, a
        precision or the visibility state changed since the last call."""
        if self._pool is None:
            raise ValueError("the store holds no segment in the decode page format (block_size 16, head_dim "
                             "64/128, group 32/64/128 or one per block and head, fp16 CUDA tensors)")
        visible = set(self.visible_segment_ids())
        flat = sorted(s.record.segment_id for s in self._segments.values()
                      if not s.paged and s.record.segment_id in visible)
        if flat:
            raise ValueError(f"segments {flat} are visible but not stored in the decode page format; "
                             "attend them through materialize_visible()")
        if not 0 <= layer < self.layers:
            raise ValueError(f"layer {layer} outside the store's {self.layers} layers")
        if not visible:
            raise RuntimeError("no resident KV blocks were selected")
        table = self._visible_table(frozenset(visible))
        batch = table.shape[0] // self.layers
        return P.PagedBatch.over(self._pool, table[layer * batch:(layer + 1) * batch])

    def _visible_table(self, visible: frozenset) -> torch.Tensor:
        key = (self._table_version, visible)
        if self._device_table is not None and self._device_table[0] == key:
            return self._device_table[1]
        keep = np.zeros(self._columns, bool)
        for seg in self._segments.values():
            if seg.paged and seg.record.segment_id in visible and seg.mode is not CacheMode.EVICTED:
                keep[seg.columns] = True
        host = np.where(keep[None, :], self._descriptors[:, :self._columns], 0)
        table = P.to_device(host, self._pool.device)
        self._device_table = (key, table)
        return table

    # --------------------------------------------------- paged segments
    def _pageable(self, seg: _Segment, key: torch.Tensor) -> bool:
        if self.block_size != P.BLOCK or not key.is_cuda or key.dtype != torch.float16:
            return False
        if seg.dim not in (64, 128) or not P.group_ok(seg.dim, self.group_size):
            return False
        if any(n * seg.dim % self.group_size for n in seg.lengths):  # a group would straddle two heads
            return False
        return self._table_geometry in (None, (seg.lead, seg.dim, key.device))

    def _add_pages(self, seg: _Segment, key: torch.Tensor, value: torch.Tensor) -> None:
        heads = seg.lead[-1]
        status, stream = _lib.status_ptr(key.device), _lib.stream_of(key.device)  # raises before any change
        if self._pool is None:
            self._pool = P.PagePool(heads, seg.dim, group=self.group_size, device=key.device)
            self._table_geometry = (seg.lead, seg.dim, key.device)
            self._descriptors = np.zeros((math.prod(seg.lead[:-1]), 64), np.int64)
        rows, nblk = self._descriptors.shape[0], len(seg.lengths)
        tokens = int(key.shape[-2])
        pad = nblk * P.BLOCK - tokens

        def rows_first(t):  # [rows, heads, padded tokens, dim], zero rows past the segment's end
            t = t.reshape(rows, heads, tokens, seg.dim)
            return torch.nn.functional.pad(t, (0, 0, 0, pad)).contiguous() if pad else t.contiguous()

        k, v = rows_first(key), rows_first(value)
        if k.data_ptr() % 16 or v.data_ptr() % 16:  # a view at an odd offset: the pack kernel reads 16-byte vectors
            k, v = k.clone(), v.clone()
        self._pool.reserve(16, rows * nblk)
        slots = self._pool.alloc_many(16, rows * nblk).reshape(rows, nblk)
        ntok = np.broadcast_to(np.array(seg.lengths, np.int64), (rows, nblk))
        desc = P.encode_array(np.full((rows, nblk), _lib.MODE_FP16), ntok, slots)
        dev = self._pool.device
        d = P.to_device(desc.reshape(-1), dev)
        _lib.call("akv_pack_pages", k.data_ptr(), v.data_ptr(), heads * nblk * P.BLOCK * seg.dim,
                  nblk * P.BLOCK * seg.dim, nblk, rows * nblk, d.data_ptr(), self._pool.arena.data_ptr(),
                  self._pool.nbytes, heads, seg.dim, self.group_size, _lib.SEM_TENSOR, status, stream)
        seg.columns = self._grow_columns(nblk)
        self._descriptors[:, seg.columns] = desc

    def _grow_columns(self, n: int) -> list[int]:
        first = self._columns
        if first + n > self._descriptors.shape[1]:
            wider = np.zeros((self._descriptors.shape[0], max(2 * self._descriptors.shape[1], first + n)), np.int64)
            wider[:, :first] = self._descriptors[:, :first]
            self._descriptors = wider
        self._columns += n
        self._table_version += 1
        return list(range(first, first + n))

    def _requantize_pages(self, seg: _Segment, mode: CacheMode) -> None:
        dev = self._pool.device
        status, stream = _lib.status_ptr(dev), _lib.stream_of(dev)  # raises before any change
        old = self._descriptors[:, seg.columns]
        offsets = old >> 8
        if mode is CacheMode.EVICTED:
            self._descriptors[:, seg.columns] = 0
        else:
            bits = _BITS[mode]
            self._pool.reserve(bits, old.size)
            fresh = self._pool.alloc_many(bits, old.size).reshape(old.shape)
            new = P.encode_array(np.full(old.shape, P.BITS_TO_MODE[bits]), ((old >> 2) & 15) + 1, fresh)
            src, dst = P.to_device(old.reshape(-1), dev), P.to_device(new.reshape(-1), dev)
            heads = self._table_geometry[0][-1]
            _lib.call("akv_repack_pages", src.data_ptr(), dst.data_ptr(), old.size, self._pool.arena.data_ptr(),
                      self._pool.nbytes, heads, seg.dim, self.group_size, _lib.SEM_TENSOR, status, stream)
            self._descriptors[:, seg.columns] = new
        # stream order: anything later written into the freed slots follows the repack
        self._pool.free_many(_BITS[seg.mode], offsets)
        self._table_version += 1

    def _unpack(self, segs: list[_Segment], dtype) -> tuple[torch.Tensor, torch.Tensor]:
        """Dense K and V of paged segments (token order), one unpack launch."""
        cols = [c for s in segs for c in s.columns]
        lengths = [n for s in segs for n in s.lengths]
        out_dtype = segs[0].dtype if dtype is None else dtype
        kernel_dtype = out_dtype if out_dtype in _KERNEL_DTYPES else torch.float32
        lead, dim, dev = self._table_geometry
        rows, heads, n = self._descriptors.shape[0], lead[-1], len(cols)
        desc = P.to_device(self._descriptors[:, cols].reshape(-1), dev)
        k = torch.empty((heads, rows * n * P.BLOCK, dim), dtype=kernel_dtype, device=dev)
        v = torch.empty_like(k)
        _lib.call("akv_unpack_pages", desc.data_ptr(), rows * n, self._pool.arena.data_ptr(), self._pool.nbytes,
                  heads, dim, self.group_size, k.data_ptr(), v.data_ptr(), _KERNEL_DTYPES[kernel_dtype],
                  _lib.status_ptr(dev), _lib.stream_of(dev))
        token = torch.from_numpy(np.concatenate([j * P.BLOCK + np.arange(t) for j, t in enumerate(lengths)])).to(dev)

        def dense(t):  # [heads, rows, n * 16, dim] -> [*lead[:-1], heads, tokens, dim]
            t = t.view(heads, rows, n * P.BLOCK, dim).index_select(2, token).transpose(0, 1)
            return t.reshape(*lead, token.numel(), dim).to(out_dtype)

        return dense(k), dense(v)

    # ---------------------------------------------------- flat segments
    def _chunk_plan(self, seg: _Segment) -> list[tuple[int, int]]:
        """(first block, count) per chunk: full blocks stacked together when their
        element count is a whole number of groups, everything else alone."""
        full = [b for b, n in enumerate(seg.lengths) if n == self.block_size]
        if full and seg.numel(full[0]) % self.group_size == 0:
            return [(0, len(full))] + [(b, 1) for b in range(len(full), len(seg.lengths))]
        return [(b, 1) for b in range(len(seg.lengths))]

    def _add_flat(self, seg: _Segment, key: torch.Tensor, value: torch.Tensor) -> None:
        seg.chunks = []
        for first, count in self._chunk_plan(seg):
            lo = first * self.block_size
            hi = lo + sum(seg.lengths[first:first + count])
            parts = []
            for t in (key, value):
                piece = t[..., lo:hi, :]
                if count > 1:  # [count, *lead, block, dim]: blocks stacked, block-major
                    piece = torch.stack(piece.split(self.block_size, dim=-2))
                parts.append(quantize_tensor(piece, CacheMode.FP16, group_size=self.group_size))
            seg.chunks.append(_Chunk(first, count, parts[0], parts[1]))

    def _requantize_flat(self, seg: _Segment, mode: CacheMode) -> None:
        for chunk in seg.chunks:
            if mode is CacheMode.EVICTED:
                chunk.key, chunk.value = (PackedTensor(mode, t.shape, t.original_dtype, None, None, t.group_size,
                                                       t.original_numel) for t in (chunk.key, chunk.value))
            else:
                chunk.key, chunk.value = (quantize_tensor(t.dequantize(), mode, group_size=self.group_size)
                                          for t in (chunk.key, chunk.value))

    def _dequantize_flat(self, seg: _Segment, dtype) -> tuple[torch.Tensor, torch.Tensor]:
        out = []
        for which in ("key", "value"):
            pieces = []
            for chunk in seg.chunks:
                t = getattr(chunk, which).dequantize(dtype=dtype)
                pieces.extend(t.unbind(0) if chunk.count > 1 else (t,))
            out.append(torch.cat(pieces, dim=-2))
        return out[0], out[1]

    # --------------------------------------------------------------- lookups
    def _get(self, segment_id: int) -> _Segment:
        try:
            return self._segments[segment_id]
        except KeyError as error:
            raise KeyError(f"unknown segment {segment_id}") from error


def _tensor_bytes(tensor: Any | None) -> int:
    return 0 if tensor is None else int(tensor.numel()) * int(tensor.element_size())
