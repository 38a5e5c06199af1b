"""Declarative block store and the flat-tensor codec, with a GPU data plane.

Drop-in for ``src/anchorkv/backend.py``: the same classes, method names,
arguments, lifecycle rules and error types/messages.  The control plane
(segments, blocks, visibility, the precision lifecycle) is host bookkeeping as
in the reference; quantization and dequantization run in CUDA kernels behind
the C ABI (akv_quantize / akv_dequantize) and are bit-exact with the
reference's torch ops (backend.py:154-226).  Tensors to quantize must live on a
CUDA device; there is no CPU compute path.
"""

from __future__ import annotations

import re
from dataclasses import dataclass, field
from enum import Enum
from typing import Any, Iterable

import torch

from . import _lib
from .policy import PRECISION_RANK, CacheMode, CachePlan, as_mode


class BackendUnavailableError(RuntimeError):
    """Raised when a required runtime dependency is unavailable."""


class LossyPromotionError(RuntimeError):
    """Raised when code attempts to restore precision that was already lost."""


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


_SEGMENT_LIST = re.compile(r'(?:segments|magic_chunks)\s*=\s*["\']([0-9,\s]+)["\']', re.IGNORECASE)


@dataclass(slots=True)
class DeclarativeAttentionParser:
    """Incremental parser of ``<focus segments="...">``, ``<local>``,
    ``<global>``, ``</focus>``, ``<anchor ...>`` and ``<archive ...>`` tags
    (backend.py:64-135).  Text may arrive in arbitrary chunks; an unfinished tag
    is kept until its ``>`` arrives and text outside tags is dropped."""

    state: DeclarativeState = field(default_factory=DeclarativeState)
    _pending: str = field(default="", init=False, repr=False)

    def feed(self, text: str) -> tuple[CacheDirective, ...]:
        self._pending += text
        found: list[CacheDirective] = []
        while True:
            open_at = self._pending.find("<")
            if open_at < 0:
                self._pending = ""
                break
            close_at = self._pending.find(">", open_at + 1)
            if close_at < 0:
                self._pending = self._pending[open_at:]
                break
            tag = self._pending[open_at + 1:close_at].strip()
            self._pending = self._pending[close_at + 1:]  # consumed even if the tag is invalid
            directive = self._interpret(tag)
            if directive is not None:
                found.append(directive)
        return tuple(found)

    def _interpret(self, tag: str) -> CacheDirective | None:
        name = tag.lower()
        if name in ("global", "/focus", "/local"):
            self._set(AttentionMode.GLOBAL, ())
            return CacheDirective(DirectiveKind.MODE, mode=AttentionMode.GLOBAL)
        if name == "local":
            self._set(AttentionMode.LOCAL, ())
            return CacheDirective(DirectiveKind.MODE, mode=AttentionMode.LOCAL)
        if name.startswith("focus"):
            ids = self._segment_ids(tag)
            self._set(AttentionMode.FOCUS, ids)
            return CacheDirective(DirectiveKind.MODE, mode=AttentionMode.FOCUS, segment_ids=ids)
        for prefix, kind in (("anchor", DirectiveKind.ANCHOR), ("archive", DirectiveKind.ARCHIVE)):
            if name.startswith(prefix):
                return CacheDirective(kind, segment_ids=self._segment_ids(tag))
        return None

    def _set(self, mode: AttentionMode, focus: tuple[int, ...]) -> None:
        self.state.mode = mode
        self.state.focus_segment_ids = focus

    @staticmethod
    def _segment_ids(tag: str) -> tuple[int, ...]:
        match = _SEGMENT_LIST.search(tag)
        if match is None:
            raise ValueError(f"declarative tag is missing a segment list: <{tag}>")
        ids: dict[int, None] = {}
        for item in match.group(1).split(","):
            ids[int(item.strip())] = None
        result = tuple(ids)
        if not result or min(result) < 0:
            raise ValueError("segment IDs must be non-negative")
        return result


# ------------------------------------------------------------------- codec
_KERNEL_DTYPES = {torch.float32: _lib.DTYPE_F32, torch.float16: _lib.DTYPE_F16,
                  torch.bfloat16: _lib.DTYPE_BF16}


@dataclass(frozen=True, slots=True)
class PackedTensor:
    """A tensor stored as FP16, symmetric INT8, or packed symmetric INT4."""

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
    """Stack a Hugging Face cache into layer-first key and value tensors."""
    legacy = past_key_values.to_legacy_cache() if hasattr(past_key_values, "to_legacy_cache") \
        else past_key_values
    layers = tuple(legacy)
    if not layers:
        raise ValueError("past_key_values must contain at least one layer")
    if any(len(layer) != 2 for layer in layers):
        raise ValueError("each legacy cache layer must contain one key and one value tensor")
    shape = layers[0][0].shape
    if any(k.shape != shape or v.shape != shape for k, v in layers):
        raise ValueError("all legacy cache tensors must share one shape")
    return torch.stack([k for k, _ in layers]), torch.stack([v for _, v in layers])


# ------------------------------------------------------------- block store
@dataclass(frozen=True, slots=True)
class KVBlock:
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
        """Convert stacked layer tensors to Hugging Face's legacy cache tuple."""
        if self.key.ndim != 5 or self.value.ndim != 5:
            raise ValueError(
                "legacy conversion requires [layers, batch, heads, tokens, head_dim] tensors")
        return tuple((self.key[i], self.value[i]) for i in range(int(self.key.shape[0])))


@dataclass(slots=True)
class DeclarativeKVCache:
    """Quantized KV blocks under declarative visibility/precision state
    (backend.py:314-601).  Segments are split into ``block_size``-token blocks
    stored FP16 on insert; a segment's blocks move down the lifecycle
    FP16 -> INT8 -> INT4 -> EVICTED, never back up."""

    block_size: int = 16
    group_size: int = 64
    archive_mode: CacheMode = CacheMode.INT4
    parser: DeclarativeAttentionParser = field(default_factory=DeclarativeAttentionParser)
    _blocks: dict[int, KVBlock] = field(default_factory=dict, init=False, repr=False)
    _segments: dict[int, SegmentRecord] = field(default_factory=dict, init=False, repr=False)
    _segment_blocks: dict[int, list[int]] = field(default_factory=dict, init=False, repr=False)
    _next_block_id: int = field(default=0, init=False, repr=False)

    def __post_init__(self) -> None:
        if self.block_size <= 0 or self.group_size <= 0:
            raise ValueError("block_size and group_size must be positive")
        self.archive_mode = as_mode(self.archive_mode)
        if self.archive_mode not in (CacheMode.INT4, CacheMode.INT8):
            raise ValueError("archive_mode must be INT4 or INT8")

    # ------------------------------------------------------------ accounting
    @property
    def resident_bytes(self) -> int:
        return sum(b.stored_bytes for b in self._blocks.values())

    @property
    def full_precision_bytes(self) -> int:
        return sum(2 * (b.key.original_numel + b.value.original_numel) for b in self._blocks.values())

    @property
    def compression_ratio(self) -> float:
        return self.full_precision_bytes / max(self.resident_bytes, 1)

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
        if any(token_start < s.token_end and s.token_start < token_end for s in self._segments.values()):
            raise ValueError("segment token ranges must not overlap")
        record = SegmentRecord(segment_id, SegmentRole(role), token_start, token_end, protected)
        ids = []
        for lo in range(0, count, self.block_size):
            hi = min(lo + self.block_size, count)
            bid = self._next_block_id
            self._next_block_id += 1
            self._blocks[bid] = KVBlock(
                bid, segment_id, token_start + lo, token_start + hi,
                quantize_tensor(key[..., lo:hi, :], CacheMode.FP16, group_size=self.group_size),
                quantize_tensor(value[..., lo:hi, :], CacheMode.FP16, group_size=self.group_size))
            ids.append(bid)
        self._segments[segment_id] = record
        self._segment_blocks[segment_id] = ids
        return record

    def segment_mode(self, segment_id: int) -> CacheMode:
        modes = {b.mode for b in self._blocks_for_segment(segment_id)}
        if len(modes) != 1:
            raise RuntimeError(f"segment {segment_id} has mixed block modes")
        return modes.pop()

    def storage_report(self) -> dict[str, object]:
        """JSON-safe physical storage and state-machine statistics."""
        ordered = sorted(self._segments.items(), key=lambda kv: kv[1].token_start)
        return {
            "full_precision_bytes": self.full_precision_bytes,
            "resident_bytes": self.resident_bytes,
            "compression_ratio": self.compression_ratio,
            "attention_mode": self.parser.state.mode.value,
            "focus_segment_ids": list(self.parser.state.focus_segment_ids),
            "visible_segment_ids": list(self.visible_segment_ids()),
            "segments": [{
                "segment_id": sid,
                "role": rec.role.value,
                "token_start": rec.token_start,
                "token_end": rec.token_end,
                "tokens": rec.token_end - rec.token_start,
                "blocks": len(self._segment_blocks[sid]),
                "mode": self.segment_mode(sid).value,
                "protected": rec.protected,
                "stored_bytes": sum(b.stored_bytes for b in self._blocks_for_segment(sid)),
            } for sid, rec in ordered],
        }

    def protect_segment(self, segment_id: int) -> None:
        record = self._get_segment(segment_id)
        if self.segment_mode(segment_id) is not CacheMode.FP16:
            raise LossyPromotionError("a quantized segment cannot be restored to lossless FP16; "
                                      "protect it before archiving")
        self._segments[segment_id] = SegmentRecord(record.segment_id, record.role, record.token_start,
                                                   record.token_end, True)

    def requantize_segment(self, segment_id: int, mode: CacheMode) -> None:
        mode = as_mode(mode)
        record = self._get_segment(segment_id)
        current = self.segment_mode(segment_id)
        if record.protected and mode is not CacheMode.FP16:
            raise ValueError(f"segment {segment_id} is protected")
        if PRECISION_RANK[mode] > PRECISION_RANK[current]:
            raise LossyPromotionError(f"cannot restore {current.value} segment {segment_id} to {mode.value}")
        if mode is current:
            return
        if current is CacheMode.EVICTED:
            raise RuntimeError("evicted segments cannot be requantized")
        updated = {}
        for block in self._blocks_for_segment(segment_id):
            key, value = block.materialize()
            updated[block.block_id] = KVBlock(
                block.block_id, block.segment_id, block.token_start, block.token_end,
                quantize_tensor(key, mode, group_size=self.group_size),
                quantize_tensor(value, mode, group_size=self.group_size))
        self._blocks.update(updated)

    def apply_directive(self, directive: CacheDirective) -> None:
        if directive.kind is DirectiveKind.MODE:
            for sid in directive.segment_ids:
                self._get_segment(sid)
        elif directive.kind is DirectiveKind.ANCHOR:
            for sid in directive.segment_ids:
                self.protect_segment(sid)
        elif directive.kind is DirectiveKind.ARCHIVE:
            for sid in directive.segment_ids:
                self.requantize_segment(sid, self.archive_mode)
        else:  # pragma: no cover - DirectiveKind is exhaustive
            raise AssertionError(f"unsupported directive: {directive.kind}")

    def apply_plan(self, plan: CachePlan) -> None:
        """Apply a plan to physical storage; validated in full before any change."""
        targets = {seg.segment_id: as_mode(seg.mode) for seg in plan.segments}
        if set(targets) != set(self._segments):
            raise ValueError("cache plan and backend must contain the same segment IDs")
        for sid, target in targets.items():
            current = self.segment_mode(sid)
            if self._segments[sid].protected and target is not CacheMode.FP16:
                raise ValueError(f"segment {sid} is protected")
            if PRECISION_RANK[target] > PRECISION_RANK[current]:
                raise LossyPromotionError(
                    f"plan cannot restore {current.value} segment {sid} to {target.value}")
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
        if state.mode is AttentionMode.GLOBAL:
            chosen = set(self._segments)
        else:
            chosen = {sid for sid, rec in self._segments.items() if rec.role in ALWAYS_VISIBLE}
            if state.mode is AttentionMode.FOCUS:
                chosen |= set(state.focus_segment_ids)
        ordered = sorted(chosen, key=lambda sid: self._segments[sid].token_start)
        return tuple(sid for sid in ordered if self.segment_mode(sid) is not CacheMode.EVICTED)

    def materialize_visible(self, *, dtype: Any | None = None, device: Any | None = None) -> MaterializedCache:
        return self.materialize_segments(self.visible_segment_ids(), dtype=dtype, device=device)

    def materialize_segments(self, segment_ids: Iterable[int], *, dtype: Any | None = None,
                             device: Any | None = None) -> MaterializedCache:
        requested = tuple(dict.fromkeys(int(s) for s in segment_ids))
        blocks = sorted((b for sid in requested for b in self._blocks_for_segment(sid)
                         if b.mode is not CacheMode.EVICTED), key=lambda b: b.token_start)
        if not blocks:
            raise RuntimeError("no resident KV blocks were selected")
        keys, values = zip(*(b.materialize(dtype=dtype, device=device) for b in blocks))
        positions = torch.cat([torch.arange(b.token_start, b.token_end, device=keys[0].device)
                               for b in blocks])
        return MaterializedCache(torch.cat(keys, dim=-2), torch.cat(values, dim=-2), positions,
                                 tuple(b.block_id for b in blocks), tuple(b.segment_id for b in blocks))

    def _get_segment(self, segment_id: int) -> SegmentRecord:
        try:
            return self._segments[segment_id]
        except KeyError as error:
            raise KeyError(f"unknown segment {segment_id}") from error

    def _blocks_for_segment(self, segment_id: int) -> list[KVBlock]:
        self._get_segment(segment_id)
        return [self._blocks[bid] for bid in self._segment_blocks[segment_id]]


def _tensor_bytes(tensor: Any | None) -> int:
    return 0 if tensor is None else int(tensor.numel()) * int(tensor.element_size())
