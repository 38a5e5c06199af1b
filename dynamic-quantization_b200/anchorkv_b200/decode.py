"""Packed single-token decode attention entry point.

Drop-in for ``src/anchorkv/triton_decode.py:85-104`` (``packed_attention``):
same arguments, same validation errors, output in the query's dtype and shape.
It also accepts a :class:`~anchorkv_b200.pool.PagedBatch` (batch of sequences
over a shared page pool), where the query is ``[batch, Hq, 1, D]``.

The work runs in sm_100a kernels behind the C ABI (akv_packed_attention): the
paged decode (persistent stream-K: every resident warp takes a contiguous range
of (sequence, KV head, page) work, bulk-copies the pages into a private
shared-memory ring, dequantises in registers into mma.sync fragments and keeps
an fp32 online softmax) and the log-sum-exp merge of the partial states (one
warp per (sequence, query head), or a CTA per row for long sequences), each
launched as a programmatic dependent of the kernel before it.
"""

from __future__ import annotations

import torch

from . import _lib
from .pool import PagedBatch, group_ok

_workspaces: dict = {}
_workspace_sizes: dict = {}


def _workspace_bytes(device: torch.device, *geometry) -> int:
    """akv_workspace_bytes for ``geometry`` on ``device``, remembered (it depends only on them)."""
    key = (device.index, geometry)
    nbytes = _workspace_sizes.get(key)
    if nbytes is None:
        if len(_workspace_sizes) > 4096:
            _workspace_sizes.clear()
        nbytes = _lib.load().akv_workspace_bytes(*geometry)
        _workspace_sizes[key] = nbytes
    return nbytes


_MAX_WORKSPACES = 64


def _workspace(device: torch.device, nbytes: int, stream: int | None = None) -> torch.Tensor:
    """The decode workspace of (device, stream), grown on demand.

    Workspaces of at most ``_MAX_WORKSPACES`` streams are kept; the oldest goes
    first (a caller that makes a stream per request would otherwise hold one
    per stream forever).  Dropping one is safe: it was allocated on its own
    stream and used only there, so the allocator reuses its memory in that
    stream's order."""
    key = (device.index, torch.cuda.current_stream(device).cuda_stream if stream is None else stream)
    ws = _workspaces.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(nbytes, 1 << 16), dtype=torch.uint8, device=device)
        _workspaces.pop(key, None)
        while len(_workspaces) >= _MAX_WORKSPACES:
            _workspaces.pop(next(iter(_workspaces)))
        _workspaces[key] = ws
    return ws


def _store_geometry(layer):
    """(arena, arena bytes, table [B, stride], seq_blocks or None, max_blocks)."""
    if isinstance(layer, PagedBatch):
        return layer.pool.arena, layer.pool.nbytes, layer.table, layer.seq_blocks, layer.max_blocks
    n = len(layer.pages)
    return layer.pool.arena, layer.pool.nbytes, layer.table.view(1, -1), None, n


def _as_table(layer):
    """A DeclarativeKVCache stands for its (single) layer's visible page table."""
    if hasattr(layer, "decode_view"):
        if layer.layers > 1:
            raise ValueError("the store holds several layers: pass store.decode_view(layer)")
        return layer.decode_view(0)
    return layer


def query_head_to_kv_head(query_head: int, *, num_query_heads: int, num_kv_heads: int) -> int:
    """The KV head a query head reads under grouped-query attention
    (heads.py:112-126): ``query_head // (num_query_heads // num_kv_heads)``.

    The decode kernel serves every query head of one KV head from the same
    pages with this map (a warp's slot holds that KV head's query heads,
    consecutive in the query); the checks and errors are the reference's."""
    if num_query_heads <= 0 or num_kv_heads <= 0:
        raise ValueError("head counts must be positive")
    if num_query_heads % num_kv_heads != 0:
        raise ValueError("num_query_heads must be divisible by num_kv_heads")
    if not 0 <= query_head < num_query_heads:
        raise ValueError("query_head is out of range")
    return query_head // (num_query_heads // num_kv_heads)


def _check_query(query, layer, splits, *, empty_ok: bool) -> int:
    """The argument checks of triton_decode.py:86-94, in its order and with its
    messages, for a page table of ``layer``; returns the batch.

    ``empty_ok`` admits a table with no pages: a shard of a sequence split over
    more ranks than it has pages decodes to an empty state (zero weight in the
    LSE merge); an output needs at least one page, as in the reference."""
    batched = isinstance(layer, PagedBatch)
    batch = layer.batch if batched else 1
    if query.dim() != 4 or query.shape[0] != batch or query.shape[2] != 1 or query.shape[-1] != layer.dim:
        raise ValueError('packed kernel supports batch=1, query length=1 only' if not batched
                         else 'query must be [batch, heads, 1, head_dim] for the page table')
    length = layer.max_blocks if batched else layer.length
    if query.dtype != torch.float16 or not query.is_cuda or (length == 0 and not empty_ok):
        raise ValueError('packed kernel requires a nonempty CUDA FP16 cache')
    if layer.dim not in (64, 128) or layer.block != 16 or not group_ok(layer.dim, layer.group):
        raise ValueError('supported geometry: block=16, group=32/64/128 or one scale per '
                         'block and head, head dim=64/128')
    if query.shape[1] % layer.heads:
        raise ValueError('query heads must be divisible by KV heads')
    if splits < 0:
        raise ValueError('splits must be non-negative')
    return batch


def packed_attention(query, layer, scale, splits=4, *, out=None):
    """Attend one query token per sequence over the layer's packed pages.

    ``layer``: a PagedLayer, a PagedBatch, or a DeclarativeKVCache of one layer
    (its visible, non-evicted blocks; ``store.decode_view(l)`` for layer l of a
    multi-layer store).
    ``query``: fp16 CUDA ``[batch, Hq, 1, D]`` (batch 1 for a PagedLayer).
    ``splits``: at least this many pieces per (sequence, KV head), merged by
    LSE (the reference's split-K knob); the decode cuts finer, down to 16 pages
    a piece, while the device has resident warps to spare (``0``: every
    resident warp).  Results do not depend on it beyond fp32 rounding.
    ``out``: an optional fp16 CUDA tensor of the query's shape on its device.
    """
    layer = _as_table(layer)
    batch = _check_query(query, layer, splits, empty_ok=False)
    heads = query.shape[1]
    if out is not None and (out.dtype != torch.float16 or tuple(out.shape) != tuple(query.shape)
                            or out.device != query.device or out.stride(-1) != 1):
        raise ValueError("out must be an FP16 tensor of the query's shape on its device, unit stride in head_dim")
    if query.stride(-1) != 1 or query.stride(1) % 8 or query.stride(0) % 8 or query.data_ptr() % 16:
        query = query.contiguous()
    arena, arena_bytes, table, seq_blocks, max_blocks = _store_geometry(layer)
    if out is None:
        out = torch.empty(query.shape, dtype=query.dtype, device=query.device)
    dev = query.device
    nbytes = _workspace_bytes(dev, batch, heads, layer.heads, layer.dim, max_blocks, splits)
    if nbytes < 0:
        raise ValueError('unsupported decode geometry')
    stream = _lib.stream_of(dev)
    ws = _workspace(dev, nbytes, stream)
    _lib.call("akv_packed_attention", arena.data_ptr(), arena_bytes, table.data_ptr(), table.stride(0),
              None if seq_blocks is None else seq_blocks.data_ptr(), max_blocks,
              query.data_ptr(), query.stride(0), query.stride(1), batch, heads, layer.heads, layer.dim,
              layer.group, float(scale), splits, out.data_ptr(), out.stride(0), out.stride(1),
              ws.data_ptr(), ws.numel(), _lib.status_ptr(dev), stream)
    return out


def decode_partial_states(query, layer, scale, splits=0):
    """Decode merged to one LSE state per (sequence, query head).

    Returns fp32 ``[batch, Hq, D + 2]`` = (acc[D], m, l) with ``m`` in base-2
    units of the scaled score, for a further merge (e.g. across GPUs holding
    contiguous shards of each sequence) with :func:`merge_states`.  The query
    is checked as :func:`packed_attention` checks it, except that a table with
    no pages is allowed (its state has zero weight in the merge)."""
    layer = _as_table(layer)
    batch = _check_query(query, layer, splits, empty_ok=True)
    heads = query.shape[1]
    query = query.contiguous()
    arena, arena_bytes, table, seq_blocks, max_blocks = _store_geometry(layer)
    dev = query.device
    nbytes = _workspace_bytes(dev, batch, heads, layer.heads, layer.dim, max_blocks, splits)
    if nbytes < 0:
        raise ValueError('unsupported decode geometry')
    stream = _lib.stream_of(dev)
    ws = _workspace(dev, nbytes, stream)
    state = torch.empty((batch, heads, layer.dim + 2), dtype=torch.float32, device=dev)
    status = _lib.status_ptr(dev)
    _lib.call("akv_decode_partials", arena.data_ptr(), arena_bytes, table.data_ptr(), table.stride(0),
              None if seq_blocks is None else seq_blocks.data_ptr(), max_blocks, query.data_ptr(),
              query.stride(0), query.stride(1), batch, heads, layer.heads, layer.dim, layer.group,
              float(scale), splits, ws.data_ptr(), ws.numel(), status, stream)
    _lib.call("akv_merge", ws.data_ptr(), batch, heads, layer.dim, None, 0, 0, state.data_ptr(), status,
              stream)
    return state


def merge_states(states: torch.Tensor) -> torch.Tensor:
    """Merge ``[n, batch, Hq, D + 2]`` LSE states (e.g. gathered from n GPUs)
    into the normalised fp16 output ``[batch, Hq, 1, D]``."""
    if states.dim() != 4 or states.dtype != torch.float32 or not states.is_cuda:
        raise ValueError("states must be a CUDA float32 tensor [n, batch, heads, head_dim + 2]")
    n, batch, heads, rs = states.shape
    states = states.contiguous()
    out = torch.empty((batch, heads, 1, rs - 2), dtype=torch.float16, device=states.device)
    _lib.call("akv_merge_states", states.data_ptr(), n, batch, heads, rs - 2, out.data_ptr(),
              out.stride(0), out.stride(1), _lib.stream_of(states.device))
    return out
