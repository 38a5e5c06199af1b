"""Sequence-sharded decode for long contexts across GPUs.

The reference splits one sequence's pages across split-K programs of one GPU
and merges their (max, sum-exp, accumulator) states by log-sum-exp
(``src/anchorkv/triton_decode.py:35-82``).  The same algebra spans GPUs here:

* each rank holds a contiguous, page-aligned shard of every sequence's pages
  (:func:`shard_range`) and decodes it locally into one LSE state per query
  head (:func:`anchorkv_b200.decode_partial_states`);
* one ``all_gather_into_tensor`` over the process group (NCCL over NVLink on
  B200; ``batch * Hq * (D + 2) * 4`` bytes per rank) collects the states;
* every rank merges them on its device (:func:`anchorkv_b200.merge_states`).

No KV page ever crosses GPUs; the collective moves only the small states.
Batched decode needs none of this: sequences are independent, so a batch is
split across ranks with no collective at all.

:class:`PeerExchange` does the same exchange without a library collective:
one kernel per call (``akv_merge_exchange``) merges this rank's partials, stores
the state into every rank's buffer over NVLink, waits (bounded) for the other
ranks' states and merges them (buffers shared through CUDA IPC).
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from .decode import (_as_table, _check_query, _store_geometry, _workspace, decode_partial_states,
                     merge_states)


def shard_range(n_blocks: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous page range ``[lo, hi)`` of ``rank`` when ``n_blocks`` pages are
    split over ``world`` ranks (the first ``n_blocks % world`` ranks get one more)."""
    if world <= 0 or not 0 <= rank < world or n_blocks < 0:
        raise ValueError("invalid shard geometry")
    base, extra = divmod(n_blocks, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def gather_states(state: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather ``[batch, Hq, D + 2]`` states from every rank -> ``[world, batch, Hq, D + 2]``."""
    world = dist.get_world_size(group)
    shape = tuple(state.shape)
    out = torch.empty((world * shape[0],) + shape[1:], dtype=state.dtype, device=state.device)
    dist.all_gather_into_tensor(out, state.contiguous(), group=group)
    return out.view((world,) + shape)


def sharded_packed_attention(query, local_store, scale, *, splits=0, group=None,
                             local_states=decode_partial_states, merge=merge_states):
    """Decode over a sequence whose pages are sharded across the ranks of ``group``.

    ``local_store`` holds this rank's shard (a :class:`~anchorkv_b200.PagedBatch`
    or :class:`~anchorkv_b200.PagedLayer`); ``query`` is replicated on every
    rank.  Returns the full-context output ``[batch, Hq, 1, D]`` on every rank.
    ``local_states`` and ``merge`` are the device kernels; they are parameters so
    the collective logic can be exercised with host stand-ins."""
    state = local_states(query, local_store, scale, splits=splits)
    return merge(gather_states(state, group))


EPOCH_MAX = 0xFFFFFFFF  # the exchange kernel's epoch is a 32-bit word; 0 marks a buffer never written


def next_epoch(epoch: int) -> int:
    """The epoch of the exchange call after one with ``epoch`` (0 before the first call).

    The kernel needs each call's epoch to be nonzero, to alternate in parity
    (the parity picks the buffer half) and to differ from the epoch two calls
    before (the stale words in that half carry it).  Counting up does all
    three until 32 bits run out; after ``0xFFFFFFFF`` (odd) the count goes on
    at 2 (even), whose half holds words tagged ``0xFFFFFFFE``.  Every rank
    applies the same rule, so their epochs stay equal."""
    return epoch + 1 if epoch < EPOCH_MAX else 2


class PeerExchange:
    """Cross-GPU LSE merge over peer memory for sequences split over the ranks
    of ``group`` (one process per GPU of one node, at most 8).

    Every rank allocates an exchange buffer (``akv_exchange_bytes``), the
    ranks trade CUDA IPC handles through the process group, and each rank
    maps the others' buffers.  :meth:`attention` then decodes this rank's
    pages and runs ``akv_merge_exchange``: the output of the whole sequence,
    on every rank, in two kernel launches and no library collective.  Every
    rank must make the same calls; :meth:`close` (collective) unmaps and frees.
    """

    def __init__(self, batch: int, q_heads: int, dim: int, group=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.batch, self.q_heads, self.dim = batch, q_heads, dim
        lib = _lib.load()
        nbytes = lib.akv_exchange_bytes(self.world, batch, q_heads, dim)
        if nbytes < 0:
            raise ValueError("unsupported exchange geometry (at most 8 ranks, head_dim 64 or 128)")
        own = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        _lib.call("akv_ipc_alloc", nbytes, ctypes.byref(own), handle)
        self._own = own.value
        self._mapped = []
        ptrs = []
        try:
            handles = [None] * self.world
            dist.all_gather_object(handles, handle.raw, group=group)
            for r, h in enumerate(handles):
                if r == self.rank:
                    ptrs.append(self._own)
                    continue
                peer = ctypes.c_void_p()
                _lib.call("akv_ipc_open", ctypes.create_string_buffer(h, 64), ctypes.byref(peer))
                self._mapped.append(peer.value)
                ptrs.append(peer.value)
        except BaseException:
            # nothing has been launched on these buffers: unmap what was mapped and
            # free this rank's buffer before the error reaches the caller (the other
            # ranks learn of it from their process group's timeout)
            for ptr in self._mapped:
                _lib.load().akv_ipc_close(ctypes.c_void_p(ptr))
            _lib.load().akv_ipc_free(ctypes.c_void_p(self._own))
            self._mapped, self._own = [], None
            raise
        self._peers = (ctypes.c_void_p * self.world)(*ptrs)
        self.epoch = 0
        dist.barrier(group=group)

    def attention(self, query, local_store, scale, *, splits=0, out=None):
        """Decode this rank's pages of each sequence and merge with the other
        ranks: the full-context output ``[batch, Hq, 1, D]`` on every rank.

        The query is checked as :func:`~anchorkv_b200.packed_attention` checks
        it (a shard with no pages is allowed); ``out``, if given, is an fp16
        tensor of the query's shape on its device."""
        if tuple(query.shape) != (self.batch, self.q_heads, 1, self.dim):
            raise ValueError("query shape differs from the exchange's geometry")
        local_store = _as_table(local_store)
        _check_query(query, local_store, splits, empty_ok=True)
        if out is not None and (out.dtype != torch.float16 or tuple(out.shape) != tuple(query.shape)
                                or out.device != query.device or out.stride(-1) != 1):
            raise ValueError("out must be an FP16 tensor of the query's shape on its device, unit stride in head_dim")
        query = query.contiguous()
        arena, arena_bytes, table, seq_blocks, max_blocks = _store_geometry(local_store)
        dev = query.device
        lib = _lib.load()
        nbytes = lib.akv_workspace_bytes(self.batch, self.q_heads, local_store.heads, self.dim, max_blocks,
                                         splits)
        if nbytes < 0:
            raise ValueError("unsupported decode geometry")
        ws = _workspace(dev, nbytes)
        if out is None:
            out = torch.empty_like(query)
        stream = _lib.stream_of(dev)
        status = _lib.status_ptr(dev)
        _lib.call("akv_decode_partials", arena.data_ptr(), arena_bytes, table.data_ptr(), table.stride(0),
                  None if seq_blocks is None else seq_blocks.data_ptr(), max_blocks, query.data_ptr(),
                  query.stride(0), query.stride(1), self.batch, self.q_heads, local_store.heads, self.dim,
                  local_store.group, float(scale), splits, ws.data_ptr(), ws.numel(), status, stream)
        self.epoch = next_epoch(self.epoch)
        _lib.call("akv_merge_exchange", ws.data_ptr(), self.batch, self.q_heads, self.dim, self._peers,
                  self.rank, self.world, self.epoch, out.data_ptr(), out.stride(0), out.stride(1), status,
                  stream)
        return out

    def close(self):
        """Collective: wait for every rank's kernels, then unmap and free."""
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for ptr in self._mapped:
            _lib.call("akv_ipc_close", ctypes.c_void_p(ptr))
        self._mapped = []
        dist.barrier(group=self.group)
        if self._own:
            _lib.call("akv_ipc_free", ctypes.c_void_p(self._own))
            self._own = None
