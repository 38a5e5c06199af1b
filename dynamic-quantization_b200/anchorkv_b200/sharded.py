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
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from .decode import decode_partial_states, merge_states


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
