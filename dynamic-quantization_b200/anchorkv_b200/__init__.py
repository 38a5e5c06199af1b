"""anchorkv_b200 -- the AnchorKV packed-KV decode path, B200-native.

Drop-in replacement for the reference's block codec, block stores and packed
decode attention (``anchorkv.backend``, ``anchorkv.packed_decode``,
``anchorkv.triton_decode``), with the data plane in hand-written sm_100a CUDA
kernels behind a C ABI (``include/anchorkv_b200.h``):

* :func:`quantize_tensor` / :func:`pack_page` and the page pack/repack kernels
  (bit-exact with the reference quantizers);
* :class:`PagedLayer` (batch one) and :class:`PagedBatch` over a shared
  :class:`PagePool` arena, :class:`DeclarativeKVCache` for segment-level
  visibility and eviction;
* :func:`packed_attention`, the paged split-K decode with an LSE merge
  (query heads served by :func:`query_head_to_kv_head`'s map), and
  :func:`decode_partial_states` / :func:`merge_states` for merging across GPUs;
  ``anchorkv_b200.sharded`` adds the NVLink exchange of one long sequence's
  shards and ``anchorkv_b200.live`` batched Hugging Face decode.
"""

from .backend import (
    AttentionMode,
    BackendUnavailableError,
    CacheDirective,
    DeclarativeAttentionParser,
    DeclarativeKVCache,
    DeclarativeState,
    DirectiveKind,
    KVBlock,
    LossyPromotionError,
    MaterializedCache,
    PackedTensor,
    SegmentRecord,
    SegmentRole,
    quantize_tensor,
    stack_legacy_cache,
)
from .decode import decode_partial_states, merge_states, packed_attention, query_head_to_kv_head
from .packed_decode import PagedLayer, QuantizedPage, dense_attention, kl_divergence, pack_page, tensor_bytes
from .policy import CacheMode, CachePlan, PlannedSegment
from .pool import PagedBatch, PagePool, pack_dense
from .sharded import gather_states, shard_range, sharded_packed_attention
from ._lib import KernelError, NativeUnavailableError, take_device_status

__version__ = "0.1.0"

__all__ = [
    "AttentionMode", "BackendUnavailableError", "CacheDirective", "CacheMode", "CachePlan",
    "DeclarativeAttentionParser", "DeclarativeKVCache", "DeclarativeState", "DirectiveKind",
    "KVBlock", "KernelError", "LossyPromotionError", "MaterializedCache", "NativeUnavailableError",
    "PackedTensor", "PagePool", "PagedBatch", "PagedLayer", "PlannedSegment", "QuantizedPage",
    "SegmentRecord", "SegmentRole", "decode_partial_states", "dense_attention", "kl_divergence",
    "merge_states", "pack_page", "packed_attention", "quantize_tensor", "stack_legacy_cache",
    "take_device_status", "tensor_bytes", "pack_dense", "shard_range", "gather_states",
    "sharded_packed_attention", "query_head_to_kv_head",
]
