"""Hugging Face decode loops over the packed store: the paged layers as a live
cache and the packed kernel as the model's attention.

Mirrors the reference's model-side integration in
``src/anchorkv/colab_experiment.py``: ``stock_cache`` / ``cache_cpu`` (:86-91),
``make_live_cache`` (:92-120), ``attention_route`` (:123-148) and
``forward_token`` (:150-155), the decode loop of ``run_policy`` (:191-214) and
``model_gate`` (:294-313), whose acceptance rule is the parity check here: over
the same stores, the packed route's logits stay within a mean per-token KL of
0.002 of the dense route's, and the FP16 paged route matches the stock model.
``controlled_decode`` is the reference's fixed-history timing harness
(``src/anchorkv/benchmark_suite.py:155-264``).

Model code (``transformers``) is imported lazily: it is needed only when a
model runs.
"""

from __future__ import annotations

from contextlib import contextmanager
from dataclasses import dataclass

import torch

from .decode import packed_attention
from .packed_decode import PagedLayer, dense_attention, kl_divergence

# Name the routed attention function is registered under.
ROUTE = "anchorkv_b200"


@dataclass
class Settings:
    """The fields of the reference's experiment settings (colab_experiment.py:21-35)
    that the live cache and the decode loop read."""

    block: int = 16
    recent_pages: int = 2
    max_new_tokens: int = 48


def stock_cache(source, device="cuda"):
    """A stock ``DynamicCache`` holding ``source`` = [(key, value)] per layer."""
    from transformers import DynamicCache

    return DynamicCache([(k.to(device), v.to(device)) for k, v in source])


def cache_cpu(cache):
    """[(key, value)] per layer of a stock cache, on the host."""
    return [(layer.keys.detach().cpu(), layer.values.detach().cpu()) for layer in cache.layers]


def make_live_cache(source, settings, protected=(), bits=4, max_tokens=None, device="cuda"):
    """A ``DynamicCache`` whose layers are :class:`PagedLayer` stores: prefilled
    from ``source``, appended to (and demoted to ``bits``) as tokens are decoded.
    ``update`` hands the new keys/values back unchanged; the routed attention
    reads the stores."""
    from transformers import DynamicCache

    if max_tokens is None:
        max_tokens = source[0][0].shape[-2] + settings.max_new_tokens + 32

    class LiveCache(DynamicCache):
        def __init__(self):
            super().__init__()
            self.stores = []
            for key, value in source:
                store = PagedLayer(key.shape[1], key.shape[-1], max_tokens, block=settings.block,
                                   archive_bits=bits, protected=protected,
                                   recent_pages=settings.recent_pages, device=device)
                store.append(key.to(device), value.to(device))
                self.stores.append(store)

        def get_seq_length(self, layer_idx=0):
            return self.stores[layer_idx].length

        def update(self, key_states, value_states, layer_idx, *args, **kwargs):
            self.stores[layer_idx].append(key_states, value_states)
            return key_states, value_states

        def report(self):
            return {"resident_bytes": sum(s.resident_bytes for s in self.stores),
                    "payload_bytes": sum(s.payload_bytes for s in self.stores),
                    "demotions": sum(s.demotions for s in self.stores),
                    "tokens": self.get_seq_length()}

    return LiveCache()


@contextmanager
def attention_route(model, cache=None, backend="dense", capture=None):
    """Route the model's attention through the stores of ``cache`` for the
    duration of the block: ``backend='packed'`` runs :func:`packed_attention`
    (the sm_100a decode kernels), ``'dense'`` the dequantise-then-attend path.
    Without a cache the stock SDPA runs (queries can still be captured).  The
    registry entry is pointed back at SDPA on exit so it keeps no cache alive."""
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS

    original = model.config._attn_implementation
    dense_interface = ALL_ATTENTION_FUNCTIONS["sdpa"]

    def attention(module, query, key, value, attention_mask, scaling, **kwargs):
        if capture is not None:
            capture[module.layer_idx] = query.detach().cpu()
        if cache is None:
            return dense_interface(module, query, key, value, attention_mask, scaling=scaling, **kwargs)
        store = cache.stores[module.layer_idx]
        if backend == "packed":
            result = packed_attention(query, store, scaling)
        else:
            result = dense_attention(query, store, scaling)
        return result.transpose(1, 2).contiguous(), None

    ALL_ATTENTION_FUNCTIONS.register(ROUTE, attention)
    model.config._attn_implementation = ROUTE
    try:
        yield
    finally:
        model.config._attn_implementation = original
        ALL_ATTENTION_FUNCTIONS.register(ROUTE, dense_interface)


def forward_token(model, cache, token, packed=False):
    """One decode step of ``token`` at the cache's current length."""
    position = cache.get_seq_length()
    return model(input_ids=torch.tensor([[token]], device=model.device), past_key_values=cache,
                 cache_position=torch.tensor([position], device=model.device),
                 attention_mask={"full_attention": None} if packed else None,
                 use_cache=True, logits_to_keep=1)


POLICY_BITS = {"paged_fp16": 16, "int8": 8, "int4": 4, "oracle": 4}


@torch.inference_mode()
def decode_logits(model, source, first_token, forced, settings, policy, protected=(), backend="packed"):
    """Logits [steps, vocab] of a decode replay: ``first_token`` then the
    ``forced`` tokens, over a stock cache (``policy='native_fp16'``) or a live
    cache demoted to the policy's bits (the loop of colab_experiment.py:191-214)."""
    native = policy == "native_fp16"
    device = model.device
    cache = stock_cache(source, device) if native else make_live_cache(
        source, settings, protected, POLICY_BITS[policy], device=device)
    logits = []
    token = first_token
    with attention_route(model, cache=None if native else cache, backend=backend):
        for step in range(len(forced)):
            output = forward_token(model, cache, token, packed=not native)
            logits.append(output.logits[0, -1].float())
            token = int(forced[step])
    return torch.stack(logits)


@torch.inference_mode()
def model_gate(model, source, first_token, forced, settings):
    """The reference's model gate (colab_experiment.py:294-313) on token ids:
    for every policy the packed route must stay within a mean KL of 0.002 of
    the dense route over the same stores, with finite logits; the FP16 paged
    route must match the stock model.  Raises AssertionError otherwise and
    returns the per-policy figures."""
    stock = decode_logits(model, source, first_token, forced, settings, "native_fp16")
    checks = []
    for policy, protected in [("paged_fp16", ()), ("int8", ()), ("int4", ()), ("oracle", (0, 2))]:
        dense = decode_logits(model, source, first_token, forced, settings, policy, protected, "dense")
        packed = decode_logits(model, source, first_token, forced, settings, policy, protected, "packed")
        discrepancy = float(kl_divergence(dense, packed).mean())
        if discrepancy > 0.002 or not torch.isfinite(packed).all():
            raise AssertionError(f"kernel/model mismatch for {policy}: KL={discrepancy}")
        if policy == "paged_fp16":
            torch.testing.assert_close(dense, stock, atol=0.05, rtol=0.01)
            if float(kl_divergence(stock, packed).mean()) > 0.002:
                raise AssertionError("FP16 packed route does not match the stock model")
        checks.append({"policy": policy, "mean_kl_dense_vs_packed": discrepancy,
                       "max_logit_error": float((dense - packed).abs().max())})
    return checks


CONTROLLED_POLICIES = ("native_fp16", "paged_fp16", "int8", "int4", "automatic", "recent", "random", "oracle")


def controlled_decode(model, source, settings, policy, input_tokens, measured_tokens, warmup_tokens=32,
                      protected=(), backend="packed"):
    """Fixed-history decode throughput and cache lifecycle
    (benchmark_suite.controlled_decode, benchmark_suite.py:155-264): the
    ``warmup_tokens`` then ``measured_tokens`` of ``input_tokens`` are appended
    one decode step at a time after the ``source`` prefix; no sampling, no
    logit transfers.  ``measured_cuda_timeline_seconds`` is device-timeline
    time between two events (launch gaps included).  Returns the reference's
    row fields."""
    import gc
    import hashlib
    import json
    import time

    total = warmup_tokens + measured_tokens
    if warmup_tokens < 0 or measured_tokens <= 0 or len(input_tokens) != total:
        raise ValueError("provide exactly warmup_tokens + measured_tokens input tokens")
    if policy not in CONTROLLED_POLICIES:
        raise ValueError("unknown policy")
    device = model.device
    gpu = device.type == "cuda"
    if not gpu and backend == "packed" and policy != "native_fp16":
        raise ValueError("packed throughput requires CUDA")
    native = policy == "native_fp16"
    bits = 16 if policy == "paged_fp16" else 8 if policy == "int8" else 4

    def synchronize():
        if gpu:
            torch.cuda.synchronize(device)

    def report(cache):
        if not native:
            return cache.report()
        size = sum(t.numel() * t.element_size() for layer in cache.layers for t in (layer.keys, layer.values))
        return {"tokens": cache.get_seq_length(), "resident_bytes": size, "payload_bytes": size, "demotions": 0}

    gc.collect()
    if gpu:
        torch.cuda.empty_cache()
    prefix = source[0][0].shape[-2]
    ids = torch.tensor([input_tokens], device=device, dtype=torch.long)
    positions = torch.arange(prefix, prefix + total, device=device)
    synchronize()
    base_allocated = torch.cuda.memory_allocated(device) if gpu else None
    if gpu:
        torch.cuda.reset_peak_memory_stats(device)
    started = time.perf_counter()
    with torch.inference_mode():
        cache = (stock_cache(source, device=device) if native else
                 make_live_cache(source, settings, protected, bits, max_tokens=prefix + total, device=device))
        synchronize()
        setup_seconds = time.perf_counter() - started
        initial = report(cache)

        def step(index):
            output = model(input_ids=ids[:, index:index + 1], past_key_values=cache,
                           cache_position=positions[index:index + 1], use_cache=True,
                           attention_mask=None if native else {"full_attention": None}, logits_to_keep=1)
            del output

        with attention_route(model, None if native else cache, backend):
            warm_started = time.perf_counter()
            for index in range(warmup_tokens):
                step(index)
            synchronize()
            warmup_seconds = time.perf_counter() - warm_started
            before = report(cache)
            setup_warmup_peak = torch.cuda.max_memory_allocated(device) if gpu else None
            if gpu:
                torch.cuda.reset_peak_memory_stats(device)
                begin = torch.cuda.Event(enable_timing=True)
                end = torch.cuda.Event(enable_timing=True)
            measured_started = time.perf_counter()
            if gpu:
                begin.record()
            for index in range(warmup_tokens, total):
                step(index)
            if gpu:
                end.record()
            synchronize()
            wall_seconds = time.perf_counter() - measured_started
            cuda_seconds = begin.elapsed_time(end) / 1000 if gpu else None
        final = report(cache)
        peak = torch.cuda.max_memory_allocated(device) if gpu else None
        end_allocated = torch.cuda.memory_allocated(device) if gpu else None
    assert final["tokens"] == prefix + total, "decode did not append the complete fixed workload"
    row = {"policy": policy, "backend": "stock_sdpa" if native else backend,
           "scope": "fixed-history throughput and cache lifecycle; not answer accuracy",
           "prefix_tokens": prefix, "warmup_tokens": warmup_tokens, "measured_tokens": measured_tokens,
           "setup_seconds": setup_seconds, "warmup_seconds": warmup_seconds,
           "measured_wall_seconds": wall_seconds, "measured_cuda_timeline_seconds": cuda_seconds,
           "steady_tokens_per_second": measured_tokens / wall_seconds,
           "setup_warmup_decode_seconds": setup_seconds + warmup_seconds + wall_seconds,
           "initial_cache": initial, "measurement_start_cache": before, "final_cache": final,
           "new_measured_demotions": final["demotions"] - before["demotions"],
           "setup_warmup_peak_allocated_bytes": setup_warmup_peak, "measured_peak_allocated_bytes": peak,
           "measured_peak_incremental_bytes": peak - base_allocated if gpu else None,
           "end_incremental_bytes": end_allocated - base_allocated if gpu else None,
           "input_sha256": hashlib.sha256(json.dumps(input_tokens).encode()).hexdigest()}
    del cache, ids, positions
    gc.collect()
    if gpu:
        torch.cuda.empty_cache()
    return row
