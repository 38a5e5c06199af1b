"""Hugging Face integration (colab_experiment.py:86-155, 294-313 of the reference):
the attention route and live cache, with the reference's model gate as parity.

No checkpoint is available offline, so the models are randomly initialised
Qwen3 architectures (fp16 on the GPU); the gate compares two attention
implementations over the same stores, which holds for any weights."""

import gc
import weakref

import pytest
import torch

from anchorkv_b200 import live


def _qwen3(head_dim, heads, kv_heads, layers, device, dtype, seed=0):
    from transformers import Qwen3Config, Qwen3ForCausalLM

    torch.manual_seed(seed)
    config = Qwen3Config(vocab_size=2048, hidden_size=heads * head_dim, intermediate_size=2 * heads * head_dim,
                         num_hidden_layers=layers, num_attention_heads=heads, num_key_value_heads=kv_heads,
                         head_dim=head_dim, max_position_embeddings=4096, attn_implementation="sdpa")
    return Qwen3ForCausalLM(config).to(device=device, dtype=dtype).eval()


@torch.inference_mode()
def test_route_without_cache_captures_queries_and_restores_registry():
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS

    model = _qwen3(32, 4, 2, 2, "cpu", torch.float32)
    ids = torch.randint(0, 2048, (1, 21), generator=torch.Generator().manual_seed(1))
    prefill = model(input_ids=ids[:, :-1], use_cache=True, logits_to_keep=1)
    source = live.cache_cpu(prefill.past_key_values)
    assert len(source) == 2 and source[0][0].shape == (1, 2, 20, 32)
    stock = model(input_ids=ids[:, -1:], past_key_values=live.stock_cache(source, "cpu"), use_cache=True,
                  logits_to_keep=1).logits
    captured = {}
    with live.attention_route(model, capture=captured):
        assert model.config._attn_implementation == live.ROUTE
        routed = live.forward_token(model, live.stock_cache(source, "cpu"), int(ids[0, -1])).logits
    assert model.config._attn_implementation == "sdpa"
    assert ALL_ATTENTION_FUNCTIONS[live.ROUTE] is ALL_ATTENTION_FUNCTIONS["sdpa"]
    assert sorted(captured) == [0, 1] and captured[0].shape == (1, 4, 1, 32)
    torch.testing.assert_close(routed, stock)


@pytest.mark.gpu
@pytest.mark.parametrize("head_dim,heads,kv_heads", [(128, 16, 8), (64, 8, 2)])
def test_model_gate_on_random_qwen3(cuda, head_dim, heads, kv_heads):
    """Packed route vs dense route (mean KL <= 0.002) for FP16 / INT8 / INT4
    stores and an INT4 store with protected pages; FP16 paged vs stock."""
    model = _qwen3(head_dim, heads, kv_heads, 4, cuda, torch.float16)
    ids = torch.randint(0, 2048, (1, 181), generator=torch.Generator().manual_seed(2))
    with torch.inference_mode():
        prefill = model(input_ids=ids[:, :-1].to(cuda), use_cache=True, logits_to_keep=1)
    source = live.cache_cpu(prefill.past_key_values)
    forced = torch.randint(0, 2048, (8,), generator=torch.Generator().manual_seed(3)).tolist()
    checks = live.model_gate(model, source, int(ids[0, -1]), forced, live.Settings())
    assert [c["policy"] for c in checks] == ["paged_fp16", "int8", "int4", "oracle"]
    assert all(c["mean_kl_dense_vs_packed"] <= 0.002 for c in checks)


@pytest.mark.gpu
def test_live_cache_appends_and_demotes_during_decode(cuda):
    model = _qwen3(128, 16, 8, 2, cuda, torch.float16)
    ids = torch.randint(0, 2048, (1, 100), generator=torch.Generator().manual_seed(4))
    with torch.inference_mode():
        prefill = model(input_ids=ids[:, :-1].to(cuda), use_cache=True, logits_to_keep=1)
        source = live.cache_cpu(prefill.past_key_values)
        cache = live.make_live_cache(source, live.Settings(), bits=4, device=cuda)
        before = cache.report()
        with live.attention_route(model, cache=cache, backend="packed"):
            token = int(ids[0, -1])
            for _ in range(40):
                token = int(live.forward_token(model, cache, token, packed=True).logits[0, -1].argmax())
    after = cache.report()
    assert after["tokens"] == before["tokens"] + 40 == 139
    assert after["demotions"] > before["demotions"]
    assert after["payload_bytes"] < 2 * 2 * 2 * 8 * 139 * 128  # below the FP16 size of two layers' K and V
    # The global attention registry keeps no closure over the cache once the
    # route has exited (colab_experiment.py:147-148): the cache is freed.
    cache_ref = weakref.ref(cache)
    del cache
    gc.collect()
    assert cache_ref() is None, "the attention registry retained the live cache"


def test_controlled_decode_validates_like_the_reference():
    model = _qwen3(32, 4, 2, 1, "cpu", torch.float32)
    source = [(torch.zeros(1, 2, 16, 32), torch.zeros(1, 2, 16, 32))]
    with pytest.raises(ValueError, match="provide exactly"):
        live.controlled_decode(model, source, live.Settings(), "int4", [1, 2, 3], 2, warmup_tokens=2)
    with pytest.raises(ValueError, match="unknown policy"):
        live.controlled_decode(model, source, live.Settings(), "int2", [1, 2, 3], 1, warmup_tokens=2)
    with pytest.raises(ValueError, match="packed throughput requires CUDA"):
        live.controlled_decode(model, source, live.Settings(), "int4", [1, 2, 3], 1, warmup_tokens=2)


@torch.inference_mode()
def test_controlled_decode_native_on_cpu():
    model = _qwen3(32, 4, 2, 2, "cpu", torch.float32)
    ids = torch.randint(0, 2048, (1, 20), generator=torch.Generator().manual_seed(5))
    source = live.cache_cpu(model(input_ids=ids, use_cache=True, logits_to_keep=1).past_key_values)
    row = live.controlled_decode(model, source, live.Settings(), "native_fp16", list(range(6)), 4,
                                 warmup_tokens=2)
    assert row["final_cache"]["tokens"] == 26 and row["measured_cuda_timeline_seconds"] is None
    assert row["backend"] == "stock_sdpa" and row["new_measured_demotions"] == 0


@pytest.mark.gpu
@pytest.mark.parametrize("prefix", [128, 256, 512])
def test_controlled_decode_packed_cache_lifecycle(cuda, prefix):
    """The fixed-history workloads at 128/256/512-token prefixes: every measured
    token is appended, archived pages are demoted on the way, and the INT4 store
    stays below the stock FP16 cache."""
    model = _qwen3(128, 16, 8, 2, cuda, torch.float16)
    ids = torch.randint(0, 2048, (1, prefix), generator=torch.Generator().manual_seed(6))
    with torch.inference_mode():
        source = live.cache_cpu(model(input_ids=ids.to(cuda), use_cache=True, logits_to_keep=1).past_key_values)
    tokens = torch.randint(0, 2048, (48,), generator=torch.Generator().manual_seed(7)).tolist()
    packed = live.controlled_decode(model, source, live.Settings(), "int4", tokens, 32, warmup_tokens=16)
    native = live.controlled_decode(model, source, live.Settings(), "native_fp16", tokens, 32, warmup_tokens=16)
    assert packed["final_cache"]["tokens"] == native["final_cache"]["tokens"] == prefix + 48
    assert packed["new_measured_demotions"] > 0
    assert packed["final_cache"]["payload_bytes"] < native["final_cache"]["payload_bytes"]
    assert packed["measured_cuda_timeline_seconds"] > 0 and packed["steady_tokens_per_second"] > 0
