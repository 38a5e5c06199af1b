"""Hugging Face decode over the packed store.

* The reference's own model-side code (colab_experiment.py:92-348 and
  benchmark_suite.py:155-264, imported unmodified from its install in
  baseline/_ref) runs with this package's PagedLayer, dense_attention and
  packed_attention substituted for its own: its kernel gate, its model gate
  (packed vs dense route, mean KL <= 0.002; FP16 paged vs stock) and its
  controlled-decode harness at 128/256/512-token prefixes.
* The batched store (anchorkv_b200.live): a batch of sequences in one page
  pool keeps, page for page, the bytes B separate PagedLayers hold, decodes to
  the same outputs, and drives a batched Qwen3 decode within the gate's KL.

No checkpoint is available offline, so models are randomly initialised Qwen3
architectures (fp16 on the GPU); the gates compare attention implementations
over the same stores, which holds for any weights."""

import gc
import weakref

import pytest
import torch

import anchorkv_b200 as akv
from anchorkv_b200 import live



def _qwen3(head_dim, heads, kv_heads, layers, device, dtype, seed=0):
    from transformers import Qwen3Config, Qwen3ForCausalLM

    torch.manual_seed(seed)
    config = Qwen3Config(vocab_size=2048, hidden_size=heads * head_dim, intermediate_size=2 * heads * head_dim,
                         num_hidden_layers=layers, num_attention_heads=heads, num_key_value_heads=kv_heads,
                         head_dim=head_dim, max_position_embeddings=4096, attn_implementation="sdpa")
    return Qwen3ForCausalLM(config).to(device=device, dtype=dtype).eval()


@pytest.fixture
def reference(reference_install, monkeypatch):
    """The reference's colab_experiment / benchmark_suite modules with this
    package substituted for its block store and kernels (a one-line import
    change for a user of the reference)."""
    from anchorkv import benchmark_suite, colab_experiment, triton_decode

    monkeypatch.setattr(colab_experiment, "PagedLayer", akv.PagedLayer)
    monkeypatch.setattr(colab_experiment, "dense_attention", akv.dense_attention)
    monkeypatch.setattr(colab_experiment, "pack_page", akv.pack_page)
    monkeypatch.setattr(triton_decode, "packed_attention", akv.packed_attention)
    return colab_experiment, benchmark_suite


class _DigitTokenizer:
    """Stand-in tokenizer for the gate's forced answer: digit d is token 100 + d."""

    eos_token_id = 7

    def __call__(self, text, add_special_tokens=False):
        return type("Encoded", (), {"input_ids": [100 + int(c) for c in text]})()

    def decode(self, ids, skip_special_tokens=True):
        return "".join(str(i - 100) if 100 <= i < 110 else "?" for i in ids)


def test_route_registry_is_restored_without_a_gpu():
    from transformers.modeling_utils import ALL_ATTENTION_FUNCTIONS

    model = _qwen3(32, 4, 2, 1, "cpu", torch.float32)
    store = type("Cache", (), {"store": None})()
    with live.paged_route(model, store):
        assert model.config._attn_implementation == live.ROUTE
    assert model.config._attn_implementation == "sdpa"
    assert ALL_ATTENTION_FUNCTIONS[live.ROUTE] is ALL_ATTENTION_FUNCTIONS["sdpa"]
    with pytest.raises(ValueError, match="archive_bits"):
        live.PagedKVStore(1, 2, 2, 64, 64, archive_bits=2, device="cpu")
    with pytest.raises(ValueError, match="geometry"):
        live.PagedKVStore(1, 2, 2, 96, 64, device="cpu")
    s = live.PagedKVStore(1, 2, 2, 64, 64, device="cpu")
    with pytest.raises(ValueError, match="CUDA"):
        s.prefill(0, torch.zeros(2, 2, 5, 64), torch.zeros(2, 2, 5, 64))


@pytest.mark.gpu
def test_reference_kernel_gate_with_this_package(cuda, reference):
    colab_experiment, _ = reference
    checks = colab_experiment.kernel_gate()
    assert len(checks) == 42 and max(c["max_error"] for c in checks) <= 3e-3


@pytest.mark.gpu
@pytest.mark.parametrize("head_dim,heads,kv_heads", [(128, 16, 8), (64, 8, 2)])
def test_reference_model_gate_with_this_package(cuda, reference, head_dim, heads, kv_heads):
    """The reference's model_gate (colab_experiment.py:294-313), unmodified, over
    this package's pages and kernels: FP16 / INT8 / INT4 / protected stores."""
    colab_experiment, _ = reference
    model = _qwen3(head_dim, heads, kv_heads, 4, cuda, torch.float16)
    ids = torch.randint(0, 2048, (181,), generator=torch.Generator().manual_seed(2)).tolist()
    case = {"ids": ids, "answer": "4821", "case_id": "random-qwen3"}
    source = colab_experiment.prefill_case(model, case)
    checks = colab_experiment.model_gate(model, _DigitTokenizer(), source, case, colab_experiment.Settings())
    assert [c["policy"] for c in checks] == ["paged_fp16", "int8", "int4", "oracle"]
    assert all(c["mean_kl_dense_vs_packed"] <= 0.002 for c in checks)


@pytest.mark.gpu
@pytest.mark.parametrize("prefix", [128, 256, 512])
def test_reference_controlled_decode_with_this_package(cuda, reference, prefix):
    """The reference's fixed-history harness (benchmark_suite.py:155-264) over
    this package's live cache at 128/256/512-token prefixes: every measured
    token is appended, archived pages are demoted on the way, and the INT4
    store stays below the stock FP16 cache."""
    colab_experiment, benchmark_suite = reference
    model = _qwen3(128, 16, 8, 2, cuda, torch.float16)
    ids = torch.randint(0, 2048, (1, prefix), generator=torch.Generator().manual_seed(6))
    with torch.inference_mode():
        out = model(input_ids=ids.to(cuda), use_cache=True, logits_to_keep=1)
        source = colab_experiment.cache_cpu(out.past_key_values)
    tokens = torch.randint(0, 2048, (48,), generator=torch.Generator().manual_seed(7)).tolist()
    settings = colab_experiment.Settings()
    packed = benchmark_suite.controlled_decode(model, source, settings, "int4", tokens, 32, warmup_tokens=16)
    native = benchmark_suite.controlled_decode(model, source, settings, "native_fp16", tokens, 32, warmup_tokens=16)
    assert packed["final_cache"]["tokens"] == native["final_cache"]["tokens"] == prefix + 48
    assert packed["new_measured_demotions"] > 0
    assert packed["final_cache"]["payload_bytes"] < native["final_cache"]["payload_bytes"]
    assert packed["measured_cuda_timeline_seconds"] > 0 and packed["steady_tokens_per_second"] > 0


@pytest.mark.gpu
@pytest.mark.parametrize("dim,archive", [(128, 4), (64, 8), (128, 16)])
def test_batched_store_holds_what_paged_layers_hold(cuda, dim, archive):
    """B sequences in one PagedKVStore against B separate PagedLayers fed the
    same tokens (a prefix, then single tokens and one 7-token chunk across page
    boundaries): the same precision per page, bit-identical dense K/V, and
    decode outputs within 1e-3 of the per-sequence packed_attention and 2e-3 of
    SDPA over the pages."""
    batch, heads, hq, prefix, steps = 3, 2, 4, 45, 40
    gen = torch.Generator().manual_seed(dim + archive)
    total = prefix + steps + 7
    k = torch.randn(batch, heads, total, dim, generator=gen).half().to(cuda)
    v = torch.randn(batch, heads, total, dim, generator=gen).half().to(cuda)
    store = live.PagedKVStore(1, batch, heads, dim, total, archive_bits=archive, recent_pages=1, protected=(1,),
                              device=cuda)
    layers = [akv.PagedLayer(heads, dim, total, archive_bits=archive, recent_pages=1, protected=(1,), device=cuda)
              for _ in range(batch)]
    store.prefill(0, k[:, :, :prefix], v[:, :, :prefix])
    for b in range(batch):
        layers[b].append(k[b:b + 1, :, :prefix], v[b:b + 1, :, :prefix])
    t = prefix
    for chunk in [1] * steps + [7]:
        store.append(0, k[:, :, t:t + chunk], v[:, :, t:t + chunk])
        for b in range(batch):
            layers[b].append(k[b:b + 1, :, t:t + chunk], v[b:b + 1, :, t:t + chunk])
        t += chunk
    assert store.lengths[0] == total
    for b in range(batch):
        assert list(store.bits(0)[b]) == [p[0].bits for p in layers[b].pages]
    assert store.demotions == sum(layer.demotions for layer in layers)
    dk, dv = store.dense(0)
    for b in range(batch):
        lk, lv = layers[b].dense()
        assert torch.equal(dk[b:b + 1], lk) and torch.equal(dv[b:b + 1], lv)
    q = torch.randn(batch, hq, 1, dim, generator=gen).half().to(cuda)
    out = akv.packed_attention(q, store.batch_view(0), dim ** -0.5)
    for b in range(batch):
        one = akv.packed_attention(q[b:b + 1], layers[b], dim ** -0.5)
        torch.testing.assert_close(out[b:b + 1], one, atol=1e-3, rtol=1e-3)
        sdpa = torch.nn.functional.scaled_dot_product_attention(
            q[b:b + 1], dk[b:b + 1].repeat_interleave(2, 1), dv[b:b + 1].repeat_interleave(2, 1), scale=dim ** -0.5)
        torch.testing.assert_close(out[b:b + 1], sdpa, atol=2e-3, rtol=1e-2)
    assert store.payload_bytes == sum(layer.payload_bytes for layer in layers)
    assert akv.take_device_status(cuda) == 0


@pytest.mark.gpu
def test_batched_decode_on_random_qwen3(cuda):
    """A batch of 4 sequences decoded together through the batched live cache
    and its attention route, the reference's model-gate rule applied to it:
    FP16 pages match the stock cache's batched decode; over INT8 / INT4 /
    protected stores the packed route stays within a mean KL of 0.002 of the
    dense route over the same pages; the route keeps no cache alive on exit."""
    model = _qwen3(128, 16, 8, 4, cuda, torch.float16)
    batch, prefix, steps = 4, 150, 24
    ids = torch.randint(0, 2048, (batch, prefix + steps), generator=torch.Generator().manual_seed(9)).to(cuda)
    with torch.inference_mode():
        out = model(input_ids=ids[:, :prefix], use_cache=True, logits_to_keep=1)
        source = [(layer.keys, layer.values) for layer in out.past_key_values.layers]

        def run(bits, backend, protected=()):
            cache = live.batched_live_cache(source, max_tokens=prefix + steps, archive_bits=bits,
                                            protected=protected, device=cuda)
            logits = []
            with live.paged_route(model, cache, backend):
                for s in range(steps):
                    logits.append(live.decode_step(model, cache, ids[:, prefix + s]).float())
            assert cache.get_seq_length() == prefix + steps
            return torch.stack(logits, 1).reshape(batch * steps, -1), cache

        from transformers import DynamicCache

        stock_cache = DynamicCache([(k.clone(), v.clone()) for k, v in source])
        stock = []
        for s in range(steps):
            o = model(input_ids=ids[:, prefix + s:prefix + s + 1], past_key_values=stock_cache, use_cache=True,
                      logits_to_keep=1)
            stock.append(o.logits[:, -1].float())
        stock = torch.stack(stock, 1).reshape(batch * steps, -1)
        fp16, _ = run(16, "packed")
        torch.testing.assert_close(fp16, stock, atol=0.05, rtol=0.01)
        assert float(akv.kl_divergence(stock, fp16).mean()) <= 0.002
        for bits, protected in ((8, ()), (4, ()), (4, (0, 2))):
            dense, _ = run(bits, "dense", protected)
            packed, cache = run(bits, "packed", protected)
            assert cache.report()["demotions"] > 0
            assert torch.isfinite(packed).all()
            assert float(akv.kl_divergence(dense, packed).mean()) <= 0.002, bits
    cache_ref = weakref.ref(cache)
    del cache
    gc.collect()
    assert cache_ref() is None, "the attention registry retained the live cache"
    assert akv.take_device_status(cuda) == 0
