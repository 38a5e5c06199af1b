"""Codec kernels on the GPU, bit for bit against the reference fixtures and the oracle."""

import json
from pathlib import Path

import numpy as np
import pytest
import torch

import anchorkv_b200 as akv
import workloads as W
from anchorkv_b200 import pool as P
from oracle import codec as OC
from paged_reference import block_values, record_bytes_expected

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
CODEC = np.load(GOLDEN / "codec.npz")
META = json.loads((GOLDEN / "codec.json").read_text())
MODE = {8: akv.CacheMode.INT8, 4: akv.CacheMode.INT4}


def _input(meta):
    raw = torch.from_numpy(CODEC[meta["input"]].copy())
    return raw.view(torch.bfloat16) if meta["dtype"] == "bfloat16" else raw


def _bytes(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.uint8).numpy().reshape(-1)


@pytest.mark.parametrize("meta", META["tensor"], ids=lambda m: m["name"])
def test_quantize_tensor_golden(cuda, meta):
    x = _input(meta).to(cuda)
    packed = akv.quantize_tensor(x, MODE[meta["bits"]], group_size=meta["group"])
    key = f"t_{meta['name']}"
    np.testing.assert_array_equal(_bytes(packed.payload), CODEC[key + "_payload"].view(np.uint8).reshape(-1))
    np.testing.assert_array_equal(_bytes(packed.scales), CODEC[key + "_scales"].view(np.uint8).reshape(-1))
    assert packed.stored_bytes == meta["stored_bytes"]
    restored = packed.dequantize()
    assert restored.dtype == x.dtype and tuple(restored.shape) == tuple(meta["shape"])
    np.testing.assert_array_equal(_bytes(restored), CODEC[key + "_deq"].view(np.uint8).reshape(-1))


@pytest.mark.parametrize("meta", META["page"], ids=lambda m: m["name"])
def test_pack_page_golden(cuda, meta):
    x = _input(meta).to(cuda)
    page = akv.pack_page(x, meta["bits"], meta["group"])
    key = f"p_{meta['name']}"
    np.testing.assert_array_equal(_bytes(page.data), CODEC[key + "_payload"].view(np.uint8).reshape(-1))
    if meta["bits"] != 16:
        np.testing.assert_array_equal(_bytes(page.scales), CODEC[key + "_scales"].view(np.uint8).reshape(-1))
    assert page.nbytes == meta["nbytes"]
    np.testing.assert_array_equal(_bytes(page.dense()), CODEC[key + "_dense"].view(np.uint8).reshape(-1))


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("group", [2048, 64, 16, 10, 1000])
def test_quantize_tensor_random_vs_oracle(cuda, dtype, bits, group):
    x = (W.outlier_kv(group + bits, (3, 4, 37, 64), signed=True).float() * 1.7).to(dtype)
    packed = akv.quantize_tensor(x.to(cuda), MODE[bits], group_size=group)
    payload, scales = OC.quantize_tensor(x.float().numpy(), bits, group)
    np.testing.assert_array_equal(_bytes(packed.payload), payload.view(np.uint8))
    np.testing.assert_array_equal(_bytes(packed.scales), scales.view(np.uint8))


def _dense_kv(seed, batch, heads, tokens, dim):
    k = W.outlier_kv(seed, (batch, heads, tokens, dim), signed=True)
    v = W.outlier_kv(seed + 1, (batch, heads, tokens, dim), signed=True)
    return k, v


@pytest.mark.parametrize("dim", [64, 128])
@pytest.mark.parametrize("group,semantics", [(2048, "tensor"), (1024, "tensor"), (64, "tensor"),
                                             (64, "page"), (32, "page"), (128, "page")])
def test_pack_pages_records_are_reference_bytes(cuda, dim, group, semantics):
    if group > 16 * dim or (semantics == "page" and dim % group):
        pytest.skip("group does not apply to this head dim")
    if group == 1024 and dim != 64 or group == 2048 and dim != 128:
        pytest.skip("per-block scale group is 16 * head_dim")
    batch, heads, tokens = 2, 4, 80
    k, v = _dense_kv(7 + dim + group, batch, heads, tokens, dim)
    bits = np.array(W.draw_modes(3 + group, batch * 5, {16: .25, 8: .25, 4: .4, 0: .1})).reshape(batch, 5)
    counts = {b: int((bits == b).sum()) + 2 for b in (16, 8, 4)}
    pool = P.PagePool(heads, dim, group=group, pages=counts, device=cuda, shuffle_seed=5)
    store = P.pack_dense(pool, k.to(cuda), v.to(cuda), bits, semantics=semantics)
    assert akv.take_device_status(cuda) == 0
    arena = pool.arena.cpu().numpy()
    table = store.table.cpu().numpy()
    for b in range(batch):
        for j in range(5):
            mode_bits, ntok, off = P.decode(int(table[b, j]))
            if bits[b, j] == 0:
                assert mode_bits is None
                continue
            assert mode_bits == bits[b, j] and ntok == 16
            rec = P.record_bytes(dim, group, mode_bits)
            for h in range(heads):
                got = arena[off + h * rec: off + (h + 1) * rec].tobytes()
                sl = slice(16 * j, 16 * j + 16)
                want = record_bytes_expected(k[b, h, sl].numpy(), v[b, h, sl].numpy(), mode_bits, group,
                                             semantics, rec)
                assert got == want, (b, j, h, mode_bits)


@pytest.mark.parametrize("dim", [64, 128])
@pytest.mark.parametrize("src_bits,dst_bits", [(16, 8), (16, 4), (8, 4), (16, 16), (8, 8)])
def test_repack_and_unpack_match_page_semantics(cuda, dim, src_bits, dst_bits):
    heads, n, group = 3, 6, 64
    k, v = _dense_kv(11 + dim + src_bits, 1, heads, 16 * n, dim)
    pool = P.PagePool(heads, dim, group=group, pages={16: 2 * n, 8: 2 * n, 4: n}, device=cuda)
    src = P.pack_dense(pool, k.to(cuda), v.to(cuda), [[src_bits] * n], semantics="page")
    offs = pool.alloc_many(dst_bits, n)
    dst_desc = torch.tensor([P.encode(dst_bits, 16, int(o)) for o in offs], dtype=torch.int64, device=cuda)
    from anchorkv_b200 import _lib
    _lib.call("akv_repack_pages", src.table.data_ptr(), dst_desc.data_ptr(), n, pool.arena.data_ptr(),
              pool.nbytes, heads, dim, group, _lib.SEM_PAGE, _lib.status_word(cuda).data_ptr(), _lib.stream_of(cuda))
    ok = torch.empty((heads, n * 16, dim), dtype=torch.float16, device=cuda)
    ov = torch.empty_like(ok)
    _lib.call("akv_unpack_pages", dst_desc.data_ptr(), n, pool.arena.data_ptr(), pool.nbytes, heads, dim,
              group, ok.data_ptr(), ov.data_ptr(), _lib.DTYPE_F16, _lib.status_word(cuda).data_ptr(),
              _lib.stream_of(cuda))
    assert akv.take_device_status(cuda) == 0
    for t, got in ((k, ok), (v, ov)):
        for j in range(n):
            sl = slice(16 * j, 16 * j + 16)
            src_vals = block_values(t[0, :, sl].numpy(), src_bits, group, "page")
            want = block_values(src_vals, dst_bits, group, "page")
            np.testing.assert_array_equal(got[:, sl].cpu().numpy().view(np.uint16), want.view(np.uint16))
