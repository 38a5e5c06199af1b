"""akv_packed_attention_static, the allocation-free decode entry point, through the C ABI.

Some callers cannot allocate device memory: hosts that reserve all of HBM up
front for their own pool (a serving engine's KV pool), latency-critical decode
loops where cudaMalloc/cudaFree would synchronize the device, and bindings that
hold raw pointers but no allocator.  For them the split-K partials live in a
fixed 8 MiB array inside the library.  This file checks, on two calls in a row,
that its output matches akv_packed_attention with a caller-owned workspace
(within the decode tolerance), and that oversize requests are refused.  It is
named so pytest collects it last.
"""

import math

import numpy as np
import pytest
import torch

import workloads as W
from anchorkv_b200 import _lib
from anchorkv_b200 import pool as P

pytestmark = pytest.mark.gpu
ATOL, RTOL = 2e-3, 1e-2


def _store(cuda, seed, batch, q_heads, kv_heads, tokens, group):
    k = W.outlier_kv(seed, (batch, kv_heads, tokens, 128))
    v = W.outlier_kv(seed + 1, (batch, kv_heads, tokens, 128))
    q = W.normal(seed + 2, (batch, q_heads, 1, 128)).to(cuda)
    nblk = tokens // 16
    bits = np.array(W.draw_modes(seed + 3, batch * nblk, {16: .15, 8: .35, 4: .4, 0: .1})).reshape(batch, nblk)
    pool = P.PagePool(kv_heads, 128, group=group, pages={b: int((bits == b).sum()) for b in (16, 8, 4)},
                      device=cuda, shuffle_seed=seed)
    return q, P.pack_dense(pool, k.to(cuda), v.to(cuda), bits, semantics="tensor" if group == 2048 else "page")


def _args(q, store, splits):
    pool, t = store.pool, store.table
    return (pool.arena.data_ptr(), pool.nbytes, t.data_ptr(), t.stride(0), store.seq_blocks.data_ptr(),
            store.max_blocks, q.data_ptr(), q.stride(0), q.stride(1), q.shape[0], q.shape[1], pool.heads,
            128, pool.group, 1 / math.sqrt(128), splits)


def _with_workspace(q, store, splits, cuda):
    lib = _lib.load()
    out = torch.empty_like(q)
    nbytes = lib.akv_workspace_bytes(q.shape[0], q.shape[1], store.pool.heads, 128, store.max_blocks, splits)
    ws = torch.empty(nbytes, dtype=torch.uint8, device=cuda)
    status = lib.akv_packed_attention(*_args(q, store, splits), out.data_ptr(), out.stride(0), out.stride(1),
                                      ws.data_ptr(), ws.numel(), None, _lib.stream_of(cuda))
    assert status == _lib.OK, _lib.status_string(status)
    return out


def _static(q, store, splits, cuda):
    lib = _lib.load()
    out = torch.empty_like(q)
    status = lib.akv_packed_attention_static(*_args(q, store, splits), out.data_ptr(), out.stride(0),
                                             out.stride(1), None, _lib.stream_of(cuda))
    assert status == _lib.OK, _lib.status_string(status)
    return out


def test_static_scratch_matches_workspace_entry_on_consecutive_calls(cuda):
    first = _store(cuda, 501, batch=4, q_heads=16, kv_heads=8, tokens=1024, group=2048)
    second = _store(cuda, 601, batch=2, q_heads=32, kv_heads=8, tokens=512, group=64)
    static_first = _static(*first, 8, cuda)
    static_second = _static(*second, 3, cuda)  # reuses the scratch the first call left behind
    torch.cuda.synchronize(cuda)
    for (q, store), splits, got in ((first, 8, static_first), (second, 3, static_second)):
        want = _with_workspace(q, store, splits, cuda)
        np.testing.assert_allclose(got.float().cpu().numpy(), want.float().cpu().numpy(), atol=ATOL, rtol=RTOL)
    again = _static(*first, 8, cuda)
    np.testing.assert_allclose(again.float().cpu().numpy(), static_first.float().cpu().numpy(),
                               atol=ATOL, rtol=RTOL)


def test_static_scratch_refuses_requests_beyond_its_size(cuda):
    lib = _lib.load()
    assert lib.akv_static_scratch_bytes() == 8 << 20
    q, store = _store(cuda, 701, batch=1, q_heads=16, kv_heads=8, tokens=64, group=2048)
    # A geometry whose partial states need more than the fixed scratch.
    batch = 1
    while lib.akv_workspace_bytes(batch, 64, 8, 128, 512, 0) <= 8 << 20:
        batch *= 2
    q = torch.zeros(batch, 64, 1, 128, dtype=torch.float16, device=cuda)
    splits = 0
    out = torch.empty_like(q)
    args = list(_args(q, store, splits))
    args[5], args[9], args[10], args[11] = 512, batch, 64, 8  # max_blocks, batch, q_heads, kv_heads
    status = lib.akv_packed_attention_static(*args, out.data_ptr(), out.stride(0), out.stride(1), None,
                                             _lib.stream_of(cuda))
    assert status == _lib.ERR_SCRATCH
    assert "8 MiB" in _lib.status_string(status)


def test_static_scratch_runs_a_long_sequence_with_the_requested_splits(cuda):
    """A single long sequence whose finer cut of the work (every resident warp)
    would need more than the fixed scratch runs with exactly `splits` pieces
    per (sequence, KV head) instead, and matches the workspace entry."""
    lib = _lib.load()
    q, store = _store(cuda, 801, batch=1, q_heads=64, kv_heads=8, tokens=32768, group=2048)
    splits = 4
    assert lib.akv_workspace_bytes(1, 64, 8, 128, store.max_blocks, splits) > lib.akv_static_scratch_bytes()
    got = _static(q, store, splits, cuda)
    want = _with_workspace(q, store, splits, cuda)
    np.testing.assert_allclose(got.float().cpu().numpy(), want.float().cpu().numpy(), atol=ATOL, rtol=RTOL)
