"""Cross-GPU LSE merge over peer memory (akv_merge_exchange, PeerExchange):
the long-context exchange of the reference's split-K merge
(triton_decode.py:70-82) across GPUs, against the oracle.

Single-GPU cases call the kernel with one rank, make its bounded wait run out
on a rank that never stores, or give it the other ranks' parts in its buffer
beforehand; the two-rank cases run as two child processes, one GPU each
(skipped with fewer GPUs), with NVLS off."""

import ctypes
import math
import os
import socket

import numpy as np
import pytest
import torch

import anchorkv_b200 as akv
import workloads as W
from anchorkv_b200 import _lib
from anchorkv_b200 import pool as P
from paged_reference import paged_decode_f64

pytestmark = pytest.mark.gpu

HQ, HKV, D, PAGES = 32, 8, 128, 300


def _sequence(seed=41):
    k = W.outlier_kv(seed, (1, HKV, 16 * PAGES, D))
    v = W.outlier_kv(seed + 1, (1, HKV, 16 * PAGES, D))
    q = W.normal(seed + 2, (1, HQ, 1, D))
    bits = np.array(W.draw_modes(seed + 3, PAGES, {16: .05, 8: .25, 4: .7}))[None]
    return k, v, q, bits


def _sequence_batch(batch, seed=141):
    k = W.outlier_kv(seed, (batch, HKV, 16 * PAGES, D))
    v = W.outlier_kv(seed + 1, (batch, HKV, 16 * PAGES, D))
    q = W.normal(seed + 2, (batch, HQ, 1, D))
    bits = np.array([W.draw_modes(seed + 3 + b, PAGES, {16: .05, 8: .25, 4: .7}) for b in range(batch)])
    return k, v, q, bits


def _store(device, k, v, bits, lo, hi):
    sub = bits[:, lo:hi]
    pool = P.PagePool(HKV, D, group=2048, pages={b: int((sub == b).sum()) for b in (16, 8, 4)}, device=device)
    return P.pack_dense(pool, k[:, :, 16 * lo:16 * hi].to(device), v[:, :, 16 * lo:16 * hi].to(device), sub)


def _buffer(world):
    lib = _lib.load()
    ptr, handle = ctypes.c_void_p(), ctypes.create_string_buffer(64)
    _lib.call("akv_ipc_alloc", lib.akv_exchange_bytes(world, 1, HQ, D), ctypes.byref(ptr), handle)
    return ptr.value


def _decode(store, q, ws, batch=1):
    lib = _lib.load()
    stream = torch.cuda.current_stream(q.device).cuda_stream
    _lib.call("akv_decode_partials", store.pool.arena.data_ptr(), store.pool.nbytes, store.table.data_ptr(),
              store.table.stride(0), store.seq_blocks.data_ptr(), store.max_blocks, q.data_ptr(), q.stride(0),
              q.stride(1), batch, HQ, HKV, D, 2048, 0.088, 0, ws.data_ptr(), ws.numel(),
              _lib.status_word(q.device).data_ptr(), stream)


def test_single_rank_exchange_equals_packed_attention(cuda):
    k, v, q, bits = _sequence()
    store = _store(cuda, k, v, bits, 0, PAGES)
    qd = q.to(cuda)
    ref = akv.packed_attention(qd, store, 0.088, splits=0)
    lib = _lib.load()
    ws = torch.empty(lib.akv_workspace_bytes(1, HQ, HKV, D, PAGES, 0), dtype=torch.uint8, device=cuda)
    own = _buffer(1)
    peers = (ctypes.c_void_p * 1)(own)
    for epoch in (1, 2, 3):
        out = torch.full_like(qd, float("nan"))
        _decode(store, qd, ws)
        _lib.call("akv_merge_exchange", ws.data_ptr(), 1, HQ, D, peers, 0, 1, epoch, out.data_ptr(), out.stride(0),
                  out.stride(1), _lib.status_word(cuda).data_ptr(), torch.cuda.current_stream(cuda).cuda_stream)
        torch.testing.assert_close(out, ref, atol=1e-3, rtol=1e-3)
    assert akv.take_device_status(cuda) == 0
    _lib.call("akv_ipc_free", ctypes.c_void_p(own))


def test_exchange_wait_runs_out_and_reports(cuda):
    """Rank 0 of a two-rank exchange whose other rank never stores: the words
    that never carry the epoch make the bounded wait give up (2 s), the status
    word reports AKV_DEV_TIMEOUT and the context stays usable."""
    k, v, q, bits = _sequence()
    store = _store(cuda, k, v, bits, 0, PAGES // 2)
    qd = q.to(cuda)
    lib = _lib.load()
    ws = torch.empty(lib.akv_workspace_bytes(1, HQ, HKV, D, store.max_blocks, 0), dtype=torch.uint8, device=cuda)
    own, silent = _buffer(2), _buffer(2)
    peers = (ctypes.c_void_p * 2)(own, silent)
    out = torch.zeros_like(qd)
    _decode(store, qd, ws)
    _lib.call("akv_merge_exchange", ws.data_ptr(), 1, HQ, D, peers, 0, 2, 1, out.data_ptr(), out.stride(0),
              out.stride(1), _lib.status_word(cuda).data_ptr(), torch.cuda.current_stream(cuda).cuda_stream)
    torch.cuda.synchronize(cuda)
    with pytest.raises(akv.KernelError, match="bounded wait"):  # the API's next call reports it
        akv.packed_attention(qd, store, 0.088)
    assert akv.take_device_status(cuda) == 0  # raising cleared the word
    assert (out == 0).all()  # nothing merged
    assert float(torch.ones(4, device=cuda).sum()) == 4.0  # the context still works
    for ptr in (own, silent):
        _lib.call("akv_ipc_free", ctypes.c_void_p(ptr))


def _tagged(values, epoch):
    """Exchange words of fp32 values: the value's bits in the low half, the epoch in the high half."""
    return (values.contiguous().view(torch.int32).to(torch.int64) & 0xFFFFFFFF) | (epoch << 32)


@pytest.mark.parametrize("world, me, batch", [(2, 0, 1), (2, 1, 1), (4, 2, 1), (8, 5, 1), (2, 1, 2), (4, 3, 4)])
def test_exchange_merges_every_rank_on_one_gpu(cuda, world, me, batch):
    """The multi-rank merge on one GPU, with no kernel waiting on another
    kernel: the other ranks' part-states are in this rank's exchange buffer
    before the call, tagged with the call's epoch, as their kernels would have
    stored them over NVLink (rank r's first part = its page range decoded to a
    state by decode_partial_states, its other parts empty).  Rank `me` decodes
    its own range and runs the exchange kernel; three epochs alternate the
    parity halves.  The output matches the oracle over the whole sequence, and
    this rank's own parts land in every rank's buffer tagged with the epoch.
    Batches of 1, 2 and 4 sequences give 32, 64 and 128 rows: four, two and one
    part-states per row."""
    from anchorkv_b200.sharded import shard_range

    k, v, q, bits = _sequence() if batch == 1 else _sequence_batch(batch)
    qd = q.to(cuda)
    lib = _lib.load()
    rows = batch * HQ
    states = {}
    for r in range(world):
        if r != me:
            lo, hi = shard_range(PAGES, r, world)
            st = akv.decode_partial_states(qd, _store(cuda, k, v, bits, lo, hi), 0.088)  # [batch, HQ, D + 2]
            states[r] = st.reshape(rows, D + 2)
    lo, hi = shard_range(PAGES, me, world)
    store = _store(cuda, k, v, bits, lo, hi)
    ws = torch.empty(lib.akv_workspace_bytes(batch, HQ, HKV, D, store.max_blocks, 0), dtype=torch.uint8,
                     device=cuda)
    nbytes = lib.akv_exchange_bytes(world, batch, HQ, D)
    splits = nbytes // (2 * world * rows * (D + 2) * 8)
    assert nbytes == 2 * world * splits * rows * (D + 2) * 8 and splits == {32: 4, 64: 2, 128: 1}[rows]
    bufs = [torch.zeros(nbytes // 8, dtype=torch.int64, device=cuda) for _ in range(world)]
    words = [b.view(2, world, splits, rows, D + 2) for b in bufs]
    peers = (ctypes.c_void_p * world)(*[b.data_ptr() for b in bufs])
    empty = torch.zeros((rows, D + 2), dtype=torch.float32, device=cuda)
    empty[:, D] = -math.inf
    oracle = paged_decode_f64(q[:, :, 0].numpy(), k.numpy(), v.numpy(), bits, 0.088, group=2048)
    for epoch in (1, 2, 3):
        par = epoch & 1
        for r, st in states.items():  # what rank r's kernel would have stored into this rank's buffer
            words[me][par, r, 0] = _tagged(st, epoch)
            for s in range(1, splits):
                words[me][par, r, s] = _tagged(empty, epoch)
        out = torch.full_like(qd, float("nan"))
        _decode(store, qd, ws, batch)
        _lib.call("akv_merge_exchange", ws.data_ptr(), batch, HQ, D, peers, me, world, epoch, out.data_ptr(),
                  out.stride(0), out.stride(1), _lib.status_word(cuda).data_ptr(),
                  torch.cuda.current_stream(cuda).cuda_stream)
        torch.cuda.synchronize(cuda)
        assert akv.take_device_status(cuda) == 0
        np.testing.assert_allclose(out.float().cpu().numpy().reshape(-1), oracle.reshape(-1), atol=2e-3, rtol=1e-2)
        for r in range(world):  # this rank's parts, in every rank's buffer, carry the epoch
            assert bool(((words[r][par, me] >> 32) == epoch).all())


def _rank_main(rank, world, port, queue, epochs=3, delay_rank=None):
    """One rank: its shard of the sequence, ``epochs`` back-to-back calls of
    PeerExchange.attention and one of the NCCL all-gather form.  Rank
    ``delay_rank`` sleeps on the host before most of its calls, so the other
    rank runs ahead by up to one call and waits for it inside the kernel."""
    try:
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        import datetime
        import time

        import torch.distributed as dist

        from anchorkv_b200.sharded import PeerExchange, shard_range, sharded_packed_attention

        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=dev)
        k, v, q, bits = _sequence()
        lo, hi = shard_range(PAGES, rank, world)
        store = _store(dev, k, v, bits, lo, hi)
        qd = q.to(dev)
        ex = PeerExchange(1, HQ, D)
        outs = []
        for e in range(epochs):
            if rank == delay_rank and e % 4 != 3:
                time.sleep(0.002 * (1 + e % 3) ** 2)  # 2, 8 or 18 ms of host delay before the launches
            outs.append(ex.attention(qd, store, 0.088))
        outs = [o.float().cpu() for o in outs]
        nccl = sharded_packed_attention(qd, store, 0.088).float().cpu()
        status = akv.take_device_status(dev)
        ex.close()
        dist.destroy_process_group()
        queue.put((rank, status, [o.numpy() for o in outs], nccl.numpy()))
    except Exception as exc:  # reported to the parent, which fails the test
        queue.put((rank, -1, repr(exc), None))


def _run_ranks(world, **kw):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, queue), kwargs=kw) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in procs:
        rank, status, outs, nccl = queue.get(timeout=240)
        results[rank] = (status, outs, nccl)
    for p in procs:
        p.join(timeout=60)
    assert all(results[r][0] == 0 for r in results), results
    return results


def _oracle():
    k, v, q, bits = _sequence()
    return paged_decode_f64(q[:, :, 0].numpy(), k.numpy(), v.numpy(), bits, 0.088, group=2048)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_rank_exchange_against_oracle():
    results = _run_ranks(2)
    oracle = _oracle()
    for r in (0, 1):
        for out in results[r][1]:
            np.testing.assert_allclose(out.reshape(-1), oracle.reshape(-1), atol=2e-3, rtol=1e-2)
    np.testing.assert_array_equal(results[0][1][0], results[1][1][0])


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_rank_exchange_with_a_delayed_rank():
    """Twelve back-to-back epochs while rank 1 sleeps on the host before most
    calls: rank 0's kernels run up to one call ahead and wait for rank 1's
    states inside the kernel.  The epoch-parity halves of the exchange buffers
    keep every call's states apart, so no wait runs out (status 0 on both
    ranks), every output is within tolerance of the oracle, both ranks agree
    bit for bit, and the NCCL all-gather form gives the same result."""
    results = _run_ranks(2, epochs=12, delay_rank=1)
    oracle = _oracle()
    for r in (0, 1):
        status, outs, nccl = results[r]
        assert len(outs) == 12
        for out in outs:
            np.testing.assert_allclose(out.reshape(-1), oracle.reshape(-1), atol=2e-3, rtol=1e-2)
            np.testing.assert_array_equal(out, outs[0])  # the same inputs every epoch
        np.testing.assert_allclose(nccl.reshape(-1), outs[0].reshape(-1), atol=1e-3, rtol=1e-3)
    np.testing.assert_array_equal(results[0][1][-1], results[1][1][-1])


def test_exchange_merges_every_rank_on_one_gpu_head_dim_64(cuda):
    """The prefilled multi-rank merge at head_dim 64 (two words per lane, 66
    words per state): 3 ranks, rank 2 here, 16 query / 4 KV heads."""
    from anchorkv_b200.sharded import shard_range

    hq, hkv, dim, pages, world, me = 16, 4, 64, 120, 3, 2
    k = W.outlier_kv(61, (1, hkv, 16 * pages, dim))
    v = W.outlier_kv(62, (1, hkv, 16 * pages, dim))
    q = W.normal(63, (1, hq, 1, dim))
    bits = np.array(W.draw_modes(64, pages, {16: .1, 8: .3, 4: .6}))[None]
    qd = q.to(cuda)

    def store(lo, hi):
        sub = bits[:, lo:hi]
        pool = P.PagePool(hkv, dim, group=16 * dim, pages={b: int((sub == b).sum()) for b in (16, 8, 4)},
                          device=cuda)
        return P.pack_dense(pool, k[:, :, 16 * lo:16 * hi].to(cuda), v[:, :, 16 * lo:16 * hi].to(cuda), sub)

    lib = _lib.load()
    states = {r: akv.decode_partial_states(qd, store(*shard_range(pages, r, world)), 0.1)[0]
              for r in range(world) if r != me}
    mine = store(*shard_range(pages, me, world))
    ws = torch.empty(lib.akv_workspace_bytes(1, hq, hkv, dim, mine.max_blocks, 0), dtype=torch.uint8, device=cuda)
    nbytes = lib.akv_exchange_bytes(world, 1, hq, dim)
    splits = nbytes // (2 * world * hq * (dim + 2) * 8)
    assert splits == 4
    bufs = [torch.zeros(nbytes // 8, dtype=torch.int64, device=cuda) for _ in range(world)]
    words = [b.view(2, world, splits, hq, dim + 2) for b in bufs]
    peers = (ctypes.c_void_p * world)(*[b.data_ptr() for b in bufs])
    empty = torch.zeros((hq, dim + 2), dtype=torch.float32, device=cuda)
    empty[:, dim] = -math.inf
    oracle = paged_decode_f64(q[:, :, 0].numpy(), k.numpy(), v.numpy(), bits, 0.1, group=16 * dim)
    stream = torch.cuda.current_stream(cuda).cuda_stream
    for epoch in (1, 2, 3):
        par = epoch & 1
        for r, st in states.items():
            words[me][par, r, 0] = _tagged(st, epoch)
            for s in range(1, splits):
                words[me][par, r, s] = _tagged(empty, epoch)
        out = torch.full_like(qd, float("nan"))
        _lib.call("akv_decode_partials", mine.pool.arena.data_ptr(), mine.pool.nbytes, mine.table.data_ptr(),
                  mine.table.stride(0), mine.seq_blocks.data_ptr(), mine.max_blocks, qd.data_ptr(), qd.stride(0),
                  qd.stride(1), 1, hq, hkv, dim, 16 * dim, 0.1, 0, ws.data_ptr(), ws.numel(),
                  _lib.status_word(cuda).data_ptr(), stream)
        _lib.call("akv_merge_exchange", ws.data_ptr(), 1, hq, dim, peers, me, world, epoch, out.data_ptr(),
                  out.stride(0), out.stride(1), _lib.status_word(cuda).data_ptr(), stream)
        torch.cuda.synchronize(cuda)
        assert akv.take_device_status(cuda) == 0
        np.testing.assert_allclose(out.float().cpu().numpy().reshape(-1), oracle.reshape(-1), atol=2e-3, rtol=1e-2)
