"""The long-context sharded decode on world-size-2 gloo CPU ranks.

Each rank holds a contiguous shard of one sequence's pages; the per-rank LSE
states are all-gathered and merged.  The device kernels are replaced by the
oracle here (host stand-ins); the collective, the shard geometry and the merge
algebra are the code under test.  A rank that raises before the collective is
reported instead of hanging the other rank (short process-group timeout)."""

import math
import os
import socket
from datetime import timedelta

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from anchorkv_b200.sharded import shard_range, sharded_packed_attention
from oracle import attention as OA


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _states_f64(q, k, v, scale):
    """Oracle LSE state per query head: (acc, m [base 2], l) like decode_partial_states."""
    hq, d = q.shape
    hkv = k.shape[0]
    g = hq // hkv
    out = np.zeros((1, hq, d + 2))
    for h in range(hq):
        if k.shape[1] == 0:
            out[0, h, d] = -np.inf
            continue
        s = (k[h // g] @ q[h]) * scale * math.log2(math.e)
        m = s.max()
        p = np.exp2(s - m)
        out[0, h, :d] = p @ v[h // g]
        out[0, h, d] = m
        out[0, h, d + 1] = p.sum()
    return torch.from_numpy(out)


def _merge_f64(states):
    st = states.numpy()
    n, b, hq, rs = st.shape
    res = np.zeros((b, hq, 1, rs - 2))
    for h in range(hq):
        parts = [(st[i, 0, h, :-2], st[i, 0, h, -2], st[i, 0, h, -1]) for i in range(n)]
        top = max(m for _, m, _ in parts)
        w = [0.0 if m == -np.inf else 2.0 ** (m - top) for _, m, _ in parts]
        num = sum(wi * a for wi, (a, _, _) in zip(w, parts))
        den = sum(wi * l for wi, (_, _, l) in zip(w, parts))
        res[0, h, 0] = num / den
    return torch.from_numpy(res)


def _worker(rank, world, port, fail_rank, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    try:
        g = torch.Generator().manual_seed(0)
        tokens, hkv, hq, d = 16 * 37, 2, 8, 64
        k = torch.randn(hkv, tokens, d, generator=g, dtype=torch.float64)
        v = torch.randn(hkv, tokens, d, generator=g, dtype=torch.float64)
        q = torch.randn(hq, d, generator=g, dtype=torch.float64)
        lo, hi = shard_range(tokens // 16, rank, world)
        shard = (k[:, 16 * lo:16 * hi].numpy(), v[:, 16 * lo:16 * hi].numpy())
        if rank == fail_rank:
            raise RuntimeError("injected failure before the collective")
        out = sharded_packed_attention(
            q.numpy(), shard, 0.125,
            local_states=lambda qq, st, sc, splits=0: _states_f64(qq, st[0], st[1], sc),
            merge=_merge_f64)
        full = OA.attention_f64(q.numpy(), k.numpy(), v.numpy(), 0.125)
        results[rank] = float(np.abs(out.numpy()[0, :, 0] - full).max())
    except Exception as e:  # noqa: BLE001 - reported to the parent
        results[rank] = f"{type(e).__name__}: {e}"
    finally:
        dist.destroy_process_group()


def _run(world, fail_rank=-1):
    ctx = mp.get_context("spawn")
    port = _free_port()
    with ctx.Manager() as mgr:
        results = mgr.dict()
        procs = [ctx.Process(target=_worker, args=(r, world, port, fail_rank, results)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
            if p.is_alive():
                p.kill()
        return dict(results)


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_lse_merge_matches_full_context(world):
    res = _run(world)
    assert len(res) == world
    for r in range(world):
        assert isinstance(res[r], float), res[r]
        assert res[r] < 1e-10


def test_shard_ranges_tile_the_sequence():
    for n in (0, 1, 7, 64, 65536, 100003):
        for world in (1, 2, 3, 8):
            ranges = [shard_range(n, r, world) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
            sizes = [hi - lo for lo, hi in ranges]
            assert max(sizes) - min(sizes) <= 1


def test_rank_failure_before_collective_is_reported_not_hung():
    res = _run(2, fail_rank=1)
    assert "injected failure" in str(res.get(1))
    assert isinstance(res.get(0), str)  # the surviving rank's collective errored out (timeout / closed peer)
