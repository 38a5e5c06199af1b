#!/usr/bin/env python
"""Benchmark of the packed mixed-precision KV decode path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload batched]
    python bench.py --impl reference_gpu   # the reference's own Triton decode beside ours (batch 1)

A step is one decode token for every sequence of the batch through all layers:
per layer, the paged split-K decode kernel and the LSE merge kernel over that
layer's page table (one launch each).  The default workload is the batched
Qwen3-0.6B attention shape: 28 layers, 16 query / 8 KV heads, head_dim 128,
batch 64, 8192-token context in 16-token pages; per page FP16 / INT8 / INT4 /
evicted = 15 / 35 / 40 / 10 %, per-block-per-KV-head fp16 scales, the page
tables a random permutation of one shared physical pool, split-K 8, fp16
N(0, 1) inputs (synthetic, seeded).  Under torchrun every rank decodes its
own batch of 64 sequences (weak scaling, no collective on the data path).

value: resident-KV GB/s of the whole job (algorithmic bytes: non-evicted page
payload + scales, plus queries and outputs, divided by the max-over-ranks
device time per step); the KV pool (25.6 GB per GPU) is far larger than L2,
so every step reads HBM.  e2e: the same metric through the public Python
entry point with the step's queries copied from pinned host memory and the
outputs read back inside the timed region.

--impl reference times the reference's PyTorch CPU path (the reference arm);
--impl reference_gpu runs the reference's own GPU decode (its Triton kernel,
installed unmodified in baseline/_ref) and ours on the same pages, at the
batch-1, group-64 shapes that kernel supports.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (str(ROOT / "dynamic-quantization_b200"), str(ROOT)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "decode-attn resident-KV GB/s (% B200 HBM peak) & tokens/s at 1/2/4/8 GPUs"
FALLBACK_HBM_GBS = 6650.0

WORKLOADS = {
    "batched": dict(
        name="batched decode, Qwen3-0.6B attention shape",
        layers=28, q_heads=16, kv_heads=8, dim=128, batch=64, tokens=8192,
        mix={16: 0.15, 8: 0.35, 4: 0.40, 0: 0.10}, splits=8, group=2048),
    # One layer of the same step (916 MB of KV, > L2; under 1 GB on the device):
    # the case full ncu captures are taken on, its launches identical to the
    # step's.
    # 36 layers x 128 sequences x 32,768 tokens, 32 query / 8 KV heads (GQA 4),
    # INT4-heavy: 220 GB of KV per step, sequences sharded across the GPUs
    # (strong scaling, no collective).  Layers cycle over as many distinct
    # stores as fit a GPU; every launch still streams its whole store from HBM.
    "large": dict(
        name="large-batch decode, Qwen3-8B-like attention shape (GQA 4)",
        layers=36, q_heads=32, kv_heads=8, dim=128, batch=128, tokens=32768,
        mix={16: 0.095, 8: 0.19, 4: 0.665, 0: 0.05}, splits=8, group=2048, strong=True, outliers=True),
    "batched_small": dict(
        name="batched decode, Qwen3-0.6B attention shape, 1 layer (profiling case)",
        layers=1, q_heads=16, kv_heads=8, dim=128, batch=64, tokens=8192,
        mix={16: 0.15, 8: 0.35, 4: 0.40, 0: 0.10}, splits=8, group=2048),
}


# One sequence of 1,048,576 tokens (65,536 pages), 32 query / 8 KV heads,
# 5/25/70 FP16/INT8/INT4, split contiguously across the GPUs (strong scaling):
# each rank decodes its shard into LSE states, NCCL all-gathers them, every
# rank merges.  A step is one layer's decode of the whole context.
LONG = dict(
    name="long-context single-sequence decode, 1,048,576 tokens, sequence-sharded",
    layers=1, q_heads=32, kv_heads=8, dim=128, batch=1, tokens=1 << 20,
    mix={16: 0.05, 8: 0.25, 4: 0.70}, group=2048)

PACK = dict(
    name="requantize/pack, 28 layers x 32 sequences x 8 KV heads x 4096 tokens x 128 dims",
    layers=28, batch=32, kv_heads=8, tokens=4096, dim=128, group=2048,
    mix={16: 0.20, 8: 0.30, 4: 0.50})
# 2 layers x 8 sequences (268 MB of fp16 input, > L2): the pack profiling case.
PACK_SMALL = dict(PACK, name="requantize/pack, 2 layers x 8 sequences (profiling case)", layers=2, batch=8)


def hbm_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def traffic_for(name: str):
    """DRAM traffic per launch of kernel case ``name`` from ``profiles/traffic.json``
    (one ncu capture each, with the command that made it), or None."""
    f = ROOT / "profiles" / "traffic.json"
    if not f.exists():
        return None
    entry = json.loads(f.read_text()).get(name)
    if not entry:
        return None
    return {"bytes_per_launch": float(entry["bytes_per_launch"]), "source": entry["source"]}


class ClockSampler:
    """nvidia-smi SM clock / throttle-reason samples while the timed region runs."""

    FIELDS = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_id: str):
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", gpu_id, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        time.sleep(0.15)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.seek(0)
        rows = [r.split(",") for r in self.file.read().strip().splitlines() if r.count(",") >= 5]
        os.unlink(self.file.name)
        if not rows:
            return None
        sm = [float(r[0]) for r in rows if r[0].strip().replace(".", "").isdigit()]
        mx = [float(r[1]) for r in rows if r[1].strip().replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if "Active" in r[2 + i] and "Not" not in r[2 + i]})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# --------------------------------------------------------------- CPU baseline
REF_DIR = ROOT / "baseline" / "_ref"


def import_reference():
    """The unmodified reference package installed in baseline/_ref: returns
    (packed_decode module, None) or (None, why it is not importable)."""
    if str(REF_DIR) not in sys.path:
        sys.path.insert(0, str(REF_DIR))
    try:
        from anchorkv import packed_decode as ref_pd
    except Exception as exc:  # not installed here, or a dependency is missing
        return None, f"reference not importable from {REF_DIR}: {type(exc).__name__}: {exc}"
    return ref_pd, None


def cpu_baseline(wl: dict, seed: int, seconds: float, calls_min: int = 3):
    """Time the reference's own CPU decode path on one sequence-layer of the
    workload for about ``seconds`` with all host cores; returns a dict.

    The reference (baseline/_ref, unmodified) holds a batch-one sequence in its
    ``PagedLayer`` (packed_decode.py:108-194) and decodes with
    ``dense_attention`` (packed_decode.py:197-203): every call dequantises all
    pages to fp16, concatenates them and runs SDPA.  Its layer has no eviction,
    so evicted blocks are left out of it, as ``materialize_segments`` drops them
    (backend.py:557-591); each kept page is demoted to the block's precision with
    ``PagedLayer.demote``.  Its pages take one scale per 64 elements (the layer
    requires groups along head_dim), the workload's one per (block, KV head):
    bytes are counted in the workload's layout, as for the GPU arm.  If the
    reference cannot be imported, the CPU restatement in oracle/baseline.py is
    timed instead and the result says so."""
    import numpy as np
    import torch

    from anchorkv_b200 import pool as P

    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    # Contexts beyond 65,536 tokens are timed on a 65,536-token contiguous slice;
    # tokens/s is scaled by the number of slices.
    blocks = min(wl["tokens"], 65536) // 16
    slices = wl["tokens"] // (blocks * 16)
    Hq, Hkv, D = wl["q_heads"], wl["kv_heads"], wl["dim"]
    keys = list(wl["mix"])
    bits = np.random.default_rng(seed).choice(np.array(keys), size=blocks, p=[wl["mix"][k] for k in keys])
    gen = torch.Generator().manual_seed(seed)
    q = torch.randn(1, Hq, 1, D, generator=gen).half()
    scale = 1 / math.sqrt(D)
    nbytes = sum(P.algorithmic_record_bytes(D, wl["group"], int(b)) * Hkv for b in bits if b) + 2 * q.numel() * 2
    ref_pd, why = import_reference()
    if ref_pd is not None:
        kept = np.nonzero(bits)[0]
        k = torch.randn(1, Hkv, blocks * 16, D, generator=gen).half()
        v = torch.randn(1, Hkv, blocks * 16, D, generator=gen).half()
        tok = torch.from_numpy((kept[:, None] * 16 + np.arange(16)[None, :]).reshape(-1))
        layer = ref_pd.PagedLayer(Hkv, D, len(tok), group=64, archive_bits=16, device="cpu")
        layer.append(k[:, :, tok], v[:, :, tok])
        for page, b in enumerate(bits[kept]):
            if b != 16:
                layer.demote(page, int(b))

        def call():
            return ref_pd.dense_attention(q, layer, scale)

        kind, what = "reference", ("the reference's PagedLayer (baseline/_ref, unmodified; group 64) + "
                                   "dense_attention")
    else:
        from oracle import baseline as OB

        pages = OB.build_sequence(seed, Hkv, D, blocks, bits, wl["group"])

        def call():
            return OB.decode_cpu(pages, q, scale)

        kind, what = "port", f"fallback, {why}: the CPU restatement oracle/baseline.decode_cpu"
    call()  # warm
    times = []
    t_end = time.perf_counter() + seconds
    while len(times) < calls_min or time.perf_counter() < t_end:
        t0 = time.perf_counter()
        call()
        times.append(time.perf_counter() - t0)
    per_call = statistics.median(times)
    calls_per_step = wl["layers"] * wl["batch"] * slices
    return {
        "gbs": nbytes / per_call / 1e9,
        "tokens_per_s": wl["batch"] / (per_call * calls_per_step),
        "cores": cores,
        "kind": kind,
        "calls": len(times),
        "seconds_per_call": per_call,
        "seconds_timed": sum(times),
        "calls_per_step": calls_per_step,
        "sample": (f"{len(times)} decode calls of {what} on one sequence-layer slice ({blocks} pages, "
                   f"{Hkv} KV heads, the workload's precision mix), median per call, {cores} threads; "
                   f"a full step is {calls_per_step} such calls"),
    }


# ------------------------------------------------------------------ GPU setup
# Device bytes the KV stores of one GPU may take (the rest holds the fp16
# staging of one layer, queries and workspaces).
STORE_BUDGET = 120e9


def layer_store_bytes(wl: dict, batch: int) -> float:
    """Expected arena bytes of one layer's store at the workload's precision mix."""
    from anchorkv_b200 import pool as P

    pages = batch * (wl["tokens"] // 16)
    per_page = sum(p * P.record_bytes(wl["dim"], wl["group"], b) * wl["kv_heads"]
                   for b, p in wl["mix"].items() if b)
    return pages * per_page


def workload_bits(wl: dict, seed: int, batch: int, distinct: int):
    """Per-page precisions (16 / 8 / 4 / 0 = evicted) of ``distinct`` layer stores."""
    import numpy as np

    rng = np.random.default_rng(seed)
    keys = list(wl["mix"])
    probs = np.array([wl["mix"][k] for k in keys])
    return [rng.choice(np.array(keys), size=(batch, wl["tokens"] // 16), p=probs) for _ in range(distinct)]


def batched_plan(wl: dict, world: int):
    """(sequences per rank, distinct layer stores per rank, arena bytes of rank 0's pool):
    what run_ours builds, worked out on the host."""
    from anchorkv_b200 import pool as P

    strong = bool(wl.get("strong"))
    B = wl["batch"] // world if strong else wl["batch"]
    distinct = max(1, min(wl["layers"], int(STORE_BUDGET // layer_store_bytes(wl, B))))
    bits = workload_bits(wl, 1234, B, distinct)
    arena = sum(int(sum((x == b).sum() for x in bits)) * wl["kv_heads"] * P.record_bytes(wl["dim"], wl["group"], b)
                for b in (16, 8, 4))
    return B, distinct, max(arena, 16)


def batched_config(wl: dict, world: int, B: int, distinct: int, arena_bytes: int) -> dict:
    """The ``config`` of a batched/large line (both arms print the same one)."""
    strong = bool(wl.get("strong"))
    return {
        "workload": wl["name"], "layers": wl["layers"], "q_heads": wl["q_heads"], "kv_heads": wl["kv_heads"],
        "head_dim": wl["dim"], "batch_per_gpu": B, "context_tokens": wl["tokens"], "page_tokens": 16,
        "precision_mix": {"fp16": wl["mix"][16], "int8": wl["mix"][8], "int4": wl["mix"][4],
                          "evicted": wl["mix"][0]},
        "scale_group": wl["group"], "split_k": wl["splits"],
        "kv_pool_gb_per_gpu": round(arena_bytes / 1e9, 2),
        "distinct_layer_stores": distinct,
        "parallelism": f"batch-sharded x{world} (independent sequences, no collective)",
        "l2": "inputs larger than L2 (KV pool >> 126 MB), no flush needed",
    } | ({"strong_scaling_total_batch": wl["batch"]} if strong else {})


def build_workload(wl: dict, device, seed: int, batch: int | None = None, distinct: int | None = None):
    """Packed stores for ``distinct`` layers (all of them by default) of ``batch``
    sequences each; layer l of the step uses store l % distinct.  Returns
    (pool, stores per layer, queries [L, batch, Hq, 1, D], KV bytes per layer)."""
    import numpy as np
    import torch

    from anchorkv_b200 import pool as P

    batch = wl["batch"] if batch is None else batch
    distinct = wl["layers"] if distinct is None else distinct
    bits = workload_bits(wl, seed, batch, distinct)
    counts = {b: int(sum((x == b).sum() for x in bits)) for b in (16, 8, 4)}
    pool = P.PagePool(wl["kv_heads"], wl["dim"], group=wl["group"], pages=counts, device=device,
                      shuffle_seed=seed, zero=False)
    gen = torch.Generator(device=device).manual_seed(seed)
    shape = (batch, wl["kv_heads"], wl["tokens"], wl["dim"])
    k = torch.empty(shape, dtype=torch.float16, device=device)
    v = torch.empty_like(k)

    def outliers(x):  # 4 channels per (sequence, head) scaled by +-8
        ch = torch.randint(0, wl["dim"], shape[:2] + (4,), generator=gen, device=device)
        sign = torch.where(torch.rand(shape[:2] + (4,), generator=gen, device=device) < 0.5, -8.0, 8.0)
        x.mul_(torch.ones(shape[:2] + (wl["dim"],), device=device).scatter_(2, ch, sign).half()[:, :, None, :])

    stores = []
    for layer_bits in bits:
        k.normal_(generator=gen)
        v.normal_(generator=gen)
        if wl.get("outliers"):
            outliers(k)
            outliers(v)
        stores.append(P.pack_dense(pool, k, v, layer_bits, semantics="tensor"))
    del k, v
    q = torch.randn((wl["layers"], batch, wl["q_heads"], 1, wl["dim"]), generator=gen,
                    device=device, dtype=torch.float32).half()
    torch.cuda.synchronize(device)
    layers = [stores[l % distinct] for l in range(wl["layers"])]
    kv_bytes = [t.resident_bytes() for t in layers]
    return pool, layers, q, kv_bytes


def run_ours(args, wl):
    import torch
    import torch.distributed as dist

    import anchorkv_b200 as akv
    from anchorkv_b200 import _lib

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    strong = bool(wl.get("strong"))
    if strong and wl["batch"] % world:
        raise SystemExit(f"{wl['batch']} sequences do not split evenly over {world} GPUs")
    B, distinct, _ = batched_plan(wl, world)  # sequences and distinct layer stores this rank holds
    pool, layers, q, kv_bytes = build_workload(wl, device, seed=1234 + rank, batch=B, distinct=distinct)
    L, Hq, D = wl["layers"], wl["q_heads"], wl["dim"]
    splits, scale = wl["splits"], 1 / math.sqrt(D)
    io_bytes = q[0].numel() * 2 * 2  # queries in + outputs out, per layer
    step_bytes = sum(kv_bytes) + L * io_bytes
    out = torch.empty_like(q)
    lib = _lib.load()
    ws_bytes = lib.akv_workspace_bytes(B, Hq, wl["kv_heads"], D, wl["tokens"] // 16, splits)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    sptr = stream.cuda_stream
    status = _lib.status_word(device)

    def attend(l):  # the C-ABI drop-in: decode, then merge (2 launches)
        t = layers[l]
        return lib.akv_packed_attention(pool.arena.data_ptr(), pool.nbytes, t.table.data_ptr(), t.table.stride(0),
                                        t.seq_blocks.data_ptr(), t.max_blocks, q[l].data_ptr(), q[l].stride(0),
                                        q[l].stride(1), B, Hq, wl["kv_heads"], D, wl["group"], scale, splits,
                                        out[l].data_ptr(), out[l].stride(0), out[l].stride(1), ws.data_ptr(),
                                        ws_bytes, status.data_ptr(), sptr)

    def step():
        for l in range(L):
            assert attend(l) == 0

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize(device)

    for _ in range(args.warmup):
        step()
    barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    gpu_id = "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
    sampler = ClockSampler(gpu_id)
    time.sleep(0.3)
    t0.record(stream)
    for i in range(args.steps):
        step()
    t1.record(stream)
    barrier()
    clocks = sampler.stop()
    ms_local = t0.elapsed_time(t1) / args.steps
    assert akv.take_device_status(device) == 0, "device status word set during the timed region"
    # The decode kernel alone (events on its stream around each launch; the
    # events break the overlap of the two launches, so this is a separate pass).
    dec_steps = max(3, args.steps // 5)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(dec_steps * L)]
    for i in range(dec_steps):
        for l in range(L):
            t = layers[l]
            ev[i * L + l][0].record(stream)
            assert lib.akv_decode_partials(pool.arena.data_ptr(), pool.nbytes, t.table.data_ptr(),
                                           t.table.stride(0), t.seq_blocks.data_ptr(), t.max_blocks,
                                           q[l].data_ptr(), q[l].stride(0), q[l].stride(1), B, Hq, wl["kv_heads"],
                                           D, wl["group"], scale, splits, ws.data_ptr(), ws_bytes,
                                           status.data_ptr(), sptr) == 0
            ev[i * L + l][1].record(stream)
    barrier()
    dec_ms_mean = sum(a.elapsed_time(b) for a, b in ev) / len(ev)

    # ---- end to end through the public API, pinned host buffers
    q_host = q.cpu().pin_memory()
    out_host = torch.empty(q.shape, dtype=q.dtype).pin_memory()
    q_dev = torch.empty_like(q)
    copies = torch.cuda.Stream(device)
    # Layers travel in groups: queries in [0], [1-4], [5-8], ...; outputs back in
    # [0-3], [4-7], ..., with the last layer alone, so the first decode waits for
    # one layer's query and the step's end for one layer's output.
    in_groups = [(0, min(1, L))] + [(g, min(g + 4, L)) for g in range(1, L, 4)]
    out_cuts = list(range(0, L - 1, 4)) + [L - 1, L] if L > 1 else [0, L]
    out_groups = [(a, b) for a, b in zip(out_cuts[:-1], out_cuts[1:]) if a < b]
    ev_in = [torch.cuda.Event() for _ in in_groups]
    ev_out = [torch.cuda.Event() for _ in out_groups]
    in_first = {g0: i for i, (g0, _) in enumerate(in_groups)}
    out_last = {g1 - 1: i for i, (_, g1) in enumerate(out_groups)}

    def e2e_step():
        # The queries go in from pinned memory on a copy stream, a group at a
        # time; a group's first layer waits for the group's copy and its outputs
        # come back as soon as the group's last merge has run.  Between the
        # other layers no stream dependency sits between the kernels, so each
        # decode still launches as a programmatic dependent of the merge before
        # it.  The step ends when the last output is on the host.
        copies.wait_stream(stream)  # the previous step is done with q_dev
        with torch.cuda.stream(copies):
            for i, (g0, g1) in enumerate(in_groups):
                q_dev[g0:g1].copy_(q_host[g0:g1], non_blocking=True)
                ev_in[i].record(copies)
        for l in range(L):
            if l in in_first:
                stream.wait_event(ev_in[in_first[l]])
            akv.packed_attention(q_dev[l], layers[l], scale, splits=splits, out=out[l])
            if l in out_last:
                ev_out[out_last[l]].record(stream)
        with torch.cuda.stream(copies):
            for i, (g0, g1) in enumerate(out_groups):
                copies.wait_event(ev_out[i])
                out_host[g0:g1].copy_(out[g0:g1], non_blocking=True)
        stream.wait_stream(copies)

    for _ in range(max(3, args.warmup)):
        e2e_step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_steps = max(10, args.steps // 4)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    barrier()
    e2e_ms_local = e0.elapsed_time(e1) / e2e_steps

    # ---- sustained: at least 1 s of back-to-back steps with its own clock record
    # (the timed region above may be a short burst at boost clocks; the 1 kW
    # power cap settles the SM clock lower within about a second)
    sus_steps = max(args.steps, int(math.ceil(args.sustained_seconds * 1e3 / max(ms_local, 1e-3))))
    barrier()
    sus_sampler = ClockSampler(gpu_id)
    time.sleep(0.3)
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record(stream)
    for _ in range(sus_steps):
        step()
    s1.record(stream)
    barrier()
    sus_clocks = sus_sampler.stop()
    sus_ms_local = s0.elapsed_time(s1) / sus_steps
    assert akv.take_device_status(device) == 0, "device status word set during the sustained region"

    times = torch.tensor([ms_local, e2e_ms_local, dec_ms_mean, sus_ms_local], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    ms, e2e_ms, dec_ms_max, sus_ms = times.tolist()
    long_leg = None if args.no_long else long_context_leg(args, device, rank, world, local)
    peak, peak_kind = hbm_peak()
    if rank == 0:
        total_bytes = step_bytes * world
        gbs = total_bytes / (ms * 1e-3) / 1e9
        tokens = B * world / (ms * 1e-3)
        achieved = (step_bytes / L) / (dec_ms_mean * 1e-3) / 1e9
        traffic = traffic_for(f"decode_streamk_{args.workload}") if not args.mix else None
        line = {
            "metric": METRIC, "value": round(gbs, 1), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "strong" if strong else "weak", "vs_baseline": None,
            "dtype": "f16 operands, f32 accumulation",
            "data": "synthetic (seeded fp16 N(0,1)" + (", 4 outlier channels per head x(+-8))" if wl.get("outliers")
                                                        else ")"),
            "config": batched_config(wl, world, B, distinct, pool.nbytes),
            "tokens_per_s": round(tokens, 1),
            "pct_of_hbm_peak": round(100 * gbs / world / peak, 2),
            "resident_bytes_per_step_per_gpu": step_bytes,
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": f"{peak_kind} hbm_gbs",
                         "kernel": "decode_streamk_kernel<128>",
                         "traffic": None if traffic is None else traffic["bytes_per_launch"],
                         "traffic_source": None if traffic is None else traffic["source"],
                         "algorithmic_bytes_per_launch": step_bytes // L,
                         "launch_ms_mean": round(dec_ms_mean, 5), "launch_ms_max_over_ranks": round(dec_ms_max, 5)},
            "e2e": {"value": round(total_bytes / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                    "ms_per_step": round(e2e_ms, 4), "tokens_per_s": round(B * world / (e2e_ms * 1e-3), 1),
                    "h2d_bytes_per_step": q.numel() * 2, "d2h_bytes_per_step": out.numel() * 2,
                    "path": "anchorkv_b200.packed_attention per layer; queries from pinned host memory and "
                            "outputs back to it on a copy stream in groups of up to 4 layers (the first query and "
                            "the last output alone), overlapping the other layers' decode"},
            "gpu_launches": args.steps * L * 2,
            "clocks": clocks,
            "sustained": {"steps": sus_steps, "seconds": round(sus_ms * sus_steps / 1e3, 3),
                          "ms_per_step": round(sus_ms, 4),
                          "value": round(total_bytes / (sus_ms * 1e-3) / 1e9, 1), "unit": "GB/s",
                          "tokens_per_s": round(B * world / (sus_ms * 1e-3), 1),
                          "pct_of_hbm_peak": round(100 * total_bytes / (sus_ms * 1e-3) / 1e9 / world / peak, 2),
                          "clocks": sus_clocks},
        }
        if long_leg is not None:
            line["long_context"] = long_leg
        if world == 1 and not args.no_cpu_baseline:
            cb = cpu_baseline(wl, seed=99, seconds=args.cpu_seconds)
            line["cpu_baseline"] = {"value": round(cb["gbs"], 4), "unit": "GB/s", "cores": cb["cores"],
                                    "kind": cb["kind"], "sample": cb["sample"],
                                    "tokens_per_s": round(cb["tokens_per_s"], 4)}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


def pack_cpu_baseline(seconds: float):
    """The reference codec (quantize_tensor per 16-token slab, restated in numpy)
    timed on the host for about ``seconds``."""
    import numpy as np

    from oracle import codec as OC

    rng = np.random.default_rng(5)
    slabs = (rng.standard_normal((64, 16, 128)) * 1.0).astype(np.float16)
    bits = rng.choice(np.array([16, 8, 4]), size=64, p=[0.2, 0.3, 0.5])
    nbytes = 0
    done = 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < seconds or done < 64:
        i = done % 64
        x = slabs[i]
        nbytes += x.nbytes
        if bits[i] == 16:
            nbytes += x.astype(np.float16).nbytes
        else:
            payload, scales = OC.quantize_tensor(x, int(bits[i]), 2048)
            nbytes += payload.nbytes + scales.nbytes
        done += 1
    dt = time.perf_counter() - t0
    return {"gbs": nbytes / dt / 1e9, "cores": 1,
            "sample": f"{done} 16x128 fp16 slabs through the numpy restatement of quantize_tensor, one core"}


def run_pack(args, wl):
    """Bulk requantize/pack of dense fp16 K/V into page records (one launch per step)."""
    import numpy as np
    import torch

    import anchorkv_b200 as akv
    from anchorkv_b200 import _lib
    from anchorkv_b200 import pool as P

    device = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(device)
    L, B, H, T, D = wl["layers"], wl["batch"], wl["kv_heads"], wl["tokens"], wl["dim"]
    nblk = T // 16
    rng = np.random.default_rng(7)
    keys = list(wl["mix"])
    bits = rng.choice(np.array(keys), size=(L * B, nblk), p=[wl["mix"][k] for k in keys])
    counts = {b: int((bits == b).sum()) for b in (16, 8, 4)}
    pool = P.PagePool(H, D, group=wl["group"], pages=counts, device=device, shuffle_seed=11, zero=False)
    codes = np.zeros_like(bits)
    offsets = np.zeros(bits.shape, np.int64)
    for b_, mode in P.BITS_TO_MODE.items():
        where = bits == b_
        offsets[where] = pool.alloc_many(b_, int(where.sum()))
        codes[where] = mode
    desc = torch.from_numpy(P.encode_array(codes, np.full(bits.shape, 16), offsets).reshape(-1)).to(device)
    gen = torch.Generator(device=device).manual_seed(3)
    src = []
    for _ in range(2):  # K and V: N(0,1) with 4 outlier channels per head scaled x(+-8)
        x = torch.empty((L * B, H, T, D), dtype=torch.float16, device=device).normal_(generator=gen)
        ch = torch.randint(0, D, (L * B, H, 4), generator=gen, device=device)
        sign = torch.where(torch.rand((L * B, H, 4), generator=gen, device=device) < 0.5, -8.0, 8.0)
        fac = torch.ones((L * B, H, D), device=device).scatter_(2, ch, sign).half()
        x.mul_(fac[:, :, None, :])
        src.append(x)
    k, v = src
    status = _lib.status_word(device)
    stream = torch.cuda.current_stream(device)
    lib = _lib.load()
    n_pages = L * B * nblk
    read = 2 * k.numel() * 2
    written = sum(counts[b] * P.algorithmic_record_bytes(D, wl["group"], b) * H for b in (16, 8, 4))

    def step():
        assert lib.akv_pack_pages(k.data_ptr(), v.data_ptr(), H * T * D, T * D, nblk, n_pages, desc.data_ptr(),
                                  pool.arena.data_ptr(), pool.nbytes, H, D, wl["group"], _lib.SEM_TENSOR,
                                  status.data_ptr(), stream.cuda_stream) == 0

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(device)
    gpu_id = "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
    sampler = ClockSampler(gpu_id)
    time.sleep(0.3)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(args.steps):
        step()
    t1.record(stream)
    torch.cuda.synchronize(device)
    clocks = sampler.stop()
    assert akv.take_device_status(device) == 0
    ms = t0.elapsed_time(t1) / args.steps
    peak, peak_kind = hbm_peak()
    gbs = (read + written) / (ms * 1e-3) / 1e9
    # e2e: one layer's K/V copied in from pinned host memory and its page records
    # (a contiguous pool of that layer's pages) copied back, every step.
    k_host = k[:B].cpu().pin_memory()
    v_host = v[:B].cpu().pin_memory()
    layer_pages = B * nblk
    lbits = bits[:B]
    e2e_pool = P.PagePool(H, D, group=wl["group"], pages={b: int((lbits == b).sum()) for b in (16, 8, 4)},
                          device=device, zero=False)
    lcodes = np.zeros_like(lbits)
    loffs = np.zeros(lbits.shape, np.int64)
    for b_, mode in P.BITS_TO_MODE.items():
        where = lbits == b_
        loffs[where] = e2e_pool.alloc_many(b_, int(where.sum()))
        lcodes[where] = mode
    ldesc = torch.from_numpy(P.encode_array(lcodes, np.full(lbits.shape, 16), loffs).reshape(-1)).to(device)
    out_host = torch.empty(e2e_pool.nbytes, dtype=torch.uint8).pin_memory()
    kd, vd = torch.empty_like(k[:B]), torch.empty_like(v[:B])

    def e2e_step():
        kd.copy_(k_host, non_blocking=True)
        vd.copy_(v_host, non_blocking=True)
        assert lib.akv_pack_pages(kd.data_ptr(), vd.data_ptr(), H * T * D, T * D, nblk, layer_pages,
                                  ldesc.data_ptr(), e2e_pool.arena.data_ptr(), e2e_pool.nbytes, H, D, wl["group"],
                                  _lib.SEM_TENSOR, status.data_ptr(), stream.cuda_stream) == 0
        out_host.copy_(e2e_pool.arena, non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(10):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(device)
    e2e_ms = e0.elapsed_time(e1) / 10
    layer_bytes = 2 * k_host.numel() * 2 + sum(
        int((lbits == b).sum()) * P.algorithmic_record_bytes(D, wl["group"], b) * H for b in (16, 8, 4))
    line = {
        "metric": "requantize/pack GB/s (read + written bytes)", "value": round(gbs, 1), "unit": "GB/s",
        "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16 in, int8/int4/f16 out",
        "data": "synthetic (seeded fp16 N(0,1), 4 outlier channels per head x(+-8))",
        "config": {"workload": wl["name"], "precision_mix": {"fp16": 0.2, "int8": 0.3, "int4": 0.5},
                   "scale_group": wl["group"], "pages": n_pages, "semantics": "quantize_tensor",
                   "l2": "inputs larger than L2 (15 GB), no flush needed"},
        "pct_of_hbm_peak": round(100 * gbs / peak, 2),
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(gbs / peak, 4), "peak_source": f"{peak_kind} hbm_gbs",
                     "kernel": "pack_pages_kernel<128,2048,tensor>",
                     "traffic": (lambda t: None if t is None else t["bytes_per_launch"])(
                         traffic_for("pack_pages_pack") if wl is PACK else None),
                     "traffic_source": (lambda t: None if t is None else t["source"])(
                         traffic_for("pack_pages_pack") if wl is PACK else None),
                     "algorithmic_bytes_per_launch": read + written, "launch_ms_mean": round(ms, 5)},
        "e2e": {"value": round(layer_bytes / (e2e_ms * 1e-3) / 1e9, 1), "unit": "GB/s", "ms_per_step": round(e2e_ms, 4),
                "h2d_bytes_per_step": 2 * k_host.numel() * 2, "d2h_bytes_per_step": e2e_pool.nbytes,
                "path": "akv_pack_pages on one layer, K/V from pinned host, records back to pinned host"},
        "gpu_launches": args.steps,
        "clocks": clocks,
    }
    if not args.no_cpu_baseline:
        cb = pack_cpu_baseline(args.cpu_seconds)
        line["cpu_baseline"] = {"value": round(cb["gbs"], 4), "unit": "GB/s", "cores": cb["cores"],
                                "kind": "port", "sample": cb["sample"]}
    print(json.dumps(line), flush=True)


def build_long_shard(wl: dict, device, rank: int, world: int):
    """This rank's contiguous page range of the long sequence, packed into its
    own pool.  The sequence (page precisions and K/V values) is the same for
    every world size: precisions come from one seed, values are drawn per
    1024-page chunk from a seed of the chunk's index."""
    import numpy as np
    import torch

    from anchorkv_b200 import pool as P
    from anchorkv_b200.sharded import shard_range

    Hkv, D = wl["kv_heads"], wl["dim"]
    nblk = wl["tokens"] // 16
    lo, hi = shard_range(nblk, rank, world)
    keys = list(wl["mix"])
    bits = np.random.default_rng(1000).choice(np.array(keys), size=(1, nblk), p=[wl["mix"][k] for k in keys])
    bits = bits[:, lo:hi]
    pool = P.PagePool(Hkv, D, group=wl["group"], pages={b: int((bits == b).sum()) for b in (16, 8, 4)},
                      device=device, shuffle_seed=rank, zero=False)
    k = torch.empty((1, Hkv, (hi - lo) * 16, D), dtype=torch.float16, device=device)
    v = torch.empty_like(k)
    chunk = 1024
    for c0 in range(lo - lo % chunk, hi, chunk):
        a, b = max(c0, lo), min(c0 + chunk, hi)
        gen = torch.Generator(device=device).manual_seed(77 + c0 // chunk)
        for dst in (k, v):
            src = torch.randn((1, Hkv, chunk * 16, D), generator=gen, device=device, dtype=torch.float16)
            dst[:, :, (a - lo) * 16:(b - lo) * 16] = src[:, :, (a - c0) * 16:(b - c0) * 16]
    store = P.pack_dense(pool, k, v, bits, semantics="tensor")
    del k, v
    torch.cuda.synchronize(device)
    return pool, store, (lo, hi)


def long_context_leg(args, device, rank: int, world: int, local: int, wl: dict = None):
    """One 1,048,576-token sequence split contiguously over the ranks (strong
    scaling): every rank decodes its page range into partial states, then one
    kernel merges them, exchanges the (max, sum, accumulator) states over NVLink
    peer memory and merges the world's states (akv_merge_exchange); on one GPU
    the decode's partials merge straight into the output.  Also times the NCCL
    form (merge to states, all_gather_into_tensor, merge_states) and checks,
    untimed, that both forms agree and that every rank holds the same output.
    Every rank must call it; returns the measurements (max over ranks)."""
    import torch
    import torch.distributed as dist

    import anchorkv_b200 as akv
    from anchorkv_b200 import _lib
    from anchorkv_b200.sharded import PeerExchange, next_epoch, sharded_packed_attention

    wl = LONG if wl is None else wl
    Hq, Hkv, D = wl["q_heads"], wl["kv_heads"], wl["dim"]
    pool, store, (lo, hi) = build_long_shard(wl, device, rank, world)
    qgen = torch.Generator(device=device).manual_seed(5)  # the same query on every rank
    q = torch.randn((1, Hq, 1, D), generator=qgen, device=device, dtype=torch.float32).half()
    kv_bytes = store.resident_bytes()
    scale = 1 / math.sqrt(D)
    lib = _lib.load()
    ws_bytes = lib.akv_workspace_bytes(1, Hq, Hkv, D, hi - lo, 0)
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=device)
    out = torch.empty_like(q)
    exchange = PeerExchange(1, Hq, D) if world > 1 else None
    stream = torch.cuda.current_stream(device)
    sptr = stream.cuda_stream
    status = _lib.status_word(device)

    def decode():
        assert lib.akv_decode_partials(pool.arena.data_ptr(), pool.nbytes, store.table.data_ptr(),
                                       store.table.stride(0), store.seq_blocks.data_ptr(), store.max_blocks,
                                       q.data_ptr(), q.stride(0), q.stride(1), 1, Hq, Hkv, D, wl["group"], scale,
                                       0, ws.data_ptr(), ws_bytes, status.data_ptr(), sptr) == 0

    def combine():
        if world == 1:  # the whole sequence is here: merge the partials straight into the output
            assert lib.akv_merge(ws.data_ptr(), 1, Hq, D, out.data_ptr(), out.stride(0), out.stride(1), None,
                                 status.data_ptr(), sptr) == 0
            return
        exchange.epoch = next_epoch(exchange.epoch)  # merge, exchange over NVLink and merge again in one kernel
        assert lib.akv_merge_exchange(ws.data_ptr(), 1, Hq, D, exchange._peers, exchange.rank, world,
                                      exchange.epoch, out.data_ptr(), out.stride(0), out.stride(1),
                                      status.data_ptr(), sptr) == 0

    def step():
        decode()
        combine()

    def nccl_step():
        if world == 1:
            return akv.merge_states(akv.decode_partial_states(q, store, scale, splits=0)[None])
        return sharded_packed_attention(q, store, scale, splits=0)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])
        torch.cuda.synchronize(device)

    def events(n):
        return [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]

    # untimed cross-checks: the peer-memory exchange against the NCCL form, and every rank's output
    step()
    out_peer = out.clone()
    out_nccl = nccl_step()
    barrier()
    checks = torch.zeros(2, dtype=torch.float64, device=device)
    checks[0] = (out_peer.float() - out_nccl.float()).abs().max()
    if world > 1:
        every = torch.empty((world,) + tuple(out_peer.shape), dtype=out_peer.dtype, device=device)
        dist.all_gather_into_tensor(every, out_peer)
        checks[1] = (every.float() - every[0:1].float()).abs().max()
        dist.all_reduce(checks, op=dist.ReduceOp.MAX)

    steps = args.steps
    for _ in range(args.warmup):
        step()
    barrier()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(steps):
        step()
    t1.record(stream)
    barrier()
    ms_local = t0.elapsed_time(t1) / steps
    ev = events(steps)  # the decode alone (events around each launch)
    for a, b in ev:
        a.record(stream)
        decode()
        b.record(stream)
    barrier()
    dec_ms = sum(a.elapsed_time(b) for a, b in ev) / steps
    ev = events(steps)  # the combining kernel alone, each after an untimed decode
    for a, b in ev:
        decode()
        a.record(stream)
        combine()
        b.record(stream)
    barrier()
    comb_ms = sum(a.elapsed_time(b) for a, b in ev) / steps
    for _ in range(3):
        nccl_step()
    barrier()
    n0, n1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n0.record(stream)
    for _ in range(steps):
        nccl_step()
    n1.record(stream)
    barrier()
    nccl_ms = n0.elapsed_time(n1) / steps

    # end to end: the query from pinned host memory, the output back to it
    q_host = q.cpu().pin_memory()
    out_host = torch.empty(q.shape, dtype=q.dtype).pin_memory()

    def e2e_step():
        q.copy_(q_host, non_blocking=True)
        step()
        out_host.copy_(out, non_blocking=True)

    for _ in range(3):
        e2e_step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2e_steps = max(10, steps // 4)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    barrier()
    e2e_ms = e0.elapsed_time(e1) / e2e_steps
    st = float(akv.take_device_status(device))
    mx = torch.tensor([ms_local, dec_ms, comb_ms, nccl_ms, e2e_ms, st], dtype=torch.float64, device=device)
    kv_all = torch.tensor([float(kv_bytes)], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        dist.all_reduce(kv_all, op=dist.ReduceOp.SUM)
        exchange.close()
    ms, dec_max, comb_max, nccl_max, e2e_max, st_max = mx.tolist()
    assert st_max == 0, f"device status word set in the long-context leg: {int(st_max)}"
    peak, peak_kind = hbm_peak()
    io = 2 * q.numel() * 2
    step_bytes = kv_all.item() + io
    res = {
        "workload": wl["name"], "context_tokens": wl["tokens"], "q_heads": Hq, "kv_heads": Hkv, "head_dim": D,
        "precision_mix": {"fp16": wl["mix"][16], "int8": wl["mix"][8], "int4": wl["mix"][4]},
        "scale_group": wl["group"], "n_gpus": world, "scaling": "strong", "steps": steps,
        "ms_per_step": round(ms, 5), "value": round(step_bytes / (ms * 1e-3) / 1e9, 1), "unit": "GB/s",
        "tokens_per_s": round(1 / (ms * 1e-3), 1),
        "pct_of_hbm_peak": round(100 * step_bytes / (ms * 1e-3) / 1e9 / world / peak, 2),
        "decode_ms_max_over_ranks": round(dec_max, 5),
        "decode_ms_rank0": round(dec_ms, 5),
        "combine_kernel": "merge_exchange_kernel (epoch-tagged NVLink peer stores, bounded waits)" if world > 1
        else "merge_wide_kernel (local partials into the output)",
        "combine_ms_max_over_ranks": round(comb_max, 5),
        "nccl_variant_ms_per_step": round(nccl_max, 5),
        "nccl_variant": "decode + merge to states + all_gather_into_tensor + merge_states" if world > 1
        else "decode + merge to states + merge_states (no collective at one GPU)",
        "collective_bytes_per_rank": Hq * (D + 2) * 4,
        "check_max_abs_peer_vs_nccl": float(checks[0]), "check_max_abs_across_ranks": float(checks[1]),
        "roofline": {"bound": "hbm", "achieved": round((kv_bytes + io) / (dec_ms * 1e-3) / 1e9, 1), "peak": peak,
                     "unit": "GB/s", "frac": round((kv_bytes + io) / (dec_ms * 1e-3) / 1e9 / peak, 4),
                     "peak_source": f"{peak_kind} hbm_gbs", "kernel": "decode_streamk_kernel<128> (rank 0)",
                     "algorithmic_bytes_per_launch": kv_bytes + io, "launch_ms_mean": round(dec_ms, 5)},
        "e2e": {"value": round(step_bytes / (e2e_max * 1e-3) / 1e9, 1), "unit": "GB/s", "ms_per_step": round(e2e_max, 5),
                "h2d_bytes_per_step": q.numel() * 2, "d2h_bytes_per_step": out.numel() * 2},
        "l2": "inputs larger than L2 (1.5 GB of KV over the ranks), no flush needed",
    }
    del pool, store, ws
    return res


def long_config(wl: dict, world: int) -> dict:
    """The ``config`` of a long-context line (both arms print the same one)."""
    return {"workload": wl["name"], "q_heads": wl["q_heads"], "kv_heads": wl["kv_heads"], "head_dim": wl["dim"],
            "context_tokens": wl["tokens"], "page_tokens": 16,
            "precision_mix": {"fp16": wl["mix"][16], "int8": wl["mix"][8], "int4": wl["mix"][4]},
            "scale_group": wl["group"],
            "parallelism": f"sequence-sharded x{world}" + (
                ", LSE states exchanged over NVLink peer memory in the merge kernel" if world > 1 else ""),
            "collective_bytes_per_rank": wl["q_heads"] * (wl["dim"] + 2) * 4,
            "l2": "inputs larger than L2 (1.5 GB of KV over the ranks), no flush needed"}


def run_long(args, wl):
    """--workload long: the long-context leg alone, as the line's headline."""
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    gpu_id = "GPU-" + str(torch.cuda.get_device_properties(device).uuid)
    sampler = ClockSampler(gpu_id)
    res = long_context_leg(args, device, rank, world, local, wl)
    clocks = sampler.stop()
    if rank == 0:
        traffic = traffic_for("decode_streamk_long")
        roof = dict(res["roofline"])
        roof["traffic"] = None if traffic is None else round(traffic["bytes_per_launch"] / world)
        roof["traffic_source"] = None if traffic is None else traffic["source"] + " (scaled by 1/n_gpus)"
        line = {
            "metric": METRIC, "value": res["value"], "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": res["ms_per_step"], "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16 operands, f32 accumulation", "data": "synthetic (seeded fp16 N(0,1))",
            "config": long_config(wl, world),
            "tokens_per_s": res["tokens_per_s"], "pct_of_hbm_peak": res["pct_of_hbm_peak"],
            "roofline": roof, "e2e": res["e2e"], "long_context": res,
            "gpu_launches": args.steps * 2, "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


def run_reference(args, wl, long=False):
    """The reference arm: the reference's own CPU decode path (``cpu_baseline``)
    on the host cores, same metric, unit and config as this repository's arm.
    A step is a bounded sample (one sequence-layer decode call of the workload,
    or a 65,536-token slice of the long sequence); ``value`` is the sample's
    resident-KV GB/s and tokens/s is extrapolated to the full workload.  Under
    torchrun only rank 0 runs."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    per_step = max(0.02, args.cpu_seconds / max(1, args.steps))
    cb = cpu_baseline(wl, seed=99, seconds=per_step * args.steps, calls_min=args.steps + args.warmup)
    if long:
        config = long_config(wl, world)
        scaling = "strong"
    else:
        B, distinct, arena = batched_plan(wl, world)
        config = batched_config(wl, world, B, distinct, arena)
        scaling = "strong" if wl.get("strong") else "weak"
    line = {
        "impl": "reference", "metric": METRIC, "value": round(cb["gbs"], 4), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "calls_timed": cb["calls"],
        "ms_per_step": round(cb["seconds_per_call"] * 1e3, 3),
        "ms_per_full_step_extrapolated": round(cb["seconds_per_call"] * cb["calls_per_step"] * 1e3, 1),
        "higher_is_better": True, "scaling": scaling, "vs_baseline": None,
        "dtype": "f16 operands (torch CPU SDPA)", "data": "synthetic (seeded fp16 N(0,1))",
        "config": config,
        "tokens_per_s": round(cb["tokens_per_s"], 4),
        "cpu_baseline": {"value": round(cb["gbs"], 4), "unit": "GB/s", "cores": cb["cores"], "kind": cb["kind"],
                         "sample": cb["sample"]},
        "e2e": {"value": round(cb["gbs"], 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "step_definition": "one decode call of one sequence-layer (a bounded sample of the full step)",
    }
    print(json.dumps(line), flush=True)


# Batch-1 shapes the reference's packed GPU kernel takes (group 64, head_dim 128):
# (query heads, KV heads, context tokens).
REF_GPU_CASES = [(16, 8, 512), (16, 8, 8192), (32, 8, 32768)]


def run_reference_gpu(args):
    """The reference's own GPU decode next to ours, one JSON line per case.

    The reference, installed unmodified in baseline/_ref, builds its PagedLayer
    (packed_decode.py:108-194) and runs its Triton packed_attention
    (triton_decode.py:85-104, default splits=4); ours builds
    anchorkv_b200.PagedLayer from the same appended K/V and runs
    anchorkv_b200.packed_attention with the same arguments.  Pages older than
    the two most recent are archived to INT4 by both.  Each call is timed with
    CUDA events over --steps calls after --warmup; bytes are the resident
    payload + scales of the layer."""
    import torch

    ref_dir = ROOT / "baseline" / "_ref"
    sys.path.insert(0, str(ref_dir))
    try:
        from anchorkv import packed_decode as ref_pd
        from anchorkv import triton_decode as ref_td
    except Exception as exc:  # not installed, or its dependencies are missing
        print(json.dumps({"impl": "reference_gpu", "unavailable": f"reference not importable from {ref_dir}: "
                                                                     f"{type(exc).__name__}: {exc}"}), flush=True)
        return
    import anchorkv_b200 as akv

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    D, group = 128, 64
    for hq, hkv, tokens in REF_GPU_CASES:
        gen = torch.Generator(device=dev).manual_seed(tokens + hq)
        k = torch.randn((1, hkv, tokens, D), generator=gen, device=dev).half()
        v = torch.randn((1, hkv, tokens, D), generator=gen, device=dev).half()
        q = torch.randn((1, hq, 1, D), generator=gen, device=dev).half()
        scale = D ** -0.5
        ref = ref_pd.PagedLayer(hkv, D, tokens, group=group, archive_bits=4, recent_pages=2, device=dev)
        ours = akv.PagedLayer(hkv, D, tokens, group=group, archive_bits=4, recent_pages=2, device=dev)
        for begin in range(0, tokens, 256):
            ref.append(k[:, :, begin:begin + 256], v[:, :, begin:begin + 256])
            ours.append(k[:, :, begin:begin + 256], v[:, :, begin:begin + 256])
        assert [p[0].bits for p in ref.pages] == [p[0].bits for p in ours.pages]

        def timed(fn):
            for _ in range(args.warmup):
                fn()
            torch.cuda.synchronize(dev)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(args.steps):
                fn()
            b.record()
            torch.cuda.synchronize(dev)
            return a.elapsed_time(b) / args.steps

        out_ref = ref_td.packed_attention(q, ref, scale)
        out_ours = akv.packed_attention(q, ours, scale)
        diff = float((out_ref.float() - out_ours.float()).abs().max())
        ms_ref = timed(lambda: ref_td.packed_attention(q, ref, scale))
        ms_ours = timed(lambda: akv.packed_attention(q, ours, scale))
        assert akv.take_device_status(dev) == 0
        nbytes = ours.payload_bytes
        line = {
            "impl": "reference_gpu", "metric": "batch-1 decode-attn resident-KV GB/s, the reference's Triton "
                                              "packed_attention and ours on the same pages",
            "unit": "GB/s", "higher_is_better": True, "steps": args.steps, "warmup": args.warmup,
            "config": {"workload": f"one sequence, {tokens} tokens, {hq} query / {hkv} KV heads, head_dim {D}, "
                                   f"group {group}, pages older than the last two archived to INT4",
                       "splits": 4, "resident_bytes": nbytes, "pages": len(ours.pages)},
            "reference": {"ms_per_call": round(ms_ref, 5), "value": round(nbytes / (ms_ref * 1e-3) / 1e9, 2)},
            "ours": {"ms_per_call": round(ms_ours, 5), "value": round(nbytes / (ms_ours * 1e-3) / 1e9, 2)},
            "max_abs_diff": diff,
        }
        print(json.dumps(line), flush=True)
        del ref, ours, k, v
        torch.cuda.empty_cache()


# ----------------------------------------------------------- live decode
LIVE_PREFIXES = (128, 256, 512)


def _qwen3_06b(device):
    """Randomly initialised Qwen3-0.6B architecture (no checkpoint offline): 28
    layers, hidden 1024, 16 query / 8 KV heads of 128, fp16."""
    import torch
    from transformers import Qwen3Config, Qwen3ForCausalLM

    torch.manual_seed(0)
    config = Qwen3Config(vocab_size=151936, hidden_size=1024, intermediate_size=3072, num_hidden_layers=28,
                         num_attention_heads=16, num_key_value_heads=8, head_dim=128,
                         max_position_embeddings=40960, tie_word_embeddings=True, attn_implementation="sdpa")
    return Qwen3ForCausalLM(config).to(device=device, dtype=torch.float16).eval()


def run_live(args):
    """Decode tokens/s of a Qwen3-0.6B-shaped model (random weights) at
    128/256/512-token prefixes, one JSON line per (arm, prefix):

    * reference: the reference's controlled_decode (benchmark_suite.py:155-264)
      with its own live cache and packed route (its PagedLayer and Triton
      kernel, installed unmodified in baseline/_ref), INT4 archive;
    * ours_dropin: the same harness with this package's PagedLayer,
      dense_attention and packed_attention substituted for the reference's;
    * stock: the harness's native_fp16 policy (transformers SDPA, FP16 cache);
    * ours_batched: this package's batched live cache (anchorkv_b200.live) at
      batch 1 and 32, INT4 archive; tokens/s counts every sequence's token.

    Each arm decodes the same fixed token history (32 warm-up, --live-tokens
    measured) after the same prefill, timed as the harness times it (wall
    clock and CUDA events around the measured steps)."""
    import torch

    import anchorkv_b200 as akv
    from anchorkv_b200 import live

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    ref_pd, why = import_reference()
    if ref_pd is None:
        print(json.dumps({"workload": "live", "unavailable": why}), flush=True)
        return
    from anchorkv import benchmark_suite as BS
    from anchorkv import colab_experiment as CE
    from anchorkv import triton_decode as TD

    model = _qwen3_06b(dev)
    settings = CE.Settings()
    warm, measured = 32, args.live_tokens
    gen = torch.Generator().manual_seed(11)
    originals = (CE.PagedLayer, CE.dense_attention, CE.pack_page, TD.packed_attention)

    def substitute(ours):
        CE.PagedLayer, CE.dense_attention, CE.pack_page, TD.packed_attention = (
            (akv.PagedLayer, akv.dense_attention, akv.pack_page, akv.packed_attention) if ours else originals)

    for prefix in LIVE_PREFIXES:
        ids = torch.randint(0, 151936, (1, prefix), generator=gen)
        tokens = torch.randint(0, 151936, (warm + measured,), generator=gen).tolist()
        with torch.inference_mode():
            out = model(input_ids=ids.to(dev), use_cache=True, logits_to_keep=1)
            source = CE.cache_cpu(out.past_key_values)
            del out
        for arm, policy, ours in (("reference", "int4", False), ("ours_dropin", "int4", True),
                                  ("stock", "native_fp16", False)):
            substitute(ours)
            try:
                row = BS.controlled_decode(model, source, settings, policy, tokens, measured, warmup_tokens=warm)
            finally:
                substitute(False)
            line = {"workload": "live controlled decode, Qwen3-0.6B shape (random weights), batch 1",
                    "arm": arm, "prefix_tokens": prefix, "batch": 1, "measured_tokens": measured,
                    "tokens_per_s": round(row["steady_tokens_per_second"], 2),
                    "cuda_timeline_tokens_per_s": round(measured / row["measured_cuda_timeline_seconds"], 2),
                    "final_payload_bytes": row["final_cache"]["payload_bytes"],
                    "new_measured_demotions": row["new_measured_demotions"]}
            print(json.dumps(line), flush=True)
        for batch in (1, 32):
            seqs = [(k.expand(batch, -1, -1, -1).contiguous().to(dev), v.expand(batch, -1, -1, -1).contiguous().to(dev))
                    for k, v in source]
            hist = torch.tensor(tokens, device=dev).view(1, -1).expand(batch, -1).contiguous()
            with torch.inference_mode():
                cache = live.batched_live_cache(seqs, max_tokens=prefix + warm + measured + 16, device=dev)
                with live.paged_route(model, cache):
                    for i in range(warm):
                        live.decode_step(model, cache, hist[:, i])
                    torch.cuda.synchronize(dev)
                    t0 = time.perf_counter()
                    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    a.record()
                    for i in range(warm, warm + measured):
                        live.decode_step(model, cache, hist[:, i])
                    b.record()
                    torch.cuda.synchronize(dev)
                    wall = time.perf_counter() - t0
            assert akv.take_device_status(dev) == 0
            line = {"workload": f"live decode, Qwen3-0.6B shape (random weights), batch {batch}",
                    "arm": "ours_batched", "prefix_tokens": prefix, "batch": batch, "measured_tokens": measured,
                    "tokens_per_s": round(batch * measured / wall, 2),
                    "cuda_timeline_tokens_per_s": round(batch * measured / (a.elapsed_time(b) / 1e3), 2),
                    "final_payload_bytes": cache.report()["payload_bytes"],
                    "demotions": cache.report()["demotions"]}
            print(json.dumps(line), flush=True)
            del cache, seqs


# --------------------------------------------------------- other kernels
def run_kernels(args):
    """Every kernel besides the decode and the pack, on a case larger than L2
    (or, for the merges, the decode's own partials, which L2 holds), timed with
    CUDA events over --steps launches after --warmup: one JSON line per kernel
    with its algorithmic bytes, achieved GB/s and fraction of the measured HBM
    peak.  --kernel NAME runs one case (the ncu captures do)."""
    import numpy as np
    import torch

    import anchorkv_b200 as akv
    from anchorkv_b200 import _lib
    from anchorkv_b200 import live as LV
    from anchorkv_b200 import pool as P

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lib = _lib.load()
    stream = torch.cuda.current_stream(dev)
    sptr = stream.cuda_stream
    status = _lib.status_word(dev).data_ptr()
    peak, peak_kind = hbm_peak()
    wanted = args.kernel
    import ctypes

    def timed(name, nbytes, fn, note):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize(dev)
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
        for a, b in ev:
            a.record(stream)
            fn()
            b.record(stream)
        torch.cuda.synchronize(dev)
        ms = sum(a.elapsed_time(b) for a, b in ev) / len(ev)
        assert akv.take_device_status(dev) == 0
        gbs = nbytes / (ms * 1e-3) / 1e9
        print(json.dumps({"workload": "kernels", "kernel": name, "launch_ms_mean": round(ms, 5),
                          "algorithmic_bytes_per_launch": int(nbytes), "achieved_gbs": round(gbs, 1),
                          "frac_of_hbm_peak": round(gbs / peak, 4), "peak": peak,
                          "peak_source": f"{peak_kind} hbm_gbs", "case": note}), flush=True)

    def want(name):
        return wanted in (None, name)

    if want("quantize_flat") or want("dequantize_flat"):
        n = 256 << 20  # 256 Mi fp16 elements (512 MB), groups of 64, INT4
        x = torch.randn(n, dtype=torch.float16, device=dev)
        payload = torch.empty(n // 2, dtype=torch.uint8, device=dev)
        scales = torch.empty(n // 64, dtype=torch.float16, device=dev)
        out = torch.empty_like(x)
        q_bytes = 2 * n + n // 2 + 2 * (n // 64)
        if want("quantize_flat"):
            timed("quantize_vec_kernel<half,4,tensor>", q_bytes,
                  lambda: _lib.call("akv_quantize", x.data_ptr(), _lib.DTYPE_F16, n, 64, 4, _lib.SEM_TENSOR,
                                    payload.data_ptr(), scales.data_ptr(), sptr),
                  "256 Mi fp16 elements to INT4, group 64 (quantize_tensor; whole power-of-two groups of "
                  "8-256 take the vector kernel)")
        if want("dequantize_flat"):
            _lib.call("akv_quantize", x.data_ptr(), _lib.DTYPE_F16, n, 64, 4, _lib.SEM_TENSOR, payload.data_ptr(),
                      scales.data_ptr(), sptr)
            timed("dequantize_vec_kernel<half,4>", q_bytes,
                  lambda: _lib.call("akv_dequantize", payload.data_ptr(), scales.data_ptr(), n, 64, 4,
                                    out.data_ptr(), _lib.DTYPE_F16, sptr),
                  "256 Mi INT4 elements to fp16, group 64 (PackedTensor.dequantize; the vector kernel)")
        del x, payload, scales, out
    if want("unpack_pages") or want("repack_pages"):
        wl = WORKLOADS["batched_small"]
        pool, layers, _, kv_bytes = build_workload(wl, dev, seed=1234, batch=16, distinct=1)
        t = layers[0]
        desc = t.table.reshape(-1).contiguous()
        npg = desc.numel()
        if want("unpack_pages"):
            ok = torch.empty((wl["kv_heads"], npg * 16, wl["dim"]), dtype=torch.float16, device=dev)
            ov = torch.empty_like(ok)
            dense = 2 * ok.numel() * 2
            timed("unpack_pages_kernel<128,2048,half>", kv_bytes[0] + dense,
                  lambda: _lib.call("akv_unpack_pages", desc.data_ptr(), npg, pool.arena.data_ptr(), pool.nbytes,
                                    wl["kv_heads"], wl["dim"], wl["group"], ok.data_ptr(), ov.data_ptr(),
                                    _lib.DTYPE_F16, status, sptr),
                  "one layer of the batched workload at 16 sequences (8192 tokens, 15/35/40/10 mix) to dense fp16")
            del ok, ov
        if want("repack_pages"):
            d = desc.cpu().numpy()
            src = d[(d & 3) == _lib.MODE_FP16]  # the FP16 pages, requantized to INT4
            pool.reserve(4, src.size)
            dst_off = pool.alloc_many(4, src.size)
            dst = P.encode_array(np.full(src.size, _lib.MODE_INT4), np.full(src.size, 16), dst_off)
            s_t, d_t = torch.from_numpy(src).to(dev), torch.from_numpy(dst).to(dev)
            nbytes = src.size * wl["kv_heads"] * (P.algorithmic_record_bytes(wl["dim"], wl["group"], 16) +
                                                 P.algorithmic_record_bytes(wl["dim"], wl["group"], 4))
            timed("pack_pages_kernel<128,2048,tensor,record>", nbytes,
                  lambda: _lib.call("akv_repack_pages", s_t.data_ptr(), d_t.data_ptr(), src.size,
                                    pool.arena.data_ptr(), pool.nbytes, wl["kv_heads"], wl["dim"], wl["group"],
                                    _lib.SEM_TENSOR, status, sptr),
                  f"{src.size} FP16 pages (8 KV heads) requantized to INT4 records (requantize_segment)")
        del pool, layers
    if want("merge_states"):
        n, batch, hq, dim = 8, 4096, 32, 128
        states = torch.randn((n, batch, hq, dim + 2), dtype=torch.float32, device=dev)
        states[..., dim] = states[..., dim].abs()
        out = torch.empty((batch, hq, 1, dim), dtype=torch.float16, device=dev)
        timed("merge_states_kernel<128>", states.numel() * 4 + out.numel() * 2,
              lambda: _lib.call("akv_merge_states", states.data_ptr(), n, batch, hq, dim, out.data_ptr(),
                                out.stride(0), out.stride(1), sptr),
              "8 states (8 GPUs' shares) of 4096 sequences x 32 query heads")
        del states, out
    if want("merge_wide") or want("merge_exchange") or want("merge_rows"):
        for name in ("merge_wide", "merge_exchange", "merge_rows"):
            if not want(name):
                continue
            if name == "merge_rows":
                wl = WORKLOADS["batched_small"]
                pool, layers, qs, _ = build_workload(wl, dev, seed=1234, distinct=1)
                store, q, hq, hkv, D, batch, splits = layers[0], qs[0], wl["q_heads"], wl["kv_heads"], wl["dim"], \
                    wl["batch"], wl["splits"]
            else:
                pool, store, _ = build_long_shard(LONG, dev, 0, 1)
                hq, hkv, D, batch, splits = LONG["q_heads"], LONG["kv_heads"], LONG["dim"], 1, 0
                q = torch.randn((1, hq, 1, D), device=dev).half()
            mb = store.max_blocks
            ws_bytes = lib.akv_workspace_bytes(batch, hq, hkv, D, mb, splits)
            ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
            out = torch.empty((batch, hq, 1, D), dtype=torch.float16, device=dev)
            _lib.call("akv_decode_partials", pool.arena.data_ptr(), pool.nbytes, store.table.data_ptr(),
                      store.table.stride(0), store.seq_blocks.data_ptr(), mb, q.data_ptr(), q.stride(0), q.stride(1),
                      batch, hq, hkv, D, 2048, 0.088, splits, ws.data_ptr(), ws_bytes, status, sptr)
            torch.cuda.synchronize(dev)
            # bytes the merge reads: the partial states the decode wrote (every contributor of every row)
            hdr = ws[:64].view(torch.int32).cpu().numpy().astype(np.int64)
            warps, rng, items, slot_heads = hdr[1], hdr[3], hdr[5], hdr[10]
            begin = np.arange(warps) * rng
            end = np.minimum(begin + rng, items * mb)
            touched = int(((end - 1) // mb - begin // mb + 1).sum())  # (warp, item) partials the merge folds
            part = touched * slot_heads * (D + 2) * 4
            if name == "merge_exchange":
                nbytes_ex = lib.akv_exchange_bytes(1, batch, hq, D)
                own = ctypes_alloc(nbytes_ex)
                peers = (ctypes.c_void_p * 1)(own)
                epoch = [0]

                def fn():
                    epoch[0] += 1
                    _lib.call("akv_merge_exchange", ws.data_ptr(), batch, hq, D, peers, 0, 1, epoch[0],
                              out.data_ptr(), out.stride(0), out.stride(1), status, sptr)

                timed("merge_exchange_kernel<128>", part + out.numel() * 2, fn,
                      "one rank's merge + exchange of the 1M-token sequence's partials (world 1: its own buffer)")
                torch.cuda.synchronize(dev)
                _lib.call("akv_ipc_free", ctypes.c_void_p(own))
            else:
                timed(f"{name}_kernel<128>", part + out.numel() * 2,
                      lambda: _lib.call("akv_merge", ws.data_ptr(), batch, hq, D, out.data_ptr(), out.stride(0),
                                        out.stride(1), None, status, sptr),
                      "the decode's partials of " + ("the 1M-token sequence (one CTA per row)" if name != "merge_rows"
                                                    else "one batched layer (one warp per row)") +
                      "; L2 holds them (written by the decode just before)")
            del pool, store, ws
    if want("append_rows"):
        batch, heads, dim = 1024, 8, 128
        store = LV.PagedKVStore(1, batch, heads, dim, 4096, device=dev)
        k = torch.randn((batch, heads, 64, dim), device=dev).half()
        store.prefill(0, k, k)
        kk = torch.randn((batch, heads, 1, dim), device=dev).half()
        tbl = store.tables[0]
        page, row = divmod(store.lengths[0], 16)
        timed("append_rows_kernel<128>", 2 * kk.numel() * 2 * 2,
              lambda: _lib.call("akv_append_rows", kk.data_ptr(), kk.data_ptr(), kk.stride(0), kk.stride(1),
                                kk.stride(2), batch, 1, 3, tbl.data_ptr(), tbl.stride(0), page - 1, None,
                                store.pool.arena.data_ptr(), store.pool.nbytes, heads, dim, status, sptr),
              "one decode token of 1024 sequences x 8 KV heads into their FP16 pages (row 3)")


def ctypes_alloc(nbytes: int) -> int:
    """A zeroed device buffer from akv_ipc_alloc (the exchange buffers' allocator)."""
    import ctypes

    from anchorkv_b200 import _lib

    ptr, handle = ctypes.c_void_p(), ctypes.create_string_buffer(64)
    _lib.call("akv_ipc_alloc", nbytes, ctypes.byref(ptr), handle)
    return ptr.value


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--gpus", type=int, default=1, help="GPUs of one node, one process each (torchrun for N > 1)")
    ap.add_argument("--steps", type=int, default=300, help="timed steps (one decode token per sequence, all layers)")
    ap.add_argument("--warmup", type=int, default=10, help="untimed steps first (at least 3)")
    ap.add_argument("--impl", choices=("ours", "reference", "reference_gpu"), default="ours",
                    help="ours: the CUDA kernels; reference: the reference's CPU decode path (timed on the "
                         "host cores); reference_gpu: the reference's own Triton decode beside ours, batch 1")
    ap.add_argument("--workload", choices=sorted(WORKLOADS) + ["long", "pack", "pack_small", "live", "kernels"],
                    default="batched",
                    help="batched (default), large, long (one 1M-token sequence), pack (requantize); "
                         "*_small: one-layer profiling cases")
    ap.add_argument("--mix", choices=("fp16", "int8", "int4"), default=None,
                    help="profiling: every page of a batched workload in this one precision")
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="seconds of CPU timing for the CPU baseline")
    ap.add_argument("--no-cpu-baseline", action="store_true", help="skip the CPU baseline (profiling runs)")
    ap.add_argument("--no-long", action="store_true",
                    help="skip the long-context leg of the batched/large runs (profiling runs)")
    ap.add_argument("--sustained-seconds", type=float, default=1.2,
                    help="seconds of back-to-back steps in the line's sustained record")
    ap.add_argument("--kernel", default=None, help="--workload kernels: run this one case (e.g. unpack_pages)")
    ap.add_argument("--live-tokens", type=int, default=64, help="--workload live: measured decode tokens")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    if args.workload == "live":
        run_live(args)
        return
    if args.workload == "kernels":
        run_kernels(args)
        return
    if args.impl == "reference_gpu":
        run_reference_gpu(args)
        return
    if args.workload in ("pack", "pack_small"):
        if args.impl == "reference":
            cb = pack_cpu_baseline(args.cpu_seconds)
            print(json.dumps({"impl": "reference", "metric": "requantize/pack GB/s (read + written bytes)",
                              "value": round(cb["gbs"], 4), "unit": "GB/s", "n_gpus": 1,
                              "higher_is_better": True, "config": {"workload": PACK["name"]},
                              "cpu_baseline": {"value": round(cb["gbs"], 4), "unit": "GB/s", "cores": cb["cores"],
                                               "kind": "port", "sample": cb["sample"]},
                              "e2e": {"value": round(cb["gbs"], 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                                      "d2h_bytes_per_step": 0}}))
        else:
            run_pack(args, PACK if args.workload == "pack" else PACK_SMALL)
        return
    if args.workload == "long":
        if args.impl == "reference":
            run_reference(args, dict(LONG, layers=1, batch=1, splits=0), long=True)
        else:
            run_long(args, LONG)
        return
    wl = WORKLOADS[args.workload]
    if args.mix:
        bits = {"fp16": 16, "int8": 8, "int4": 4}[args.mix]
        wl = dict(wl, name=f"{wl['name']}, all pages {args.mix}", mix={b: float(b == bits) for b in (16, 8, 4, 0)})
    if args.impl == "reference":
        run_reference(args, wl)
    else:
        run_ours(args, wl)


if __name__ == "__main__":
    main()
