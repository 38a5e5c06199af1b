"""Seeded synthetic inputs shared by the fixture generator and the tests.

Everything is drawn from a CPU ``torch.Generator`` so the same seed gives the
same bytes here and on any machine running the same torch build; fixtures store
a sha256 of the inputs so a test can prove it regenerated them exactly.

Shapes and distributions follow the packed-decode workloads: fp16 N(0, 1) K/V
with 4 outlier channels per KV head scaled x8, fp16 N(0, 1) queries, per-block
precision drawn from a seed.
"""

from __future__ import annotations

import hashlib

import torch

FP16, INT8, INT4, EVICTED = 16, 8, 4, 0


def generator(seed: int) -> torch.Generator:
    return torch.Generator().manual_seed(int(seed))


def outlier_kv(seed: int, shape, n_outliers: int = 4, factor: float = 8.0,
               signed: bool = False) -> torch.Tensor:
    """fp16 ``[..., heads, tokens, dim]`` N(0,1) with outlier channels per head."""
    g = generator(seed)
    x = torch.randn(tuple(shape), generator=g)
    heads, dim = shape[-3], shape[-1]
    for h in range(heads):
        channels = torch.randperm(dim, generator=g)[:n_outliers]
        for c in channels.tolist():
            f = factor
            if signed and torch.rand((), generator=g).item() < 0.5:
                f = -factor
            x[..., h, :, c] *= f
    return x.half()


def normal(seed: int, shape, dtype=torch.float16) -> torch.Tensor:
    return torch.randn(tuple(shape), generator=generator(seed)).to(dtype)


def draw_modes(seed: int, count: int, mix) -> list[int]:
    """Per-block precision from a seed.  ``mix`` maps mode -> probability, in order
    FP16, INT8, INT4, EVICTED (missing modes have probability 0)."""
    u = torch.rand(count, generator=generator(seed)).tolist()
    order = [FP16, INT8, INT4, EVICTED]
    edges = []
    acc = 0.0
    for m in order:
        acc += float(mix.get(m, 0.0))
        edges.append((acc, m))
    out = []
    for x in u:
        for edge, m in edges:
            if x < edge:
                out.append(m)
                break
        else:
            out.append(edges[-1][1])
    return out


def sha256(*tensors) -> str:
    h = hashlib.sha256()
    for t in tensors:
        h.update(t.detach().cpu().contiguous().view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


# Single-layer parity workload: 16 query heads, 8 KV heads, head_dim 128,
# batch 1, 512 tokens in 16-token blocks, 25/25/50 FP16/INT8/INT4 per block with
# per-block-per-KV-head scales (group = 16 * 128), softmax scale 1/sqrt(128).
PARITY = dict(q_heads=16, kv_heads=8, dim=128, tokens=512, block=16, group=2048,
              mix={FP16: 0.25, INT8: 0.25, INT4: 0.5})


def parity_workload(seed: int = 2026):
    p = PARITY
    k = outlier_kv(seed, (1, p["kv_heads"], p["tokens"], p["dim"]))
    v = outlier_kv(seed + 1, (1, p["kv_heads"], p["tokens"], p["dim"]))
    q = normal(seed + 2, (1, p["q_heads"], 1, p["dim"]))
    modes = draw_modes(seed + 3, p["tokens"] // p["block"], p["mix"])
    return q, k, v, modes


def gate_workload(dim: int, length: int, seed: int):
    """One case of the reference's kernel gate (colab_experiment.py:271-291):
    2 KV heads, 4 query heads, fp16 N(0,1)."""
    k = normal(seed, (1, 2, length, dim))
    v = normal(seed + 1, (1, 2, length, dim))
    q = normal(seed + 2, (1, 4, 1, dim))
    return q, k, v


GATE_DIMS = (64, 128)
GATE_LENGTHS = (1, 15, 16, 17, 33, 65, 97)
GATE_BITS = (4, 8, 16)


def gate_seed(dim: int, length: int, bits: int) -> int:
    return 1000 * dim + 10 * length + bits


# Declarative-store scenarios in the decode page format (fp16 K/V, 16-token
# blocks).  Each segment is (segment id, token start, tokens, role); ``steps``
# run in order, then each of ``views`` (directive text fed to the store) gives
# one recorded state.  "mixed" holds one segment whose partial block a scale
# group would straddle (37 tokens x head_dim 64, group 128), which cannot be a
# page record and stays flat.
DECLARATIVE = [
    dict(name="slab_4d", lead=(1, 8), dim=128, group=2048, q_heads=16, seed=501,
         segments=[(0, 0, 16, "sink"), (1, 16, 32, "scaffold"), (2, 48, 64, "context"), (3, 112, 48, "context"),
                   (4, 176, 80, "context"), (5, 256, 32, "response")],
         steps=[("requantize", 2, "int8"), ("requantize", 2, "int4"), ("requantize", 3, "int4"),
                ("requantize", 4, "int8"), ("feed", '<anchor segments="0">'), ("requantize", 1, "evicted")],
         views=["", '<focus segments="3">', "<local>", "</local>"]),
    dict(name="rows_5d", lead=(2, 3, 4), dim=64, group=64, q_heads=8, seed=777,
         segments=[(0, 0, 37, "sink"), (1, 40, 21, "context"), (2, 61, 16, "context"), (3, 90, 45, "context"),
                   (4, 135, 9, "response")],
         steps=[("requantize", 1, "int8"), ("requantize", 1, "int4"), ("requantize", 3, "int8"),
                ("feed", '<archive segments="2">'), ("requantize", 0, "int8")],
         views=["", '<focus segments="1,3">', "<local>"]),
    dict(name="rows_g32_d128", lead=(2, 4), dim=128, group=32, q_heads=8, seed=913,
         segments=[(0, 0, 33, "scaffold"), (1, 33, 50, "context"), (2, 83, 7, "response")],
         steps=[("requantize", 1, "int4"), ("requantize", 0, "int8")],
         views=["", "<local>"]),
    dict(name="mixed", lead=(2, 4), dim=64, group=128, q_heads=8, seed=1201,
         segments=[(0, 0, 32, "sink"), (1, 32, 37, "context"), (2, 69, 48, "response")],
         steps=[("requantize", 1, "int8"), ("requantize", 2, "int4")],
         views=["", "<local>"]),
]


def declarative_inputs(spec):
    """K/V per segment (fp16, ``lead + (tokens, dim)``) and one query per layer
    (``[batch, q_heads, 1, dim]``)."""
    kv = {}
    for sid, _, tokens, _ in spec["segments"]:
        shape = tuple(spec["lead"]) + (tokens, spec["dim"])
        kv[sid] = (outlier_kv(spec["seed"] + 10 * sid, shape), outlier_kv(spec["seed"] + 10 * sid + 1, shape))
    lead = tuple(spec["lead"])
    layers, batch = (lead[0], lead[1]) if len(lead) == 3 else (1, lead[0])
    q = [normal(spec["seed"] + 1000 + layer, (batch, spec["q_heads"], 1, spec["dim"])) for layer in range(layers)]
    return kv, q
