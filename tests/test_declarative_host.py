"""DeclarativeKVCache's control plane against the reference's own, on CPU, over random programs.

Each program builds the same segments in the reference's ``DeclarativeKVCache``
(backend.py:314-601, installed unmodified in baseline/_ref) and in this
package's, then applies the same random stream of operations to both:
requantizations (including promotions and evictions), anchors, plans, and
declarative text fed in arbitrary pieces (tags split across calls, unknown
ids, malformed segment lists, stray angle brackets), with reads interleaved.
Every operation must end the same way on both (the same result, or an error
of the same type and message), and after each one the storage reports and
the visible segments must agree.  Materialised K/V are compared bit for bit:
CPU tensors take the flat-segment path, whose codec calls run the oracle here
(bit-exact with the reference).  Paged segments and their page table are
compared with the reference on the GPU (tests/test_gpu_declarative.py).
"""

import numpy as np
import pytest
import torch

import anchorkv_b200 as akv
from host_codec import use_oracle_codec

MODES = ("fp16", "int8", "int4", "evicted")
ROLES = ("sink", "scaffold", "context", "response")


@pytest.fixture
def reference(reference_install, monkeypatch):
    from anchorkv import backend, policy

    use_oracle_codec(monkeypatch)
    return backend, policy


def _norm(x):
    """A comparable form of a result from either implementation."""
    if isinstance(x, torch.Tensor):
        return ("tensor", x.dtype, tuple(x.shape), x.contiguous().view(torch.uint8).reshape(-1).tolist()
                if x.dtype != torch.int64 else x.tolist())
    if hasattr(x, "block_ids") and hasattr(x, "positions"):  # MaterializedCache
        return ("materialized", _norm(x.key), _norm(x.value), _norm(x.positions), x.block_ids, x.segment_ids)
    if hasattr(x, "kind") and hasattr(x, "segment_ids"):  # CacheDirective
        return ("directive", x.kind.value, None if x.mode is None else x.mode.value, x.segment_ids)
    if hasattr(x, "role") and hasattr(x, "token_start"):  # SegmentRecord
        return ("record", x.segment_id, x.role.value, x.token_start, x.token_end, x.protected)
    if hasattr(x, "value") and type(x).__name__ in ("CacheMode", "SegmentRole", "AttentionMode"):
        return ("enum", x.value)
    if isinstance(x, tuple):
        return tuple(_norm(v) for v in x)
    return x


def _outcome(fn):
    try:
        return ("ok", _norm(fn()))
    except Exception as error:  # the type name and message must agree, not the class object
        return ("error", type(error).__name__, str(error))


class _Program:
    def __init__(self, seed, ref_backend, ref_policy):
        self.rng = np.random.default_rng(seed)
        self.RB, self.RPol = ref_backend, ref_policy
        rng = self.rng
        self.block = int(rng.choice([2, 3, 4, 16]))
        self.group = int(rng.choice([2, 4, 8, 16, 64]))
        archive = str(rng.choice(["int4", "int8"]))
        self.layers = int(rng.choice([0, 2]))  # 0: 4-D segments
        self.dtype = [torch.float32, torch.float16, torch.bfloat16][int(rng.integers(3))]
        self.ref = self.RB.DeclarativeKVCache(block_size=self.block, group_size=self.group,
                                              archive_mode=self.RPol.CacheMode(archive))
        self.ours = akv.DeclarativeKVCache(block_size=self.block, group_size=self.group,
                                           archive_mode=akv.CacheMode(archive))
        self.ids, self.cursor, self.gen = [], 0, torch.Generator().manual_seed(seed)

    def tensors(self, tokens):
        shape = ((self.layers,) if self.layers else ()) + (1, 2, tokens, 8)
        return (torch.randn(shape, generator=self.gen).to(self.dtype),
                torch.randn(shape, generator=self.gen).to(self.dtype))

    def both(self, fn):
        a, b = _outcome(lambda: fn(self.ref, self.RB, self.RPol)), _outcome(lambda: fn(self.ours, akv, akv))
        assert a == b, (a, b)
        return a

    def some_ids(self):
        pool = self.ids + [97]  # an id no segment has
        n = int(self.rng.integers(1, 4))
        return [int(self.rng.choice(pool)) for _ in range(n)]

    def add(self):
        rng = self.rng
        sid = int(rng.choice(self.ids)) if self.ids and rng.random() < 0.1 else len(self.ids) + 10 * int(rng.integers(2))
        tokens = int(rng.integers(0 if rng.random() < 0.05 else 1, 21))
        start = self.cursor + int(rng.integers(0, 3)) - (2 if rng.random() < 0.1 else 0)
        role, protected = str(rng.choice(ROLES)), bool(rng.random() < 0.15)
        k, v = self.tensors(max(tokens, 1))
        k, v = k[..., :tokens, :], v[..., :tokens, :]
        res = self.both(lambda c, M, Pm: c.add_segment(sid, k, v, token_start=start, role=M.SegmentRole(role),
                                                      protected=protected))
        if res[0] == "ok":
            self.ids.append(sid)
            self.cursor = start + tokens

    def text(self):
        rng = self.rng
        ids = ", ".join(str(i) for i in self.some_ids())
        pieces = [f'<focus segments="{ids}">', "</focus>", "<local>", "</local>", "<global>",
                  f"<anchor segments='{ids}'>", f'<archive segments="{ids}">', "<focus>",
                  f"<FOCUS magic_chunks='{ids}'>", '<archive segments="1,,2">', "<focus segments='-1'>",
                  "plain words ", "<", ">", "a < b", "< local >", "<unknown tag>", "<anchor segments=\"\">"]
        text = "".join(str(rng.choice(pieces)) for _ in range(int(rng.integers(1, 4))))
        cut = int(rng.integers(0, len(text) + 1))  # a tag may arrive in two pieces
        return text[:cut], text[cut:]

    def step(self):
        rng = self.rng
        op = int(rng.integers(11))
        if op == 0 or not self.ids:
            self.add()
        elif op in (1, 2):
            sid, mode = int(rng.choice(self.ids + [97])), str(rng.choice(MODES))
            self.both(lambda c, M, Pm: c.requantize_segment(sid, Pm.CacheMode(mode)))
        elif op == 3:
            sid = int(rng.choice(self.ids + [97]))
            self.both(lambda c, M, Pm: c.protect_segment(sid))
        elif op in (4, 5):
            for part in self.text():
                self.both(lambda c, M, Pm: c.feed_declarations(part))
        elif op == 6:
            ids = list(self.ids)
            if rng.random() < 0.2 and ids:
                ids.pop()
            modes = [str(rng.choice(MODES)) for _ in ids]
            self.both(lambda c, M, Pm: c.apply_plan(Pm.CachePlan(
                tuple(Pm.PlannedSegment(i, Pm.CacheMode(m), 0, 0.0, "r") for i, m in zip(ids, modes)), 0, 0, 0)))
        elif op == 7:
            dtype = [None, torch.float32, torch.float16, torch.bfloat16][int(rng.integers(4))]
            self.both(lambda c, M, Pm: c.materialize_visible(dtype=dtype))
        elif op == 8:
            ids = self.some_ids() + self.some_ids()
            self.both(lambda c, M, Pm: c.materialize_segments(ids))
        elif op == 9:
            sid = int(rng.choice(self.ids + [97]))
            self.both(lambda c, M, Pm: c.segment_mode(sid))
        else:
            self.both(lambda c, M, Pm: c.visible_segment_ids())
        self.both(lambda c, M, Pm: c.storage_report())
        self.both(lambda c, M, Pm: (c.resident_bytes, c.full_precision_bytes, c.compression_ratio))
        self.both(lambda c, M, Pm: (c.parser.state.mode.value, c.parser.state.focus_segment_ids))


@pytest.mark.parametrize("seed", range(40))
def test_random_programs_match_the_reference(reference, seed):
    program = _Program(seed, *reference)
    for _ in range(int(program.rng.integers(3, 6))):
        program.add()
    for _ in range(40):
        program.step()
    if program.layers:  # the legacy cache view of 5-D segments
        program.both(lambda c, M, Pm: c.materialize_visible().to_legacy_cache())


PARSER_PIECES = ["<", ">", "<<", ">>", "focus", "FOCUS", "Focus", "/focus", "local", "/local", "global", "anchor",
                 "archive", " ", "  ", "segments", "magic_chunks", "SEGMENTS", "=", " = ", '"', "'", "1", "2", "17",
                 ",", ", ", "-", "x", "\n", "<focus segments=\"3\">", "</focus>", "<archive segments='4,5'>",
                 "<anchor segments=\"2, 2\">", "< global >", "<local/>", "<focusx segments=\"1\">", "<>",
                 "<local>", "< LOCAL >", "</local>", "<focus segments=\"1,,2\">", "<archive segments=\"-3\">",
                 "<anchor magic_chunks='0'>"]


@pytest.mark.parametrize("seed", range(30))
def test_parser_fuzz_matches_the_reference(reference, seed):
    """Random streams of tag fragments, fed in random chunks, give the same directives,
    errors and parser state after every chunk as the reference's parser."""
    RB, _ = reference
    rng = np.random.default_rng(1000 + seed)
    ours, ref = akv.DeclarativeAttentionParser(), RB.DeclarativeAttentionParser()
    for _ in range(60):
        chunk = "".join(str(rng.choice(PARSER_PIECES)) for _ in range(int(rng.integers(1, 6))))
        a = _outcome(lambda: ref.feed(chunk))
        b = _outcome(lambda: ours.feed(chunk))
        assert a == b, (chunk, a, b)
        assert (ref.state.mode.value, ref.state.focus_segment_ids) == \
            (ours.state.mode.value, ours.state.focus_segment_ids), chunk
