"""The cross-GPU exchange's ordering argument, checked on a model on the CPU.

merge_exchange_kernel (csrc/akv_decode.cu) moves every value as one 64-bit word
that carries the epoch of the call that wrote it, into slot [epoch & 1][source
rank] of every rank's buffer; a rank's call e reads the words of [e & 1][*]
once they all carry e.  The stream gives two orderings: a rank's decode of call
e + 1 starts only after its exchange grid of call e has completed, and its
exchange of e + 1 only after that decode.

The model runs W ranks through E calls under random interleavings.  Each word
store lands on its own (64-bit stores are single-copy atomic, nothing more is
assumed about their order), each rank's wait polls its own buffer, and a call
completes once every word it needs carried its epoch.  With two parity halves
no schedule deadlocks and every word a rank merges is the value that the
source rank wrote in the same call.  With one half the model finds the race
the halves remove: a fast rank's next call overwrites a word that a slower
rank has not read yet, which then waits for a tag that never comes back."""

import random

import pytest

WORDS = 3  # words per (source rank, row): enough to let the stores of one state land apart


def value(src, epoch, word):
    return (src * 1000 + epoch) * 10 + word


def run(world, epochs, halves, seed, tags=None):
    """Returns None if every call of every rank completed with the right values,
    else a string naming the first violation (a wrong value or a stuck wait).

    ``tags[e]`` is the epoch word call ``e`` (1-based) passes to the kernel
    (default: ``e``); the kernel compares tags only, so the model records each
    word's call beside its tag to see whether a matching tag ever names the
    wrong call."""
    rng = random.Random(seed)
    tags = list(range(epochs + 1)) if tags is None else tags
    buf = [[[[(0, 0, 0)] * WORDS for _ in range(world)] for _ in range(halves)] for _ in range(world)]
    call = [0] * world           # last completed call per rank
    phase = ["idle"] * world     # idle -> stored (publishing) -> done
    pending = [None] * world     # word stores of the current call not yet landed
    seen = [None] * world        # words of the current call read so far
    while True:
        actions = []
        for r in range(world):
            if call[r] == epochs:
                continue
            e = call[r] + 1
            if phase[r] == "idle":
                actions.append(("start", r))
            elif phase[r] == "stored":
                if pending[r]:
                    actions.append(("land", r))
                if any(v is None for v in seen[r]):
                    actions.append(("poll", r))
                if not pending[r] and all(v is not None for v in seen[r]):
                    actions.append(("finish", r))
        if not actions:
            if all(c == epochs for c in call):
                return None
            stuck = [r for r in range(world) if call[r] < epochs]
            return f"deadlock: ranks {stuck} wait for words that never carry their epoch"
        kind, r = rng.choice(actions)
        e = call[r] + 1
        half = tags[e] % halves
        if kind == "start":  # the decode of call e ran; the exchange kernel begins storing
            pending[r] = [(p, w) for p in range(world) for w in range(WORDS)]
            rng.shuffle(pending[r])
            seen[r] = [None] * (world * WORDS)
            phase[r] = "stored"
        elif kind == "land":  # one word store reaches rank p's buffer
            p, w = pending[r].pop()
            buf[p][half][r][w] = (e, tags[e], value(r, e, w))
        elif kind == "poll":  # the waiting CTA reads one word of its own buffer
            idx = rng.choice([i for i, v in enumerate(seen[r]) if v is None])
            src, w = divmod(idx, WORDS)
            writer, tag, v = buf[r][half][src][w]
            if tag == tags[e]:  # what the kernel checks
                if writer != e or v != value(src, e, w):
                    return f"rank {r} call {e} read {v} from rank {src}'s call {writer}, expected {value(src, e, w)}"
                seen[r][idx] = v
            elif writer > e:
                return f"deadlock: rank {r} call {e} finds rank {src}'s word already at call {writer}"
        elif kind == "finish":  # the grid completes; the next decode may start
            call[r] = e
            phase[r] = "idle"


@pytest.mark.parametrize("world", [2, 3, 4, 8])
def test_two_parity_halves_never_mix_calls_or_stall(world):
    for seed in range(400 if world < 8 else 60):
        assert run(world, epochs=7, halves=2, seed=seed) is None, seed


def test_one_half_lets_a_fast_rank_overwrite_an_unread_word():
    failures = [run(2, epochs=7, halves=1, seed=s) for s in range(400)]
    assert any(f is not None for f in failures)
    assert all(f is None or f.startswith("deadlock") for f in failures)


def _host_tags(first, epochs):
    """Epoch words of calls 1..epochs as PeerExchange issues them, the first being ``first``."""
    from anchorkv_b200.sharded import next_epoch

    tags = [0, first]
    while len(tags) <= epochs:
        tags.append(next_epoch(tags[-1]))
    return tags


def test_epochs_that_run_out_of_32_bits_keep_the_halves_apart():
    """Across the wrap of the 32-bit epoch (0xFFFFFFFF, then 2, 3, ...) calls still
    alternate halves and never take a word of another call for their own."""
    tags = _host_tags(0xFFFFFFFC, 9)
    assert tags[1:] == [0xFFFFFFFC, 0xFFFFFFFD, 0xFFFFFFFE, 0xFFFFFFFF, 2, 3, 4, 5, 6]
    assert all(t != 0 for t in tags[1:])
    for world in (2, 3, 4):
        for seed in range(300):
            assert run(world, epochs=9, halves=2, seed=seed, tags=tags) is None, (world, seed)


def test_a_wrap_that_repeats_a_parity_is_caught():
    """Wrapping 0xFFFFFFFF to 1 would put two consecutive calls in one half, the race
    the halves exist to remove; the model finds it."""
    tags = [0, 0xFFFFFFFE, 0xFFFFFFFF, 1, 2, 3, 4, 5]
    failures = [run(2, epochs=7, halves=2, seed=s, tags=tags) for s in range(400)]
    assert any(f is not None for f in failures)
