"""akv_merge_states (merge_states): n LSE states per (sequence, query head) row,
as gathered from n GPUs, merged into the normalised output, against the
oracle's float64 log-sum-exp merge (the algebra of triton_decode.py:70-82).

The states' maxima are base-2 units of the scaled score; the oracle's are
natural-log, so they are converted (2^(m - top) = e^(m ln 2 - top ln 2))."""

import math

import numpy as np
import pytest
import torch

import anchorkv_b200 as akv
from oracle import attention as OA

pytestmark = pytest.mark.gpu


def _states(n, batch, heads, dim, seed):
    g = np.random.default_rng(seed)
    acc = g.standard_normal((n, batch, heads, dim)) * g.uniform(0.1, 50, (n, batch, heads, 1))
    m = g.uniform(-30, 30, (n, batch, heads))
    l = g.uniform(0.5, 200, (n, batch, heads))
    empty = g.random((n, batch, heads)) < 0.15  # empty shares: max -inf, weight 0
    m[empty] = -np.inf
    l[empty] = 0.0
    acc[empty] = 0.0
    if n > 1:
        m[:, 0, 0] = -np.inf  # one row with every share empty
        l[:, 0, 0] = 0.0
        acc[:, 0, 0] = 0.0
    st = np.concatenate([acc, m[..., None], l[..., None]], axis=-1).astype(np.float32)
    return st


@pytest.mark.parametrize("dim", [64, 128])
@pytest.mark.parametrize("n", [1, 3, 8, 9, 40])
def test_merge_states_against_oracle(cuda, n, dim):
    batch, heads = 5, 6
    st = _states(n, batch, heads, dim, seed=n * 131 + dim)
    out = akv.merge_states(torch.from_numpy(st).to(cuda)).float().cpu().numpy()  # [batch, heads, 1, dim]
    for b in range(batch):
        for h in range(heads):
            parts = [(st[s, b, h, :dim].astype(np.float64), float(st[s, b, h, dim]) * math.log(2.0),
                      float(st[s, b, h, dim + 1])) for s in range(n)]
            want = OA.lse_merge_f64(parts)
            np.testing.assert_allclose(out[b, h, 0], want, atol=2e-3, rtol=1e-2)
    if n > 1:
        assert (out[0, 0] == 0).all()  # every share empty: zeros
