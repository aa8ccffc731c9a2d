"""Host-side checks of the n-gram order argument (no GPU): the T shape per
order, invalid orders rejected before any device call, and the oracle's
closure reading T by its rank exactly as tree_ops.py:28-40 carries cand /
pc / ppc."""
import numpy as np
import pytest

from oracle import builder as OB


def test_pmi_step_shape_per_order():
    from dforktree_b200 import kernels as K
    assert K.pmi_step_shape(2) == (16, 16)
    assert K.pmi_step_shape(3) == (16, 16, 16)
    assert K.pmi_step_shape(4) == (16, 16, 16, 16)
    for bad in (1, 5, 0):
        with pytest.raises(ValueError):
            K.pmi_step_shape(bad)


def test_ngram_path_fn_rejects_unknown_order():
    from dforktree_b200 import tree_ops as TO
    with pytest.raises(ValueError):
        TO.ngram_path_fn(None, 5, None, None, None, None, None, 0.3, 0.6)


def test_oracle_closure_indexes_t_by_order():
    rng = np.random.default_rng(0)
    S, M, W = 4, 16, 5
    lp = rng.standard_normal((S, M)).astype(np.float32)
    rest = rng.standard_normal(S).astype(np.float32)
    cand = rng.integers(0, M, W)
    pc = rng.integers(0, M, W)
    ppc = rng.integers(0, M, W)
    al = rng.random(W) < 0.5
    for order in (2, 3, 4):
        T = rng.standard_normal((S - 1,) + (M,) * order).astype(np.float32)
        fn = OB.path_scores(T, lp, rest, 0.3, 0.6)
        s = 2
        got = fn(s, cand, pc, ppc, al)
        for w in range(W):
            idx = {2: (cand[w],), 3: (pc[w], cand[w]), 4: (ppc[w], pc[w], cand[w])}[order]
            t = T[s - 1][idx]
            lam = np.float32(0.3 if al[w] else 0.6)
            x = (lp[s] + (lam * t).astype(np.float32)).astype(np.float32)
            m = max(x.max(), rest[s])
            lse = np.float32(np.log(np.exp(x - m).sum(dtype=np.float32) + np.exp(rest[s] - m)) + m)
            np.testing.assert_allclose(got[w], x - lse, rtol=1e-5, atol=1e-5)
