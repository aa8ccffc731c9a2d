"""The fork-aware closure at n-gram orders 2 and 4 on the device
(tree_ops.ngram_path_fn's `order`, tree_ops.py:55-66; the Builder itself uses
order 3, fc1_builder.py:31).

* the dense PMI tensor T of each order against the reference's own T (a
  seeded sample kept in the golden fixture) and against the whole oracle T,
  within 1e-5;
* the tree_ops mirror (score -> ngram_path_fn -> beam_tree -> tree_struct)
  against the reference's beam over that T, bit-exact barring classified fp32
  score ties;
* the batched score+build at order 4 against the oracle per request;
* a probe that misses for the key 0 (context trigram (0, 0, 0) absent) backs
  off like the reference's searchsorted lookup (ngram_gpu.py:28-33).
"""
import os

import numpy as np
import pytest
import torch

from oracle import builder as OB
from oracle import ngram as ON
from tests.golden import cases

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from dforktree_b200 import build
    build.build()


def _gold(name):
    return np.load(os.path.join(GOLD, name + ".npz"))


def _np(t):
    return t.detach().cpu().numpy()


def _ng(table):
    from dforktree_b200.ngram_gpu import NGramGPU
    return NGramGPU(table, DEV, beta3=60.0)


def _tie_gap(trace, W, N):
    gaps = []
    for t in trace[:-1] + [trace[-1][:N]]:
        t = t[: W + 1]
        t = t[np.isfinite(t)]
        if t.size > 1:
            gaps.append(np.min(np.abs(np.diff(t)) / np.maximum(np.abs(t[:-1]), 1.0)))
    return min(gaps) if gaps else np.inf


def _check_tree(got, ref, keys, trace, N, name):
    bad = [k for k in keys if not np.array_equal(np.asarray(got[k]), np.asarray(ref[k]))]
    if bad:
        gap = _tie_gap(trace, max(N - 1, 16), N)
        assert gap < 1e-5, f"{name}: tree differs in {bad} (no fp32 tie: gap {gap:.2e})"
        pytest.xfail(f"{name}: fp32 score tie (relative gap {gap:.2e}) flips {bad}")


@pytest.mark.parametrize("case", cases.ORDER_CASES, ids=lambda c: c["name"])
def test_pmi_dense_other_orders(case):
    from dforktree_b200 import kernels as K
    g = _gold(case["name"])
    table, _, root, pre1 = cases.order_inputs(case)
    ng = _ng(table)
    ids = torch.from_numpy(g["ids"]).to(DEV)[None].int()
    T = K.pmi_dense(ng.table, ids, torch.tensor([root], device=DEV), torch.tensor([pre1], device=DEV),
                    status=ng.status, order=case["order"])
    assert tuple(T.shape) == (1,) + tuple(g["T_shape"])
    Tn = _np(T)[0]
    np.testing.assert_allclose(Tn.reshape(-1)[g["T_index"]], g["T_sample"], rtol=1e-5, atol=1e-5)
    ref = OB.dense_pmi(ON.NGramOracle(table, beta3=60.0), case["order"], g["ids"], pre1, root)
    np.testing.assert_allclose(Tn, ref, rtol=1e-5, atol=1e-5)
    assert ng.device_status() == 0


@pytest.mark.parametrize("case", cases.ORDER_CASES, ids=lambda c: c["name"])
def test_tree_ops_other_orders_match_reference(case):
    from dforktree_b200 import kernels as K
    from dforktree_b200 import tree_ops as TO
    g = _gold(case["name"])
    table, logits, root, pre1 = cases.order_inputs(case)
    ng = _ng(table)
    S, N = case["S"], case["N"]
    lp, ids, rest = K.score(torch.from_numpy(logits).to(DEV))
    np.testing.assert_array_equal(_np(ids)[0], g["ids"])
    lp0, rest0 = lp[0], rest[0]
    c0 = lp0[0] - torch.logsumexp(torch.cat((lp0[0], rest0[:1])), 0)          # fc1_builder.py:29
    rt, p1 = torch.tensor([root], device=DEV), torch.tensor([pre1], device=DEV)
    fn = TO.ngram_path_fn(ng, case["order"], ids[0], lp0, rest0, p1, rt, 0.3, 0.6)
    assert fn.order == case["order"] and tuple(fn.T.shape[1:]) == tuple(g["T_shape"])
    ss, cand, parent, flags = TO.beam_tree(c0, None, N, 99, case["chain_first"], fn, S=S, root=rt)
    parent_full = torch.cat((torch.tensor([-1], device=DEV), parent + 1))
    anc, depth, cidx = TO.tree_struct(parent_full)
    got = dict(ss=_np(ss), cand=_np(cand), flags=_np(flags), parent=_np(parent_full), anc=_np(anc),
               depth=_np(depth), cidx=_np(cidx), tokens=np.concatenate([[root], g["ids"][_np(ss), _np(cand)]]))
    trace = []
    OB.builder_run(logits, root, pre1, ON.NGramOracle(table, beta3=60.0), N=N, chain_first=case["chain_first"],
                   order=case["order"], trace=trace)
    _check_tree(got, {k: g[k] for k in got}, tuple(got), trace, N, case["name"])
    assert ng.device_status() == 0


def test_score_build_order4_batched_matches_oracle():
    from dforktree_b200 import kernels as K
    from dforktree_b200 import synth
    case = next(c for c in cases.ORDER_CASES if c["order"] == 4 and not c["chain_first"])
    table, logits0, root0, pre10 = cases.order_inputs(case)
    ng = _ng(table)
    ong = ON.NGramOracle(table, beta3=60.0)
    S, V, N, B = case["S"], case["V"], case["N"], 3
    logits = [logits0] + [synth.make_logits(S, V, seed=900 + r) for r in range(1, B)]
    rng = np.random.default_rng(3)
    roots = [root0] + [int(x) for x in synth.zipf_ids(rng, B - 1, V)]
    pre1s = [pre10] + [int(x) for x in synth.zipf_ids(rng, B - 1, V)]
    lt = torch.from_numpy(np.stack(logits)).to(DEV)
    rt = torch.tensor(roots, device=DEV)
    p1 = torch.tensor(pre1s, device=DEV)
    ws = K.score_build_workspace(B, S, V, N, device=DEV, order=4)
    assert ws.numel() > B * (S - 1) * 16 ** 4 * 4
    out = K.tree_outputs(B, S, N, DEV)
    K.score_build(ng.table, lt, rt, p1, N, ws, out, status=ng.status, order=4)
    with pytest.raises(Exception):
        K.score_build(ng.table, lt, rt, None, N, ws, out, order=4)       # order 4 reads pre1: required
    torch.cuda.synchronize()
    for r in range(B):
        trace = []
        ref = OB.builder_run(logits[r], roots[r], pre1s[r], ong, N=N, order=4, trace=trace)
        got = {k: _np(out[k][r]) for k in ("tokens", "parent", "depth", "anc", "cidx", "nxt", "sib")}
        _check_tree(got, ref, tuple(got), trace, N, f"request {r}")
    assert ng.device_status() == 0


def test_p4_backs_off_when_the_zero_context_is_absent():
    """keys3 without the key 0: the context trigram (0, 0, 0) is absent, so
    p4(0, 0, 0, c) = (0 + beta4 p3) / (0 + beta4) even though quadgram rows
    of trigram rank 0 exist (n4c[0] > 0) -- a lookup that took a miss for a
    hit on key 0 would read them."""
    from dforktree_b200.ngram_gpu import NGramGPU
    V = 8
    k2 = np.array([0 * V + 5, 1 * V + 2, 2 * V + 3], np.int64)
    k3 = np.array([(1 * V + 2) * V + 3, (2 * V + 3) * V + 4], np.int64)
    k4 = np.array([0 * V + 5, 1 * V + 1], np.int64)                 # rank-0 trigram followed by 5; rank 1 by 1
    table = dict(V=np.int64(V), N=np.int64(40), keys=k2, cab=np.array([4, 6, 7], np.int64),
                 prev=np.array([4, 6, 7, 0, 0, 0, 0, 0], np.int64), nxt=np.array([0, 0, 6, 7, 0, 4, 0, 0], np.int64),
                 keys3=k3, c3=np.array([3, 2], np.int64), keys3c=np.array([1 * V + 2, 2 * V + 3], np.int64),
                 n3c=np.array([3, 2], np.int64), keys4=k4, c4=np.array([9, 5], np.int64),
                 n4c=np.array([9, 5], np.int64))
    ng = NGramGPU(table, DEV, beta3=60.0)
    ong = ON.NGramOracle(table, beta3=60.0)
    z = np.array([0, 0, 1, 1, 0], np.int64)
    a = np.array([0, 0, 2, 2, 1], np.int64)
    b = np.array([0, 0, 3, 3, 2], np.int64)
    c = np.array([5, 1, 5, 1, 3], np.int64)
    t = lambda x: torch.from_numpy(x).to(DEV)
    np.testing.assert_array_equal(_np(ng.p4(t(z), t(a), t(b), t(c))), ong.p4(z, a, b, c))
    np.testing.assert_allclose(_np(ng.pmi(4, t(z), t(a), t(b), t(c))), ong.pmi(4, z, a, b, c), rtol=1e-5, atol=1e-5)
    assert ng.device_status() == 0
