"""GPU parity of every sm_100a kernel against the reference goldens and the
CPU oracle.  Bars (north star): tree tokens / parents bit-exact barring fp32
score ties (classified below), PMI within 1e-5, GDN outputs and committed
states within 2e-2 (bf16) / 1e-3 (fp32) relative to the largest magnitude.
"""
import os

import numpy as np
import pytest
import torch

from oracle import builder as OB
from oracle import gdn as OG
from oracle import ngram as ON
from tests.golden import cases

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DEV = "cuda"


def _gold(name):
    return np.load(os.path.join(GOLD, name + ".npz"))


def _np(t):
    return t.detach().cpu().numpy()


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from dforktree_b200 import build
    build.build()


def _ng(table, beta3=60.0):
    from dforktree_b200.ngram_gpu import NGramGPU
    return NGramGPU(table, DEV, beta3=beta3)


# ------------------------------------------------------------------ n-gram --
def test_ngram_eval_matches_reference_golden():
    g = _gold("ngram_small")
    table = cases.ngram_table()
    z, a, b, c = (torch.from_numpy(x).to(DEV) for x in cases.ngram_queries(int(table["V"])))
    for name, b3 in (("b20", 20.0), ("b60", 60.0)):
        ng = _ng(table, b3)
        np.testing.assert_array_equal(_np(ng.pn), g["pn"])
        np.testing.assert_array_equal(_np(ng.p2(b, c)), g[f"p2_{name}"])
        np.testing.assert_array_equal(_np(ng.p3(a, b, c)), g[f"p3_{name}"])
        np.testing.assert_array_equal(_np(ng.p4(z, a, b, c)), g[f"p4_{name}"])
        for order in (2, 3, 4):
            np.testing.assert_allclose(_np(ng.pmi(order, z, a, b, c)), g[f"pmi{order}_{name}"], rtol=1e-5,
                                       atol=1e-5)
        assert ng.device_status() == 0


def test_ngram_broadcast_shapes_and_bad_token_status():
    table = cases.ngram_table()
    ng = _ng(table)
    V = int(table["V"])
    a = torch.arange(4, device=DEV)[:, None, None]
    b = torch.arange(5, device=DEV)[None, :, None]
    c = torch.arange(6, device=DEV)[None, None, :]
    out = ng.pmi(3, None, a, b, c)
    assert out.shape == (4, 5, 6)
    ref = ON.NGramOracle(table, beta3=60.0).pmi(3, None, _np(a), _np(b), _np(c))
    np.testing.assert_allclose(_np(out), ref, rtol=1e-5, atol=1e-5)
    assert ng.device_status() == 0
    ng.p2(torch.tensor([3], device=DEV), torch.tensor([V + 5], device=DEV))
    assert ng.device_status() & 1  # DFT_DEV_BAD_TOKEN, raised without a fault


def test_table_rejects_unsorted_keys():
    from dforktree_b200 import kernels as K
    from dforktree_b200._lib import DFTError
    from dforktree_b200.ngram_gpu import load_npz_arrays
    t = load_npz_arrays(cases.ngram_table())
    t["keys"] = t["keys"][::-1].copy()
    with pytest.raises(DFTError, match="unsorted"):
        K.Table(t)


# ------------------------------------------------------------------- score --
@pytest.mark.parametrize("case", cases.BUILDER_CASES[:4], ids=lambda c: c["name"])
def test_score_matches_oracle(case):
    from dforktree_b200 import kernels as K
    _, logits, _, _ = cases.builder_inputs(case)
    lp, ids, rest = K.score(torch.from_numpy(logits).to(DEV))
    olp, oids, orest, _ = OB.score(logits)
    np.testing.assert_array_equal(_np(ids)[0], oids)
    np.testing.assert_allclose(_np(lp)[0], olp, rtol=2e-6, atol=2e-6)
    # rest = log(1 - sum exp(lp)) is ill-conditioned when the top-16 mass is ~1:
    # compare the out-of-list mass itself
    np.testing.assert_allclose(np.exp(_np(rest)[0]), np.exp(orest), rtol=1e-4, atol=2e-6)


def test_score_full_vocab_and_bf16():
    from dforktree_b200 import kernels as K
    x = np.stack([cases.config0_inputs(s, table={})[1] for s in (0, 1)])   # table unused
    xt = torch.from_numpy(x).to(DEV)
    lp, ids, rest = K.score(xt)
    for b in range(2):
        olp, oids, orest, _ = OB.score(x[b])
        np.testing.assert_array_equal(_np(ids)[b], oids)
        np.testing.assert_allclose(_np(lp)[b], olp, rtol=2e-6, atol=3e-6)
        np.testing.assert_allclose(_np(rest)[b], orest, rtol=1e-5, atol=1e-5)
    xb = xt.to(torch.bfloat16)
    lp, ids, rest = K.score(xb)
    olp, oids, orest, _ = OB.score(_np(xb[0].float()))
    # bf16 logits have many exact ties: compare the selected values, not the order of equal ones
    np.testing.assert_allclose(np.sort(_np(xb[0].float())[np.arange(24)[:, None], _np(ids)[0]], 1),
                               np.sort(_np(xb[0].float())[np.arange(24)[:, None], oids], 1))
    np.testing.assert_allclose(_np(lp)[0], olp, rtol=2e-6, atol=3e-6)


def test_score_unaligned_rows():
    """Row starts off a 16-byte boundary exercise the scalar head/tail path."""
    from dforktree_b200 import kernels as K
    rng = np.random.default_rng(5)
    V = 5003
    x = (rng.standard_normal((3, V)) * 3).astype(np.float32)
    xt = torch.from_numpy(np.concatenate([np.zeros(1, np.float32), x.reshape(-1)])).to(DEV)[1:].view(3, V)
    lp, ids, rest = K.score(xt)
    olp, oids, orest, _ = OB.score(x)
    np.testing.assert_array_equal(_np(ids)[0], oids)
    np.testing.assert_allclose(_np(lp)[0], olp, rtol=2e-6, atol=2e-6)


# ---------------------------------------------------------- score + build --
def _tie_gap(trace, W, N):
    """Smallest relative gap between adjacent keys the reference's top-k calls
    rank (per step: the top W+1; final: the top N)."""
    gaps = []
    for t in trace[:-1]:
        t = t[: W + 1]
        t = t[np.isfinite(t)]
        if t.size > 1:
            gaps.append(np.min(np.abs(np.diff(t)) / np.maximum(np.abs(t[:-1]), 1.0)))
    t = trace[-1][:N]
    t = t[np.isfinite(t)]
    if t.size > 1:
        gaps.append(np.min(np.abs(np.diff(t)) / np.maximum(np.abs(t[:-1]), 1.0)))
    return min(gaps) if gaps else np.inf


def _assert_tree(got, ref, trace=None, N=32, name=""):
    keys = ("tokens", "parent", "depth", "anc", "cidx", "nxt", "sib")
    bad = [k for k in keys if not np.array_equal(np.asarray(got[k]), np.asarray(ref[k]))]
    if not bad:
        return
    if trace is not None:
        gap = _tie_gap(trace, max(N - 1, 16), N)
        if gap < 1e-5:
            pytest.xfail(f"{name}: fp32 score tie (relative gap {gap:.2e}) flips {bad}")
    raise AssertionError(f"{name}: tree differs in {bad}")


@pytest.mark.parametrize("case", cases.BUILDER_CASES, ids=lambda c: c["name"])
def test_builder_matches_reference_golden(case, monkeypatch):
    from dforktree_b200.fc1_builder import Builder
    monkeypatch.setenv("FC1_CHAIN_FIRST", "1" if case["chain_first"] else "0")
    g = _gold(case["name"])
    table, logits, root, pre1 = cases.builder_inputs(case)
    lt = torch.from_numpy(logits).to(DEV)
    ng = _ng(table) if case["ngram"] else None
    bld = Builder(lt, ngram=case["ngram"], ng=ng, n=case["N"])
    tree, depth, parent, anc, nxt, sib = bld(lt, torch.tensor([root], device=DEV), torch.tensor([pre1], device=DEV))
    got = dict(tokens=_np(tree)[0], parent=_np(parent), depth=_np(depth), anc=_np(anc), cidx=_np(bld.cidx),
               nxt=_np(nxt), sib=_np(sib))
    trace = []
    OB.builder_run(logits, root, pre1, ON.NGramOracle(table, beta3=60.0) if case["ngram"] else None, N=case["N"],
                   chain_first=case["chain_first"], trace=trace)
    _assert_tree(got, {k: g[k] for k in got}, trace, case["N"], case["name"])
    assert bld.device_status() == 0


def test_pmi_dense_matches_reference_golden():
    from dforktree_b200 import kernels as K
    for case in [c for c in cases.BUILDER_CASES if c["ngram"]][:3]:
        g = _gold(case["name"])
        table, _, root, pre1 = cases.builder_inputs(case)
        ng = _ng(table)
        ids = torch.from_numpy(g["ids"]).to(DEV)[None].int()
        T = K.pmi_dense(ng.table, ids, torch.tensor([root], device=DEV), torch.tensor([pre1], device=DEV))
        np.testing.assert_allclose(_np(T)[0], g["T"], rtol=1e-5, atol=1e-5)


def test_builder_batched_matches_oracle_per_request():
    """One batched launch over 8 requests (config 1 semantics at V=2048)."""
    from dforktree_b200.fc1_builder import Builder
    base = dict(cases.BUILDER_CASES[0])
    table, _, _, _ = cases.builder_inputs(base)
    ng = _ng(table)
    ong = ON.NGramOracle(table, beta3=60.0)
    B = 8
    logits, roots, pre1s = [], [], []
    for r in range(B):
        c = dict(base, seed=500 + r)
        _, lg, rt, p1 = cases.builder_inputs(c)
        logits.append(lg)
        roots.append(rt)
        pre1s.append(p1)
    lt = torch.from_numpy(np.stack(logits)).to(DEV)
    bld = Builder(lt, ng=ng, n=32)
    tree, depth, parent, anc, nxt, sib = bld(lt, torch.tensor(roots, device=DEV), torch.tensor(pre1s, device=DEV))
    for r in range(B):
        trace = []
        ref = OB.builder_run(logits[r], roots[r], pre1s[r], ong, N=32, trace=trace)
        got = dict(tokens=_np(tree)[r], parent=_np(parent)[r], depth=_np(depth)[r], anc=_np(anc)[r],
                   cidx=_np(bld.cidx)[r], nxt=_np(nxt)[r], sib=_np(sib)[r])
        _assert_tree(got, ref, trace, 32, f"req{r}")


@pytest.fixture(scope="module")
def config0_table():
    c = cases.CONFIG0
    from dforktree_b200 import synth
    return synth.make_ngram_table(c["V"], c["nb"], c["nt"], seed=c["table_seed"])


def test_builder_config0_full_vocab_matches_reference(config0_table):
    from dforktree_b200.fc1_builder import Builder
    ng = _ng(config0_table)
    for seed in cases.CONFIG0_SEEDS:
        g = _gold(f"config0_seed{seed}")
        _, logits, root, pre1 = cases.config0_inputs(seed, config0_table)
        lt = torch.from_numpy(logits).to(DEV)
        bld = Builder(lt, ng=ng, n=32, graph=False)
        tree, depth, parent, anc, nxt, sib = bld(lt, torch.tensor([root], device=DEV),
                                                 torch.tensor([pre1], device=DEV))
        got = dict(tokens=_np(tree)[0], parent=_np(parent), depth=_np(depth), cidx=_np(bld.cidx), nxt=_np(nxt),
                   sib=_np(sib), anc=_np(anc))
        ref = {k: g[k] for k in ("tokens", "parent", "depth", "cidx", "nxt", "sib")}
        ref["anc"] = OB.tree_struct(g["parent"], 4)[0]
        _assert_tree(got, ref, None, 32, f"config0 seed {seed}")


# ------------------------------------------------------------ tree utilities --
def test_tree_struct_and_accept_greedy_random():
    from dforktree_b200 import kernels as K
    from dforktree_b200 import synth
    rng = np.random.default_rng(7)
    for N in (1, 2, 16, 32, 64):
        B = 6
        par = np.stack([synth.random_tree_parents(N, rng, chain_p=0.5 * (b % 2)) for b in range(B)])
        anc, depth, cidx, nxt, sib = K.tree_struct(torch.from_numpy(par).to(DEV))
        for b in range(B):
            oa, od, oc = OB.tree_struct(par[b], 4)
            on, osb = OB.next_and_sibling(par[b])
            np.testing.assert_array_equal(_np(anc)[b], oa)
            np.testing.assert_array_equal(_np(depth)[b], od)
            np.testing.assert_array_equal(_np(cidx)[b], oc)
            np.testing.assert_array_equal(_np(nxt)[b], on)
            np.testing.assert_array_equal(_np(sib)[b], osb)
        tokens = rng.integers(0, 5, (B, N))
        target = rng.integers(0, 5, (B, N))
        P = 24
        path, alen, last, bonus = K.accept_greedy(*(torch.from_numpy(x).to(DEV) for x in (tokens,)), nxt, sib,
                                                  torch.from_numpy(target).to(DEV), P)
        for b in range(B):
            cur, acc = 0, [0]
            while True:
                ch = [v for v in range(1, N) if par[b][v] == cur]
                hit = [v for v in ch if tokens[b][v] == target[b][cur]]
                if not hit:
                    break
                cur = hit[0]
                acc.append(cur)
            exp = np.full(P, -1)
            exp[:min(len(acc), P)] = acc[:P]
            np.testing.assert_array_equal(_np(path)[b], exp)
            assert int(alen[b]) == len(acc) and int(last[b]) == cur and int(bonus[b]) == target[b][cur]


# -------------------------------------------------------------------- conv --
@pytest.mark.parametrize("case", cases.CONV_CASES, ids=lambda c: c["name"])
def test_conv_matches_reference_golden(case):
    from dforktree_b200 import fc1_conv, tree_kernels
    g = _gold(case["name"])
    parent, x, cs, w, bias = cases.conv_inputs(case)
    N, Cn = x.shape
    cidx = torch.from_numpy(g["cidx"]).to(DEV)
    xt = torch.from_numpy(x.T.copy()).to(DEV)[None]                   # [1, C, N] channels-first
    iw = torch.zeros(case["dst_slots"], N, Cn, 3, device=DEV)
    y = fc1_conv.conv(torch.from_numpy(cs).to(DEV), xt, torch.from_numpy(w).to(DEV), torch.from_numpy(bias).to(DEV),
                      cidx, torch.tensor([case["slot"]], device=DEV), torch.tensor([case["dst"]], device=DEV), iw)
    np.testing.assert_allclose(_np(y)[0], g["y"], rtol=1e-6, atol=1e-6)
    np.testing.assert_array_equal(_np(iw), g["iw"])
    y2 = tree_kernels.tree_conv_fused(torch.from_numpy(cs[case["slot"]]).to(DEV), torch.from_numpy(x).to(DEV), cidx,
                                      torch.from_numpy(w).to(DEV), torch.from_numpy(bias).to(DEV))
    np.testing.assert_allclose(_np(y2), g["y_fused"], rtol=1e-6, atol=1e-6)


# --------------------------------------------------------------------- GDN --
def _rel(a, b):
    return float(np.abs(np.asarray(a, np.float64) - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.mark.parametrize("case", cases.GDN_CASES, ids=lambda c: c["name"])
def test_gdn_verify_matches_reference_golden(case):
    from dforktree_b200 import tree_kernels
    g = _gold(case["name"])
    d = cases.gdn_inputs(case)
    N, Hk, Hv, D = case["N"], case["Hk"], case["Hv"], case["D"]
    pool = torch.from_numpy(d["pool"]).to(DEV)
    keys = torch.zeros(Hv, N, D, device=DEV)
    values = torch.zeros(Hv, N, D, device=DEV)
    gains = torch.zeros(Hv, N, device=DEV)
    A_log = torch.from_numpy(d["A_log"]).to(DEV)
    o = tree_kernels.tree_gdn_split(torch.from_numpy(d["y"]).to(DEV), torch.from_numpy(d["a"]).to(DEV),
                                    torch.from_numpy(d["b"]).to(DEV), A_log, torch.from_numpy(d["dt_bias"]).to(DEV),
                                    pool[0].transpose(-1, -2), torch.from_numpy(d["anc"]).to(DEV), Hk, Hv, D, D,
                                    aux=(keys, values, gains), neg_exp_A=-A_log.exp(),
                                    state_indices=torch.tensor([case["slot"]], dtype=torch.int32, device=DEV),
                                    state_slot_stride=pool.stride(0))
    assert _rel(_np(o), g["o"]) < 1e-3
    assert _rel(_np(keys), g["k"]) < 1e-5
    assert _rel(_np(values), g["vn"]) < 1e-3
    np.testing.assert_allclose(_np(gains), g["G"], rtol=1e-5, atol=1e-5)


def test_gdn_verify_batched_qwen_shape_fp32_and_bf16():
    """B requests x (Hk=16, Hv=32, D=128) with random trees vs the oracle."""
    from dforktree_b200 import kernels as K
    B, N, Hk, Hv, D = 3, 32, 16, 32, 128
    ins = [cases.gdn_inputs(dict(N=N, Hk=Hk, Hv=Hv, D=D, slots=1, seed=900 + r, chain_p=0.6 * (r % 2)))
           for r in range(B)]
    for d in ins[1:]:                                   # one layer: shared gate parameters
        d["A_log"], d["dt_bias"] = ins[0]["A_log"], ins[0]["dt_bias"]
    pool = torch.from_numpy(np.concatenate([d["pool"] for d in ins])).to(DEV)         # slot r = request r
    A_log = torch.from_numpy(ins[0]["A_log"]).to(DEV)
    dtb = torch.from_numpy(ins[0]["dt_bias"]).to(DEV)
    anc = torch.from_numpy(np.stack([d["anc"] for d in ins])).to(DEV)
    for dt, tol in ((torch.float32, 1e-3), (torch.bfloat16, 2e-2)):
        y = torch.from_numpy(np.stack([d["y"] for d in ins])).to(DEV).to(dt)
        a = torch.from_numpy(np.stack([d["a"] for d in ins])).to(DEV).to(dt)
        b = torch.from_numpy(np.stack([d["b"] for d in ins])).to(DEV).to(dt)
        ak = torch.zeros(B, Hk, N, D, device=DEV)
        av = torch.zeros(B, Hv, N, D, device=DEV)
        ag = torch.zeros(B, Hv, N, device=DEV)
        o = K.gdn_tree_verify(y, a, b, A_log, dtb, anc, pool, Hk, Hv, aux_k=ak, aux_vn=av, aux_g=ag,
                              aux_k_per_v=False)
        for r in range(B):
            d = ins[r]
            oo, ok, ovn, oG = OG.tree_gdn(_np(y[r].float()), _np(a[r].float()), _np(b[r].float()), d["A_log"],
                                          d["dt_bias"], d["pool"], 0, d["anc"], Hk, Hv, D, D)
            assert _rel(_np(o[r].float()), oo) < tol, (dt, r)
            assert _rel(_np(av[r]), ovn) < 1e-3, (dt, r)
            assert _rel(_np(ak[r]), ok[::2]) < 1e-5
            np.testing.assert_allclose(_np(ag[r]), oG, rtol=1e-5, atol=1e-5)


# ------------------------------------------------------------------ commit --
@pytest.mark.parametrize("case", cases.COMMIT_CASES, ids=lambda c: c["name"])
def test_commit_matches_reference_golden(case):
    from dforktree_b200 import fc1_fused, tree_kernels
    g = _gold(case["name"])
    d = cases.commit_inputs(case)
    L_, NN = case["L"], case["NN"]
    H = cases.COMMIT_HEADS_STORED
    temporal = torch.from_numpy(d["state"]).to(DEV)
    K_, V_, G_ = (torch.from_numpy(d[k]).to(DEV) for k in ("K", "Vn", "G"))
    anc = torch.from_numpy(d["anc"]).to(DEV)
    path = torch.from_numpy(d["path"]).to(DEV)[None]
    inter = torch.zeros(L_, 2, NN, 32, 128, 128, device=DEV)
    fc1_fused.snapshots(temporal, K_, V_, G_, anc, path, torch.from_numpy(d["ends"]).to(DEV),
                        torch.tensor([case["slot"]], device=DEV), torch.tensor([1], device=DEV), inter)
    for e, u in enumerate(d["ends"]):
        if u < 0:
            continue
        got = _np(inter[:, 1, u, :H])
        np.testing.assert_allclose(got, g[f"end{e}"], rtol=1e-5, atol=1e-5)
    assert not torch.any(inter[:, 0]).item()
    plen = int((d["path"] >= 0).sum())
    st = temporal[:, case["slot"], :H].transpose(-1, -2).contiguous()            # K-major [L, H, DK, DV]
    tree_kernels.closed_commit(st, K_[:, :H].contiguous(), V_[:, :H].contiguous(), G_[:, :H].contiguous(),
                               path[0, :plen], torch.tensor([plen - 1], device=DEV))
    if plen <= 16:
        np.testing.assert_allclose(_np(st), g["closed"], rtol=1e-5, atol=1e-5)
    else:  # the reference kernel truncates at 16 nodes; this one commits the whole chain
        for l in range(L_):
            for h in range(H):
                ref = OG.snapshot(d["state"][l, case["slot"], h], d["K"][l, h], d["Vn"][l, h], d["G"][l, h], d["anc"],
                                  d["path"][:plen], int(d["path"][plen - 1]))
                np.testing.assert_allclose(_np(st)[l, h].T, ref, rtol=1e-5, atol=1e-5)


def test_verify_then_commit_equals_recurrence():
    """verify (aux) -> in-place commit along a root-to-leaf path == the per-node
    gated delta rule state at the leaf (Hk=16, Hv=32, batched)."""
    from dforktree_b200 import kernels as K
    B, N, Hk, Hv, D = 2, 32, 16, 32, 128
    ins = [cases.gdn_inputs(dict(N=N, Hk=Hk, Hv=Hv, D=D, slots=1, seed=950 + r, chain_p=0.8)) for r in range(B)]
    for d in ins[1:]:
        d["A_log"], d["dt_bias"] = ins[0]["A_log"], ins[0]["dt_bias"]
    pool = torch.from_numpy(np.concatenate([d["pool"] for d in ins])).to(DEV)
    pool0 = pool.clone()
    A_log = torch.from_numpy(ins[0]["A_log"]).to(DEV)
    dtb = torch.from_numpy(ins[0]["dt_bias"]).to(DEV)
    anc = torch.from_numpy(np.stack([d["anc"] for d in ins])).to(DEV)
    y = torch.from_numpy(np.stack([d["y"] for d in ins])).to(DEV)
    a = torch.from_numpy(np.stack([d["a"] for d in ins])).to(DEV)
    b = torch.from_numpy(np.stack([d["b"] for d in ins])).to(DEV)
    ak = torch.zeros(1, B, Hk, N, D, device=DEV)
    av = torch.zeros(1, B, Hv, N, D, device=DEV)
    ag = torch.zeros(1, B, Hv, N, device=DEV)
    K.gdn_tree_verify(y, a, b, A_log, dtb, anc, pool, Hk, Hv, aux_k=ak[0], aux_vn=av[0], aux_g=ag[0],
                      aux_k_per_v=False)
    P = 24
    paths = np.full((B, P), -1)
    for r in range(B):
        p = ins[r]["path"][:P]
        paths[r, :len(p)] = p
    ends = torch.from_numpy(np.array([[paths[r][(paths[r] >= 0).sum() - 1]] for r in range(B)])).to(DEV)
    st_in = pool.unsqueeze(0)
    st_out = torch.as_strided(pool, (1, B, 1, Hv, D, D), (0, pool.stride(0), 0, pool.stride(1), pool.stride(2), 1))
    K.gdn_commit(st_in, st_out, ak, av, ag, anc, torch.from_numpy(paths).to(DEV), ends, Hk, Hv, aux_k_per_v=False)
    for r in range(B):
        d = ins[r]
        _, S = OG.naive_recurrence(d["y"], d["a"], d["b"], d["A_log"], d["dt_bias"], d["pool"], 0, d["parent"], Hk,
                                   Hv, D, D)
        u = int(ends[r, 0])
        ref = np.transpose(S[:, u], (0, 2, 1))                                   # [Hv, Dv, Dk]
        assert _rel(_np(pool[r]), ref) < 1e-3
    assert not torch.equal(pool, pool0)
