"""Pin the CPU oracle against golden vectors produced by the reference itself.

The fixtures under tests/golden/ were written by make_golden.py from the
reference's own code (torch CPU + Triton interpreter).  These tests need no
GPU and run in the CPU suite.
"""
import os

import numpy as np
import pytest

from oracle import builder, gdn, ngram
from tests.golden import cases

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load(name):
    return np.load(os.path.join(GOLD, name + ".npz"))


def test_ngram_oracle_matches_reference():
    g = _load("ngram_small")
    table = cases.ngram_table()
    z, a, b, c = cases.ngram_queries(int(table["V"]))
    np.testing.assert_allclose(g["checksum"], cases.checksum(table["keys"], table["keys3"], table["keys4"], z, a, b, c))
    for name, b3 in (("b20", 20.0), ("b60", 60.0)):
        ng = ngram.NGramOracle(table, beta3=b3)
        np.testing.assert_array_equal(ng.pn, g["pn"])
        # p2/p3/p4 use + * / only: bit-exact
        np.testing.assert_array_equal(ng.p2(b, c), g[f"p2_{name}"])
        np.testing.assert_array_equal(ng.p3(a, b, c), g[f"p3_{name}"])
        np.testing.assert_array_equal(ng.p4(z, a, b, c), g[f"p4_{name}"])
        for order in (2, 3, 4):
            # pmi differs only by the last ulp of log between libraries
            np.testing.assert_allclose(ng.pmi(order, z, a, b, c), g[f"pmi{order}_{name}"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("case", cases.BUILDER_CASES, ids=lambda c: c["name"])
def test_builder_oracle_matches_reference(case):
    g = _load(case["name"])
    table, logits, root, pre1 = cases.builder_inputs(case)
    np.testing.assert_allclose(g["checksum"], cases.checksum(logits, table["keys"], table["keys3"], [root, pre1]))
    ng = ngram.NGramOracle(table, beta3=60.0) if case["ngram"] else None
    out = builder.builder_run(logits, root, pre1, ng, N=case["N"], chain_first=case["chain_first"])
    for key in ("tokens", "parent", "depth", "anc", "cidx", "nxt", "sib", "ids"):
        np.testing.assert_array_equal(out[key], g[key], err_msg=key)
    np.testing.assert_allclose(out["lp"], g["lp"], rtol=1e-5, atol=2e-6)
    if case["ngram"]:
        np.testing.assert_allclose(out["T"], g["T"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("case", cases.ORDER_CASES, ids=lambda c: c["name"])
def test_builder_oracle_other_orders_match_reference(case):
    """ngram_path_fn at orders 2 and 4 (tree_ops.py:59-64) and the beam over
    it: T (a seeded sample of its entries) and the whole tree."""
    g = _load(case["name"])
    table, logits, root, pre1 = cases.order_inputs(case)
    np.testing.assert_allclose(g["checksum"], cases.checksum(logits, table["keys"], table["keys3"],
                                                             table.get("keys4", np.zeros(0)), [root, pre1]))
    ng = ngram.NGramOracle(table, beta3=60.0)
    out = builder.builder_run(logits, root, pre1, ng, N=case["N"], chain_first=case["chain_first"],
                              order=case["order"])
    assert out["T"].shape == tuple(g["T_shape"]) == (case["S"] - 1,) + (16,) * case["order"]
    np.testing.assert_array_equal(g["T_index"], cases.order_t_sample(out["T"].shape))
    np.testing.assert_allclose(out["T"].reshape(-1)[g["T_index"]], g["T_sample"], rtol=1e-5, atol=1e-5)
    for key in ("tokens", "parent", "depth", "anc", "cidx", "ids", "ss", "cand"):
        np.testing.assert_array_equal(out[key], g[key], err_msg=key)
    np.testing.assert_array_equal(out["flags"], g["flags"])


@pytest.mark.slow
@pytest.mark.parametrize("seed", cases.CONFIG0_SEEDS)
def test_builder_oracle_config0_full_vocab(seed):
    g = _load(f"config0_seed{seed}")
    table, logits, root, pre1 = cases.config0_inputs(seed, _config0_table())
    np.testing.assert_allclose(
        g["checksum"], cases.checksum(logits, table["keys"][:100000], table["keys3"][:100000], [root, pre1]))
    out = builder.builder_run(logits, root, pre1, ngram.NGramOracle(table, beta3=60.0), N=32)
    for key in ("tokens", "parent", "depth", "cidx", "nxt", "sib", "ids"):
        np.testing.assert_array_equal(out[key], g[key], err_msg=key)


_TABLE0 = {}


def _config0_table():
    if "t" not in _TABLE0:
        c = cases.CONFIG0
        from dforktree_b200 import synth
        _TABLE0["t"] = synth.make_ngram_table(c["V"], c["nb"], c["nt"], seed=c["table_seed"])
    return _TABLE0["t"]


@pytest.mark.parametrize("case", cases.GDN_CASES, ids=lambda c: c["name"])
def test_gdn_oracle_matches_reference(case):
    g = _load(case["name"])
    d = cases.gdn_inputs(case)
    np.testing.assert_allclose(g["checksum"], cases.checksum(d["y"], d["a"], d["b"], d["pool"], d["anc"]))
    o, k, vn, G = gdn.tree_gdn(d["y"], d["a"], d["b"], d["A_log"], d["dt_bias"], d["pool"], case["slot"],
                               d["anc"], case["Hk"], case["Hv"], case["D"], case["D"])
    sc = np.abs(g["o"]).max()
    assert np.abs(o - g["o"]).max() <= 1e-5 * sc
    np.testing.assert_allclose(k, g["k"], rtol=1e-6, atol=1e-7)
    assert np.abs(vn - g["vn"]).max() <= 1e-5 * np.abs(g["vn"]).max()
    np.testing.assert_allclose(G, g["G"], rtol=1e-5, atol=1e-6)
    if "o_fused" in g:
        assert np.abs(g["o_fused"] - g["o"]).max() <= 1e-5 * sc
    # independent per-node recurrence
    on, _ = gdn.naive_recurrence(d["y"], d["a"], d["b"], d["A_log"], d["dt_bias"], d["pool"], case["slot"],
                                 d["parent"], case["Hk"], case["Hv"], case["D"], case["D"])
    assert np.abs(on - g["o"]).max() <= 1e-5 * sc


@pytest.mark.parametrize("case", cases.CONV_CASES, ids=lambda c: c["name"])
def test_conv_oracle_matches_reference(case):
    g = _load(case["name"])
    parent, x, cs, w, bias = cases.conv_inputs(case)
    np.testing.assert_allclose(g["checksum"], cases.checksum(x, cs, w, bias))
    _, _, cidx = builder.tree_struct(parent, 4)
    np.testing.assert_array_equal(cidx, g["cidx"])
    y, win = gdn.tree_conv(x, cs[case["slot"]], w, bias, cidx)
    np.testing.assert_array_equal(y, g["y"])
    np.testing.assert_array_equal(y, g["y_fused"])
    np.testing.assert_array_equal(win, g["iw"][case["dst"]])


@pytest.mark.parametrize("case", cases.COMMIT_CASES, ids=lambda c: c["name"])
def test_commit_oracle_matches_reference(case):
    g = _load(case["name"])
    d = cases.commit_inputs(case)
    np.testing.assert_allclose(g["checksum"], cases.checksum(d["state"], d["K"], d["Vn"], d["G"], d["path"]))
    H = cases.COMMIT_HEADS_STORED
    for e, u in enumerate(d["ends"]):
        if u < 0:
            assert not np.any(g[f"end{e}"])
            continue
        for l in range(case["L"]):
            for h in range(H):
                s = gdn.snapshot(d["state"][l, case["slot"], h], d["K"][l, h], d["Vn"][l, h], d["G"][l, h],
                                 d["anc"], d["path"], int(u))
                np.testing.assert_allclose(s, g[f"end{e}"][l, h], rtol=1e-5, atol=1e-6)
    plen = int((d["path"] >= 0).sum())
    st = gdn.closed_commit(d["state"][:, case["slot"], :H].transpose(0, 1, 3, 2), d["K"][:, :H], d["Vn"][:, :H],
                           d["G"][:, :H], d["path"][:plen], plen - 1)
    np.testing.assert_allclose(st, g["closed"], rtol=1e-5, atol=1e-6)


def test_commit_closed_form_equals_recurrence():
    """Closed-form commit along the accepted path == the per-node recurrence."""
    case = dict(cases.GDN_CASES[-1])
    d = cases.gdn_inputs(case)
    Hk, Hv, D = case["Hk"], case["Hv"], case["D"]
    o, k, vn, G = gdn.tree_gdn(d["y"], d["a"], d["b"], d["A_log"], d["dt_bias"], d["pool"], case["slot"], d["anc"],
                               Hk, Hv, D, D)
    _, S = gdn.naive_recurrence(d["y"], d["a"], d["b"], d["A_log"], d["dt_bias"], d["pool"], case["slot"],
                                d["parent"], Hk, Hv, D, D)
    u = int(d["path"][-1])
    for h in range(Hv):
        s = gdn.snapshot(d["pool"][case["slot"], h], k[h], vn[h], G[h], d["anc"], d["path"], u)
        ref = S[h, u].T
        assert np.abs(s - ref).max() <= 1e-4 * np.abs(ref).max()


@pytest.mark.parametrize("case", cases.ATTN_CASES, ids=lambda c: c["name"])
def test_attention_oracle_matches_flashinfer_golden(case):
    """oracle/attn.py against flashinfer's own paged prefill (fa2, page size 1,
    the plugin's custom mask, one request per plan as fc1_plan.py plans it),
    fixtures written by tests/golden/make_attn_golden.py.  flashinfer rounds P
    to bf16 before P.V and its output to bf16; the fp32 restatement agrees
    within 1e-2 of the largest magnitude."""
    from oracle import attn as OA
    g = np.load(os.path.join(GOLD, case["name"] + ".npz"))
    d = cases.attn_inputs(case)
    np.testing.assert_allclose(g["checksum"], cases.checksum(d["q"], d["k"], d["v"], d["kv_indices"], d["anc"]))
    ref = (g["o_bf16"].astype(np.uint32) << 16).view(np.float32)
    o = OA.tree_attention(d["q"], d["k"], d["v"], d["kv_indptr"], d["kv_indices"], d["anc"])
    assert np.abs(o - ref).max() <= 1e-2 * np.abs(ref).max()
