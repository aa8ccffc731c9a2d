"""Tree-masked attention verify (dft_tree_attn) against the CPU oracle: the
mask of fc1_branch64.py:39 over a paged KV cache (page size 1, scattered
slots), grouped-query heads, key splits and the single-split path, ragged
prefixes, rescaling of the running max, and bad slot indices.  Bar: bf16
output within 2e-2 of the largest magnitude (north-star bf16 tolerance)."""
import numpy as np
import pytest
import torch

from oracle import attn as OA
from oracle import builder as OB

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL = 2e-2


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from dforktree_b200 import build
    build.build()


def _np(t):
    return t.detach().float().cpu().numpy()


def _case(B, N, Hq, Hkv, plens, seed, slots=None, q_scale=1.0, growing=False):
    from dforktree_b200 import synth
    rng = np.random.default_rng(seed)
    lens = [p + N for p in plens]
    total = sum(lens)
    slots = slots or total + 97
    perm = rng.permutation(slots)[:total].astype(np.int32)   # scattered pages (page size 1)
    indptr = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    anc = np.stack([OB.tree_struct(synth.random_tree_parents(N, rng), 4)[0] for _ in range(B)])
    g = torch.Generator(device=DEV)
    g.manual_seed(seed)
    D = 256
    q = (torch.randn(B, N, Hq, D, device=DEV, generator=g) * q_scale).to(torch.bfloat16)
    k = torch.randn(slots, Hkv, D, device=DEV, generator=g)
    if growing:
        # key norms rising along each request's context: the running max grows tile after tile
        ramp = torch.zeros(slots, device=DEV)
        for b in range(B):
            idx = torch.from_numpy(perm[indptr[b]:indptr[b + 1]].astype(np.int64)).to(DEV)
            ramp[idx] = torch.linspace(0.2, 3.0, idx.numel(), device=DEV)
        k = k * ramp[:, None, None]
    k = k.to(torch.bfloat16)
    v = torch.randn(slots, Hkv, D, device=DEV, generator=g).to(torch.bfloat16)
    return dict(q=q, k=k, v=v, indptr=torch.from_numpy(indptr).to(DEV), indices=torch.from_numpy(perm).to(DEV),
                anc=torch.from_numpy(anc).to(DEV), max_len=max(lens))


def _run(c, status=None, **kw):
    from dforktree_b200 import kernels as K
    return K.tree_attention(c["q"], c["k"], c["v"], c["indptr"], c["indices"], c["anc"], max_kv_len=c["max_len"],
                            status=status, **kw)


def _ref(c, sm_scale=None):
    return OA.tree_attention(_np(c["q"]), _np(c["k"]), _np(c["v"]), _np(c["indptr"]).astype(np.int64),
                             _np(c["indices"]).astype(np.int64), _np(c["anc"]), sm_scale)


def _rel(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.mark.parametrize("B,N,Hq,Hkv,plens", [
    (3, 32, 16, 4, [100, 3000, 37]),      # Qwen3.5 attention heads, splits > 1 (8: 12 pairs, 48 tiles)
    (2, 32, 16, 4, [5, 20]),              # <= 64 keys: one split, direct output
    (2, 16, 16, 4, [300, 64]),            # N = 16: query rows 64..127 padded
    (2, 32, 8, 4, [200, 129]),            # G = 2
    (1, 7, 16, 2, [450]),                 # G = 8, ragged N
    (4, 32, 16, 4, [0, 1, 63, 64]),       # prefix lengths at tile edges (0 = tree only)
])
def test_tree_attention_matches_oracle(B, N, Hq, Hkv, plens):
    c = _case(B, N, Hq, Hkv, plens, seed=B * 100 + N + Hq + sum(plens))
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    o = _run(c, status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    got, ref = _np(o), _ref(c)
    assert np.isfinite(got).all()
    assert _rel(got, ref) < TOL, _rel(got, ref)


def test_tree_attention_rescales_growing_scores_and_custom_scale():
    c = _case(2, 32, 16, 4, [900, 1500], seed=7, q_scale=2.0, growing=True)
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    o = _run(c, status=st, sm_scale=0.11)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    got, ref = _np(o), _ref(c, 0.11)
    assert _rel(got, ref) < TOL, _rel(got, ref)


def test_tree_mask_is_applied():
    """A tree key hidden from a node must not leak into its output: giving a
    non-ancestor's value row a huge value changes only the nodes that see it."""
    c = _case(1, 32, 16, 4, [40], seed=11)
    o0 = _np(_run(c))
    anc = _np(c["anc"])[0]
    m = int(np.argmax(anc.sum(0) == 1)) if (anc.sum(0) == 1).any() else 31   # a leaf: visible to itself only
    slot = int(_np(c["indices"])[40 + m])
    c["v"][slot] = 50.0
    o1 = _np(_run(c))
    changed = np.abs(o1 - o0).max(axis=(2, 3)) > 1e-3
    assert np.array_equal(changed[0], anc[:, m] > 0.5)


def test_bad_slot_sets_status_without_fault():
    c = _case(2, 32, 16, 4, [70, 10], seed=3)
    c["indices"][5] = c["k"].shape[0] + 10
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    o = _run(c, status=st)
    torch.cuda.synchronize()
    assert int(st.item()) & 4
    assert np.isfinite(_np(o)).all()


def test_tree_attention_bench_shape_sampled_requests():
    """Batch 64, 4K-token prefixes, Qwen3.5 attention heads (the bench's
    attention workload); two requests checked against the oracle."""
    B, N = 64, 32
    c = _case(B, N, 16, 4, [4096] * B, seed=21)
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    o = _run(c, status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    got = _np(o)
    assert np.isfinite(got).all()
    for b in (0, 37):
        lo, hi = int(c["indptr"][b]), int(c["indptr"][b + 1])
        idx = c["indices"][lo:hi].long()
        sub = dict(q=c["q"][b:b + 1], k=c["k"][idx], v=c["v"][idx],
                   indptr=torch.tensor([0, hi - lo], device=DEV), indices=torch.arange(hi - lo, device=DEV),
                   anc=c["anc"][b:b + 1], max_len=hi - lo)
        assert _rel(got[b:b + 1], _ref(sub)) < TOL


def test_wrapper_plan_run_with_plugin_custom_mask():
    """plan / run with the mask built as fc1_branch64.py:39 does (ones over the
    prefix, anc over the tree), flattened per request, q as [B*n, Hq, D]."""
    from dforktree_b200.tree_attn import TreeAttentionWrapper
    c = _case(2, 32, 16, 4, [300, 77], seed=5)
    lens = [332, 109]
    mask = torch.cat([torch.cat((torch.ones(32, Lb - 32, dtype=torch.bool, device=DEV), c["anc"][b].bool()), 1).flatten()
                      for b, Lb in enumerate(lens)])
    w = TreeAttentionWrapper(DEV).plan(c["indptr"], c["indices"], 16, 4, 256, n=32, custom_mask=mask,
                                       kv_lens_host=lens)
    o = w.run(c["q"].view(64, 16, 256), (c["k"], c["v"]))
    torch.cuda.synchronize()
    assert o.shape == (64, 16, 256) and w.device_status() == 0
    assert _rel(_np(o).reshape(2, 32, 16, 256), _ref(c)) < TOL


@pytest.mark.skipif(__import__("os").environ.get("DFT_TEST_FLASHINFER") != "1",
                    reason="opt-in (DFT_TEST_FLASHINFER=1): JIT-builds flashinfer's prefill kernel on the box")
def test_tree_attention_matches_flashinfer_custom_mask():
    """Pin against the library the reference plugin verifies through: flashinfer's
    paged prefill (fa2, page size 1) planned as fc1_plan.py:16-33 plans it, with
    the fc1_branch64.py:39 mask [ones(n, prefix) | anc], one request per plan."""
    flashinfer = pytest.importorskip("flashinfer")
    B, N, HQ, HKV, D = 2, 32, 16, 4, 256
    c = _case(B, N, HQ, HKV, [700, 45], seed=31)
    ours = _np(_run(c))
    ws = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=DEV)
    for b in range(B):
        lo, hi = int(c["indptr"][b]), int(c["indptr"][b + 1])
        Lb = hi - lo
        mask = torch.cat((torch.ones(N, Lb - N, dtype=torch.bool, device=DEV), c["anc"][b].bool()), 1).flatten()
        w = flashinfer.BatchPrefillWithPagedKVCacheWrapper(ws, "NHD", backend="fa2")
        w.plan(torch.tensor([0, N], dtype=torch.int32, device=DEV), torch.tensor([0, Lb], dtype=torch.int32, device=DEV),
               c["indices"][lo:hi].to(torch.int32), torch.ones(1, dtype=torch.int32, device=DEV), HQ, HKV, D, 1,
               custom_mask=mask, q_data_type=torch.bfloat16, kv_data_type=torch.bfloat16)
        ref = w.run(c["q"][b], (c["k"].unsqueeze(1), c["v"].unsqueeze(1)))
        torch.cuda.synchronize()
        assert _rel(ours[b], _np(ref)) < TOL, (b, _rel(ours[b], _np(ref)))


@pytest.mark.parametrize("case", __import__("tests.golden.cases", fromlist=["ATTN_CASES"]).ATTN_CASES,
                         ids=lambda c: c["name"])
def test_tree_attention_matches_flashinfer_golden(case):
    """dft_tree_attn against flashinfer's own paged prefill output (fa2, page
    size 1, the fc1_branch64.py:39 mask, planned as fc1_plan.py:16-33 plans it;
    fixtures from tests/golden/make_attn_golden.py), GQA ratios 1 / 2 / 4 / 8,
    ragged prefixes, N = 16 and 32; bf16 bar 2e-2."""
    import os

    from tests.golden import cases
    g = np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", case["name"] + ".npz"))
    d = cases.attn_inputs(case)
    t = lambda x: torch.from_numpy(x).to(DEV)
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    from dforktree_b200 import kernels as K
    o = K.tree_attention(t(d["q"]).to(torch.bfloat16), t(d["k"]).to(torch.bfloat16), t(d["v"]).to(torch.bfloat16),
                         t(d["kv_indptr"]), t(d["kv_indices"]), t(d["anc"]), status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    ref = (g["o_bf16"].astype(np.uint32) << 16).view(np.float32)
    assert _rel(_np(o), ref) < TOL
