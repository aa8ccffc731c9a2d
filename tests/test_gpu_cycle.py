"""GPU: the tcgen05 GDN verifier (fused tree conv) and the batched cycle.

* fused conv + verify == separate conv launch + verify (same arithmetic);
* tcgen05 path vs the CUDA-core path vs the CPU oracle at the Qwen3.5 head
  shape, fp32 and bf16 activations;
* one DraftTreeCycle step (score -> build -> conv+verify per layer -> greedy
  accept -> in-place commit) against the oracle chain, request by request.
"""
import numpy as np
import pytest
import torch

from oracle import builder as OB
from oracle import gdn as OG
from oracle import ngram as ON

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from dforktree_b200 import build
    build.build()


def _np(t):
    return t.detach().float().cpu().numpy()


def _rel(a, b):
    return float(np.abs(np.asarray(a, np.float64) - b).max() / max(np.abs(b).max(), 1e-30))


def _layer_inputs(B, N, Hk, Hv, D, seed, dtype, chain_p=0.5):
    from dforktree_b200 import kernels as K
    from dforktree_b200 import synth
    rng = np.random.default_rng(seed)
    C = 2 * Hk * D + Hv * D
    par = np.stack([synth.random_tree_parents(N, rng, chain_p=chain_p * (b % 2)) for b in range(B)])
    parent = torch.from_numpy(par).to(DEV)
    anc, depth, cidx, nxt, sib = K.tree_struct(parent)
    g = torch.Generator(device=DEV)
    g.manual_seed(seed)
    x = torch.randn(B, N, C, device=DEV, generator=g).to(dtype)
    conv_state = torch.randn(B, C, 3, device=DEV, generator=g).to(dtype)
    weight = (torch.randn(C, 4, device=DEV, generator=g) * 0.5).to(dtype)
    a = torch.randn(B, N, Hv, device=DEV, generator=g).to(dtype)
    b = torch.randn(B, N, Hv, device=DEV, generator=g).to(dtype)
    pool = torch.randn(B, Hv, D, D, device=DEV, generator=g) * 0.02
    A_log = torch.randn(Hv, device=DEV, generator=g) * 0.5
    dtb = torch.randn(Hv, device=DEV, generator=g) * 0.5
    return dict(par=par, anc=anc, cidx=cidx, x=x, conv_state=conv_state, weight=weight, a=a, b=b, pool=pool,
                A_log=A_log, dtb=dtb)


def _verify(d, Hk, Hv, y=None, conv=False, force_simt=False, status=None):
    from dforktree_b200 import kernels as K
    B, N = d["a"].shape[:2]
    ak = torch.zeros(B, Hk, N, 128, device=DEV)
    av = torch.zeros(B, Hv, N, 128, device=DEV)
    ag = torch.zeros(B, Hv, N, device=DEV)
    cv = dict(x=d["x"], conv_state=d["conv_state"], weight=d["weight"], cidx=d["cidx"]) if conv else None
    o = K.gdn_tree_verify(y, d["a"], d["b"], d["A_log"], d["dtb"], d["anc"], d["pool"], Hk, Hv, aux_k=ak,
                          aux_vn=av, aux_g=ag, aux_k_per_v=False, conv=cv, force_simt=force_simt, status=status,
                          o=torch.empty(B, N, Hv, 128, dtype=d["x"].dtype, device=DEV))
    return o, ak, av, ag


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_fused_conv_verify_equals_separate_conv_then_verify(dtype):
    from dforktree_b200 import kernels as K
    Hk, Hv = 16, 32
    d = _layer_inputs(4, 32, Hk, Hv, 128, seed=31, dtype=dtype)
    y = K.tree_conv(d["x"], d["conv_state"], d["weight"], None, d["cidx"])
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    ref = _verify(d, Hk, Hv, y=y, status=st)
    got = _verify(d, Hk, Hv, conv=True, status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    for r, g_ in zip(ref, got):
        assert torch.equal(r, g_)


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-3), (torch.bfloat16, 2e-2)])
@pytest.mark.parametrize("N", [32, 20, 1])
def test_tensor_core_verify_matches_simt_and_oracle(dtype, tol, N):
    from dforktree_b200 import kernels as K
    Hk, Hv, D = 16, 32, 128
    d = _layer_inputs(3, N, Hk, Hv, D, seed=40 + N, dtype=dtype)
    y = K.tree_conv(d["x"], d["conv_state"], d["weight"], None, d["cidx"])
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    tc = _verify(d, Hk, Hv, y=y, status=st)
    si = _verify(d, Hk, Hv, y=y, force_simt=True)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    assert _rel(_np(tc[0]), _np(si[0])) < tol
    assert _rel(_np(tc[2]), _np(si[2])) < 1e-3
    assert _rel(_np(tc[1]), _np(si[1])) < 1e-5
    for r in range(3):
        anc = _np(d["anc"][r])
        oo, ok, ovn, oG = OG.tree_gdn(_np(y[r]), _np(d["a"][r]), _np(d["b"][r]), _np(d["A_log"]), _np(d["dtb"]),
                                      _np(d["pool"]), r, anc, Hk, Hv, D, D)
        assert _rel(_np(tc[0][r]), oo) < tol, r
        assert _rel(_np(tc[2][r]), ovn) < 1e-3, r
        np.testing.assert_allclose(_np(tc[3][r]), oG, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("N", [32, 17])
def test_tensor_core_verify_many_units_per_cta(N):
    """B = 20 requests x 16 k-heads = 320 work units, so every persistent CTA
    loops over two or three units (state / tile prefetch across units)."""
    from dforktree_b200 import kernels as K
    Hk, Hv = 16, 32
    d = _layer_inputs(20, N, Hk, Hv, 128, seed=90 + N, dtype=torch.bfloat16)
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    tc = _verify(d, Hk, Hv, conv=True, status=st)
    y = K.tree_conv(d["x"], d["conv_state"], d["weight"], None, d["cidx"])
    si = _verify(d, Hk, Hv, y=y, force_simt=True)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    assert _rel(_np(tc[0]), _np(si[0])) < 2e-2
    assert _rel(_np(tc[2]), _np(si[2])) < 1e-3
    assert _rel(_np(tc[1]), _np(si[1])) < 1e-5
    np.testing.assert_allclose(_np(tc[3]), _np(si[3]), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("conv", [True, False])
def test_overlapped_layer_launches_equal_ordinary_launches(conv):
    """Programmatic dependent launch (overlap_prev): layers launched back to
    back, each overlapping the previous layer's verify, give bit-identical
    outputs to ordinary launches -- including a shared o buffer (each layer's
    writes wait for the previous layer) and the y-input path whose activation
    TMA is issued after the wait."""
    from dforktree_b200 import kernels as K
    Hk, Hv, L, B = 16, 32, 4, 40
    layers = [_layer_inputs(B, 32, Hk, Hv, 128, seed=300 + l, dtype=torch.bfloat16) for l in range(L)]
    for d in layers[1:]:   # one tree per cycle, as in the plugin
        d["anc"], d["cidx"] = layers[0]["anc"], layers[0]["cidx"]
    ys = [None if conv else K.tree_conv(d["x"], d["conv_state"], d["weight"], None, d["cidx"]) for d in layers]
    st = torch.zeros(1, dtype=torch.int32, device=DEV)

    def run(overlap, o_shared=None):
        # every buffer allocated up front: nothing is queued between the launches
        outs = [(o_shared if o_shared is not None else torch.empty(B, 32, Hv, 128, dtype=torch.bfloat16, device=DEV),
                 torch.zeros(B, Hk, 32, 128, device=DEV), torch.zeros(B, Hv, 32, 128, device=DEV),
                 torch.zeros(B, Hv, 32, device=DEV)) for _ in layers]
        cvs = [dict(x=d["x"], conv_state=d["conv_state"], weight=d["weight"], cidx=d["cidx"]) if conv else None
               for d in layers]
        torch.cuda.synchronize()
        for l, d in enumerate(layers):
            o, ak, av, ag = outs[l]
            K.gdn_tree_verify(ys[l], d["a"], d["b"], d["A_log"], d["dtb"], d["anc"], d["pool"], Hk, Hv, aux_k=ak,
                              aux_vn=av, aux_g=ag, aux_k_per_v=False, conv=cvs[l], status=st, o=o,
                              overlap_prev=overlap and l > 0)
            if not overlap:
                torch.cuda.synchronize()
        return outs

    ref = run(False)
    torch.cuda.synchronize()
    got = run(True)
    torch.cuda.synchronize()
    o_shared = torch.empty(B, 32, Hv, 128, dtype=torch.bfloat16, device=DEV)
    shared = run(True, o_shared)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    for l in range(L):
        for r, g_ in zip(ref[l], got[l]):
            assert torch.equal(r, g_), l
        for r, g_ in zip(ref[l][1:], shared[l][1:]):
            assert torch.equal(r, g_), l
    assert torch.equal(o_shared, ref[-1][0])


def test_cycle_step_matches_oracle_chain():
    """One batched cycle (B=4, 2 GDN layers, V=2048) request by request."""
    from dforktree_b200 import kernels as K
    from dforktree_b200 import synth
    from dforktree_b200.cycle import CycleConfig, DraftTreeCycle
    from dforktree_b200.ngram_gpu import load_npz_arrays
    V, S, N, B, Ls = 2048, 24, 32, 4, 2
    table = synth.make_ngram_table(V, 60000, 200000, seed=77)
    cfg = CycleConfig(B=B, S=S, V=V, N=N, layers=Ls)
    cyc = DraftTreeCycle(cfg, K.Table(load_npz_arrays(table), beta3=60.0), DEV, seed=5)
    pool0 = cyc.pool.clone()
    cs0 = cyc.conv_state.clone()
    logits = np.stack([synth.make_logits(S, V, seed=600 + r) for r in range(B)])
    lt = torch.from_numpy(logits).to(DEV)
    root = torch.tensor([11, 22, 33, 44], device=DEV)
    pre1 = torch.tensor([1, 2, 3, 4], device=DEV)
    g = torch.Generator(device=DEV)
    g.manual_seed(9)
    x = torch.randn(Ls, B, N, cfg.C, device=DEV, generator=g).to(torch.bfloat16)
    a = torch.randn(Ls, B, N, cfg.Hv, device=DEV, generator=g).to(torch.bfloat16)
    b = torch.randn(Ls, B, N, cfg.Hv, device=DEV, generator=g).to(torch.bfloat16)
    acc_len = torch.tensor([1, 3, 6, 24], device=DEV)

    def target_fn(tree):
        nx = tree["nxt"]
        tgt = torch.gather(tree["tokens"], 1, nx.clamp(min=0))
        keep = (nx >= 0) & (tree["depth"] + 1 < acc_len[:, None])
        return torch.where(keep, tgt, torch.full_like(tgt, -1))

    cyc.step(lt, root, pre1, x, a, b, target_fn)
    torch.cuda.synchronize()
    assert int(cyc.status.item()) == 0
    ong = ON.NGramOracle(table, beta3=60.0)
    path = cyc.path.cpu().numpy()
    for r in range(B):
        tr = OB.builder_run(logits[r], int(root[r]), int(pre1[r]), ong, N=N)
        assert np.array_equal(cyc.tree["tokens"][r].cpu().numpy(), tr["tokens"])
        assert np.array_equal(cyc.tree["parent"][r].cpu().numpy(), tr["parent"])
        # accepted path: first-child chain, length min(acc_len, chain depth)
        p = [0]
        while len(p) < int(acc_len[r]) and tr["nxt"][p[-1]] >= 0:
            p.append(int(tr["nxt"][p[-1]]))
        assert list(path[r][: len(p)]) == p and np.all(path[r][len(p):] == -1)
        for l in range(Ls):
            xr = _np(x[l, r])
            y, _ = OG.tree_conv(xr, _np(cs0[l, r]), _np(cyc.conv_w[l]), None, tr["cidx"])
            y = _np(torch.from_numpy(y).to(torch.bfloat16))      # the conv output is stored in x's dtype
            o, k, vn, G = OG.tree_gdn(y, _np(a[l, r]), _np(b[l, r]), _np(cyc.A_log[l]), _np(cyc.dt_bias[l]),
                                      _np(pool0[l]), r, tr["anc"], cfg.Hk, cfg.Hv, 128, 128)
            for h in range(cfg.Hv):
                ref = OG.snapshot(_np(pool0[l, r, h]), k[h], vn[h], G[h], tr["anc"], path[r], p[-1])
                assert _rel(_np(cyc.pool[l, r, h]), ref) < 1e-3, (r, l, h)
            # conv-window commit: taps 1..3 of the last accepted node (old state columns or new inputs)
            cols = tr["cidx"][p[-1], 1:]
            src = [_np(cs0[l, r])[:, c] if c < 3 else xr[c - 3] for c in cols]
            np.testing.assert_array_equal(_np(cyc.conv_state[l, r]), np.stack(src, 1))


@pytest.mark.parametrize("dtype,C", [(torch.float32, 1000), (torch.bfloat16, 1000), (torch.bfloat16, 1024)])
def test_conv_commit_slots_skips_and_bad_index(dtype, C):
    """Conv-window commit through the C ABI: per layer and request the state
    takes taps 1..3 of node last[b] (state columns or new inputs, by cidx);
    last < 0 leaves it untouched; slots map requests to pool rows.  bf16 with
    C % 8 == 0 runs the packed 16-byte kernel, the rest the general one."""
    from dforktree_b200 import kernels as K
    from dforktree_b200 import synth
    Ls, B, N, slots_n = 3, 5, 32, 9
    rng = np.random.default_rng(21)
    cidx = np.stack([OB.tree_struct(synth.random_tree_parents(N, rng), 4)[2] for _ in range(B)])
    g = torch.Generator(device=DEV)
    g.manual_seed(4)
    x = torch.randn(Ls, B, N, C, device=DEV, generator=g).to(dtype)
    cs = torch.randn(Ls, slots_n, C, 3, device=DEV, generator=g).to(dtype)
    slots = torch.tensor([7, 0, 3, 8, 5], device=DEV)
    last = torch.tensor([0, 31, -1, 17, 5], device=DEV)
    cs0 = _np(cs.float())
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    K.conv_commit(x, cs, torch.from_numpy(cidx).to(DEV), last, slots=slots, status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    got, xs = _np(cs.float()), _np(x.float())
    want = cs0.copy()
    for l in range(Ls):
        for bi in range(B):
            u = int(last[bi])
            if u < 0:
                continue
            s = int(slots[bi])
            for j, col in enumerate(cidx[bi, u, 1:]):
                want[l, s, :, j] = cs0[l, s, :, col] if col < 3 else xs[l, bi, col - 3]
    np.testing.assert_array_equal(got, want)
    # a last-node index past the tree raises BAD_INDEX and writes nothing for that request
    cs1 = cs.clone()
    K.conv_commit(x, cs, torch.from_numpy(cidx).to(DEV), torch.tensor([-1, -1, 40, -1, -1], device=DEV),
                  slots=slots, status=st)
    torch.cuda.synchronize()
    assert int(st.item()) & 4
    assert torch.equal(cs, cs1)
