"""GPU: the tcgen05 GDN verifier for trees of 33..64 nodes (the plugin's
default FC1_TREE_N = 64, fc1_fused.py:4) against the CUDA-core verifier and
the CPU oracle.

* outputs o within 2e-2 (bf16), vn within 1e-3, k_hat / G within 1e-5, for
  random trees, chain-like trees and one 64-node chain (depth 63: 64 levels
  of the depth-level solve);
* fused conv + verify == separate conv launch + verify, bit for bit;
* 640 work units on the persistent CTAs (state / tile prefetch across units);
* back-to-back layers overlapped by programmatic dependent launch equal
  ordinary launches;
* k-head ratio 1 and per-v-head k_hat rows.
"""
import numpy as np
import pytest
import torch

from oracle import gdn as OG
from tests.test_gpu_cycle import _layer_inputs, _np, _rel, _verify

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from dforktree_b200 import build
    build.build()


def _with_chain(d, r):
    """Make request r a single chain 0 <- 1 <- ... <- N-1."""
    from dforktree_b200 import kernels as K
    N = d["a"].shape[1]
    par = d["par"].copy()
    par[r] = np.arange(-1, N - 1)
    anc, _, cidx, _, _ = K.tree_struct(torch.from_numpy(par).to(DEV))
    d.update(par=par, anc=anc, cidx=cidx)
    return d


@pytest.mark.parametrize("N", [64, 48, 33])
def test_verify64_matches_simt_and_oracle(N):
    from dforktree_b200 import kernels as K
    Hk, Hv, D = 16, 32, 128
    d = _with_chain(_layer_inputs(3, N, Hk, Hv, D, seed=500 + N, dtype=torch.bfloat16), 2)
    y = K.tree_conv(d["x"], d["conv_state"], d["weight"], None, d["cidx"])
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    tc = _verify(d, Hk, Hv, y=y, status=st)
    si = _verify(d, Hk, Hv, y=y, force_simt=True)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    assert _rel(_np(tc[0]), _np(si[0])) < 2e-2
    assert _rel(_np(tc[2]), _np(si[2])) < 1e-3
    assert _rel(_np(tc[1]), _np(si[1])) < 1e-5
    for r in range(3):
        anc = _np(d["anc"][r])
        oo, ok, ovn, oG = OG.tree_gdn(_np(y[r]), _np(d["a"][r]), _np(d["b"][r]), _np(d["A_log"]), _np(d["dtb"]),
                                      _np(d["pool"]), r, anc, Hk, Hv, D, D)
        assert _rel(_np(tc[0][r]), oo) < 2e-2, r
        assert _rel(_np(tc[2][r]), ovn) < 1e-3, r
        assert _rel(_np(tc[1][r]), ok[:: Hv // Hk]) < 1e-5, r
        np.testing.assert_allclose(_np(tc[3][r]), oG, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("N", [64, 40])
def test_verify64_fused_conv_equals_separate_conv(N):
    from dforktree_b200 import kernels as K
    Hk, Hv = 16, 32
    d = _layer_inputs(4, N, Hk, Hv, 128, seed=600 + N, dtype=torch.bfloat16)
    y = K.tree_conv(d["x"], d["conv_state"], d["weight"], None, d["cidx"])
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    ref = _verify(d, Hk, Hv, y=y, status=st)
    got = _verify(d, Hk, Hv, conv=True, status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    for r, g_ in zip(ref, got):
        assert torch.equal(r, g_)


def test_verify64_many_units_per_cta():
    """B = 20 requests x 32 v-heads = 640 work units: every persistent CTA
    loops over four or five units."""
    from dforktree_b200 import kernels as K
    Hk, Hv = 16, 32
    d = _layer_inputs(20, 64, Hk, Hv, 128, seed=700, dtype=torch.bfloat16)
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


def test_verify64_overlapped_layers_equal_ordinary_launches():
    from dforktree_b200 import kernels as K
    Hk, Hv, L, B, N = 16, 32, 3, 24, 64
    layers = [_layer_inputs(B, N, Hk, Hv, 128, seed=800 + l, dtype=torch.bfloat16) for l in range(L)]
    for d in layers[1:]:
        d["anc"], d["cidx"] = layers[0]["anc"], layers[0]["cidx"]
    st = torch.zeros(1, dtype=torch.int32, device=DEV)

    def run(overlap):
        outs = [(torch.empty(B, N, Hv, 128, dtype=torch.bfloat16, device=DEV), torch.zeros(B, Hk, N, 128, device=DEV),
                 torch.zeros(B, Hv, N, 128, device=DEV), torch.zeros(B, Hv, N, device=DEV)) for _ in layers]
        cvs = [dict(x=d["x"], conv_state=d["conv_state"], weight=d["weight"], cidx=d["cidx"]) for d in layers]
        torch.cuda.synchronize()
        for l, d in enumerate(layers):
            o, ak, av, ag = outs[l]
            K.gdn_tree_verify(None, d["a"], d["b"], d["A_log"], d["dtb"], d["anc"], d["pool"], Hk, Hv, aux_k=ak,
                              aux_vn=av, aux_g=ag, aux_k_per_v=False, conv=cvs[l], status=st, o=o,
                              overlap_prev=overlap and l > 0)
            if not overlap:
                torch.cuda.synchronize()
        return outs

    ref = run(False)
    torch.cuda.synchronize()
    got = run(True)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    for l in range(L):
        for r, g_ in zip(ref[l], got[l]):
            assert torch.equal(r, g_), l


def test_verify64_head_ratio_one_and_per_v_khat():
    from dforktree_b200 import kernels as K
    Hk = Hv = 8
    D, N, B = 128, 64, 2
    d = _layer_inputs(B, N, Hk, Hv, D, seed=900, dtype=torch.bfloat16)
    y = K.tree_conv(d["x"], d["conv_state"], d["weight"], None, d["cidx"])
    st = torch.zeros(1, dtype=torch.int32, device=DEV)
    ak = torch.zeros(B, Hv, N, D, device=DEV)
    o = K.gdn_tree_verify(y, d["a"], d["b"], d["A_log"], d["dtb"], d["anc"], d["pool"], Hk, Hv, aux_k=ak,
                          aux_k_per_v=True, status=st, o=torch.empty(B, N, Hv, D, dtype=torch.bfloat16, device=DEV))
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    for r in range(B):
        oo, ok, _, _ = OG.tree_gdn(_np(y[r]), _np(d["a"][r]), _np(d["b"][r]), _np(d["A_log"]), _np(d["dtb"]),
                                   _np(d["pool"]), r, _np(d["anc"][r]), Hk, Hv, D, D)
        assert _rel(_np(o[r]), oo) < 2e-2, r
        assert _rel(_np(ak[r]), ok) < 1e-5, r
