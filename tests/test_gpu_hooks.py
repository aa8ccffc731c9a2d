"""The plugin hooks driven the way SGLang and the reference's verify_branch
drive them, with stand-in objects shaped like SGLang's arguments.

Per tree size (32: tensor-core verifier; 64: the plugin's default size):
1. the reference's bare-name imports resolve to this package
   (fc1_plugin.alias_reference_modules), and verify_branch's lines
   fc1_branch64.py:18-30 run as written: Builder(logits) -> the tree ->
   fc1_fused.CTX.anc / CTX.cidx;
2. per GDN layer, the conv hook (`causal_conv1d_update`, fc1_conv.py:33-45)
   then the verify hook (`TritonGDNKernel.target_verify`, fc1_fused.py:59-75)
   with SGLang's keyword arguments (ssm_states, cache_indices,
   intermediate_state_indices, conv_state_indices, intermediate_conv_window);
3. the commit hook (`commit_mamba_states_after_verify`, fc1_fused.py:77-87)
   with a stand-in target worker / request pool and SGLang's
   `_verify_commit_step_indices`, writing intermediate_ssm for the last
   accepted node and a tracked node.
Outputs are compared with the CPU oracle on a tree that is not a chain.
"""
import types

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


@pytest.mark.parametrize("NN", [32, 64])
def test_hooks_with_sglang_shaped_arguments(NN, monkeypatch, tmp_path):
    from dforktree_b200 import fc1_conv, fc1_fused, fc1_plugin, synth
    monkeypatch.setenv("FC1_TREE_N", str(NN))
    monkeypatch.setattr(fc1_fused, "NN", NN)
    monkeypatch.setattr(fc1_fused, "CTX", None)
    V, S, Hk, Hv, D = 2048, 24, 16, 32, 128
    C = 2 * Hk * D + Hv * D
    table = synth.make_ngram_table(V, 60000, 200000, seed=5)
    path = tmp_path / "ngram.npz"
    np.savez(path, **table)
    monkeypatch.setenv("FC1_NGRAM_PATH", str(path))
    monkeypatch.setenv("FC1_CHAIN_FIRST", "0")
    prev = fc1_plugin.alias_reference_modules()
    try:
        import fc1_builder
        import fc1_fused as bare_fused
        assert bare_fused is fc1_fused and fc1_builder.__name__ == "dforktree_b200.fc1_builder"
        # ---- fc1_branch64.py:18-30, as written
        logits_np = synth.make_logits(S, V, seed=31)
        logits = torch.from_numpy(logits_np).to(DEV)
        root, pre1 = torch.tensor([[17]], device=DEV), torch.tensor([3], device=DEV)
        w = types.SimpleNamespace()
        w.fc1_builder = fc1_builder.Builder(logits, compile_build=False)
        tree, depth, parent, anc, nxt, sib = w.fc1_builder(logits, root[:, 0], pre1)
        bare_fused.set_tree(anc, w.fc1_builder.cidx)      # CTX is created by the hooks in a server; here on first use
        bare_fused.CTX.anc.copy_(anc)
        bare_fused.CTX.cidx.copy_(w.fc1_builder.cidx)
    finally:
        fc1_plugin.restore_modules(prev)
    ong = ON.NGramOracle(table, beta3=60.0)
    ref_tree = OB.builder_run(logits_np, 17, 3, ong, N=NN)
    assert np.array_equal(_np(tree)[0], ref_tree["tokens"]) and np.array_equal(_np(parent), ref_tree["parent"])
    assert int(depth.max()) >= 2, "the test wants a tree that is not a chain of first children"
    anc_np, cidx_np = ref_tree["anc"], ref_tree["cidx"]
    assert np.array_equal(_np(fc1_fused.CTX.anc), anc_np)
    assert np.array_equal(fc1_fused.CTX.cidx.cpu().numpy(), cidx_np)

    # ---- SGLang-shaped state: 3 request slots, 2 intermediate slots, 24 GDN layers in the pools
    L_pool, n_layers, slot, inter_slot = 24, 2, 2, 1
    g = torch.Generator(device=DEV)
    g.manual_seed(7)
    ssm = torch.randn(L_pool, 3, Hv, D, D, device=DEV, generator=g) * 0.02          # temporal [L, slots, H, V, K]
    ssm0 = ssm.clone()
    inter_ssm = torch.zeros(L_pool, 2, NN, Hv, D, D, device=DEV)                   # [L, slots, NN, H, V, K]
    conv_states = [torch.randn(3, C, 3, device=DEV, generator=g).to(torch.bfloat16) for _ in range(n_layers)]
    iw = [torch.zeros(2, NN, C, 3, dtype=torch.bfloat16, device=DEV) for _ in range(n_layers)]
    weights = [(torch.randn(C, 4, device=DEV, generator=g) * 0.5).to(torch.bfloat16) for _ in range(n_layers)]
    A_logs = [torch.randn(Hv, device=DEV, generator=g) * 0.5 for _ in range(n_layers)]
    dt_biases = [torch.randn(Hv, device=DEV, generator=g) * 0.5 for _ in range(n_layers)]
    xs = [torch.randn(1, C, NN, device=DEV, generator=g).to(torch.bfloat16) for _ in range(n_layers)]
    a_s = [torch.randn(1, NN, Hv, device=DEV, generator=g).to(torch.bfloat16) for _ in range(n_layers)]
    b_s = [torch.randn(1, NN, Hv, device=DEV, generator=g).to(torch.bfloat16) for _ in range(n_layers)]
    idx = lambda i: torch.tensor([i], dtype=torch.int32, device=DEV)

    def no_fallback(*a, **k):
        raise AssertionError("the hook fell back to SGLang's original")

    conv_hook = fc1_conv.make_hook(no_fallback)
    orig_commit_calls = []
    fused, fused_commit = fc1_fused.make_hooks(no_fallback, lambda *a: orig_commit_calls.append(a),
                                               lambda batch, accept_index, accept_lens, draft_token_num:
                                               (last_t, track_t))
    outs, ys = [], []
    for l in range(n_layers):
        y = conv_hook(xs[l], conv_states[l], weights[l], None, "silu", conv_state_indices=idx(slot),
                      intermediate_state_indices=idx(inter_slot), intermediate_conv_window=iw[l])
        assert y.shape == (1, C, NN)
        ys.append(y[0].t().clone())                        # [NN, C]: the verify's input (CTX.current_mixed)
        q = torch.empty(1, NN, Hk, D, device=DEV)          # shape carriers: the hook reads CTX.current_mixed
        v = torch.empty(1, NN, Hv, D, device=DEV)
        o = fused(None, A_logs[l], dt_biases[l], q, q, v, a_s[l], b_s[l], cache_steps=NN,
                  intermediate_state_indices=idx(inter_slot), ssm_states=ssm[l], cache_indices=idx(slot))
        outs.append(o)
    # acceptance: a root-to-leaf path through a depth-2 node
    u = int(np.nonzero(ref_tree["depth"] == int(ref_tree["depth"].max()))[0][0])
    p = [u]
    while ref_tree["parent"][p[-1]] >= 0:
        p.append(int(ref_tree["parent"][p[-1]]))
    p = p[::-1]
    track = int(ref_tree["nxt"][0])                         # another node to snapshot (first child of the root)
    accept_index = torch.full((1, 24), -1, dtype=torch.int64, device=DEV)
    accept_index[0, :len(p)] = torch.tensor(p, device=DEV)
    last_t = torch.tensor([p[-1]], device=DEV)
    track_t = torch.tensor([track], device=DEV)
    pool = types.SimpleNamespace(
        get_speculative_mamba2_params_all_layers=lambda: types.SimpleNamespace(temporal=ssm,
                                                                               intermediate_ssm=inter_ssm),
        get_mamba_indices=lambda rpi: idx(slot).long())
    worker = types.SimpleNamespace(model_runner=types.SimpleNamespace(req_to_token_pool=pool))
    batch = types.SimpleNamespace(req_pool_indices=torch.tensor([0], device=DEV))
    fused_commit(worker, batch, torch.tensor([len(p)], device=DEV), accept_index, NN)
    torch.cuda.synchronize()
    assert len(orig_commit_calls) == 1                      # SGLang's own commit still runs after the snapshots

    for l in range(n_layers):
        x_nc = _np(xs[l][0]).T                              # [NN, C]
        cs0 = _np(conv_states[l][slot])
        yy, win = OG.tree_conv(x_nc, cs0, _np(weights[l]), None, cidx_np)
        np.testing.assert_array_equal(_np(iw[l][inter_slot]), win)
        # the conv output is stored in bf16: within one bf16 ulp (2^-7 relative) of the fp32 oracle
        yg = _np(ys[l])
        np.testing.assert_allclose(yg, yy, rtol=2.0 ** -7, atol=1e-6)
        # verify and commit checked on the hook's own y, so that a bf16 rounding
        # flip of y (1 ulp = 0.4 %) does not count against the fp32 stages
        oo, k, vn, G = OG.tree_gdn(yg, _np(a_s[l][0]), _np(b_s[l][0]), _np(A_logs[l]), _np(dt_biases[l]),
                                   _np(ssm0[l]), slot, anc_np, Hk, Hv, D, D)
        assert _rel(_np(outs[l][0]), oo) < 2e-2, (NN, l)
        for end in (p[-1], track):
            for h in range(Hv):
                ref = OG.snapshot(_np(ssm0[l, slot, h]), k[h], vn[h], G[h], anc_np, np.asarray(p), end)
                assert _rel(_np(inter_ssm[l, inter_slot, end, h]), ref) < 1e-3, (NN, l, end, h)
    assert torch.equal(ssm, ssm0)                           # the temporal pool is only read
