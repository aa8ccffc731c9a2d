"""Generate the golden fixtures from the reference implementation itself.

Run in a container that has the reference sources (never on the GPU box):

    python tests/golden/make_golden.py --ref <reference checkout>/dforktree

The reference modules are imported from their own sources: `ngram_gpu`,
`tree_ops` and `fc1_builder` run as torch CPU code; the Triton kernels of
`tree_kernels`, `fc1_block_inverse`, `fc1_conv` and `fc1_fused` run under
`TRITON_INTERPRET=1` on CPU tensors (exact float32 dots).

The one piece the reference does not ship -- the closure returned by
`tree_ops.ngram_path_fn` (tree_ops.py:66 returns an undefined `fn`) -- is
supplied by `oracle.reference_shim.reconstructed_fn`, which is the
reconstruction the oracle and the CUDA path implement; the reference's own code computes the PMI tensor T
it closes over, the beam search and the tree structure.

Inputs are rebuilt from seeds by `tests/golden/cases.py`; each fixture stores
outputs and an input checksum.
"""
from __future__ import annotations

import argparse
import os
import sys
import tempfile

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import reference_shim  # noqa: E402
from tests.golden import cases  # noqa: E402


def _load_reference(ref_dir: str):
    return reference_shim.load_reference(ref_dir)


def _table_file(table: dict) -> str:
    fd, path = tempfile.mkstemp(suffix=".npz")
    os.close(fd)
    np.savez(path, **table)
    return path


def _patch_path_fn(mods):
    return reference_shim.patch_path_fn(mods)


def gen_ngram(mods, out_dir):
    import torch
    NG = mods["ngram_gpu"].NGramGPU
    table = cases.ngram_table()
    path = _table_file(table)
    try:
        ng = NG(path, "cpu")
        ng3 = NG(path, "cpu", beta3=60.0)
    finally:
        os.unlink(path)
    z, a, b, c = cases.ngram_queries(int(table["V"]))
    t = lambda x: torch.from_numpy(x)
    res = {}
    for name, g in (("b20", ng), ("b60", ng3)):
        res[f"p2_{name}"] = g.p2(t(b), t(c)).numpy()
        res[f"p3_{name}"] = g.p3(t(a), t(b), t(c)).numpy()
        res[f"p4_{name}"] = g.p4(t(z), t(a), t(b), t(c)).numpy()
        for order in (2, 3, 4):
            res[f"pmi{order}_{name}"] = g.pmi(order, t(z), t(a), t(b), t(c)).numpy()
    res["pn"] = ng.pn.numpy()
    res["checksum"] = cases.checksum(table["keys"], table["keys3"], table["keys4"], z, a, b, c)
    np.savez_compressed(os.path.join(out_dir, "ngram_small.npz"), **res)
    print("ngram_small", {k: v.shape for k, v in res.items()})


def _run_builder(mods, captured, table, logits, root, pre1, N, chain_first, ngram):
    import torch
    FB = mods["fc1_builder"]
    NG = mods["ngram_gpu"].NGramGPU
    b = FB.Builder.__new__(FB.Builder)          # Builder.__init__ needs CUDA graphs
    b.n = N
    b.slots = logits.shape[0]
    b.chain_first = chain_first
    b.logits = torch.from_numpy(logits.copy())
    b.root = torch.tensor([root], dtype=torch.long)
    b.pre1 = torch.tensor([pre1], dtype=torch.long)
    if ngram:
        path = _table_file(table)
        try:
            b.ng = NG(path, "cpu", beta3=60.0)   # fc1_builder.py:17
        finally:
            os.unlink(path)
    else:
        b.ng = None
    captured.clear()
    b.run()
    lp, ids = torch.log_softmax(b.logits.float(), -1).topk(16, -1)
    out = dict(tokens=b.tokens.numpy(), parent=b.parent.numpy(), depth=b.depth.numpy(),
               anc=b.anc.numpy(), cidx=b.cidx.numpy(), nxt=b.nxt.numpy(), sib=b.sib.numpy(),
               lp=lp.numpy(), ids=ids.numpy())
    if ngram:
        out["T"] = captured["T"].numpy()
    return out


def gen_builder(mods, captured, out_dir, with_config0=True):
    for case in cases.BUILDER_CASES:
        table, logits, root, pre1 = cases.builder_inputs(case)
        out = _run_builder(mods, captured, table, logits, root, pre1, case["N"], case["chain_first"], case["ngram"])
        out["checksum"] = cases.checksum(logits, table["keys"], table["keys3"], [root, pre1])
        np.savez_compressed(os.path.join(out_dir, case["name"] + ".npz"), **out)
        print(case["name"], out["tokens"][:8], out["parent"][:8])
    if with_config0:
        table = None
        for seed in cases.CONFIG0_SEEDS:
            table, logits, root, pre1 = cases.config0_inputs(seed, table)
            out = _run_builder(mods, captured, table, logits, root, pre1, cases.CONFIG0["N"], False, True)
            keep = {k: out[k] for k in ("tokens", "parent", "depth", "cidx", "nxt", "sib", "lp", "ids")}
            keep["checksum"] = cases.checksum(logits, table["keys"][:100000], table["keys3"][:100000], [root, pre1])
            np.savez_compressed(os.path.join(out_dir, f"config0_seed{seed}.npz"), **keep)
            print("config0", seed, out["tokens"][:8], out["parent"][:8])


def gen_orders(mods, captured, out_dir):
    """tree_ops.ngram_path_fn at n-gram orders 2 and 4 and the reference's
    beam_tree / tree_struct over it: the steps of Builder.run
    (fc1_builder.py:27-40) with the order argument changed.  Keeps a seeded
    sample of T (cases.order_t_sample) and the whole tree."""
    import torch
    TO = mods["tree_ops"]
    NG = mods["ngram_gpu"].NGramGPU
    for case in cases.ORDER_CASES:
        table, logits, root, pre1 = cases.order_inputs(case)
        path = _table_file(table)
        try:
            ng = NG(path, "cpu", beta3=60.0)
        finally:
            os.unlink(path)
        S, N = case["S"], case["N"]
        lp, ids = torch.log_softmax(torch.from_numpy(logits).float(), -1).topk(16, -1)
        rest = torch.log((1 - lp.exp().sum(-1)).clamp(1e-06, 1.0))
        c0 = lp[0] - torch.logsumexp(torch.cat((lp[0], rest[:1])), 0)
        captured.clear()
        fn = TO.ngram_path_fn(ng, case["order"], ids, lp, rest, torch.tensor([pre1]), torch.tensor([root]), 0.3, 0.6)
        ss, cand, parent, flags = TO.beam_tree(c0, None, N, 99, case["chain_first"], fn, S=S)
        parent_full = torch.cat((torch.tensor([-1]), parent + 1))
        anc, depth, cidx = TO.tree_struct(parent_full, 4)
        T = captured["T"].numpy()
        sel = cases.order_t_sample(T.shape)
        out = dict(ids=ids.numpy(), lp=lp.numpy(), T_index=sel, T_sample=T.reshape(-1)[sel],
                   T_shape=np.asarray(T.shape), ss=ss.numpy(), cand=cand.numpy(), flags=flags.numpy(),
                   parent=parent_full.numpy(), depth=depth.numpy(), anc=anc.numpy(), cidx=cidx.numpy(),
                   tokens=torch.cat((torch.tensor([root]), ids[ss, cand])).numpy(),
                   checksum=cases.checksum(logits, table["keys"], table["keys3"], table.get("keys4", np.zeros(0)),
                                           [root, pre1]))
        np.savez_compressed(os.path.join(out_dir, case["name"] + ".npz"), **out)
        print(case["name"], T.shape, out["tokens"][:8], out["parent"][:8])


def gen_gdn(mods, out_dir):
    import torch
    TK = mods["tree_kernels"]
    for case in cases.GDN_CASES:
        d = cases.gdn_inputs(case)
        N, Hk, Hv, D = case["N"], case["Hk"], case["Hv"], case["D"]
        pool = torch.from_numpy(d["pool"].copy())
        state = pool[0].transpose(-1, -2)
        keys = torch.zeros(Hv, N, D)
        values = torch.zeros(Hv, N, D)
        gains = torch.zeros(Hv, N)
        A_log = torch.from_numpy(d["A_log"])
        neg = -A_log.float().exp()
        o = TK.tree_gdn_split(torch.from_numpy(d["y"]), torch.from_numpy(d["a"]), torch.from_numpy(d["b"]),
                              A_log, torch.from_numpy(d["dt_bias"]), state, torch.from_numpy(d["anc"]),
                              Hk, Hv, D, D, aux=(keys, values, gains), neg_exp_A=neg,
                              state_indices=torch.tensor([case["slot"]], dtype=torch.int32),
                              state_slot_stride=pool.stride(0))
        res = dict(o=o.numpy(), k=keys.numpy(), vn=values.numpy(), G=gains.numpy(),
                   checksum=cases.checksum(d["y"], d["a"], d["b"], d["pool"], d["anc"]))
        if N <= 32 and int(d["anc"].sum(1).max()) <= 16:
            # the reference's single-kernel Neumann variant (exact for <= 16-node chains)
            S0 = pool[case["slot"]].transpose(-1, -2).contiguous()
            of = TK.tree_gdn_fused(torch.from_numpy(d["y"]), torch.from_numpy(d["a"]), torch.from_numpy(d["b"]),
                                   A_log, torch.from_numpy(d["dt_bias"]), S0, torch.from_numpy(d["anc"]),
                                   Hk, Hv, D, D)
            res["o_fused"] = of.numpy()
        np.savez_compressed(os.path.join(out_dir, case["name"] + ".npz"), **res)
        print(case["name"], float(np.abs(res["o"]).max()))


def gen_conv(mods, out_dir):
    import torch
    import triton
    FC = mods["fc1_conv"]
    TK = mods["tree_kernels"]
    TO = mods["tree_ops"]
    for case in cases.CONV_CASES:
        parent, x, conv_state, weight, bias = cases.conv_inputs(case)
        N, C = case["N"], case["C"]
        _, _, cidx = TO.tree_struct(torch.from_numpy(parent), 4)
        cidx32 = cidx.int().contiguous()
        cs = torch.from_numpy(conv_state.copy())
        xt = torch.from_numpy(x.T.copy())[None]                     # [1, C, N] channels-first
        iw = torch.zeros(case["dst_slots"], N, C, 3)
        out = torch.empty(1, N, C)
        w = torch.from_numpy(weight)
        bt = torch.from_numpy(bias)
        FC.conv[(N, triton.cdiv(C, 256))](cs, xt, w, bt, cidx32, torch.tensor([case["slot"]]),
                                          torch.tensor([case["dst"]]), iw, out, C, *cs.stride(),
                                          xt.stride(1), xt.stride(2), *iw.stride(), BIAS=True, BC=256)
        y2 = TK.tree_conv_fused(cs[case["slot"]], torch.from_numpy(x), cidx32, w, bt, BC=256)
        res = dict(y=out[0].numpy(), iw=iw.numpy(), y_fused=y2.numpy(), cidx=cidx.numpy(),
                   checksum=cases.checksum(x, conv_state, weight, bias))
        np.savez_compressed(os.path.join(out_dir, case["name"] + ".npz"), **res)
        print(case["name"], float(np.abs(res["y"]).max()))


def gen_commit(mods, out_dir):
    import torch
    FF = mods["fc1_fused"]
    TK = mods["tree_kernels"]
    H = cases.COMMIT_HEADS_STORED
    for case in cases.COMMIT_CASES:
        d = cases.commit_inputs(case)
        L, NN = case["L"], case["NN"]
        temporal = torch.from_numpy(d["state"])
        K, Vn, G = torch.from_numpy(d["K"]), torch.from_numpy(d["Vn"]), torch.from_numpy(d["G"])
        anc = torch.from_numpy(d["anc"])
        path = torch.from_numpy(d["path"])[None]
        res = {}
        for e, u in enumerate(d["ends"]):
            # one end per launch into a [L, 1, 1, 32, 128, 128] output (u-stride 0)
            out = torch.zeros(L, 1, 1, 32, 128, 128)
            ends = torch.tensor([int(u), -1])
            st = list(out.stride())
            st[2] = 0
            FF.snapshots[(L * 32, 4, 8)](temporal, K, Vn, G, anc, path, ends,
                                         torch.tensor([case["slot"]]), torch.tensor([0]), out,
                                         NN, path.shape[1], *temporal.stride(), *st)
            res[f"end{e}"] = out[:, 0, 0, :H].numpy()
        # closed_commit over the accepted chain, K-major states (<= 16 nodes loaded)
        plen = int((d["path"] >= 0).sum())
        src = torch.from_numpy(d["path"][:plen].astype(np.int64))
        st_kv = torch.from_numpy(d["state"][:, case["slot"], :H].transpose(0, 1, 3, 2).copy())
        TK.closed_commit(st_kv, K[:, :H].contiguous(), Vn[:, :H].contiguous(), G[:, :H].contiguous(),
                         src, torch.tensor([plen - 1]))
        res["closed"] = st_kv.numpy()
        res["checksum"] = cases.checksum(d["state"], d["K"], d["Vn"], d["G"], d["path"])
        np.savez_compressed(os.path.join(out_dir, case["name"] + ".npz"), **res)
        print(case["name"], d["ends"], float(np.abs(res["end0"]).max()))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("DFORKTREE_REF"),
                    help="the reference's dforktree/ source directory (or set DFORKTREE_REF)")
    ap.add_argument("--out", default=HERE)
    ap.add_argument("--only", default="")
    ap.add_argument("--no-config0", action="store_true")
    args = ap.parse_args()
    if not args.ref:
        ap.error("give the reference's dforktree/ directory with --ref or DFORKTREE_REF")
    mods = _load_reference(args.ref)
    captured = _patch_path_fn(mods)
    only = set(args.only.split(",")) if args.only else {"ngram", "builder", "orders", "gdn", "conv", "commit"}
    if "ngram" in only:
        gen_ngram(mods, args.out)
    if "builder" in only:
        gen_builder(mods, captured, args.out, with_config0=not args.no_config0)
    if "orders" in only:
        gen_orders(mods, captured, args.out)
    if "gdn" in only:
        gen_gdn(mods, args.out)
    if "conv" in only:
        gen_conv(mods, args.out)
    if "commit" in only:
        gen_commit(mods, args.out)


if __name__ == "__main__":
    main()
