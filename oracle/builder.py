"""Oracle: scoring, fork-aware closure, beam tree search, tree structure.

Test infrastructure only.  numpy float32 restatement of
  * `Builder.run`                 -- fc1_builder.py:26-47
  * `tree_ops.beam_tree`          -- tree_ops.py:7-53
  * `tree_ops.ngram_path_fn`      -- tree_ops.py:55-66 (T construction)
  * `tree_ops.tree_struct`        -- tree_ops.py:68-89

Conventions shared with the CUDA path (both differ from torch only where torch
leaves an order unspecified):
  * top-k returns values in descending order, exact ties broken by the lower
    flat index first;
  * argmax returns the first maximal index (as torch documents).

PARITY-UNPINNED piece: the reference ships `ngram_path_fn` without the closure
it returns (`return fn` with `fn` undefined, tree_ops.py:66).  `path_scores`
restates its reconstruction: for beam w at step s with parent candidate
`cand[w]`, grandparent candidate `pc[w]` and flag `al[w]` ("every ancestor was
the drafter's top-1"):
    x[w, l]  = lp[s, l] + lam(al[w]) * T[s-1, pc[w], cand[w], l]
    lam      = lam_a if al[w] else lam_p
    lc[w, l] = x[w, l] - logsumexp([x[w, :], rest[s]])
i.e. PMI evidence from the branch's last two tokens with the larger weight
(lam_p) after the branch leaves the top-1 path, renormalised together with the
out-of-list mass `rest[s]` exactly like the no-n-gram branch of Builder.run
(fc1_builder.py:35-36).  For the other orders `ngram_path_fn` accepts
(tree_ops.py:59-64) the same closure reads the context its T spans:
T[s-1, cand[w], l] for order 2 and T[s-1, ppc[w], pc[w], cand[w], l] for
order 4, `ppc` being the great-grandparent candidate beam_tree carries for it
(tree_ops.py:24, 40).
"""
from __future__ import annotations

import numpy as np

F32 = np.float32
NEG = F32(-np.inf)


def _topk_desc(x: np.ndarray, k: int):
    """Top-k of a 1-D array: values descending, ties -> lower index first."""
    x = np.asarray(x)
    order = np.lexsort((np.arange(x.size), -x.astype(np.float64)))[:k]
    return x[order], order


def _logsumexp_lastdim(x: np.ndarray) -> np.ndarray:
    # torch.logsumexp: amax, infinite max replaced by 0, log(sum(exp(x-m))) + m
    m = np.max(x, axis=-1, keepdims=True)
    m = np.where(np.isinf(m), F32(0), m).astype(np.float32)
    s = np.sum(np.exp((x - m).astype(np.float32)), axis=-1, keepdims=True, dtype=np.float32)
    return (np.log(s) + m).astype(np.float32)


def _row_topk(x: np.ndarray, M: int):
    """Row-wise top-M of a [S, V] array (descending, ties -> lower index)."""
    S, V = x.shape
    part = np.argpartition(-x, M - 1, axis=1)[:, :M]
    thr = np.take_along_axis(x, part, 1).min(axis=1)
    ids = np.empty((S, M), np.int64)
    for s in range(S):
        above = np.nonzero(x[s] > thr[s])[0]
        tie = np.nonzero(x[s] == thr[s])[0]
        cand = np.concatenate([above, tie[: M - above.size]])
        v = x[s, cand]
        o = np.lexsort((cand, -v.astype(np.float64)))
        ids[s] = cand[o]
    return ids


def score(logits: np.ndarray, M: int = 16):
    """fc1_builder.py:27-29: lp, ids = topk(log_softmax(logits)); rest; c0."""
    x = np.asarray(logits, np.float32)
    m = x.max(axis=-1, keepdims=True)
    sh = (x - m).astype(np.float32)
    lse = np.log(np.sum(np.exp(sh), axis=-1, keepdims=True, dtype=np.float32)).astype(np.float32)
    lp_full = (sh - lse).astype(np.float32)
    ids = _row_topk(lp_full, M)
    lp = np.take_along_axis(lp_full, ids, 1).astype(np.float32)
    rest = np.log(np.clip(F32(1) - np.sum(np.exp(lp), axis=-1, dtype=np.float32), F32(1e-6), F32(1.0))).astype(np.float32)
    c0 = (lp[0] - _logsumexp_lastdim(np.concatenate([lp[0], rest[:1]]))).astype(np.float32)
    return lp, ids, rest, c0


def dense_pmi(ng, order: int, ids: np.ndarray, pre1: int, root: int) -> np.ndarray:
    """tree_ops.py:56-65: the dense PMI tensor T over E = [pre1; root; ids]."""
    S, M = ids.shape
    E = np.concatenate([np.full((1, M), pre1, np.int64), np.full((1, M), root, np.int64),
                        ids.astype(np.int64)], 0)
    ch = E[3:S + 2]
    if order == 2:
        T = ng.pmi(2, None, None, E[2:S + 1][:, :, None], ch[:, None, :])
    elif order == 3:
        T = ng.pmi(3, None, E[1:S][:, :, None, None], E[2:S + 1][:, None, :, None], ch[:, None, None, :])
    else:
        T = ng.pmi(4, E[0:S - 1][:, :, None, None, None], E[1:S][:, None, :, None, None],
                   E[2:S + 1][:, None, None, :, None], ch[:, None, None, None, :])
    return np.asarray(T, np.float32)


def path_scores(T: np.ndarray, lp: np.ndarray, rest: np.ndarray, lam_a: float, lam_p: float):
    """Reconstructed fork-aware closure fn(s, cand, pc, ppc, al) -> lc [W, M]
    (PARITY-UNPINNED, see module docstring).  The order follows from T
    [S-1] + (M,) * order: cand, pc, ppc are the beam's candidates at
    positions s-1, s-2, s-3, i.e. the order-4 context, so order 2 reads
    T[s-1][cand], order 3 T[s-1][pc, cand], order 4 T[s-1][ppc, pc, cand]."""
    la, lpn = F32(lam_a), F32(lam_p)
    order = T.ndim - 1

    def fn(s, cand, pc, ppc, al):
        Ts = T[s - 1]
        t = Ts[cand] if order == 2 else (Ts[pc, cand] if order == 3 else Ts[ppc, pc, cand])   # [W, M]
        lam = np.where(al, la, lpn).astype(np.float32)[:, None]
        x = (lp[s][None, :] + (lam * t).astype(np.float32)).astype(np.float32)
        r = np.broadcast_to(rest[s], (x.shape[0], 1)).astype(np.float32)
        return (x - _logsumexp_lastdim(np.concatenate([x, r], -1))).astype(np.float32)

    return fn


def beam_tree(c0, logc, N, lmax, chain_first=True, path_fn=None, S=None, trace=None):
    """tree_ops.py:7-53 in numpy.  `trace` (a list) receives per-step keys for
    tie classification in tests."""
    S = logc.shape[0] + 1 if logc is not None else S
    M = c0.shape[0]
    W = max(N - 1, M)
    assert W >= M and lmax >= 1
    BIG = F32(10000.0 if chain_first else 0.0)
    arM = np.arange(M)
    top0 = arM == int(np.argmax(c0))
    pad = W - M
    sc = np.concatenate([c0.astype(np.float32), np.full(pad, NEG, np.float32)])
    fl = np.concatenate([top0, np.zeros(pad, bool)])
    lv = np.concatenate([(~top0).astype(np.int64), np.full(pad, lmax + 1, np.int64)])
    cand = np.concatenate([arM, np.zeros(pad, np.int64)])
    par = np.full(W, -1, np.int64)
    al = np.concatenate([arM == 0, np.zeros(pad, bool)])
    pc = np.zeros(W, np.int64)
    ppc = np.zeros(W, np.int64)
    key = np.where((lv <= lmax) & (sc > NEG), (sc + BIG * fl.astype(np.float32)).astype(np.float32), NEG)
    keys, pars, cands, fls = [key], [par], [cand], [fl]
    for s in range(1, S):
        lc = logc[s - 1].astype(np.float32)[cand] if path_fn is None else path_fn(s, cand, pc, ppc, al).astype(np.float32)
        is_top = arM[None, :] == np.argmax(lc, -1)[:, None]
        sc_c = (sc[:, None] + lc).astype(np.float32)
        fl_c = fl[:, None] & is_top
        lv_c = lv[:, None] + (~is_top).astype(np.int64)
        ok = (lv_c <= lmax) & (key[:, None] > NEG)
        key_c = np.where(ok, (sc_c + BIG * fl_c.astype(np.float32)).astype(np.float32), NEG)
        if trace is not None:
            trace.append(np.sort(key_c.reshape(-1))[::-1].copy())
        key, idx = _topk_desc(key_c.reshape(-1), W)
        p_, c_ = idx // M, idx % M
        sc, fl, lv = sc_c.reshape(-1)[idx], fl_c.reshape(-1)[idx], lv_c.reshape(-1)[idx]
        pc, ppc, al = cand[p_], pc[p_], al[p_] & (c_ == 0)
        par, cand = p_, c_
        keys.append(key)
        pars.append(par)
        cands.append(cand)
        fls.append(fl)
    K, Pb, Cb, Fb = np.stack(keys), np.stack(pars), np.stack(cands), np.stack(fls)
    kflat = K.reshape(-1)
    if trace is not None:
        trace.append(np.sort(kflat)[::-1].copy())
    _, gi = _topk_desc(kflat, N - 1)
    ss, bi = gi // W, gi % W
    order = np.argsort(ss * W + np.arange(N - 1), kind="stable")
    ss, bi = ss[order], bi[order]
    inv = np.zeros((S, W), np.int64)
    inv[ss, bi] = np.arange(1, N)
    pb = Pb[ss, bi]
    parent = np.where(ss == 0, 0, inv[np.maximum(ss - 1, 0), np.maximum(pb, 0)]) - 1
    return ss, Cb[ss, bi], parent, Fb[ss, bi], K


def tree_struct(parent_full: np.ndarray, Kc: int):
    """tree_ops.py:68-89: ancestor matrix (incl. self), depth, conv columns."""
    N = parent_full.shape[0]
    ar = np.arange(N)
    P = np.zeros((N, N), np.float32)
    P[ar[1:], np.maximum(parent_full[1:], 0)] = 1.0
    I = np.eye(N, dtype=np.float32)
    Anc, Pk = I + P, P @ P
    for _ in range(4):
        Anc = Anc @ (I + Pk)
        Pk = Pk @ Pk
    Anc = (Anc > 0.5).astype(np.float32)
    depth = Anc.sum(1).astype(np.int64) - 1
    cols, Pr = [], I
    for r in range(Kc):
        if r > 0:
            Pr = Pr @ P
        a_r = np.argmax(Pr, 1)
        cols.append(np.where(r <= depth, Kc - 1 + a_r, Kc - 1 - (r - depth)))
    cidx = np.stack(cols[::-1], 1).astype(np.int64)
    return Anc, depth, cidx


def next_and_sibling(parent_full: np.ndarray):
    """fc1_builder.py:41-47: first child (`nxt`) and next sibling (`sib`)."""
    n = parent_full.shape[0]
    u = np.arange(n)
    children = (parent_full[None, :] == u[:, None]) & (u[None, :] > 0)
    nxt = np.where(children, u[None, :], n).min(-1)
    sibling = (parent_full[:, None] == parent_full[None, :]) & (u[None, :] > u[:, None])
    sib = np.where(sibling, u[None, :], n).min(-1)
    return np.where(nxt < n, nxt, -1), np.where(sib < n, sib, -1)


def builder_run(logits, root: int, pre1: int, ng=None, N: int = 32, chain_first: bool = False,
                lam_a: float = 0.3, lam_p: float = 0.6, M: int = 16, lmax: int = 99,
                order: int = 3, trace=None) -> dict:
    """fc1_builder.py:26-47 (`Builder.run`) for one request."""
    logits = np.asarray(logits, np.float32)
    S = logits.shape[0]
    lp, ids, rest, c0 = score(logits, M)
    T = None
    if ng is not None:
        T = dense_pmi(ng, order, ids, pre1, root)
        fn, logc = path_scores(T, lp, rest, lam_a, lam_p), None
    else:
        fn = None
        base = np.broadcast_to(lp[1:, None, :], (S - 1, M, M)).astype(np.float32)
        r = np.broadcast_to(rest[1:, None, None], (S - 1, M, 1)).astype(np.float32)
        logc = (base - _logsumexp_lastdim(np.concatenate([base, r], -1))).astype(np.float32)
    ss, cand, parent, flags, K = beam_tree(c0, logc, N, lmax, chain_first, fn, S=S, trace=trace)
    parent_full = np.concatenate([[-1], parent + 1]).astype(np.int64)
    anc, depth, cidx = tree_struct(parent_full, 4)
    tokens = np.concatenate([[root], ids[ss, cand]]).astype(np.int64)
    nxt, sib = next_and_sibling(parent_full)
    return dict(lp=lp, ids=ids, rest=rest, c0=c0, T=T, ss=ss, cand=cand, flags=flags, keys=K,
                parent=parent_full, anc=anc, depth=depth, cidx=cidx, tokens=tokens, nxt=nxt, sib=sib)
