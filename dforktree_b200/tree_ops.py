"""`tree_ops` with the reference's interface (tree_ops.py:7-89).

`beam_tree`, `ngram_path_fn` and `tree_struct` keep their signatures; the
per-step Python closure of the reference becomes a `PathFn` descriptor that
the device beam kernel evaluates itself (one CTA per request, all steps in
shared memory).  Inputs may carry a leading batch dimension.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import kernels as K


@dataclass
class PathFn:
    """The fork-aware scoring closure of `ngram_path_fn` (tree_ops.py:55-66),
    as data: the dense PMI tensor T [B, S-1] + (M,) * order, drafter lp
    [B, S, M], out-of-list mass rest [B, S], ids [B, S, M] and the two
    weights.  The reference ships the function without its closure; the
    device kernel evaluates  lc = x - logsumexp([x, rest[s]]),
    x = lp[s] + (lam_a if on-top-1-path else lam_p) * t  with the closure
    arguments cand, pc, ppc (the beam's candidates at positions s-1, s-2,
    s-3) indexing T by order: t = T[s-1, cand] (2), T[s-1, pc, cand] (3),
    T[s-1, ppc, pc, cand] (4)."""
    T: torch.Tensor
    lp: torch.Tensor
    rest: torch.Tensor
    ids: torch.Tensor
    lam_a: float
    lam_p: float
    order: int = 3


def ngram_path_fn(ng, order, ids, lp, rest, pre1, root, lam_a, lam_p) -> PathFn:
    """tree_ops.py:55-66: builds T for n-gram order 2, 3 or 4 on the device
    (order 4 reads pre1 as E[0]; the reference's torch.cat needs it for every
    order, the device kernels of orders 2 and 3 never read it)."""
    if order not in (2, 3, 4):
        raise ValueError(f"n-gram order must be 2, 3 or 4, not {order}")
    b3 = ids.dim() == 2
    ids_b = ids.unsqueeze(0) if b3 else ids
    lp_b = lp.unsqueeze(0) if b3 else lp
    rest_b = rest.unsqueeze(0) if b3 else rest
    B = ids_b.shape[0]
    T = K.pmi_dense(ng.table, ids_b, root.reshape(B), None if pre1 is None else pre1.reshape(B), ng.status,
                    order=order)
    return PathFn(T, lp_b.float().contiguous(), rest_b.float().contiguous(), ids_b, lam_a, lam_p, order)


def beam_tree(c0, logc, N, lmax, chain_first=True, path_fn: PathFn = None, S=None, root=None):
    """tree_ops.py:7-53.  Returns (ss, cand, parent, flags) like the
    reference (node 1..N-1 order, parent -1 = root), batched if c0 is [B, M]."""
    batched = c0.dim() == 2
    c0b = c0 if batched else c0.unsqueeze(0)
    B, M = c0b.shape
    dev = c0b.device
    if path_fn is not None:
        lp, rest, ids, T = path_fn.lp, path_fn.rest, path_fn.ids, path_fn.T
        la, lpn = path_fn.lam_a, path_fn.lam_p
        logc_b = None
    else:
        logc_b = logc if logc.dim() == 4 else logc.unsqueeze(0)
        S = logc_b.shape[1] + 1
        lp = torch.zeros(B, S, M, dtype=torch.float32, device=dev)
        rest = torch.zeros(B, S, dtype=torch.float32, device=dev)
        ids = torch.zeros(B, S, M, dtype=torch.int32, device=dev)
        T, la, lpn = None, 0.3, 0.6
    rt = torch.zeros(B, dtype=torch.int64, device=dev) if root is None else root.reshape(B).to(torch.int64)
    out = K.beam_build(lp, ids, rest, rt, N, T=T, logc=None if logc_b is None else logc_b.float().contiguous(),
                       c0=c0b.float().contiguous(), lmax=lmax, chain_first=chain_first, lam_a=la, lam_p=lpn)
    parent = out["parent"][:, 1:] - 1
    res = (out["ss"], out["cand"], parent, out["flags"].bool())
    return res if batched else tuple(x[0] for x in res)


def tree_struct(parent_full, Kc=4):
    """tree_ops.py:68-89: (Anc [N,N] f32, depth [N] i64, cidx [N,4] i64)."""
    if Kc != 4:
        raise NotImplementedError("conv width 4 (Qwen3.5 GDN) only")
    batched = parent_full.dim() == 2
    anc, depth, cidx, _, _ = K.tree_struct(parent_full if batched else parent_full.unsqueeze(0))
    return (anc, depth, cidx) if batched else (anc[0], depth[0], cidx[0])
