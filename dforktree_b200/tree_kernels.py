"""`tree_kernels` with the reference's interface (tree_kernels.py:86-208).

`tree_gdn_split` / `tree_gdn_fused` -> dft_gdn_tree_verify (one kernel, exact
triangular inverse for any N <= 64; the reference's fused variant truncates
the inverse at 16 ancestors, this one does not), `tree_conv_fused` ->
dft_tree_conv, `closed_commit` -> dft_gdn_commit.  Single-request calls as in
the reference; the batched forms live in `kernels`.
"""
from __future__ import annotations

import torch

from . import kernels as K


def available():
    return torch.cuda.is_available()


def tree_conv_fused(conv_state, mixed0, cidx, w2, bias, BC=1024):
    """tree_kernels.py:86-93: conv_state [C, KC-1], mixed0 [N, C], cidx [N, 4]."""
    N, Cn = mixed0.shape
    cs = conv_state.unsqueeze(0)                                    # one slot
    y = K.tree_conv(mixed0.unsqueeze(0), cs, w2, bias, cidx.unsqueeze(0))
    return y[0]


def tree_gdn_split(y, aa0, bb0, A_log, dt_bias, S0, Anc, Hk, Hv, Dk, Dv, scale=None, BV=64, num_warps=8, aux=None,
                   neg_exp_A=None, state_indices=None, state_slot_stride=0):
    """tree_kernels.py:193-208.  S0 is the [Hv, Dk, Dv] view of slot 0 of a pool
    (pool[0].transpose(-1, -2), fc1_fused.py:63); state_indices[0] selects the
    slot at `state_slot_stride` elements apart.  Returns o [N, Hv, Dv] in y.dtype
    and fills aux = (k [Hv, N, Dk], vn [Hv, N, Dv], G [Hv, N]) when given."""
    N = y.shape[0]
    aa0 = aa0 if aa0.stride(-1) == 1 else aa0.contiguous()
    bb0 = bb0 if bb0.stride(-1) == 1 else bb0.contiguous()
    if aa0.stride() != bb0.stride():
        aa0, bb0 = aa0.contiguous(), bb0.contiguous()
    # pool element (slot, h, v, k) = S0[h, k, v] + slot * state_slot_stride
    s_h, s_k, s_v = S0.stride()
    strides = (int(state_slot_stride) if state_indices is not None else 0, s_h, s_v, s_k)
    # slots addressable from S0's base (bounds the state TMA)
    avail = S0.untyped_storage().nbytes() // S0.element_size() - S0.storage_offset()
    nslots = max(1, avail // int(state_slot_stride)) if state_indices is not None and state_slot_stride else 1
    slots = None
    if state_indices is not None:
        slots = state_indices.reshape(-1)[:1].to(torch.int64)
    o = torch.empty(1, N, Hv, Dv, dtype=y.dtype, device=y.device)
    ak = av = ag = None
    if aux is not None:
        ak, av, ag = aux[0].unsqueeze(0), aux[1].unsqueeze(0), aux[2].unsqueeze(0)
    K.gdn_tree_verify(y.unsqueeze(0), aa0.unsqueeze(0), bb0.unsqueeze(0), A_log, dt_bias, Anc.unsqueeze(0), S0, Hk,
                      Hv, Dk, Dv, state_slots=slots, scale=scale, neg_exp_A=neg_exp_A, o=o, aux_k=ak, aux_vn=av,
                      aux_g=ag, aux_k_per_v=True, pool_strides=strides, pool_nslots=nslots)
    return o[0]


def tree_gdn_fused(y, aa0, bb0, A_log, dt_bias, S0, Anc, Hk, Hv, Dk, Dv, scale=None, BV=16, num_warps=4, aux=None,
                   neg_exp_A=None):
    """tree_kernels.py:95-108 (single state S0 [Hv, Dk, Dv]); exact for any depth."""
    return tree_gdn_split(y, aa0, bb0, A_log, dt_bias, S0, Anc, Hk, Hv, Dk, Dv, scale=scale, aux=aux,
                          neg_exp_A=neg_exp_A)


def closed_commit(states, keys, values, gains, src, n):
    """tree_kernels.py:129-132: in place over K-major states [L, H, DK, DV] along
    the chain src[0..n].  Commits the whole chain (the reference kernel loads at
    most 16 path nodes)."""
    L_, H, DK, DV = states.shape
    N = keys.shape[2]
    nn = int(n.reshape(-1)[0]) if torch.is_tensor(n) else int(n)
    path = src.reshape(-1)[: nn + 1].to(torch.int64).reshape(1, -1)
    ends = path[:, -1:].clone()
    anc = torch.ones(1, N, N, dtype=torch.float32, device=states.device)   # a chain: every node is an ancestor
    # states (l, h, k, v) viewed as (l, slot=1, h, v, k)
    st = states.unsqueeze(1).transpose(-1, -2)
    out = torch.as_strided(states, (L_, 1, 1, H, DV, DK),
                           (states.stride(0), 0, 0, states.stride(1), states.stride(3), states.stride(2)))
    K.gdn_commit(st, out, keys.unsqueeze(1), values.unsqueeze(1), gains.unsqueeze(1), anc, path, ends, Hk=H, Hv=H,
                 aux_k_per_v=True, Dk=DK, Dv=DV)
    return states
