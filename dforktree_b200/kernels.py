"""Thin torch-facing wrappers over the C ABI (one function per entry point).

Tensors must be CUDA tensors on the current device; every call is launched
on the current torch stream and never synchronises.  Shapes follow the
batched C ABI: requests first.
"""
from __future__ import annotations

import ctypes as C
import os

import torch

from . import _lib as L


def _status_ptr(status):
    return None if status is None else status.data_ptr()


# ------------------------------------------------------------------ table --
class Table:
    """Device n-gram hash tables (owner of a dft_table handle)."""

    def __init__(self, arrays: dict, beta2=20.0, beta3=20.0, beta4=20.0, clip=10.0, max_load=0.35,
                 device=None):
        lib = L.lib()
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        g = lambda k: arrays.get(k)
        t = lambda x, dt: None if x is None else torch.as_tensor(x).to(device=dev, dtype=dt).contiguous()
        keys, cab = t(g("keys"), torch.int64), t(g("cab"), torch.float32)
        prev, pn = t(g("prev"), torch.float32), t(g("pn"), torch.float32)
        k3, c3 = t(g("keys3"), torch.int64), t(g("c3"), torch.float32)
        k3c, n3c = t(g("keys3c"), torch.int64), t(g("n3c"), torch.float32)
        k4, c4, n4c = t(g("keys4"), torch.int64), t(g("c4"), torch.float32), t(g("n4c"), torch.float32)
        n = lambda x: 0 if x is None else int(x.numel())
        d = L.TableDesc(V=int(arrays["V"]), keys=L.ptr(keys), cab=L.ptr(cab), n_bigram=n(keys), prev=L.ptr(prev),
                        pn=L.ptr(pn), keys3=L.ptr(k3), c3=L.ptr(c3), n_trigram=n(k3), keys3c=L.ptr(k3c),
                        n3c=L.ptr(n3c), n_ctx3=n(k3c), keys4=L.ptr(k4), c4=L.ptr(c4), n_quad=n(k4),
                        n4c=L.ptr(n4c), beta2=beta2, beta3=beta3, beta4=beta4, clip=clip, max_load=max_load)
        h = C.c_void_p()
        with torch.cuda.device(dev):
            L.check(lib.dft_table_create(C.byref(d), C.byref(h), L.stream_handle()), "dft_table_create")
        self.handle = h
        self.V = int(arrays["V"])
        self.device = dev
        self.betas = (beta2, beta3, beta4, clip)

    @classmethod
    def load(cls, path, device=None, params=None):
        """Table from a cached file written by `save` (no npz parse, no hash build).
        `params` = (beta2, beta3, beta4, clip) overrides the saved parameters."""
        lib = L.lib()
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        h = C.c_void_p()
        with torch.cuda.device(dev):
            L.check(lib.dft_table_load(os.fsencode(path), C.byref(h), L.stream_handle()), "dft_table_load")
        self = cls.__new__(cls)
        self.handle, self.device = h, dev
        self.V = self.info()["V"]
        self.betas = None
        if params is not None:
            self.set_params(*params)
        return self

    def save(self, path):
        """Write the built tables to `path` (see dft_table_save)."""
        with torch.cuda.device(self.device):
            L.check(L.load().dft_table_save(self.handle, os.fsencode(path), L.stream_handle()), "dft_table_save")

    def set_params(self, beta2, beta3, beta4, clip):
        L.check(L.load().dft_table_set_params(self.handle, beta2, beta3, beta4, clip), "dft_table_set_params")
        self.betas = (beta2, beta3, beta4, clip)

    def marginals(self):
        """(prev [V], pn [V]) fp32 device copies of the table's marginals."""
        prev = torch.empty(self.V, dtype=torch.float32, device=self.device)
        pn = torch.empty_like(prev)
        with torch.cuda.device(self.device):
            L.check(L.load().dft_table_copy_marginals(self.handle, prev.data_ptr(), pn.data_ptr(),
                                                      L.stream_handle()), "dft_table_copy_marginals")
        return prev, pn

    def info(self):
        v = [C.c_int64() for _ in range(5)]
        L.check(L.load().dft_table_info(self.handle, *[C.byref(x) for x in v]), "dft_table_info")
        return dict(V=v[0].value, pair_slots=v[1].value, trip_slots=v[2].value, quad_slots=v[3].value,
                    bytes=v[4].value)

    def close(self):
        if getattr(self, "handle", None) is not None and self.handle.value:
            L.load().dft_table_destroy(self.handle)
            self.handle = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def ngram_eval(table: Table, order: int, what: int, z, a, b, c, status=None) -> torch.Tensor:
    """Elementwise p (what=0) or PMI (what=1) over broadcast id tensors."""
    lib = L.lib()
    ids = [x for x in (z, a, b, c) if x is not None]
    shape = torch.broadcast_shapes(*[x.shape for x in ids])
    flat = lambda x: None if x is None else x.to(torch.int64).expand(shape).contiguous().reshape(-1)
    fz, fa, fb, fc = flat(z), flat(a), flat(b), flat(c)
    out = torch.empty(shape, dtype=torch.float32, device=fb.device)
    L.check(lib.dft_ngram_eval(table.handle, order, what, L.ptr(fz), L.ptr(fa), L.ptr(fb), L.ptr(fc),
                               fb.numel(), out.data_ptr(), _status_ptr(status), L.stream_handle()),
            "dft_ngram_eval")
    return out


# ---------------------------------------------------------- score + build --
def build_params(B, S, V, N, M=16, lmax=99, chain_first=False, use_ngram=True, lam_a=0.3, lam_p=0.6, order=3):
    return L.BuildParams(B=B, S=S, V=V, M=M, N=N, lmax=lmax, chain_first=int(bool(chain_first)),
                         use_ngram=int(bool(use_ngram)), lam_a=lam_a, lam_p=lam_p, pmi_order=order)


def pmi_step_shape(order: int, M: int = 16):
    """Shape of T per (request, step) for the closure's n-gram order."""
    if order not in (2, 3, 4):
        raise ValueError(f"n-gram order must be 2, 3 or 4, not {order}")
    return (M,) * order


def _logits_view(logits: torch.Tensor):
    if logits.dim() == 2:
        logits = logits.unsqueeze(0)
    if logits.stride(-1) != 1:
        logits = logits.contiguous()
    B, S, V = logits.shape
    return logits, B, S, V, logits.stride(0), logits.stride(1)


def score(logits: torch.Tensor, M: int = 16):
    """lp [B,S,M] f32, ids [B,S,M] i32, rest [B,S] f32 (fc1_builder.py:27-28)."""
    lib = L.lib()
    x, B, S, V, sb, ss = _logits_view(logits)
    p = build_params(B, S, V, N=32, M=M)
    lp = torch.empty(B, S, M, dtype=torch.float32, device=x.device)
    ids = torch.empty(B, S, M, dtype=torch.int32, device=x.device)
    rest = torch.empty(B, S, dtype=torch.float32, device=x.device)
    L.check(lib.dft_score(C.byref(p), x.data_ptr(), L.dtype_code(x), sb, ss, lp.data_ptr(), ids.data_ptr(),
                          rest.data_ptr(), L.stream_handle()), "dft_score")
    return lp, ids, rest


def pmi_dense(table: Table, ids: torch.Tensor, root: torch.Tensor, pre1: torch.Tensor = None, status=None,
              order: int = 3):
    """Dense PMI T over E = [pre1; root; ids] (tree_ops.py:56-65): [B, S-1, M, M]
    for order 2, [B, S-1, M, M, M] for order 3, [B, S-1, M, M, M, M] for
    order 4 (which reads pre1 as E[0] and requires it)."""
    lib = L.lib()
    B, S, M = ids.shape
    step = pmi_step_shape(order, M)
    if order == 4 and pre1 is None:
        raise L.DFTError("order-4 PMI needs pre1 (E[0])")
    ids = ids.to(torch.int32).contiguous()
    root = root.reshape(B).to(torch.int64).contiguous()
    pre1 = None if pre1 is None else pre1.reshape(B).to(torch.int64).contiguous()
    p = build_params(B, S, table.V, N=32, M=M, order=order)
    T = torch.empty(B, S - 1, *step, dtype=torch.float32, device=ids.device)
    L.check(lib.dft_pmi_dense(table.handle, C.byref(p), ids.data_ptr(), root.data_ptr(), L.ptr(pre1),
                              T.data_ptr(), _status_ptr(status), L.stream_handle()), "dft_pmi_dense")
    return T


def tree_outputs(B, S, N, device, W=None, extras=True):
    W = max(N - 1, 16) if W is None else W
    o = dict(tokens=torch.empty(B, N, dtype=torch.int64, device=device),
             parent=torch.empty(B, N, dtype=torch.int64, device=device),
             depth=torch.empty(B, N, dtype=torch.int64, device=device),
             anc=torch.empty(B, N, N, dtype=torch.float32, device=device),
             nxt=torch.empty(B, N, dtype=torch.int64, device=device),
             sib=torch.empty(B, N, dtype=torch.int64, device=device),
             cidx=torch.empty(B, N, 4, dtype=torch.int64, device=device))
    if extras:
        o.update(ss=torch.empty(B, N - 1, dtype=torch.int64, device=device),
                 cand=torch.empty(B, N - 1, dtype=torch.int64, device=device),
                 flags=torch.empty(B, N - 1, dtype=torch.uint8, device=device),
                 keys=torch.empty(B, S, W, dtype=torch.float32, device=device))
    return o


def _tree_struct_out(o: dict) -> L.TreeOut:
    return L.TreeOut(**{k: L.ptr(o.get(k)) for k in ("tokens", "parent", "depth", "anc", "nxt", "sib", "cidx",
                                                       "ss", "cand", "flags", "keys")})


def beam_build(lp, ids, rest, root, N, T=None, logc=None, c0=None, lmax=99, chain_first=False, lam_a=0.3,
               lam_p=0.6, out=None, status=None, V=None):
    """The n-gram order of the closure follows from T's rank: T [B, S-1]
    + (M,) * order."""
    lib = L.lib()
    B, S, M = lp.shape
    use_ngram = T is not None
    order = 3
    if use_ngram:
        order = T.dim() - 2
        if T.shape != (B, S - 1, *pmi_step_shape(order, M)) or not T.is_contiguous():
            raise L.DFTError(f"T must be a contiguous [B, S-1] + (M,) * order tensor, got {tuple(T.shape)}")
    p = build_params(B, S, V or 1 << 20, N, M, lmax, chain_first, use_ngram, lam_a, lam_p, order)
    out = tree_outputs(B, S, N, lp.device) if out is None else out
    to = _tree_struct_out(out)
    L.check(lib.dft_beam_build(C.byref(p), lp.contiguous().data_ptr(), ids.to(torch.int32).contiguous().data_ptr(),
                               rest.contiguous().data_ptr(), L.ptr(T), L.ptr(logc), L.ptr(c0),
                               root.reshape(B).to(torch.int64).contiguous().data_ptr(), C.byref(to),
                               _status_ptr(status), L.stream_handle()), "dft_beam_build")
    return out


def score_build_workspace(B, S, V, N, use_ngram=True, M=16, device=None, order=3) -> torch.Tensor:
    p = build_params(B, S, V, N, M, use_ngram=use_ngram, order=order)
    nbytes = L.load().dft_score_build_workspace_bytes(C.byref(p))
    if nbytes < 0:
        raise L.DFTError("unsupported score_build shape")
    return torch.empty(max(nbytes, 1), dtype=torch.uint8, device=device)


def score_build(table, logits, root, pre1, N, workspace, out, lmax=99, chain_first=False, use_ngram=True,
                lam_a=0.3, lam_p=0.6, status=None, order=3):
    """Builder.run (fc1_builder.py:26-47) for a batch: three launches.  `order`
    is the n-gram order of the closure (the Builder's is 3); the workspace
    must be sized for the same order."""
    lib = L.lib()
    x, B, S, V, sb, ss = _logits_view(logits)
    p = build_params(B, S, V, N, 16, lmax, chain_first, use_ngram, lam_a, lam_p, order)
    to = _tree_struct_out(out)
    L.check(lib.dft_score_build(None if table is None else table.handle, C.byref(p), x.data_ptr(), L.dtype_code(x),
                                sb, ss, root.data_ptr(), L.ptr(pre1), workspace.data_ptr(), C.byref(to),
                                _status_ptr(status), L.stream_handle()), "dft_score_build")
    return out


def score_build_static(table, logits, root, pre1, N, out, lmax=99, chain_first=False, use_ngram=True, lam_a=0.3,
                       lam_p=0.6, status=None, order=3):
    """score_build without a workspace: the library's fixed-size device
    scratch (dft_score_build_static); for callers that cannot allocate."""
    lib = L.lib()
    x, B, S, V, sb, ss = _logits_view(logits)
    p = build_params(B, S, V, N, 16, lmax, chain_first, use_ngram, lam_a, lam_p, order)
    to = _tree_struct_out(out)
    L.check(lib.dft_score_build_static(None if table is None else table.handle, C.byref(p), x.data_ptr(),
                                       L.dtype_code(x), sb, ss, root.data_ptr(), L.ptr(pre1), C.byref(to),
                                       _status_ptr(status), L.stream_handle()), "dft_score_build_static")
    return out


def tree_struct(parent: torch.Tensor, status=None):
    """anc [B,N,N], depth, cidx [B,N,4], nxt, sib for parent [B,N] (root first)."""
    lib = L.lib()
    if parent.dim() == 1:
        parent = parent.unsqueeze(0)
    parent = parent.to(torch.int64).contiguous()
    B, N = parent.shape
    dev = parent.device
    anc = torch.empty(B, N, N, dtype=torch.float32, device=dev)
    depth = torch.empty(B, N, dtype=torch.int64, device=dev)
    cidx = torch.empty(B, N, 4, dtype=torch.int64, device=dev)
    nxt = torch.empty(B, N, dtype=torch.int64, device=dev)
    sib = torch.empty(B, N, dtype=torch.int64, device=dev)
    L.check(lib.dft_tree_struct(B, N, parent.data_ptr(), anc.data_ptr(), depth.data_ptr(), cidx.data_ptr(),
                                nxt.data_ptr(), sib.data_ptr(), _status_ptr(status), L.stream_handle()),
            "dft_tree_struct")
    return anc, depth, cidx, nxt, sib


def accept_greedy(tokens, nxt, sib, target, P, status=None, out=None):
    """Greedy tree acceptance; returns (path [B,P], accept_len, last, bonus)."""
    lib = L.lib()
    B, N = tokens.shape
    dev = tokens.device
    if out is None:
        out = (torch.empty(B, P, dtype=torch.int64, device=dev), torch.empty(B, dtype=torch.int64, device=dev),
               torch.empty(B, dtype=torch.int64, device=dev), torch.empty(B, dtype=torch.int64, device=dev))
    path, alen, last, bonus = out
    c = lambda t: t.to(torch.int64).contiguous()
    tokens, nxt, sib, target = c(tokens), c(nxt), c(sib), c(target)
    L.check(lib.dft_accept_greedy(B, N, P, tokens.data_ptr(), nxt.data_ptr(), sib.data_ptr(), target.data_ptr(),
                                  path.data_ptr(), alen.data_ptr(), last.data_ptr(), bonus.data_ptr(),
                                  _status_ptr(status), L.stream_handle()), "dft_accept_greedy")
    return path, alen, last, bonus


# -------------------------------------------------------------- tree conv --
def tree_conv(x, conv_state, weight, bias, cidx, state_slots=None, y=None, iw=None, iw_slots=None, status=None):
    """x [B, N, C] (any strides, channel stride given), conv_state [slots, C, 3],
    weight [C, 4], cidx [B, N, 4] -> y [B, N, C] (fc1_conv.py:8-27)."""
    lib = L.lib()
    B, N, Cn = x.shape
    if y is None:
        y = torch.empty(B, N, Cn, dtype=x.dtype, device=x.device)
    assert y.stride(2) == 1
    w = weight.reshape(Cn, 4).contiguous()
    cidx = cidx.reshape(B, N, 4).to(torch.int64).contiguous()
    a = L.ConvArgs(B=B, N=N, C=Cn, x=x.data_ptr(), x_dtype=L.dtype_code(x), x_sb=x.stride(0), x_sn=x.stride(1),
                   x_sc=x.stride(2), conv_state=conv_state.data_ptr(), cs_dtype=L.dtype_code(conv_state),
                   cs_ss=conv_state.stride(0), cs_sc=conv_state.stride(1), cs_st=conv_state.stride(2),
                   state_slots=L.ptr(state_slots), weight=w.data_ptr(), w_dtype=L.dtype_code(w),
                   bias=L.ptr(None if bias is None else bias.to(w.dtype).contiguous()), cidx=cidx.data_ptr(),
                   y=y.data_ptr(), y_dtype=L.dtype_code(y), y_sb=y.stride(0), y_sn=y.stride(1),
                   iw=L.ptr(iw), iw_dtype=L.dtype_code(iw) if iw is not None else 0,
                   iw_sd=iw.stride(0) if iw is not None else 0, iw_sn=iw.stride(1) if iw is not None else 0,
                   iw_sc=iw.stride(2) if iw is not None else 0, iw_sj=iw.stride(3) if iw is not None else 0,
                   iw_slots=L.ptr(iw_slots))
    keep = (w, cidx, bias)
    L.check(lib.dft_tree_conv(C.byref(a), _status_ptr(status), L.stream_handle()), "dft_tree_conv")
    del keep
    return y


def conv_commit(x, conv_state, cidx, last, slots=None, status=None):
    """Conv-window commit: conv_state [.., slots, C, 3] of each request takes the
    window (taps 1..3) of its last accepted node `last` [B] (< 0: unchanged).
    x [B, N, C] or [L, B, N, C] pre-conv inputs (channel stride 1); conv_state
    [slots, C, 3] or [L, slots, C, 3]; cidx [B, N, 4].  In place."""
    lib = L.lib()
    if x.dim() == 3:
        x = x.unsqueeze(0)
        conv_state = conv_state.unsqueeze(0)
    Ln, B, N, Cn = x.shape
    assert x.stride(3) == 1 and conv_state.shape[0] == Ln
    assert conv_state.shape[2:] == (Cn, 3) and cidx.numel() == B * N * 4 and last.numel() == B
    assert slots is not None or conv_state.shape[1] >= B
    cidx = cidx.reshape(B, N, 4).to(torch.int64).contiguous()
    last = last.reshape(B).to(torch.int64).contiguous()
    slots = None if slots is None else slots.reshape(B).to(torch.int64).contiguous()
    a = L.ConvCommitArgs(L=Ln, B=B, N=N, C=Cn, x=x.data_ptr(), x_dtype=L.dtype_code(x), x_sl=x.stride(0),
                         x_sb=x.stride(1), x_sn=x.stride(2), conv_state=conv_state.data_ptr(),
                         cs_dtype=L.dtype_code(conv_state), cs_sl=conv_state.stride(0), cs_ss=conv_state.stride(1),
                         cs_sc=conv_state.stride(2), cs_st=conv_state.stride(3), slots=L.ptr(slots),
                         cidx=cidx.data_ptr(), last=last.data_ptr())
    keep = (cidx, last, slots)
    L.check(lib.dft_conv_commit(C.byref(a), _status_ptr(status), L.stream_handle()), "dft_conv_commit")
    del keep


# -------------------------------------------------------- GDN tree verify --
def gdn_tree_verify(y, a, b, A_log, dt_bias, anc, pool, Hk, Hv, Dk=128, Dv=128, state_slots=None, scale=None,
                    neg_exp_A=None, o=None, aux_k=None, aux_vn=None, aux_g=None, aux_k_per_v=True, status=None,
                    pool_strides=None, pool_nslots=None, conv=None, force_simt=False, overlap_prev=False):
    """Batched tree GDN verify.

    y [B, N, 2*Hk*Dk + Hv*Dv] (last stride 1) -- or None with conv = dict(x=[B, N, C]
    pre-conv inputs, conv_state=[slots, C, 3], weight=[C, 4], bias=None|[C],
    cidx=[B, N, 4], conv_slots=None|[B]) to fuse the tree conv;
    a, b [B, N, Hv] (last stride 1);
    pool [slots, Hv, Dv, Dk] (any strides; `pool_strides` = (slot, h, v, k)
    element strides overrides pool.stride() for views torch cannot express);
    anc [B, N, N] f32; o [B, N, Hv, Dv].
    aux_k [B, Hv or Hk, N, Dk], aux_vn [B, Hv, N, Dv], aux_g [B, Hv, N].
    overlap_prev: programmatic dependent launch -- the caller guarantees that
    the kernel queued just before this call writes none of pool, anc, the conv
    state / weights / columns and the slot maps (the previous layer's verify
    does not); dropped when an argument needs a conversion here (that copy
    would be the kernel just before).
    """
    lib = L.lib()
    ref = y if y is not None else conv["x"]
    B, N, _ = ref.shape
    assert ref.stride(2) == 1 and a.stride(2) == 1 and b.stride(2) == 1 and a.stride() == b.stride()
    if o is None:
        o = torch.empty(B, N, Hv, Dv, dtype=ref.dtype, device=ref.device)
    assert o.stride(3) == 1
    anc_in = anc
    anc = anc.reshape(B, N, N).to(torch.float32).contiguous()
    converted = anc.data_ptr() != anc_in.data_ptr()
    if scale is None:
        scale = Dk ** -0.5
    A_log_f = None if A_log is None else A_log.to(torch.float32).contiguous()
    neg = None if neg_exp_A is None else neg_exp_A.to(torch.float32).contiguous()
    dtb = dt_bias.contiguous()
    ps = tuple(pool.stride()) if pool_strides is None else tuple(int(x) for x in pool_strides)
    nslots = int(pool.shape[0]) if pool_nslots is None and pool_strides is None else int(pool_nslots or 0)
    cv = None
    keep_cv = ()
    if conv is not None:
        x = conv["x"]
        cs = conv["conv_state"]
        w = conv["weight"].reshape(-1, 4).contiguous()
        bias = conv.get("bias")
        bias = None if bias is None else bias.to(w.dtype).contiguous()
        cidx = conv["cidx"].reshape(B, N, 4).to(torch.int64).contiguous()
        cslots = conv.get("conv_slots")
        cslots = None if cslots is None else cslots.to(torch.int64).contiguous()
        converted = converted or w.data_ptr() != conv["weight"].data_ptr() or \
            cidx.data_ptr() != conv["cidx"].data_ptr() or \
            (bias is not None and bias.data_ptr() != conv["bias"].data_ptr()) or \
            (cslots is not None and cslots.data_ptr() != conv["conv_slots"].data_ptr())
        cv = L.GdnConvArgs(x=x.data_ptr(), x_dtype=L.dtype_code(x), x_sb=x.stride(0), x_sn=x.stride(1),
                           conv_state=cs.data_ptr(), cs_dtype=L.dtype_code(cs), cs_ss=cs.stride(0),
                           cs_sc=cs.stride(1), cs_st=cs.stride(2), conv_slots=L.ptr(cslots), weight=w.data_ptr(),
                           w_dtype=L.dtype_code(w), bias=L.ptr(bias), cidx=cidx.data_ptr())
        keep_cv = (w, bias, cidx, cslots)
    args = L.GdnArgs(B=B, N=N, Hk=Hk, Hv=Hv, Dk=Dk, Dv=Dv, scale=float(scale),
                     y=L.ptr(y), y_dtype=L.dtype_code(y) if y is not None else 0,
                     y_sb=y.stride(0) if y is not None else 0, y_sn=y.stride(1) if y is not None else 0,
                     a=a.data_ptr(), bg=b.data_ptr(), ab_dtype=L.dtype_code(a), ab_sb=a.stride(0), ab_sn=a.stride(1),
                     A_log=L.ptr(A_log_f), neg_exp_A=L.ptr(neg), dt_bias=dtb.data_ptr(), dtb_dtype=L.dtype_code(dtb),
                     anc=anc.data_ptr(), pool=pool.data_ptr(), p_ss=ps[0], p_sh=ps[1], p_sv=ps[2], p_sk=ps[3],
                     p_nslots=nslots, state_slots=L.ptr(state_slots),
                     o=o.data_ptr(), o_dtype=L.dtype_code(o), o_sb=o.stride(0), o_sn=o.stride(1), o_sh=o.stride(2),
                     aux_k=L.ptr(aux_k), aux_k_per_v=int(bool(aux_k_per_v)),
                     ak_sb=aux_k.stride(0) if aux_k is not None else 0,
                     ak_sh=aux_k.stride(1) if aux_k is not None else 0,
                     ak_sn=aux_k.stride(2) if aux_k is not None else 0,
                     aux_vn=L.ptr(aux_vn), av_sb=aux_vn.stride(0) if aux_vn is not None else 0,
                     av_sh=aux_vn.stride(1) if aux_vn is not None else 0,
                     av_sn=aux_vn.stride(2) if aux_vn is not None else 0,
                     aux_g=L.ptr(aux_g), ag_sb=aux_g.stride(0) if aux_g is not None else 0,
                     ag_sh=aux_g.stride(1) if aux_g is not None else 0,
                     conv=C.pointer(cv) if cv is not None else None, force_simt=int(bool(force_simt)),
                     overlap_prev=int(bool(overlap_prev) and not converted))
    keep = (anc, A_log_f, neg, dtb, keep_cv, cv)
    rc = lib.dft_gdn_tree_verify(C.byref(args), _status_ptr(status), L.stream_handle())
    del keep
    if rc == L.DFT_ERR_UNSUPPORTED and conv is not None:
        # the fused conv lives in the tensor-core path (bf16 x and conv state):
        # otherwise run the tree conv as its own launch, then the verify
        yc = tree_conv(conv["x"], conv["conv_state"], conv["weight"], conv.get("bias"), conv["cidx"],
                       state_slots=conv.get("conv_slots"), status=status)
        return gdn_tree_verify(yc, a, b, A_log, dt_bias, anc, pool, Hk, Hv, Dk, Dv, state_slots=state_slots,
                               scale=scale, neg_exp_A=neg_exp_A, o=o, aux_k=aux_k, aux_vn=aux_vn, aux_g=aux_g,
                               aux_k_per_v=aux_k_per_v, status=status, pool_strides=pool_strides,
                               pool_nslots=pool_nslots, force_simt=force_simt)
    L.check(rc, "dft_gdn_tree_verify")
    return o


# ------------------------------------------------------------------ commit --
def gdn_commit(state_in, state_out, aux_k, aux_vn, aux_g, anc, path, ends, Hk, Hv, slots_in=None, slots_out=None,
               aux_k_per_v=True, status=None, Dk=128, Dv=128):
    """Closed-form commit (fc1_fused.py:27-49) over layers and requests.

    state_in [L, slots, Hv, Dv, Dk] (any strides); state_out [L, dst, U, Hv, Dv, Dk]
    where U is the node axis (stride 0 -> write into the slot itself);
    aux_k [L, B, H*, N, Dk], aux_vn [L, B, Hv, N, Dv], aux_g [L, B, Hv, N];
    anc [B, N, N]; path [B, P] (-1 padded); ends [B, E] (-1 = skip).
    """
    lib = L.lib()
    Lr, B, _, N, _ = aux_vn.shape
    P = path.shape[1]
    E = ends.shape[1]
    if state_out.dim() != 6 or state_in.dim() != 5:
        raise L.DFTError("gdn_commit: state_in is [L, slots, Hv, Dv, Dk], state_out [L, dst, nodes, Hv, Dv, Dk]")
    if state_out.shape[2] < N and state_out.stride(2) != 0:
        raise L.DFTError("gdn_commit: the node axis of state_out must cover all N nodes or have stride 0")
    if state_out.stride(2) == 0 and E > 1:
        raise L.DFTError("gdn_commit: several ends cannot share one output slot (node stride 0)")
    anc = anc.reshape(B, N, N).to(torch.float32).contiguous()
    path = path.to(torch.int64).contiguous()
    ends = ends.to(torch.int64).contiguous()
    si, so = state_in.stride(), state_out.stride()
    args = L.CommitArgs(L=Lr, B=B, N=N, Hk=Hk, Hv=Hv, Dk=Dk, Dv=Dv, P=P, E=E,
                        state_in=state_in.data_ptr(), si_sl=si[0], si_ss=si[1], si_sh=si[2], si_sv=si[3], si_sk=si[4],
                        state_out=state_out.data_ptr(), so_sl=so[0], so_ss=so[1], so_su=so[2], so_sh=so[3],
                        so_sv=so[4], so_sk=so[5], slots_in=L.ptr(slots_in), slots_out=L.ptr(slots_out),
                        aux_k=aux_k.data_ptr(), aux_k_per_v=int(bool(aux_k_per_v)), ak_sl=aux_k.stride(0),
                        ak_sb=aux_k.stride(1), ak_sh=aux_k.stride(2), ak_sn=aux_k.stride(3),
                        aux_vn=aux_vn.data_ptr(), av_sl=aux_vn.stride(0), av_sb=aux_vn.stride(1),
                        av_sh=aux_vn.stride(2), av_sn=aux_vn.stride(3),
                        aux_g=aux_g.data_ptr(), ag_sl=aux_g.stride(0), ag_sb=aux_g.stride(1), ag_sh=aux_g.stride(2),
                        anc=anc.data_ptr(), path=path.data_ptr(), ends=ends.data_ptr())
    keep = (anc, path, ends)
    L.check(lib.dft_gdn_commit(C.byref(args), _status_ptr(status), L.stream_handle()), "dft_gdn_commit")
    del keep
    return state_out


# ----------------------------------------------------- tree-masked attention --
def tree_attn_args(q, k_cache, v_cache, kv_indptr, kv_indices, anc, max_kv_len, sm_scale=None, o=None):
    """(ctypes args, o, kept tensors) for dft_tree_attn; shapes as tree_attention."""
    B, N, Hq, D = q.shape
    slots, Hkv, Dk = k_cache.shape
    if v_cache.shape != k_cache.shape or v_cache.stride() != k_cache.stride() or Dk != D:
        raise L.DFTError("tree_attention: k_cache / v_cache must both be [slots, Hkv, D] with equal strides")
    if q.stride(3) != 1 or k_cache.stride(2) != 1:
        raise L.DFTError("tree_attention: the head dim must be contiguous")
    if o is None:
        o = torch.empty(B, N, Hq, D, dtype=q.dtype, device=q.device)
    kv_indptr = kv_indptr.to(torch.int32).contiguous()
    kv_indices = kv_indices.to(torch.int32).contiguous()
    anc = anc.reshape(B, N, N).to(torch.float32).contiguous()
    a = L.TreeAttnArgs(B=B, N=N, Hq=Hq, Hkv=Hkv, D=D, q=q.data_ptr(), q_sb=q.stride(0), q_sn=q.stride(1),
                       q_sh=q.stride(2), k_cache=k_cache.data_ptr(), v_cache=v_cache.data_ptr(),
                       kv_st=k_cache.stride(0), kv_sh=k_cache.stride(1), n_slots=slots,
                       kv_indptr=kv_indptr.data_ptr(), kv_indices=kv_indices.data_ptr(), anc=anc.data_ptr(),
                       anc_sb=N * N, sm_scale=float(D ** -0.5 if sm_scale is None else sm_scale),
                       max_kv_len=int(max_kv_len), o=o.data_ptr(), o_sb=o.stride(0), o_sn=o.stride(1),
                       o_sh=o.stride(2))
    return a, o, (kv_indptr, kv_indices, anc)


def tree_attention(q, k_cache, v_cache, kv_indptr, kv_indices, anc, max_kv_len=None, sm_scale=None, o=None,
                   workspace=None, status=None):
    """Tree-masked attention verify: q [B, N, Hq, D] bf16; k_cache / v_cache
    [slots, Hkv, D] bf16 (page size 1); request b's keys are
    kv_indices[kv_indptr[b]:kv_indptr[b+1]] (prefix first, then the N tree
    nodes); anc [B, N, N] ancestor-or-self.  max_kv_len: host-known bound on
    the per-request key count (read from kv_indptr, with a sync, if None).
    Returns o [B, N, Hq, D]."""
    lib = L.lib()
    if max_kv_len is None:
        ptr = kv_indptr.to(torch.int64)
        max_kv_len = int((ptr[1:] - ptr[:-1]).max().item())
    a, o, keep = tree_attn_args(q, k_cache, v_cache, kv_indptr, kv_indices, anc, max_kv_len, sm_scale, o)
    need = lib.dft_tree_attn_workspace_bytes(C.byref(a))
    if need < 0:
        raise L.DFTError("tree_attention: shape outside the tensor-core path (D = 256, G in {1,2,4,8}, N*G <= 128)")
    if need > 0 and (workspace is None or workspace.numel() * workspace.element_size() < need):
        workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    L.check(lib.dft_tree_attn(C.byref(a), None if need == 0 else workspace.data_ptr(), _status_ptr(status),
                              L.stream_handle()), "dft_tree_attn")
    del keep
    return o
