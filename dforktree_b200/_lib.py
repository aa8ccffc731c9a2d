"""ctypes binding of the C ABI in include/dforktree_b200.h.

The shared library is built in-tree (`python -m dforktree_b200.build`).  There
is no fallback: if the library or a CUDA device is missing, every op raises.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libdforktree_b200.so")

DFT_F32, DFT_BF16, DFT_F16 = 0, 1, 2
DFT_OK, DFT_ERR_INVALID, DFT_ERR_UNSUPPORTED = 0, 1, 2
DFT_ERR_TABLE, DFT_ERR_IO = 4, 7
DEV_BAD_TOKEN, DEV_PROBE_LIMIT, DEV_BAD_INDEX, DEV_TIMEOUT = 1, 2, 4, 8

_DTYPES = {torch.float32: DFT_F32, torch.bfloat16: DFT_BF16, torch.float16: DFT_F16}

i32, i64, f32, vp = C.c_int32, C.c_int64, C.c_float, C.c_void_p


class DFTError(RuntimeError):
    def __init__(self, msg, status=None):
        super().__init__(msg)
        self.status = status


class TableDesc(C.Structure):
    _fields_ = [("V", i64),
                ("keys", vp), ("cab", vp), ("n_bigram", i64),
                ("prev", vp), ("pn", vp),
                ("keys3", vp), ("c3", vp), ("n_trigram", i64),
                ("keys3c", vp), ("n3c", vp), ("n_ctx3", i64),
                ("keys4", vp), ("c4", vp), ("n_quad", i64),
                ("n4c", vp),
                ("beta2", f32), ("beta3", f32), ("beta4", f32), ("clip", f32),
                ("max_load", f32)]


class BuildParams(C.Structure):
    _fields_ = [("B", i32), ("S", i32), ("V", i32), ("M", i32), ("N", i32), ("lmax", i32),
                ("chain_first", i32), ("use_ngram", i32), ("lam_a", f32), ("lam_p", f32), ("pmi_order", i32)]


class TreeOut(C.Structure):
    _fields_ = [("tokens", vp), ("parent", vp), ("depth", vp), ("anc", vp), ("nxt", vp), ("sib", vp),
                ("cidx", vp), ("ss", vp), ("cand", vp), ("flags", vp), ("keys", vp)]


class ConvArgs(C.Structure):
    _fields_ = [("B", i32), ("N", i32), ("C", i32),
                ("x", vp), ("x_dtype", i32), ("x_sb", i64), ("x_sn", i64), ("x_sc", i64),
                ("conv_state", vp), ("cs_dtype", i32), ("cs_ss", i64), ("cs_sc", i64), ("cs_st", i64),
                ("state_slots", vp),
                ("weight", vp), ("w_dtype", i32),
                ("bias", vp),
                ("cidx", vp),
                ("y", vp), ("y_dtype", i32), ("y_sb", i64), ("y_sn", i64),
                ("iw", vp), ("iw_dtype", i32), ("iw_sd", i64), ("iw_sn", i64), ("iw_sc", i64), ("iw_sj", i64),
                ("iw_slots", vp)]


class ConvCommitArgs(C.Structure):
    _fields_ = [("L", i32), ("B", i32), ("N", i32), ("C", i32),
                ("x", vp), ("x_dtype", i32), ("x_sl", i64), ("x_sb", i64), ("x_sn", i64),
                ("conv_state", vp), ("cs_dtype", i32), ("cs_sl", i64), ("cs_ss", i64), ("cs_sc", i64), ("cs_st", i64),
                ("slots", vp), ("cidx", vp), ("last", vp)]


class TreeAttnArgs(C.Structure):
    _fields_ = [("B", i32), ("N", i32), ("Hq", i32), ("Hkv", i32), ("D", i32),
                ("q", vp), ("q_sb", i64), ("q_sn", i64), ("q_sh", i64),
                ("k_cache", vp), ("v_cache", vp), ("kv_st", i64), ("kv_sh", i64), ("n_slots", i64),
                ("kv_indptr", vp), ("kv_indices", vp), ("anc", vp), ("anc_sb", i64),
                ("sm_scale", f32), ("max_kv_len", i32),
                ("o", vp), ("o_sb", i64), ("o_sn", i64), ("o_sh", i64)]


class GdnConvArgs(C.Structure):
    _fields_ = [("x", vp), ("x_dtype", i32), ("x_sb", i64), ("x_sn", i64),
                ("conv_state", vp), ("cs_dtype", i32), ("cs_ss", i64), ("cs_sc", i64), ("cs_st", i64),
                ("conv_slots", vp), ("weight", vp), ("w_dtype", i32), ("bias", vp), ("cidx", vp)]


class GdnArgs(C.Structure):
    _fields_ = [("B", i32), ("N", i32), ("Hk", i32), ("Hv", i32), ("Dk", i32), ("Dv", i32),
                ("scale", f32),
                ("y", vp), ("y_dtype", i32), ("y_sb", i64), ("y_sn", i64),
                ("a", vp), ("bg", vp), ("ab_dtype", i32), ("ab_sb", i64), ("ab_sn", i64),
                ("A_log", vp), ("neg_exp_A", vp),
                ("dt_bias", vp), ("dtb_dtype", i32),
                ("anc", vp),
                ("pool", vp), ("p_ss", i64), ("p_sh", i64), ("p_sv", i64), ("p_sk", i64), ("p_nslots", i64),
                ("state_slots", vp),
                ("o", vp), ("o_dtype", i32), ("o_sb", i64), ("o_sn", i64), ("o_sh", i64),
                ("aux_k", vp), ("aux_k_per_v", i32), ("ak_sb", i64), ("ak_sh", i64), ("ak_sn", i64),
                ("aux_vn", vp), ("av_sb", i64), ("av_sh", i64), ("av_sn", i64),
                ("aux_g", vp), ("ag_sb", i64), ("ag_sh", i64),
                ("conv", C.POINTER(GdnConvArgs)), ("force_simt", i32), ("overlap_prev", i32)]


class CommitArgs(C.Structure):
    _fields_ = [("L", i32), ("B", i32), ("N", i32), ("Hk", i32), ("Hv", i32), ("Dk", i32), ("Dv", i32),
                ("P", i32), ("E", i32),
                ("state_in", vp), ("si_sl", i64), ("si_ss", i64), ("si_sh", i64), ("si_sv", i64), ("si_sk", i64),
                ("state_out", vp), ("so_sl", i64), ("so_ss", i64), ("so_su", i64), ("so_sh", i64), ("so_sv", i64),
                ("so_sk", i64),
                ("slots_in", vp), ("slots_out", vp),
                ("aux_k", vp), ("aux_k_per_v", i32), ("ak_sl", i64), ("ak_sb", i64), ("ak_sh", i64), ("ak_sn", i64),
                ("aux_vn", vp), ("av_sl", i64), ("av_sb", i64), ("av_sh", i64), ("av_sn", i64),
                ("aux_g", vp), ("ag_sl", i64), ("ag_sb", i64), ("ag_sh", i64),
                ("anc", vp), ("path", vp), ("ends", vp)]


# exported entry points: name -> (restype, argtypes)
SIGNATURES = {
    "dft_status_string": (C.c_char_p, [C.c_int]),
    "dft_version": (C.c_int, []),
    "dft_table_create": (C.c_int, [C.POINTER(TableDesc), C.POINTER(vp), vp]),
    "dft_table_destroy": (C.c_int, [vp]),
    "dft_table_info": (C.c_int, [vp, C.POINTER(i64), C.POINTER(i64), C.POINTER(i64), C.POINTER(i64),
                                 C.POINTER(i64)]),
    "dft_table_set_params": (C.c_int, [vp, f32, f32, f32, f32]),
    "dft_table_copy_marginals": (C.c_int, [vp, vp, vp, vp]),
    "dft_table_save": (C.c_int, [vp, C.c_char_p, vp]),
    "dft_table_load": (C.c_int, [C.c_char_p, C.POINTER(vp), vp]),
    "dft_ngram_eval": (C.c_int, [vp, C.c_int, C.c_int, vp, vp, vp, vp, i64, vp, vp, vp]),
    "dft_score": (C.c_int, [C.POINTER(BuildParams), vp, i32, i64, i64, vp, vp, vp, vp]),
    "dft_pmi_dense": (C.c_int, [vp, C.POINTER(BuildParams), vp, vp, vp, vp, vp, vp]),
    "dft_beam_build": (C.c_int, [C.POINTER(BuildParams), vp, vp, vp, vp, vp, vp, vp, C.POINTER(TreeOut), vp, vp]),
    "dft_score_build_workspace_bytes": (i64, [C.POINTER(BuildParams)]),
    "dft_score_build": (C.c_int, [vp, C.POINTER(BuildParams), vp, i32, i64, i64, vp, vp, vp, C.POINTER(TreeOut),
                                  vp, vp]),
    "dft_score_build_static_capacity": (i64, []),
    "dft_score_build_static": (C.c_int, [vp, C.POINTER(BuildParams), vp, i32, i64, i64, vp, vp, C.POINTER(TreeOut),
                                         vp, vp]),
    "dft_tree_struct": (C.c_int, [i32, i32, vp, vp, vp, vp, vp, vp, vp, vp]),
    "dft_accept_greedy": (C.c_int, [i32, i32, i32, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp]),
    "dft_tree_conv": (C.c_int, [C.POINTER(ConvArgs), vp, vp]),
    "dft_conv_commit": (C.c_int, [C.POINTER(ConvCommitArgs), vp, vp]),
    "dft_tree_attn_workspace_bytes": (i64, [C.POINTER(TreeAttnArgs)]),
    "dft_tree_attn": (C.c_int, [C.POINTER(TreeAttnArgs), vp, vp, vp]),
    "dft_gdn_tree_verify": (C.c_int, [C.POINTER(GdnArgs), vp, vp]),
    "dft_gdn_commit": (C.c_int, [C.POINTER(CommitArgs), vp, vp]),
}

_lib = None
_lock = threading.Lock()


def load(path: str = LIB_PATH):
    """Load the shared library (no device needed) and bind every entry point."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise DFTError(f"{path} is missing: build it with `python -m dforktree_b200.build`")
        lib = C.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def lib():
    """The library for a compute call: requires a CUDA device (no CPU path)."""
    if not torch.cuda.is_available():
        raise DFTError("dforktree_b200 ops need a CUDA device (sm_100a); there is no CPU fallback")
    return load()


def check(rc: int, what: str):
    if rc != 0:
        msg = load().dft_status_string(rc).decode()
        raise DFTError(f"{what} failed: {msg} (status {rc})", rc)


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise DFTError(f"unsupported dtype {t.dtype}") from None


def ptr(t) -> int | None:
    return None if t is None else t.data_ptr()


def stream_handle(device=None) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def require_cuda(*tensors):
    for t in tensors:
        if t is not None and not t.is_cuda:
            raise DFTError("dforktree_b200 ops take CUDA tensors; there is no CPU fallback")
