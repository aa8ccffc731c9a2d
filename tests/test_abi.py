"""C-ABI checks that need no GPU: the library loads, exports every entry point
declared in include/dforktree_b200.h, and the ctypes structs match the C
layout (sizes and field offsets from a gcc-compiled probe of the header)."""
import ctypes
import os
import re
import subprocess

import pytest

from dforktree_b200 import _lib as L

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "dforktree_b200.h")


def _declared():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"DFT_API\s+[\w\s\*]+?\b(dft_\w+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    if not os.path.exists(L.LIB_PATH):
        from dforktree_b200 import build
        build.build()
    return L.load()


def test_library_exports_every_declared_symbol(lib):
    names = _declared()
    assert len(names) >= 16
    for n in names:
        assert hasattr(lib, n), n
    assert set(names) == set(L.SIGNATURES), "ctypes signatures must cover the header exactly"


def test_status_strings_and_version(lib):
    assert lib.dft_version() >= 10000
    assert lib.dft_status_string(0) == b"ok"
    assert b"invalid" in lib.dft_status_string(1)


def test_invalid_arguments_are_rejected_on_the_host(lib):
    # null pointers are rejected before any CUDA call (no device needed)
    assert lib.dft_table_create(None, None, None) == 1
    p = L.BuildParams(B=1, S=24, V=1000, M=15, N=32, lmax=99, use_ngram=1)
    assert lib.dft_score_build_workspace_bytes(ctypes.byref(p)) == -1      # M must be 16
    p.M = 16
    p.N = 65
    assert lib.dft_score_build_workspace_bytes(ctypes.byref(p)) == -1      # N <= 64
    p.N = 32
    assert lib.dft_score_build_workspace_bytes(ctypes.byref(p)) >= 23 * 4096 * 4
    # the closure's n-gram order: 0 (= 3), 2, 3, 4; T grows by M per order
    ws = {}
    for order in (0, 2, 3, 4):
        p.pmi_order = order
        ws[order] = lib.dft_score_build_workspace_bytes(ctypes.byref(p))
    T3 = 23 * 16 ** 3 * 4
    assert ws[0] == ws[3] and ws[4] - ws[3] >= 15 * T3 - 256 and ws[3] - ws[2] >= 15 * T3 // 16 - 256
    p.pmi_order = 5
    assert lib.dft_score_build_workspace_bytes(ctypes.byref(p)) == -1
    fake = 1 << 20
    assert lib.dft_pmi_dense(fake, ctypes.byref(p), fake, fake, None, fake, None, None) == 1   # order 5
    p.pmi_order = 4
    assert lib.dft_pmi_dense(fake, ctypes.byref(p), fake, fake, None, fake, None, None) == 1   # order 4 needs pre1
    p.pmi_order = 0
    assert lib.dft_gdn_tree_verify(None, None, None) == 1
    assert lib.dft_gdn_commit(None, None, None) == 1
    # in-place commit (zero end stride) with two end nodes would race on one tile:
    # rejected from the arguments alone (the pointers are never dereferenced)
    ca = L.CommitArgs(L=1, B=1, N=32, Hk=16, Hv=32, Dk=128, Dv=128, P=24, E=2, state_in=fake, state_out=fake,
                      so_su=0, aux_k=fake, aux_vn=fake, aux_g=fake, anc=fake, path=fake, ends=fake)
    assert lib.dft_gdn_commit(ctypes.byref(ca), None, None) == 1
    assert lib.dft_tree_conv(None, None, None) == 1
    assert lib.dft_conv_commit(None, None, None) == 1
    assert lib.dft_tree_attn(None, None, None, None) == 1
    assert lib.dft_tree_attn_workspace_bytes(None) == -1
    assert lib.dft_table_save(None, b"x", None) == 1
    assert lib.dft_table_load(None, None, None) == 1
    assert lib.dft_table_set_params(None, 20.0, 60.0, 20.0, 10.0) == 1
    assert lib.dft_table_copy_marginals(None, None, None, None) == 1
    assert b"table file" in lib.dft_status_string(7)


_PROBE = r"""
#include <stddef.h>
#include <stdio.h>
#include "dforktree_b200.h"
#define F(T, f) printf(#T " " #f " %zu\n", offsetof(T, f));
int main(void) {
  printf("dft_table_desc SIZE %zu\n", sizeof(dft_table_desc));
  printf("dft_build_params SIZE %zu\n", sizeof(dft_build_params));
  printf("dft_tree_out SIZE %zu\n", sizeof(dft_tree_out));
  printf("dft_conv_args SIZE %zu\n", sizeof(dft_conv_args));
  printf("dft_gdn_args SIZE %zu\n", sizeof(dft_gdn_args));
  printf("dft_commit_args SIZE %zu\n", sizeof(dft_commit_args));
  printf("dft_conv_commit_args SIZE %zu\n", sizeof(dft_conv_commit_args));
  F(dft_conv_commit_args, cs_st) F(dft_conv_commit_args, last) F(dft_conv_commit_args, x_sn)
  printf("dft_tree_attn_args SIZE %zu\n", sizeof(dft_tree_attn_args));
  F(dft_tree_attn_args, q) F(dft_tree_attn_args, n_slots) F(dft_tree_attn_args, sm_scale)
  F(dft_tree_attn_args, max_kv_len) F(dft_tree_attn_args, o) F(dft_tree_attn_args, o_sh)
  F(dft_table_desc, max_load) F(dft_table_desc, n4c) F(dft_build_params, lam_p) F(dft_build_params, pmi_order)
  F(dft_conv_args, iw_slots) F(dft_conv_args, y_dtype) F(dft_gdn_args, ag_sh) F(dft_gdn_args, pool)
  F(dft_gdn_args, aux_k_per_v) F(dft_gdn_args, overlap_prev) F(dft_commit_args, ends) F(dft_commit_args, aux_k_per_v) F(dft_commit_args, so_sk)
  return 0;
}
"""


def test_ctypes_layout_matches_header(tmp_path):
    src = tmp_path / "probe.c"
    src.write_text(_PROBE)
    exe = tmp_path / "probe"
    r = subprocess.run(["gcc", "-std=c99", "-I", os.path.dirname(HEADER), str(src), "-o", str(exe)],
                       capture_output=True, text=True)
    if r.returncode != 0:
        pytest.skip("gcc unavailable: " + r.stderr[:200])
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    structs = {"dft_table_desc": L.TableDesc, "dft_build_params": L.BuildParams, "dft_tree_out": L.TreeOut,
               "dft_conv_args": L.ConvArgs, "dft_gdn_args": L.GdnArgs, "dft_commit_args": L.CommitArgs,
               "dft_conv_commit_args": L.ConvCommitArgs, "dft_tree_attn_args": L.TreeAttnArgs}
    for line in out:
        if not line:
            continue
        name, field, val = line.split()
        cls = structs[name]
        if field == "SIZE":
            assert ctypes.sizeof(cls) == int(val), name
        else:
            assert getattr(cls, field).offset == int(val), (name, field)


def test_table_file_header_is_checked_before_any_device_work(lib, tmp_path):
    # missing, empty, foreign and inconsistent headers are rejected on the host (no device needed)
    h = ctypes.c_void_p()
    assert lib.dft_table_load(str(tmp_path / "missing.dftt").encode(), ctypes.byref(h), None) == 7
    cases = [b"", b"DFTTABLE" + b"\0" * 40, b"NOTATABL" + b"\0" * 120]
    import struct
    hdr = struct.pack("<8sII5q4fQQ5Q", b"DFTTABLE", 1, 0, 1000, 1024, 0, 0, 0, 20.0, 60.0, 20.0, 10.0,
                      12345, 0, 0, 0, 0, 0, 0)
    assert len(hdr) == 128
    cases.append(hdr)                                           # payload size disagrees with the slots
    cases.append(hdr[:8] + struct.pack("<I", 2) + hdr[12:])     # unknown version
    for i, blob in enumerate(cases):
        p = tmp_path / f"h{i}.dftt"
        p.write_bytes(blob)
        assert lib.dft_table_load(str(p).encode(), ctypes.byref(h), None) == 7, i
        assert not h.value


def test_tree_attention_split_plan():
    """Key splits of dft_tree_attn (host logic, no device): one split -- no
    partials workspace -- when the (request, kv-head) pairs already fill the
    SMs (batch 64 x 4 kv-heads with 4K prefixes), several for a few requests
    with long prefixes (their partials need a workspace), and none for short
    prefixes, where a unit's fixed cost outweighs the parallelism.  The
    pointers are placeholders: the plan reads only the shapes and strides."""
    from dforktree_b200 import _lib as L
    lib = L.load()
    fake = 0x10000
    D, Hq, Hkv, N = 256, 16, 4, 32

    def ws(B, max_len):
        a = L.TreeAttnArgs(B=B, N=N, Hq=Hq, Hkv=Hkv, D=D, q=fake, q_sb=N * Hq * D, q_sn=Hq * D, q_sh=D,
                           k_cache=fake, v_cache=fake, kv_st=Hkv * D, kv_sh=D, n_slots=1 << 20,
                           kv_indptr=fake, kv_indices=fake, anc=fake, anc_sb=N * N, sm_scale=0.0625,
                           max_kv_len=max_len, o=fake, o_sb=N * Hq * D, o_sn=Hq * D, o_sh=D)
        return lib.dft_tree_attn_workspace_bytes(ctypes.byref(a))

    assert ws(64, 4096 + N) == 0            # 256 pairs: one split
    assert ws(1, 4096 + N) > 0              # 4 pairs, 65 key tiles: split
    assert ws(2, 100 + N) == 0              # 3 key tiles: one split
