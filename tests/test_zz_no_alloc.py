"""dft_score_build_static: the allocation-free score + build entry point.

Some callers cannot call cudaMalloc: a plugin running inside a serving
engine's decode step, whose device memory belongs to the engine's static
pools and to torch's caching allocator, or a C host that binds only this ABI
and has no device allocator.  For them the library keeps the score + build
scratch in one fixed-size device array.  This test calls that entry point
through the C ABI and checks its trees against dft_score_build (the
workspace entry point) on two calls in a row with different inputs -- the
shared array keeps the previous call's contents, which must not leak into
the next result -- and that shapes above the array's capacity are rejected.
The file is named to be collected last.
"""
import ctypes as C

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _setup():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from dforktree_b200 import build
    build.build()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    return dev


def _static_call(lib, L, K, table, p, logits, root, pre1, got, status):
    to = K._tree_struct_out(got)
    return lib.dft_score_build_static(None if table is None else table.handle, C.byref(p), logits.data_ptr(),
                                      L.DFT_F32, logits.stride(0), logits.stride(1), root.data_ptr(),
                                      L.ptr(pre1), C.byref(to), status.data_ptr(), L.stream_handle())


def _compare(B, S, V, N, use_ngram, seed):
    """Two calls in a row of dft_score_build_static against dft_score_build on
    fresh inputs each time; trees must be identical and no status bit set."""
    from dforktree_b200 import _lib as L
    from dforktree_b200 import kernels as K
    from dforktree_b200 import synth
    from dforktree_b200.ngram_gpu import load_npz_arrays

    dev = _setup()
    lib = L.lib()
    table = None
    if use_ngram:
        table = K.Table(load_npz_arrays(synth.make_ngram_table(V, 60000, 200000, seed=seed)), beta3=60.0, device=dev)
    g = torch.Generator(device=dev)
    for call in range(2):
        g.manual_seed(1000 * seed + call)
        logits = torch.randn(B, S, V, device=dev, generator=g) * 3.0
        peak = torch.randint(0, V, (B, S), device=dev, generator=g)
        logits.view(-1, V)[torch.arange(B * S, device=dev), peak.view(-1)] += 6.0
        root = torch.randint(0, V, (B,), device=dev, generator=g)
        pre1 = torch.randint(0, V, (B,), device=dev, generator=g)
        st_ref = torch.zeros(1, dtype=torch.int32, device=dev)
        st = torch.zeros(1, dtype=torch.int32, device=dev)
        ws = K.score_build_workspace(B, S, V, N, use_ngram=use_ngram, device=dev)
        ref = K.tree_outputs(B, S, N, dev)
        K.score_build(table, logits, root, pre1, N, ws, ref, use_ngram=use_ngram, status=st_ref)
        got = {k: torch.full_like(v, 7) for k, v in ref.items()}
        p = K.build_params(B, S, V, N, use_ngram=use_ngram)
        rc = _static_call(lib, L, K, table, p, logits, root, pre1, got, st)
        assert rc == 0, lib.dft_status_string(rc)
        torch.cuda.synchronize()
        assert int(st_ref.item()) == 0 and int(st.item()) == 0
        for k in ref:
            assert torch.equal(ref[k], got[k]), (B, S, use_ngram, call, k)
    return lib, L, K, table, logits, root, pre1


def test_static_score_build_matches_workspace_entry_point():
    """Small batch with the n-gram closure, then a shape above the capacity,
    which is rejected before any launch."""
    lib, L, K, table, logits, root, pre1 = _compare(4, 24, 2048, 32, True, seed=21)
    assert lib.dft_score_build_static_capacity() == 32 << 20
    dev = logits.device
    p = K.build_params(96, 24, 2048, 32)
    out = K.tree_outputs(1, 24, 32, dev)
    st = torch.zeros(1, dtype=torch.int32, device=dev)
    rc = _static_call(lib, L, K, table, p, logits, root, pre1, out, st)
    assert rc == 6 and b"static scratch" in lib.dft_status_string(rc)


def test_static_score_build_at_capacity_shape():
    """64 requests at S = 24, the shape the 32 MiB array is sized for (its
    dense PMI tensor alone is 24.1 MB); the vocabulary stays small because the
    scratch does not depend on it."""
    from dforktree_b200 import kernels as K
    from dforktree_b200 import _lib as L
    B, S, N = 64, 24, 32
    p = K.build_params(B, S, 2048, N)
    assert L.lib().dft_score_build_workspace_bytes(C.byref(p)) > 24_000_000
    _compare(B, S, 2048, N, True, seed=22)


@pytest.mark.parametrize("B,S", [(8, 24), (3, 1)])
def test_static_score_build_without_ngram_and_single_position(B, S):
    """The branches where no PMI tensor is written: the no-n-gram builder
    (fc1_builder.py:35-36) and a one-position draft (no PMI launch)."""
    _compare(B, S, 2048, 32 if S > 1 else 8, S == 1, seed=23 + S)
