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


def test_static_score_build_matches_workspace_entry_point():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from dforktree_b200 import build
    build.build()
    from dforktree_b200 import _lib as L
    from dforktree_b200 import kernels as K
    from dforktree_b200 import synth
    from dforktree_b200.ngram_gpu import load_npz_arrays

    lib = L.lib()
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    assert lib.dft_score_build_static_capacity() == 32 << 20
    V, S, N, B = 2048, 24, 32, 4
    table = K.Table(load_npz_arrays(synth.make_ngram_table(V, 60000, 200000, seed=21)), beta3=60.0, device=dev)
    for call in range(2):
        logits = torch.from_numpy(np.stack([synth.make_logits(S, V, seed=100 * call + r) for r in range(B)])).to(dev)
        root = torch.tensor([3 + call, 9, 27, 81], dtype=torch.int64, device=dev)
        pre1 = torch.tensor([1, 2, 3, 4 + call], dtype=torch.int64, device=dev)
        ws = K.score_build_workspace(B, S, V, N, device=dev)
        ref = K.tree_outputs(B, S, N, dev)
        K.score_build(table, logits, root, pre1, N, ws, ref)
        got = {k: torch.full_like(v, 7) for k, v in ref.items()}
        p = K.build_params(B, S, V, N)
        to = K._tree_struct_out(got)
        rc = lib.dft_score_build_static(table.handle, C.byref(p), logits.data_ptr(), L.DFT_F32, logits.stride(0),
                                        logits.stride(1), root.data_ptr(), pre1.data_ptr(), C.byref(to), None,
                                        L.stream_handle())
        assert rc == 0, lib.dft_status_string(rc)
        torch.cuda.synchronize()
        for k in ref:
            assert torch.equal(ref[k], got[k]), (call, k)
    # shapes whose scratch exceeds the fixed array are rejected before any launch
    p = K.build_params(96, S, V, N)
    out = K.tree_outputs(1, S, N, dev)
    rc = lib.dft_score_build_static(table.handle, C.byref(p), logits.data_ptr(), L.DFT_F32, logits.stride(0),
                                    logits.stride(1), root.data_ptr(), pre1.data_ptr(), C.byref(K._tree_struct_out(out)),
                                    None, L.stream_handle())
    assert rc == 6 and b"static scratch" in lib.dft_status_string(rc)
