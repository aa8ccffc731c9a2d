"""Cached binary n-gram table (dft_table_save / dft_table_load): a table loaded
from the file answers every lookup exactly like the table it was saved from
(pinned to the reference's own golden vectors), re-saves byte-identically, and
truncated, damaged or foreign files are rejected with DFT_ERR_IO."""
import filecmp
import os
import time

import numpy as np
import pytest
import torch

from tests.golden import cases

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
DEV = "cuda"


def _np(t):
    return t.detach().cpu().numpy()


@pytest.fixture(scope="module")
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from dforktree_b200 import build
    build.build()


@pytest.mark.gpu
def test_cached_table_matches_reference_golden(_cuda, tmp_path):
    from dforktree_b200.ngram_gpu import NGramGPU, is_cached_table
    g = np.load(os.path.join(GOLD, "ngram_small.npz"))
    table = cases.ngram_table()
    z, a, b, c = (torch.from_numpy(x).to(DEV) for x in cases.ngram_queries(int(table["V"])))
    path = str(tmp_path / "small.dftt")
    NGramGPU(table, DEV, beta3=20.0).save(path)
    assert is_cached_table(path)
    for name, b3 in (("b20", 20.0), ("b60", 60.0)):
        ng = NGramGPU(path, DEV, beta3=b3)          # parameters come from the caller, not the file
        assert ng.has4
        np.testing.assert_array_equal(_np(ng.pn), g["pn"])
        np.testing.assert_array_equal(_np(ng.p2(b, c)), g[f"p2_{name}"])
        np.testing.assert_array_equal(_np(ng.p3(a, b, c)), g[f"p3_{name}"])
        np.testing.assert_array_equal(_np(ng.p4(z, a, b, c)), g[f"p4_{name}"])
        for order in (2, 3, 4):
            np.testing.assert_allclose(_np(ng.pmi(order, z, a, b, c)), g[f"pmi{order}_{name}"], rtol=1e-5,
                                       atol=1e-5)
        assert ng.device_status() == 0


@pytest.mark.gpu
def test_cached_table_resaves_byte_identical_and_equals_built(_cuda, tmp_path):
    from dforktree_b200 import kernels as K
    from dforktree_b200.ngram_gpu import load_npz_arrays
    arrays = load_npz_arrays(cases.ngram_table())
    built = K.Table(arrays, 20.0, 60.0, 20.0, 10.0)
    p1, p2 = str(tmp_path / "a.dftt"), str(tmp_path / "b.dftt")
    built.save(p1)
    loaded = K.Table.load(p1)
    assert loaded.info() == built.info() and loaded.betas is None
    loaded.save(p2)
    assert filecmp.cmp(p1, p2, shallow=False)
    prev, pn = loaded.marginals()
    np.testing.assert_array_equal(_np(prev), np.asarray(arrays["prev"], np.float32))
    np.testing.assert_array_equal(_np(pn), arrays["pn"])
    # dense PMI of the score+build path through both tables
    rng = np.random.default_rng(5)
    V = int(arrays["V"])
    ids = torch.from_numpy(rng.integers(0, V, (3, 24, 16), dtype=np.int32)).to(DEV)
    root = torch.from_numpy(rng.integers(0, V, 3)).to(DEV)
    np.testing.assert_array_equal(_np(K.pmi_dense(built, ids, root)), _np(K.pmi_dense(loaded, ids, root)))


@pytest.mark.gpu
def test_damaged_truncated_and_foreign_files_are_rejected(_cuda, tmp_path):
    from dforktree_b200 import _lib as L
    from dforktree_b200 import kernels as K
    from dforktree_b200.ngram_gpu import load_npz_arrays
    good = str(tmp_path / "good.dftt")
    K.Table(load_npz_arrays(cases.ngram_table())).save(good)
    raw = open(good, "rb").read()
    bad = []
    flipped = bytearray(raw)
    flipped[len(raw) // 2] ^= 0x40                    # payload bit flip -> checksum
    bad.append(bytes(flipped))
    bad.append(raw[: len(raw) - 4])                   # truncated payload
    bad.append(raw[:100])                             # truncated header
    bad.append(raw + b"\0" * 16)                      # trailing bytes
    bad.append(b"NOTATABL" + raw[8:])                 # foreign magic
    hdr = bytearray(raw)
    hdr[24:32] = (1000).to_bytes(8, "little")         # pair_slots not a power of two
    bad.append(bytes(hdr))
    for i, blob in enumerate(bad):
        p = str(tmp_path / f"bad{i}.dftt")
        open(p, "wb").write(blob)
        with pytest.raises(L.DFTError) as e:
            K.Table.load(p)
        assert e.value.status == L.DFT_ERR_IO, i
    with pytest.raises(L.DFTError) as e:
        K.Table.load(str(tmp_path / "missing.dftt"))
    assert e.value.status == L.DFT_ERR_IO
    # a save into a missing directory fails without leaving a partial file
    with pytest.raises(L.DFTError) as e:
        K.Table.load(good).save(str(tmp_path / "no" / "such" / "dir.dftt"))
    assert e.value.status == L.DFT_ERR_IO


@pytest.mark.gpu
def test_ngram_cache_argument_builds_once_then_loads(_cuda, tmp_path, monkeypatch):
    from dforktree_b200 import ngram_gpu as NG
    table = cases.ngram_table()
    cache = str(tmp_path / "cache.dftt")
    first = NG.NGramGPU(table, DEV, beta3=60.0, cache=cache)
    assert os.path.exists(cache) and not os.path.exists(cache + ".partial")
    calls = []
    real = NG.load_npz_arrays
    monkeypatch.setattr(NG, "load_npz_arrays", lambda p: calls.append(p) or real(p))
    second = NG.NGramGPU(table, DEV, beta3=60.0, cache=cache)
    assert calls == []                                # served from the cache, no npz read
    z, a, b, c = (torch.from_numpy(x).to(DEV) for x in cases.ngram_queries(int(table["V"]), n=2000, seed=3))
    for order in (2, 3, 4):
        np.testing.assert_array_equal(_np(first.pmi(order, z, a, b, c)), _np(second.pmi(order, z, a, b, c)))
    # a damaged cache is rebuilt from the npz and rewritten
    raw = bytearray(open(cache, "rb").read())
    raw[-1] ^= 1
    open(cache, "wb").write(bytes(raw))
    third = NG.NGramGPU(table, DEV, beta3=60.0, cache=cache)
    assert len(calls) == 1
    np.testing.assert_array_equal(_np(first.p3(a, b, c)), _np(third.p3(a, b, c)))
    NG.NGramGPU(table, DEV, beta3=60.0, cache=cache)  # intact again
    assert len(calls) == 1


@pytest.mark.gpu
def test_config0_table_round_trip_and_load_time(_cuda, tmp_path):
    """Full-vocabulary config-0 table (2M bigram, 8M trigram keys): build from
    arrays vs. load from the cached file; the loaded table re-saves identically."""
    from dforktree_b200 import kernels as K
    from dforktree_b200 import synth
    from dforktree_b200.ngram_gpu import load_npz_arrays
    c = cases.CONFIG0
    arrays = load_npz_arrays(synth.make_ngram_table(c["V"], c["nb"], c["nt"], seed=c["table_seed"]))
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    built = K.Table(arrays, 20.0, 60.0, 20.0, 10.0)
    torch.cuda.synchronize()
    t_build = time.perf_counter() - t0
    p1, p2 = str(tmp_path / "c0.dftt"), str(tmp_path / "c0b.dftt")
    built.save(p1)
    t0 = time.perf_counter()
    loaded = K.Table.load(p1)
    t_load = time.perf_counter() - t0
    loaded.save(p2)
    assert filecmp.cmp(p1, p2, shallow=False)
    print(f"config0 table: {os.path.getsize(p1) / 2**20:.0f} MiB, build from arrays {t_build * 1e3:.0f} ms, "
          f"load from cache {t_load * 1e3:.0f} ms")
    rng = np.random.default_rng(9)
    q = [torch.from_numpy(rng.integers(-1, c["V"], 200000)).to(DEV) for _ in range(4)]
    for order in (2, 3):
        np.testing.assert_array_equal(_np(K.ngram_eval(built, order, 1, None, *q[1:])),
                                      _np(K.ngram_eval(loaded, order, 1, None, *q[1:])))
