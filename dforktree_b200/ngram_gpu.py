"""`NGramGPU` with the reference's interface (ngram_gpu.py:6-70), backed by
open-addressed HBM hash tables and the dft_ngram_eval / dft_pmi_dense kernels.

Same constructor (npz path or dict in the reference schema, device, betas,
clip) and the same p2 / p3 / p4 / pmi methods over broadcastable id tensors.
"""
from __future__ import annotations

import os

import numpy as np
import torch

from . import _lib as L
from . import kernels as K


def load_npz_arrays(path_or_arrays) -> dict:
    """Arrays of the reference npz schema (ngram_gpu.py:9-25) as numpy."""
    if isinstance(path_or_arrays, dict):
        z = path_or_arrays
        files = set(z.keys())
    else:
        z = np.load(path_or_arrays)
        files = set(z.files)
    need = {"V", "N", "keys", "cab", "prev", "nxt"}
    missing = need - files
    if missing:
        raise KeyError(f"n-gram table is missing {sorted(missing)}")
    out = {k: np.asarray(z[k]) for k in files}
    V = int(out["V"])
    N = float(out["N"])
    # pn in float64 then cast, exactly as ngram_gpu.py:16
    out["pn"] = ((out["nxt"].astype(np.float64) + 1.0) / (N + V)).astype(np.float32)
    if "keys3" not in files:
        out.pop("c3", None)
    if "keys3c" not in files:
        out.pop("n3c", None)
    if "keys4" not in files:
        for k in ("c4", "n4c"):
            out.pop(k, None)
    return out


TABLE_MAGIC = b"DFTTABLE"


def is_cached_table(path) -> bool:
    """True when `path` is a file written by `NGramGPU.save` / `dft_table_save`."""
    if isinstance(path, dict) or not isinstance(path, (str, bytes, os.PathLike)):
        return False
    try:
        with open(path, "rb") as f:
            return f.read(8) == TABLE_MAGIC
    except OSError:
        return False


class NGramGPU:
    """Drop-in for dforktree.ngram_gpu.NGramGPU.

    `path` is the reference's npz (or a dict of its arrays) or a cached table
    file.  With `cache=<file>`, an intact cached table there is loaded instead
    of the npz; a missing or damaged one is rebuilt from the npz and written
    back.  Either way the smoothing parameters are the ones passed here.
    """

    def __init__(self, path, dev, beta2=20.0, beta3=20.0, beta4=20.0, clip=10.0, max_load=0.35, cache=None):
        self.beta2, self.beta3, self.beta4, self.clip = beta2, beta3, beta4, clip
        dev = torch.device(dev)
        if dev.type != "cuda":
            raise RuntimeError("NGramGPU needs a CUDA device; there is no CPU path")
        self.device = dev
        params = (beta2, beta3, beta4, clip)
        self.table = None
        with torch.cuda.device(dev):
            for src in ([path] if is_cached_table(path) else []) + ([cache] if cache is not None else []):
                if src is not None and os.path.exists(src):
                    try:
                        self.table = K.Table.load(src, device=dev, params=params)
                        break
                    except L.DFTError as e:
                        if e.status != L.DFT_ERR_IO or src is path:
                            raise
            if self.table is not None:
                self.prev, self.pn = self.table.marginals()
                self.has4 = self.table.info()["quad_slots"] > 0
            else:
                arrays = load_npz_arrays(path)
                self.pn = torch.from_numpy(arrays["pn"]).to(dev)
                self.prev = torch.from_numpy(np.asarray(arrays["prev"]).astype(np.float32)).to(dev)
                self.has4 = "keys4" in arrays
                self.table = K.Table(arrays, beta2, beta3, beta4, clip, max_load, device=dev)
                if cache is not None:
                    self.table.save(cache)
            self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.V = self.table.V

    def save(self, path):
        """Write this table as a cached table file (loads with NGramGPU(path, dev))."""
        self.table.save(path)

    def _t(self, x):
        if x is None:
            return None
        return torch.as_tensor(x, device=self.device)

    def p2(self, b, c):
        return K.ngram_eval(self.table, 2, 0, None, None, self._t(b), self._t(c), self.status)

    def p3(self, a, b, c):
        return K.ngram_eval(self.table, 3, 0, None, self._t(a), self._t(b), self._t(c), self.status)

    def p4(self, z, a, b, c):
        return K.ngram_eval(self.table, 4, 0, self._t(z), self._t(a), self._t(b), self._t(c), self.status)

    def pmi(self, order, z, a, b, c):
        if order == 2:
            return K.ngram_eval(self.table, 2, 1, None, None, self._t(b), self._t(c), self.status)
        if order == 3:
            return K.ngram_eval(self.table, 3, 1, None, self._t(a), self._t(b), self._t(c), self.status)
        return K.ngram_eval(self.table, 4, 1, self._t(z), self._t(a), self._t(b), self._t(c), self.status)

    def device_status(self) -> int:
        """Bits raised by lookups so far (DFT_DEV_*); reads the device (syncs)."""
        return int(self.status.item())
