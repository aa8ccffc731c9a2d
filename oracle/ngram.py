"""Oracle: n-gram PMI lookup and smoothing (test infrastructure only).

Restates `dforktree/ngram_gpu.py` of the reference in numpy float32:
  * table load            -- ngram_gpu.py:8-26
  * exact-match lookup    -- ngram_gpu.py:28-37 (`_index`, `_look`)
  * p2 / p3 / p4 / pmi    -- ngram_gpu.py:39-70
Every arithmetic step keeps the reference's order of float32 operations
(separate multiply and add, IEEE division), so the only differences to the
reference are the last-ulp differences of `log` between libraries.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32


class NGramOracle:
    """numpy restatement of `NGramGPU` (ngram_gpu.py:6-70)."""

    def __init__(self, z, beta2=20.0, beta3=20.0, beta4=20.0, clip=10.0):
        # ngram_gpu.py:9-25
        f = set(z.keys()) if isinstance(z, dict) else set(z.files)
        A = lambda x, dt: np.ascontiguousarray(np.asarray(x).astype(dt))
        self.V = int(z["V"])
        N = float(z["N"])
        self.k2, self.c2 = A(z["keys"], np.int64), A(z["cab"], np.float32)
        self.prev = A(z["prev"], np.float32)
        # pn computed in float64 then cast (ngram_gpu.py:16)
        self.pn = A((np.asarray(z["nxt"]).astype(np.float64) + 1.0) / (N + self.V), np.float32)
        e = lambda dt: np.zeros(0, dt)
        self.k3 = A(z["keys3"], np.int64) if "keys3" in f else e(np.int64)
        self.c3 = A(z["c3"], np.float32) if "keys3" in f else e(np.float32)
        self.k3c = A(z["keys3c"], np.int64) if "keys3c" in f else e(np.int64)
        self.n3c = A(z["n3c"], np.float32) if "keys3c" in f else e(np.float32)
        self.has4 = "keys4" in f
        self.k4 = A(z["keys4"], np.int64) if self.has4 else e(np.int64)
        self.c4 = A(z["c4"], np.float32) if self.has4 else e(np.float32)
        self.n4c = A(z["n4c"], np.float32) if self.has4 else np.zeros(max(len(self.k3), 1), np.float32)
        self.beta2, self.beta3, self.beta4, self.clip = F32(beta2), F32(beta3), F32(beta4), F32(clip)

    @staticmethod
    def _index(keys, q):
        # ngram_gpu.py:28-33: searchsorted + equality test, miss -> -1
        q = np.asarray(q, np.int64)
        if keys.shape[0] == 0:
            return np.full_like(q, -1)
        idx = np.minimum(np.searchsorted(keys, q.reshape(-1)), keys.shape[0] - 1).reshape(q.shape)
        return np.where(keys[idx] == q, idx, -1)

    def _look(self, keys, vals, q):
        # ngram_gpu.py:35-37
        i = self._index(keys, q)
        if vals.shape[0] == 0:
            return np.zeros(np.shape(q), np.float32)
        return np.where(i >= 0, vals[np.maximum(i, 0)], F32(0)).astype(np.float32)

    def _pn(self, c):
        # torch indexing wraps negative indices; mirror that for pn[c]
        c = np.asarray(c, np.int64)
        return self.pn[np.where(c < 0, c + self.V, c)]

    def p2(self, b, c):
        # ngram_gpu.py:39-42
        b = np.asarray(b, np.int64)
        c = np.asarray(c, np.int64)
        n = self._look(self.k2, self.c2, b * self.V + c)
        nb = np.where(b >= 0, self.prev[np.maximum(b, 0)], F32(0)).astype(np.float32)
        return ((n + self.beta2 * self._pn(c)) / (nb + self.beta2)).astype(np.float32)

    def p3(self, a, b, c):
        # ngram_gpu.py:44-51
        V = self.V
        a = np.asarray(a, np.int64)
        b = np.asarray(b, np.int64)
        c = np.asarray(c, np.int64)
        ok = (a >= 0) & (b >= 0)
        q = np.where(ok, a * V + b, -1)
        nab = self._look(self.k3c, self.n3c, q)
        q3 = np.where(ok, (a * V + b) * V + c, -1)
        nabc = self._look(self.k3, self.c3, q3)
        return ((nabc + self.beta3 * self.p2(b, c)) / (nab + self.beta3)).astype(np.float32)

    def p4(self, z, a, b, c):
        # ngram_gpu.py:53-61
        V = self.V
        z = np.asarray(z, np.int64)
        a = np.asarray(a, np.int64)
        b = np.asarray(b, np.int64)
        c = np.asarray(c, np.int64)
        ok = (z >= 0) & (a >= 0) & (b >= 0)
        q = np.where(ok, (z * V + a) * V + b, -1)
        i3 = self._index(self.k3, q)
        n4 = np.where(i3 >= 0, self.n4c[np.maximum(i3, 0)], F32(0)).astype(np.float32)
        q4 = np.where(i3 >= 0, i3 * V + c, -1)
        n4c_ = self._look(self.k4, self.c4, q4)
        return ((n4c_ + self.beta4 * self.p3(a, b, c)) / (n4 + self.beta4)).astype(np.float32)

    def pmi(self, order, z, a, b, c):
        # ngram_gpu.py:63-70
        if order == 2:
            p = self.p2(b, c)
        elif order == 3:
            p = self.p3(a, b, c)
        else:
            p = self.p4(z, a, b, c)
        return np.clip(np.log(p) - np.log(self._pn(c)), -self.clip, self.clip).astype(np.float32)
