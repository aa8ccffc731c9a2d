"""Seeded synthetic inputs for the draft-tree cycle.

The reference's real n-gram table (`ngram_counts.npz`) and drafter are not
available, so every benchmark and parity case runs on seeded synthetic data
with the shapes and value distributions the benchmark configs name:

* n-gram table in the reference npz schema (`ngram_gpu.py:8-26`): sorted int64
  keys `b*V+c` / `(a*V+b)*V+c`, float counts, `prev`/`nxt` marginals, total
  `N`, trigram contexts `keys3c`/`n3c`, optional order-4 `keys4`/`c4`/`n4c`.
  Token ids follow a discrete power law with exponent s=1.1 (inverse-CDF
  sampling, k = floor(U^(-1/(s-1))), the continuous approximation of Zipf(s)),
  folded into [0, V).  Counts are Zipf-distributed integers clipped to
  [1, 1e5].
* drafter logits 3*N(0,1) with one peaked token (+6) per position.
* GDN tree inputs (config 2): random topology, L2-normalised q/k, N(0,1) v,
  gates from N(0,1) raw inputs, state N(0, 0.02).

Pure numpy; deterministic for a given seed on any machine.
"""
from __future__ import annotations

import numpy as np

__all__ = [
    "zipf_ids", "make_ngram_table", "make_logits", "random_tree_parents",
    "make_gdn_inputs", "random_root_to_leaf_path",
]


def zipf_ids(rng: np.random.Generator, n: int, V: int, s: float = 1.1) -> np.ndarray:
    """Power-law token ids in [0, V): k = floor(U^(-1/(s-1))), folded mod V."""
    u = 1.0 - rng.random(n)
    k = np.floor(u ** (-1.0 / (s - 1.0)))
    return np.fmod(k - 1.0, float(V)).astype(np.int64)


def _sorted_unique(x: np.ndarray) -> np.ndarray:
    x = np.sort(x)
    if x.size == 0:
        return x
    keep = np.empty(x.size, dtype=bool)
    keep[0] = True
    np.not_equal(x[1:], x[:-1], out=keep[1:])
    return x[keep]


def _distinct_keys(rng, target: int, draw) -> np.ndarray:
    """Exactly `target` distinct keys (sorted) from the sampler `draw(n)`."""
    keys = np.zeros(0, np.int64)
    need = target
    for _ in range(64):
        keys = _sorted_unique(np.concatenate([keys, draw(int(need * 1.3) + 16)]))
        if keys.size >= target:
            break
        need = target - keys.size
    if keys.size < target:
        raise ValueError(f"could not draw {target} distinct keys (got {keys.size})")
    if keys.size > target:
        pick = np.sort(rng.permutation(keys.size)[:target])
        keys = keys[pick]
    return keys


def _zipf_counts(rng, n: int, s: float = 1.1, cmax: float = 1e5) -> np.ndarray:
    u = 1.0 - rng.random(n)
    k = np.floor(u ** (-1.0 / (s - 1.0)))
    return np.clip(k, 1.0, cmax).astype(np.int32)


def make_ngram_table(V: int, n_bigram: int, n_trigram: int, seed: int = 0,
                     s: float = 1.1, cmax: float = 1e5, n_quad: int = 0) -> dict:
    """Synthetic n-gram table in the reference's npz schema.

    Returns a dict with the keys `NGramGPU.__init__` reads
    (`ngram_gpu.py:9-25`): V, N, keys, cab, prev, nxt, keys3, c3, keys3c,
    n3c and, when n_quad > 0, keys4, c4, n4c.
    """
    rng = np.random.default_rng(seed)
    if n_bigram > V * V or n_trigram > V ** 3:
        raise ValueError("more distinct n-grams requested than exist")
    k2 = _distinct_keys(rng, n_bigram, lambda n: zipf_ids(rng, n, V, s) * V + zipf_ids(rng, n, V, s))
    c2 = _zipf_counts(rng, n_bigram, s, cmax)
    b2, c2i = k2 // V, k2 % V
    prev = np.bincount(b2, weights=c2, minlength=V).astype(np.int64)
    nxt = np.bincount(c2i, weights=c2, minlength=V).astype(np.int64)
    out = dict(V=np.int64(V), N=np.int64(int(c2.sum())), keys=k2, cab=c2, prev=prev, nxt=nxt)
    if n_trigram:
        k3 = _distinct_keys(
            rng, n_trigram,
            lambda n: (zipf_ids(rng, n, V, s) * V + zipf_ids(rng, n, V, s)) * V + zipf_ids(rng, n, V, s))
        c3 = _zipf_counts(rng, n_trigram, s, cmax)
        ctx = k3 // V
        keys3c = _sorted_unique(ctx)
        n3c = np.zeros(keys3c.size, np.int64)
        np.add.at(n3c, np.searchsorted(keys3c, ctx), c3)
        out.update(keys3=k3, c3=c3, keys3c=keys3c, n3c=n3c)
        if n_quad:
            # order-4 rows: key = i3*V + c where i3 indexes the context trigram in keys3
            k4 = _distinct_keys(rng, n_quad, lambda n: rng.integers(0, k3.size, n) * V + zipf_ids(rng, n, V, s))
            c4 = _zipf_counts(rng, n_quad, s, cmax)
            n4c = np.zeros(k3.size, np.int64)
            np.add.at(n4c, k4 // V, c4)
            out.update(keys4=k4, c4=c4, n4c=n4c)
    return out


def make_logits(S: int, V: int, seed: int, peak: float = 6.0, sigma: float = 3.0,
                s: float = 1.1) -> np.ndarray:
    """Drafter logits [S, V] float32: sigma*N(0,1), +peak on one token per position.

    The peaked token is drawn from the same power law as the table's ids so
    that drafted paths meet the n-gram table.
    """
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((S, V), dtype=np.float32) * np.float32(sigma))
    pk = zipf_ids(rng, S, V, s)
    x[np.arange(S), pk] += np.float32(peak)
    return x


def random_tree_parents(N: int, rng: np.random.Generator, max_depth: int = 24,
                        chain_p: float = 0.0) -> np.ndarray:
    """Parent array (root = -1): each node's parent uniform over earlier nodes,
    redrawn while the depth bound would be exceeded (config 2).  With
    chain_p > 0 a node extends the previous node with that probability, which
    gives deep, chain-like trees."""
    parent = np.full(N, -1, np.int64)
    depth = np.zeros(N, np.int64)
    for n in range(1, N):
        while True:
            p = n - 1 if (chain_p > 0 and rng.random() < chain_p) else int(rng.integers(0, n))
            if depth[p] + 1 <= max_depth:
                break
        parent[n] = p
        depth[n] = depth[p] + 1
    return parent


def ancestors_from_parents(parent: np.ndarray) -> np.ndarray:
    """Anc[i, j] = 1 when j is i or an ancestor of i (float32)."""
    N = parent.shape[0]
    anc = np.zeros((N, N), np.float32)
    for i in range(N):
        j = i
        while j >= 0:
            anc[i, j] = 1.0
            j = int(parent[j])
    return anc


def random_root_to_leaf_path(parent: np.ndarray, rng: np.random.Generator) -> np.ndarray:
    """A random root-to-leaf node path (root first)."""
    N = parent.shape[0]
    has_child = np.zeros(N, bool)
    has_child[parent[1:]] = True
    leaves = np.nonzero(~has_child)[0]
    u = int(rng.choice(leaves))
    path = []
    while u >= 0:
        path.append(u)
        u = int(parent[u])
    return np.array(path[::-1], np.int64)


def make_gdn_inputs(N: int, Hk: int, Hv: int, D: int, seed: int, slots: int = 1,
                    max_depth: int = 24, dtype=np.float32, chain_p: float = 0.0) -> dict:
    """Config-2 single-layer tree-verify inputs (batch 1).

    y = [q | k | v] per node with q,k L2-normalised rows and v ~ N(0,1);
    gates realised through the reference API as a ~ N(0,1), A_log = 0,
    dt_bias = 0 (so g = -softplus(a)) and b ~ N(0,1) (beta = sigmoid(b));
    state pool [slots, Hv, Dv, Dk] float32 ~ N(0, 0.02).
    """
    rng = np.random.default_rng(seed)
    parent = random_tree_parents(N, rng, max_depth, chain_p)
    q = rng.standard_normal((N, Hk, D)).astype(np.float32)
    k = rng.standard_normal((N, Hk, D)).astype(np.float32)
    q /= np.linalg.norm(q, axis=-1, keepdims=True)
    k /= np.linalg.norm(k, axis=-1, keepdims=True)
    v = rng.standard_normal((N, Hv, D)).astype(np.float32)
    y = np.concatenate([q.reshape(N, -1), k.reshape(N, -1), v.reshape(N, -1)], 1).astype(dtype)
    a = rng.standard_normal((N, Hv)).astype(np.float32)
    b = rng.standard_normal((N, Hv)).astype(np.float32)
    pool = (rng.standard_normal((slots, Hv, D, D)) * 0.02).astype(np.float32)
    return dict(parent=parent, anc=ancestors_from_parents(parent), y=y, a=a, b=b,
                A_log=np.zeros(Hv, np.float32), dt_bias=np.zeros(Hv, np.float32),
                pool=pool, path=random_root_to_leaf_path(parent, rng))
