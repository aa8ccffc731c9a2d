"""Seeded input generators for the golden cases.

`make_golden.py` feeds these inputs to the reference code and stores the
outputs (plus an input checksum) under `tests/golden/*.npz`; the tests rebuild
the same inputs from the same seeds, so large inputs need not be committed.
numpy's PCG64 streams are identical on every machine.
"""
from __future__ import annotations

import numpy as np

from dforktree_b200 import synth

# ---------------------------------------------------------------- n-gram ----
NGRAM_CASE = dict(V=300, n_bigram=6000, n_trigram=12000, n_quad=3000, seed=11)


def ngram_table():
    c = NGRAM_CASE
    return synth.make_ngram_table(c["V"], c["n_bigram"], c["n_trigram"], seed=c["seed"], n_quad=c["n_quad"])


def ngram_queries(V: int, n: int = 6000, seed: int = 12):
    """Random (z, a, b, c) with some invalid (-1) context ids and some c = -1
    (torch wraps pn[-1]; the key arithmetic aliases, both mirrored)."""
    rng = np.random.default_rng(seed)
    z = synth.zipf_ids(rng, n, V)
    a = synth.zipf_ids(rng, n, V)
    b = synth.zipf_ids(rng, n, V)
    c = synth.zipf_ids(rng, n, V)
    for arr, frac in ((z, 0.05), (a, 0.05), (b, 0.05), (c, 0.01)):
        arr[rng.random(n) < frac] = -1
    return z, a, b, c


# --------------------------------------------------------------- builder ----
# (name, V, S, N, table sizes, chain_first, use_ngram, seed)
BUILDER_CASES = [
    dict(name="b_v2048_s24_n32", V=2048, S=24, N=32, nb=60000, nt=200000, chain_first=False, ngram=True, seed=100),
    dict(name="b_v2048_s24_n32_s2", V=2048, S=24, N=32, nb=60000, nt=200000, chain_first=False, ngram=True, seed=101),
    dict(name="b_v2048_s23_n32_s3", V=2048, S=23, N=32, nb=60000, nt=200000, chain_first=False, ngram=True, seed=102),
    dict(name="b_v1024_s24_n16", V=1024, S=24, N=16, nb=40000, nt=150000, chain_first=False, ngram=True, seed=103),
    dict(name="b_v1024_s12_n64", V=1024, S=12, N=64, nb=40000, nt=150000, chain_first=False, ngram=True, seed=104),
    dict(name="b_v2048_s24_n32_chain", V=2048, S=24, N=32, nb=60000, nt=200000, chain_first=True, ngram=True, seed=105),
    dict(name="b_v2048_s24_n32_nongram", V=2048, S=24, N=32, nb=60000, nt=200000, chain_first=False, ngram=False, seed=106),
]

# The closure at n-gram orders 2 and 4 (tree_ops.ngram_path_fn's `order`,
# tree_ops.py:59-64; the Builder itself uses 3).  Order-4 tables carry
# quadgram rows; small V keeps the trees' contexts inside the tables.
ORDER_CASES = [
    dict(name="o2_v1024_s16_n32", order=2, V=1024, S=16, N=32, nb=40000, nt=150000, nq=0, chain_first=False,
         seed=200),
    dict(name="o4_v256_s10_n32", order=4, V=256, S=10, N=32, nb=20000, nt=120000, nq=400000, chain_first=False,
         seed=201),
    dict(name="o4_v512_s8_n64_chain", order=4, V=512, S=8, N=64, nb=30000, nt=150000, nq=300000, chain_first=True,
         seed=202),
]
ORDER_T_SAMPLE = 20000    # T entries kept per fixture (a seeded sample of the full tensor)


def order_inputs(case: dict):
    rng = np.random.default_rng(case["seed"])
    V, S = case["V"], case["S"]
    table = synth.make_ngram_table(V, case["nb"], case["nt"], seed=case["seed"] + 7, n_quad=case["nq"])
    logits = synth.make_logits(S, V, seed=case["seed"] + 13)
    hot = synth.zipf_ids(rng, S * 8, V).reshape(S, 8)
    logits[np.arange(S)[:, None], hot] += np.float32(9.0)
    root = int(synth.zipf_ids(rng, 1, V)[0])
    pre1 = int(synth.zipf_ids(rng, 1, V)[0])
    return table, logits, root, pre1


def order_t_sample(shape, seed: int = 5):
    """Flat indices of the T entries a fixture keeps (sorted, distinct)."""
    n = int(np.prod(shape))
    k = min(ORDER_T_SAMPLE, n)
    return np.sort(np.random.default_rng(seed).choice(n, k, replace=False))


# Full config-0 vocabulary (V = 248,320, 2M bigram + 8M trigram keys).
CONFIG0 = dict(V=248320, nb=2_000_000, nt=8_000_000, table_seed=0, S=24, N=32)
CONFIG0_SEEDS = [0, 1]


def builder_inputs(case: dict):
    rng = np.random.default_rng(case["seed"])
    V, S = case["V"], case["S"]
    table = synth.make_ngram_table(V, case["nb"], case["nt"], seed=case["seed"] + 7)
    logits = synth.make_logits(S, V, seed=case["seed"] + 13)
    # make a fraction of candidates hit the table: boost some table-frequent tokens
    hot = synth.zipf_ids(rng, S * 8, V).reshape(S, 8)
    logits[np.arange(S)[:, None], hot] += np.float32(9.0)
    root = int(synth.zipf_ids(rng, 1, V)[0])
    pre1 = int(synth.zipf_ids(rng, 1, V)[0])
    return table, logits, root, pre1


def config0_inputs(seed: int, table=None):
    c = CONFIG0
    if table is None:
        table = synth.make_ngram_table(c["V"], c["nb"], c["nt"], seed=c["table_seed"])
    logits = synth.make_logits(c["S"], c["V"], seed=1000 + seed)
    rng = np.random.default_rng(2000 + seed)
    root = int(synth.zipf_ids(rng, 1, c["V"])[0])
    pre1 = int(synth.zipf_ids(rng, 1, c["V"])[0])
    return table, logits, root, pre1


# ------------------------------------------------------------------- GDN ----
GDN_CASES = [
    dict(name="g_n32_hk2_hv4", N=32, Hk=2, Hv=4, D=128, slots=3, slot=1, seed=200),
    dict(name="g_n16_hk2_hv4", N=16, Hk=2, Hv=4, D=128, slots=2, slot=0, seed=201),
    dict(name="g_n64_hk1_hv2", N=64, Hk=1, Hv=2, D=128, slots=2, slot=1, seed=202),
    dict(name="g_n32_hk2_hv2_r1", N=32, Hk=2, Hv=2, D=128, slots=1, slot=0, seed=203),
    dict(name="g_n32_deep", N=32, Hk=2, Hv=4, D=128, slots=2, slot=1, seed=204, chain_p=0.85),
]


def gdn_inputs(case: dict):
    d = synth.make_gdn_inputs(case["N"], case["Hk"], case["Hv"], case["D"], seed=case["seed"],
                              slots=case["slots"], chain_p=case.get("chain_p", 0.0))
    rng = np.random.default_rng(case["seed"] + 1)
    # non-trivial decay parameters so A_log / dt_bias paths are exercised
    d["A_log"] = (rng.standard_normal(case["Hv"]) * 0.5).astype(np.float32)
    d["dt_bias"] = (rng.standard_normal(case["Hv"]) * 0.5).astype(np.float32)
    return d


CONV_CASES = [
    dict(name="c_n32_c1024", N=32, C=1024, slots=3, slot=2, dst_slots=2, dst=1, seed=300),
    dict(name="c_n16_c640", N=16, C=640, slots=1, slot=0, dst_slots=1, dst=0, seed=301),
]


def conv_inputs(case: dict):
    rng = np.random.default_rng(case["seed"])
    N, C = case["N"], case["C"]
    parent = synth.random_tree_parents(N, rng)
    x = rng.standard_normal((N, C)).astype(np.float32)
    conv_state = rng.standard_normal((case["slots"], C, 3)).astype(np.float32)
    weight = (rng.standard_normal((C, 4)) * 0.5).astype(np.float32)
    bias = (rng.standard_normal(C) * 0.1).astype(np.float32)
    return parent, x, conv_state, weight, bias


# ---------------------------------------------------------------- commit ----
# snapshots (fc1_fused.py:27-49) hard-codes 32 heads x 128 x 128.
COMMIT_CASES = [
    dict(name="s_l2_nn32", L=2, NN=32, BS=24, slots=2, slot=1, seed=400),
    dict(name="s_l1_nn64", L=1, NN=64, BS=24, slots=1, slot=0, seed=401),
    dict(name="s_l1_nn32_deep", L=1, NN=32, BS=24, slots=2, slot=0, seed=402, chain_p=0.9),
]
COMMIT_HEADS_STORED = 4


def commit_inputs(case: dict):
    rng = np.random.default_rng(case["seed"])
    L, NN, BS = case["L"], case["NN"], case["BS"]
    parent = synth.random_tree_parents(NN, rng, chain_p=case.get("chain_p", 0.0))
    anc = synth.ancestors_from_parents(parent)
    path = synth.random_root_to_leaf_path(parent, rng)
    state = (rng.standard_normal((L, case["slots"], 32, 128, 128), dtype=np.float32) * np.float32(0.02))
    K = rng.standard_normal((L, 32, NN, 128), dtype=np.float32)
    K /= np.linalg.norm(K, axis=-1, keepdims=True)
    Vn = rng.standard_normal((L, 32, NN, 128), dtype=np.float32)
    G = -np.cumsum(np.abs(rng.standard_normal((L, 32, NN), dtype=np.float32)) * np.float32(0.1), -1).astype(np.float32)
    path_pad = np.full(BS, -1, np.int64)
    path_pad[:min(len(path), BS)] = path[:BS]
    last = int(path[min(len(path), BS) - 1])
    # the second end (Mamba track node): an ancestor on the path, or -1
    track = int(path[len(path) // 2]) if len(path) > 2 else -1
    return dict(parent=parent, anc=anc, path=path_pad, ends=np.array([last, track], np.int64),
                state=state, K=K.astype(np.float32), Vn=Vn, G=G)


def checksum(*arrays) -> np.ndarray:
    """float64 sums of each array (detects generator drift)."""
    return np.array([float(np.asarray(a, np.float64).sum()) for a in arrays], np.float64)


# ------------------------------------------------------ tree attention ------
# flashinfer's paged prefill (fa2, page size 1) with the plugin's custom mask
# (fc1_branch64.py:39), one request per plan as fc1_plan.py:16-33 plans it.
# Grouped-query ratios 1/2/4/8, ragged prefixes, trees of 16 and 32 nodes.
ATTN_CASES = [
    dict(name="attn_g4_n32", Hq=16, Hkv=4, N=32, prefixes=[700, 45], seed=400),
    dict(name="attn_g2_n32", Hq=8, Hkv=4, N=32, prefixes=[128, 1000, 7], seed=401),
    dict(name="attn_g1_n16", Hq=4, Hkv=4, N=16, prefixes=[300], seed=402),
    dict(name="attn_g8_n16", Hq=16, Hkv=2, N=16, prefixes=[513, 64], seed=403),
]
ATTN_D = 256


def _bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 to the nearest bfloat16 (ties to even), kept as float32."""
    u = np.ascontiguousarray(x, np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000
    return u.astype(np.uint32).view(np.float32)


def attn_inputs(case):
    """q [B, N, Hq, D]; k / v caches [slots, Hkv, D] (bf16 values as float32);
    request b's keys are kv_indices[kv_indptr[b]:kv_indptr[b+1]] in shuffled
    slots, its prefix first and its N tree nodes last; anc [B, N, N] of random
    trees (config-2 topology)."""
    rng = np.random.default_rng(case["seed"])
    N, Hq, Hkv, D = case["N"], case["Hq"], case["Hkv"], ATTN_D
    lens = [p + N for p in case["prefixes"]]
    B, total = len(lens), sum(lens)
    slots = total + 13
    kv_indices = rng.permutation(slots)[:total].astype(np.int32)
    kv_indptr = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    anc = np.stack([synth.ancestors_from_parents(synth.random_tree_parents(N, rng)) for _ in range(B)])
    q = _bf16(rng.standard_normal((B, N, Hq, D), dtype=np.float32))
    k = _bf16(rng.standard_normal((slots, Hkv, D), dtype=np.float32))
    v = _bf16(rng.standard_normal((slots, Hkv, D), dtype=np.float32))
    return dict(q=q, k=k, v=v, kv_indptr=kv_indptr, kv_indices=kv_indices, anc=anc)
