"""Oracle: tree-masked attention verify -- TEST INFRASTRUCTURE ONLY.

numpy float32 restatement of what the plugin asks of the gated full-attention
layers during tree verification:
  * the mask, `fc1_branch64.py:39`:
        mask = cat(ones(n, prefix_len), anc.bool()), one row per tree node
  * the plan, `fc1_plan.py:16-33`: one request, qo_indptr = [0, n],
    kv_indptr = [0, prefix_len + n], page size 1, the mask bit-packed
    little-endian row-major (`flashinfer.packbits(mask.flatten(), 'little')`)
  * the attention it plans, flashinfer's paged prefill with a custom mask
    (third-party: flashinfer, the version SGLang 0.5.22 pins; not under the
    reference tree).  Its published algorithm, restated here:
        o[i, hq] = sum_j softmax_j(q[i, hq] . k[j, hq // G] * sm_scale,
                                   masked where mask[i, j] is false) v[j, hq // G]
    with G = num_qo_heads / num_kv_heads and sm_scale = head_dim ** -0.5 by
    default; keys are the KV-cache rows kv_indices[kv_indptr[b]:kv_indptr[b+1]],
    the request's prefix first and its n tree tokens last, in node order.
Parity is pinned by the call sites above (no reference test or golden vector
covers this path; the GPU tests compare against this restatement).
"""
from __future__ import annotations

import numpy as np


def _f(x):
    return np.asarray(x, np.float32)


def tree_mask(anc, prefix_len):
    """fc1_branch64.py:39: [n, prefix_len + n] boolean mask of one request."""
    anc = np.asarray(anc) > 0.5
    n = anc.shape[0]
    return np.concatenate([np.ones((n, prefix_len), bool), anc], 1)


def tree_attention(q, k_cache, v_cache, kv_indptr, kv_indices, anc, sm_scale=None):
    """q [B, N, Hq, D]; k_cache / v_cache [slots, Hkv, D]; kv_indptr [B + 1];
    anc [B, N, N].  Returns o [B, N, Hq, D] float32 (fp32 arithmetic on the
    given values; pass bf16-rounded inputs to model a bf16 run)."""
    q, kc, vc = _f(q), _f(k_cache), _f(v_cache)
    B, N, Hq, D = q.shape
    Hkv = kc.shape[1]
    G = Hq // Hkv
    scale = np.float32(D ** -0.5 if sm_scale is None else sm_scale)
    ptr = np.asarray(kv_indptr, np.int64)
    idx_all = np.asarray(kv_indices, np.int64)
    out = np.zeros((B, N, Hq, D), np.float32)
    for b in range(B):
        idx = idx_all[ptr[b]:ptr[b + 1]]
        L = idx.shape[0]
        mask = tree_mask(np.asarray(anc)[b], L - N)              # [N, L]
        for h in range(Hkv):
            K = kc[idx, h]                                       # [L, D]
            V = vc[idx, h]
            Qg = q[b, :, h * G:(h + 1) * G].reshape(N * G, D)    # rows node-major
            s = (Qg @ K.T) * scale                               # [N*G, L]
            s = np.where(np.repeat(mask, G, 0), s, -np.inf)
            s = s - s.max(1, keepdims=True)
            p = np.exp(s)
            p /= p.sum(1, keepdims=True)
            out[b, :, h * G:(h + 1) * G] = (p @ V).reshape(N, G, D)
    return out
