"""Oracle: tree conv, Gated-DeltaNet tree verifier, closed-form commit.

Test infrastructure only.  numpy float32 restatement of
  * `fc1_conv.conv` (plugin tree conv + window write)  -- fc1_conv.py:8-27
  * `tree_kernels._tree_conv_kernel`                    -- tree_kernels.py:17-33
  * `tree_kernels._tree_prepare`                        -- tree_kernels.py:136-164
  * `fc1_block_inverse.invert{16,32,64}`                -- fc1_block_inverse.py:10-83
    (restated as the exact triangular inverse (I + A)^-1 they compute)
  * `tree_kernels._tree_finish` / `tree_gdn_split`      -- tree_kernels.py:167-208
  * `fc1_fused.snapshots` (plugin closed-form commit)   -- fc1_fused.py:27-49
  * `tree_kernels._closed_commit`                       -- tree_kernels.py:111-132
plus an independent per-node gated delta-rule recurrence used to cross-check
the closed forms.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32


def _f(x):
    return np.asarray(x, np.float32)


def tree_conv(x, conv_state, weight, bias, cidx):
    """fc1_conv.py:8-27 for one request.

    x [N, C] new-token inputs, conv_state [C, 3], weight [C, 4], bias [C] or
    None, cidx [N, 4] conv columns (col < 3 -> conv_state[:, col], else
    x[col - 3]).  Returns y [N, C] = SiLU(sum_j w[:, j] * val_j + bias) and
    the window taps val_1..3 as [N, C, 3] (the `intermediate_conv_window`).
    """
    x, cs, w = _f(x), _f(conv_state), _f(weight)
    N, C = x.shape
    acc = np.zeros((N, C), np.float32)
    win = np.zeros((N, C, 3), np.float32)
    for j in range(4):
        col = np.asarray(cidx)[:, j]
        val = np.where((col < 3)[:, None], cs[:, np.clip(col, 0, 2)].T, x[np.clip(col - 3, 0, N - 1)])
        acc = (acc + (val * w[:, j][None, :]).astype(np.float32)).astype(np.float32)
        if j > 0:
            win[:, :, j - 1] = val
    if bias is not None:
        acc = (acc + _f(bias)[None, :]).astype(np.float32)
    y = (acc / (F32(1) + np.exp(-acc))).astype(np.float32)
    return y, win


def gdn_prepare(y, a, b, A_log, dt_bias, anc, Hk, Hv, Dk, scale=None, neg_exp_A=None):
    """tree_kernels.py:136-164 for all v-heads: q, k (L2-normalised), G, beta, A."""
    y, a, b, anc = _f(y), _f(a), _f(b), _f(anc)
    N = y.shape[0]
    R = Hv // Hk
    KD = Hk * Dk
    scale = F32(Dk ** -0.5 if scale is None else scale)
    q = np.zeros((Hv, N, Dk), np.float32)
    k = np.zeros((Hv, N, Dk), np.float32)
    G = np.zeros((Hv, N), np.float32)
    beta = np.zeros((Hv, N), np.float32)
    A = np.zeros((Hv, N, N), np.float32)
    isanc = anc > 0.5
    offd = ~np.eye(N, dtype=bool)
    for h in range(Hv):
        hk = h // R
        qh = y[:, hk * Dk:(hk + 1) * Dk]
        kh = y[:, KD + hk * Dk:KD + (hk + 1) * Dk]
        qh = (qh * (F32(1) / np.sqrt(np.sum(qh * qh, 1, dtype=np.float32) + F32(1e-6)))[:, None] * scale).astype(np.float32)
        kh = (kh * (F32(1) / np.sqrt(np.sum(kh * kh, 1, dtype=np.float32) + F32(1e-6)))[:, None]).astype(np.float32)
        ah = a[:, h] + _f(dt_bias)[h]
        sp = np.where(ah > 20.0, ah, np.log(F32(1) + np.exp(np.minimum(ah, F32(20))))).astype(np.float32)
        dec = _f(neg_exp_A)[h] if neg_exp_A is not None else -np.exp(_f(A_log)[h])
        g = (dec * sp).astype(np.float32)
        bt = (F32(1) / (F32(1) + np.exp(-b[:, h]))).astype(np.float32)
        Gh = (anc * g[None, :]).sum(1, dtype=np.float32)
        D = np.exp(np.where(isanc, Gh[:, None] - Gh[None, :], -np.inf)).astype(np.float32)
        A[h] = np.where(isanc & offd, ((kh * bt[:, None]) @ kh.T) * D, 0.0)
        q[h], k[h], G[h], beta[h] = qh, kh, Gh, bt
    return q, k, G, beta, A


def unit_lower_inverse(A):
    """(I + A)^-1 for strictly lower-triangular A (fc1_block_inverse.py:10-83
    computes this by 16x16 forward substitution and a block merge)."""
    A = _f(A)
    N = A.shape[-1]
    X = np.zeros_like(A)
    for i in range(N):
        row = -A[..., i, :i, None] * X[..., :i, :]          # -sum_m A[i,m] X[m,:]
        X[..., i, :] = row.sum(-2, dtype=np.float32)
        X[..., i, i] = 1.0
    return X


def gdn_finish(y, pool, slot, anc, q, k, G, beta, X, Hk, Hv, Dk, Dv):
    """tree_kernels.py:167-191: U, Wk, vn = U - Wk S0, o = (q e^G) S0 + (q k^T . D) vn."""
    y, anc = _f(y), _f(anc)
    N = y.shape[0]
    KD = Hk * Dk
    o = np.zeros((N, Hv, Dv), np.float32)
    vn = np.zeros((Hv, N, Dv), np.float32)
    isanc = anc > 0.5
    for h in range(Hv):
        D = np.exp(np.where(isanc, G[h][:, None] - G[h][None, :], -np.inf)).astype(np.float32)
        eG = np.exp(G[h]).astype(np.float32)
        v = y[:, 2 * KD + h * Dv:2 * KD + (h + 1) * Dv]
        U = X[h] @ (v * beta[h][:, None])
        Wk = X[h] @ (k[h] * beta[h][:, None] * eG[:, None])
        S0 = _f(pool)[slot, h].T                            # pool is V-major [Dv, Dk]
        vn[h] = U - Wk @ S0
        Pq = (q[h] @ k[h].T) * D
        o[:, h, :] = (q[h] * eG[:, None]) @ S0 + Pq @ vn[h]
    return o, vn


def tree_gdn(y, a, b, A_log, dt_bias, pool, slot, anc, Hk, Hv, Dk, Dv, scale=None, neg_exp_A=None):
    """tree_kernels.py:193-208 (`tree_gdn_split`): returns o [N, Hv, Dv] and the
    saved aux (k [Hv, N, Dk], vn [Hv, N, Dv], G [Hv, N])."""
    q, k, G, beta, A = gdn_prepare(y, a, b, A_log, dt_bias, anc, Hk, Hv, Dk, scale, neg_exp_A)
    X = unit_lower_inverse(A)
    o, vn = gdn_finish(y, pool, slot, anc, q, k, G, beta, X, Hk, Hv, Dk, Dv)
    return o, k, vn, G


def snapshot(S0_vk, K, Vn, G, anc, path, u):
    """fc1_fused.py:27-49 for one (layer, head) and end node u.

    S0_vk [Dv, Dk] (V-major state), K [NN, Dk], Vn [NN, Dv], G [NN],
    anc [NN, NN], path [BS] node ids (-1 pad).  Returns S_u as [Dv, Dk]:
    e^{G_u} S0 + sum_{t in path, t anc-or-self of u} e^{G_u - G_t} vn_t k_t^T.
    """
    path = np.asarray(path)
    ids = np.maximum(path, 0)
    on = (path >= 0) & (np.asarray(anc)[max(u, 0), ids] > 0)
    gn = F32(G[u])
    w = np.exp(np.where(on, gn - _f(G)[ids], -np.inf)).astype(np.float32)
    kk = _f(K)[ids] * w[:, None]
    upd = kk.T @ _f(Vn)[ids]                                 # [Dk, Dv]
    return (_f(S0_vk) * np.exp(gn) + upd.T).astype(np.float32)


def closed_commit(states_kv, keys, values, gains, src, n):
    """tree_kernels.py:111-132 (in place, K-major states [L, H, DK, DV]);
    loads at most BT=16 path nodes like the reference kernel."""
    st = _f(states_kv).copy()
    L, H, DK, DV = st.shape
    src = np.asarray(src)
    n = int(n)
    u = int(src[n])
    t = np.arange(16)
    sel = t <= n
    ids = np.where(sel, src[np.minimum(t, len(src) - 1)], 0)
    for l in range(L):
        for h in range(H):
            gn = F32(gains[l, h, u])
            w = np.exp(np.where(sel, gn - _f(gains)[l, h, ids], -np.inf)).astype(np.float32)
            kk = _f(keys)[l, h, ids] * w[:, None]            # [16, DK]
            st[l, h] = st[l, h] * np.exp(gn) + kk.T @ _f(values)[l, h, ids]
    return st


def naive_recurrence(y, a, b, A_log, dt_bias, pool, slot, parent, Hk, Hv, Dk, Dv, scale=None):
    """Independent cross-check: per-node gated delta rule along each node's
    root path, S_i = e^{g_i} S_p + beta_i k_i (v_i - e^{g_i} S_p^T k_i)^T,
    o_i = S_i^T q_i.  Returns o [N, Hv, Dv] and the states S_i [Hv, N, Dk, Dv]
    (float64)."""
    y = np.asarray(y, np.float64)
    N = y.shape[0]
    R = Hv // Hk
    KD = Hk * Dk
    scale = Dk ** -0.5 if scale is None else scale
    o = np.zeros((N, Hv, Dv))
    S = np.zeros((Hv, N, Dk, Dv))
    for h in range(Hv):
        hk = h // R
        S0 = np.asarray(pool, np.float64)[slot, h].T
        for i in range(N):
            q = y[i, hk * Dk:(hk + 1) * Dk]
            k = y[i, KD + hk * Dk:KD + (hk + 1) * Dk]
            q = q / np.sqrt((q * q).sum() + 1e-6) * scale
            k = k / np.sqrt((k * k).sum() + 1e-6)
            v = y[i, 2 * KD + h * Dv:2 * KD + (h + 1) * Dv]
            ah = float(a[i, h]) + float(dt_bias[h])
            sp = ah if ah > 20 else np.log1p(np.exp(ah))
            g = -np.exp(float(A_log[h])) * sp
            bt = 1.0 / (1.0 + np.exp(-float(b[i, h])))
            Sp = S0 if parent[i] < 0 else S[h, parent[i]]
            Sd = np.exp(g) * Sp
            S[h, i] = Sd + bt * np.outer(k, v - Sd.T @ k)
            o[i, h] = S[h, i].T @ q
    return o, S
