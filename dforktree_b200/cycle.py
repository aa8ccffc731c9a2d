"""Batched draft-tree cycle on one GPU: score -> build -> (tree conv + GDN
verify) per GDN layer, tree-masked attention per gated full-attention layer
(in the model's layer order) -> greedy acceptance -> closed-form commit.

This is the B200-native form of what the plugin does per decode step for one
request (fc1_branch64.verify_branch: Builder at :25, the patched conv and
target_verify per layer inside run_eagle_verify at :44, fused_commit after
acceptance), for B requests at once and without the target model's
projections / attention (those stay in the serving stack).

State layout in HBM (one GPU holds whole requests; requests shard across GPUs):
  pool      [L, B, Hv, Dv, Dk] fp32   recurrent state, V-major like SGLang's pool
  conv_state[L, B, C, 3]             conv window (C = 2*Hk*Dk + Hv*Dv)
  aux_k     [L, B, Hk, N, Dk] fp32    normalised keys saved by verify (per k-head)
  aux_vn    [L, B, Hv, N, Dv] fp32    delta-rule values saved by verify
  aux_g     [L, B, Hv, N]     fp32    ancestor-cumulative gates
  k_cache / v_cache [La, slots, Hkv, Da] bf16   per attention layer, page size 1:
            request b's keys are slots kv_indices[kv_indptr[b]:kv_indptr[b+1]],
            its prefix first and its N tree tokens last
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from . import kernels as K


@dataclass
class CycleConfig:
    B: int = 64           # requests per GPU
    S: int = 24           # drafter positions
    V: int = 248320       # vocabulary
    N: int = 32           # tree nodes incl. root
    layers: int = 24      # GDN layers (Qwen3.5-9B: 24 of 32)
    Hk: int = 16
    Hv: int = 32
    D: int = 128
    P: int = 24           # longest accepted path kept (draft block)
    lam_a: float = 0.3
    lam_p: float = 0.6
    chain_first: bool = False   # FC1_CHAIN_FIRST (fc1_builder.py:12): top-1 chain first
    # gated full-attention layers (Qwen3.5: every 4th layer; 0 = GDN layers only)
    attn_layers: int = 0
    Hq: int = 16
    Hkv: int = 4
    Da: int = 256
    prefix: int = 4096    # prior context per request in the KV cache

    @property
    def layer_kinds(self):
        """'gdn' / 'attn' per model layer in order: three GDN layers, then one
        attention layer, repeated (attention layers beyond that pattern last)."""
        kinds, g, a = [], 0, 0
        while g < self.layers or a < self.attn_layers:
            if a < self.attn_layers and (g == self.layers or (len(kinds) + 1) % 4 == 0):
                kinds.append("attn")
                a += 1
            else:
                kinds.append("gdn")
                g += 1
        return kinds

    @property
    def C(self):
        return 2 * self.Hk * self.D + self.Hv * self.D


class DraftTreeCycle:
    """Static buffers for one GPU's batch; `step()` launches one cycle on the
    current stream without synchronising."""

    def __init__(self, cfg: CycleConfig, table: K.Table, device, act_dtype=torch.bfloat16, seed: int = 0):
        self.cfg = c = cfg
        self.table = table
        dev = torch.device(device)
        self.device = dev
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        Ls, B, N, D = c.layers, c.B, c.N, c.D
        # per-layer parameters (random init of the GDN layer shape)
        self.conv_w = (torch.randn(Ls, c.C, 4, device=dev, generator=g) * 0.5).to(act_dtype)
        self.A_log = (torch.randn(Ls, c.Hv, device=dev, generator=g) * 0.5).float()
        self.neg_exp_A = -self.A_log.exp()
        self.dt_bias = (torch.randn(Ls, c.Hv, device=dev, generator=g) * 0.5).float()
        # request state
        self.conv_state = torch.randn(Ls, B, c.C, 3, device=dev, generator=g).to(act_dtype)
        self.pool = torch.randn(Ls, B, c.Hv, D, D, device=dev, generator=g) * 0.02
        self.aux_k = torch.zeros(Ls, B, c.Hk, N, D, device=dev)
        self.aux_vn = torch.zeros(Ls, B, c.Hv, N, D, device=dev)
        self.aux_g = torch.zeros(Ls, B, c.Hv, N, device=dev)
        # per-cycle buffers
        self.ws = K.score_build_workspace(B, c.S, c.V, N, use_ngram=True, device=dev)
        self.tree = K.tree_outputs(B, c.S, N, dev, extras=False)
        self.y = torch.empty(B, N, c.C, dtype=act_dtype, device=dev)
        self.o = torch.empty(B, N, c.Hv, D, dtype=act_dtype, device=dev)
        self.path = torch.empty(B, c.P, dtype=torch.int64, device=dev)
        self.accept_len = torch.empty(B, dtype=torch.int64, device=dev)
        self.last = torch.empty(B, dtype=torch.int64, device=dev)
        self.bonus = torch.empty(B, dtype=torch.int64, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        # commit writes S_u back into each request's own slot (node stride 0)
        p = self.pool
        self.pool_out = torch.as_strided(p, (Ls, B, 1, c.Hv, D, D),
                                         (p.stride(0), p.stride(1), 0, p.stride(2), p.stride(3), p.stride(4)))
        self.launches_per_step = 3 + Ls + 1 + 1 + 1
        if c.attn_layers:
            self._init_attention(g)

    def _init_attention(self, g):
        """KV caches of the attention layers (random prefix + tree keys in
        shuffled page-size-1 slots) and the plan, made once: the plan reads the
        tree's ancestor matrix from its buffer at every run."""
        from .tree_attn import TreeAttentionWrapper
        c, dev = self.cfg, self.device
        keys = c.prefix + c.N
        slots = c.B * keys
        self.kv_indices = torch.randperm(slots, device=dev, generator=g).to(torch.int32)
        self.kv_indptr = (torch.arange(c.B + 1, device=dev) * keys).to(torch.int32)
        self.k_cache = torch.empty(c.attn_layers, slots, c.Hkv, c.Da, dtype=torch.bfloat16, device=dev)
        self.v_cache = torch.empty_like(self.k_cache)
        for j in range(c.attn_layers):
            self.k_cache[j] = torch.randn(slots, c.Hkv, c.Da, device=dev, generator=g)
            self.v_cache[j] = torch.randn(slots, c.Hkv, c.Da, device=dev, generator=g)
        self.attn = TreeAttentionWrapper(dev).plan(self.kv_indptr, self.kv_indices, c.Hq, c.Hkv, c.Da, n=c.N,
                                                   anc=self.tree["anc"], kv_lens_host=[keys] * c.B)
        self.attn.status = self.status
        self.o_attn = torch.empty(c.B, c.N, c.Hq, c.Da, dtype=torch.bfloat16, device=dev)
        self.launches_per_step += c.attn_layers * 2

    # -- stages --------------------------------------------------------------
    def build(self, logits, root, pre1):
        c = self.cfg
        K.score_build(self.table, logits, root, pre1, c.N, self.ws, self.tree, chain_first=c.chain_first,
                      lam_a=c.lam_a, lam_p=c.lam_p, status=self.status)

    def attend_layer(self, j, q):
        """Tree-masked attention verify of attention layer j: q [B, N, Hq, Da]
        against the request's prefix and its tree keys (mask of
        fc1_branch64.py:39); output in self.o_attn."""
        return self.attn.run(q, (self.k_cache[j], self.v_cache[j]), out=self.o_attn)

    def verify_layer(self, l, x, a, b):
        """Tree conv fused into the GDN tree verify of layer l (one launch).
        From layer 1 on the launch overlaps the previous layer's verify (which
        writes none of this layer's states, conv state, weights or tree); layer
        0 follows the tree build."""
        c = self.cfg
        conv = dict(x=x, conv_state=self.conv_state[l], weight=self.conv_w[l], cidx=self.tree["cidx"])
        K.gdn_tree_verify(None, a, b, None, self.dt_bias[l], self.tree["anc"], self.pool[l], c.Hk, c.Hv, c.D, c.D,
                          neg_exp_A=self.neg_exp_A[l], o=self.o, aux_k=self.aux_k[l], aux_vn=self.aux_vn[l],
                          aux_g=self.aux_g[l], aux_k_per_v=False, status=self.status, conv=conv,
                          overlap_prev=l > 0)

    def verify_layer_unfused(self, l, x, a, b):
        """Separate tree conv launch, then the verify (the plugin's hook order)."""
        c = self.cfg
        K.tree_conv(x, self.conv_state[l], self.conv_w[l], None, self.tree["cidx"], y=self.y, status=self.status)
        K.gdn_tree_verify(self.y, a, b, None, self.dt_bias[l], self.tree["anc"], self.pool[l], c.Hk, c.Hv, c.D, c.D,
                          neg_exp_A=self.neg_exp_A[l], o=self.o, aux_k=self.aux_k[l], aux_vn=self.aux_vn[l],
                          aux_g=self.aux_g[l], aux_k_per_v=False, status=self.status)

    def accept(self, target):
        K.accept_greedy(self.tree["tokens"], self.tree["nxt"], self.tree["sib"], target, self.cfg.P,
                        status=self.status, out=(self.path, self.accept_len, self.last, self.bonus))

    def commit(self, x=None):
        """Closed-form state commit of every layer; with the cycle's pre-conv
        inputs x [L, B, N, C], also the conv-window commit (each layer's conv
        state takes the last accepted node's window)."""
        c = self.cfg
        K.gdn_commit(self.pool, self.pool_out, self.aux_k, self.aux_vn, self.aux_g, self.tree["anc"], self.path,
                     self.last.view(-1, 1), c.Hk, c.Hv, aux_k_per_v=False, status=self.status)
        if x is not None:
            K.conv_commit(x, self.conv_state, self.tree["cidx"], self.last, status=self.status)

    def verify(self, x, a, b, q=None):
        """Every layer in model order: tree conv + GDN verify per GDN layer
        (each launch overlapping the previous layer's tail), tree attention
        per attention layer (q [La, B, N, Hq, Da])."""
        l = j = 0
        for kind in self.cfg.layer_kinds:
            if kind == "gdn":
                self.verify_layer(l, x[l], a[l], b[l])
                l += 1
            else:
                self.attend_layer(j, q[j])
                j += 1

    def step(self, logits, root, pre1, x, a, b, target_fn, q=None):
        """One cycle.  x [L, B, N, C], a / b [L, B, N, Hv]; q [La, B, N, Hq, Da]
        when the cycle has attention layers; target_fn(tree) -> the target
        model's token per node [B, N] (int64)."""
        self.build(logits, root, pre1)
        self.verify(x, a, b, q)
        self.accept(target_fn(self.tree))
        self.commit(x)
