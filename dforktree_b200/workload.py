"""Synthetic inputs of the draft-tree cycle at the benchmark configurations.

The reference's n-gram table, drafter checkpoints and prompts are not
available, so seeded stand-ins with the configurations' shapes and value
distributions are used (one generator for the bench and its parity tests):

* drafter logits [B, S, V] fp32: 3 * N(0, 1) with one peaked token (+6) per
  position (config 0, per request);
* root / previous tokens uniform over V;
* per GDN layer the pre-conv activations x [B, N, C] and the gate inputs
  a, b [B, N, Hv] (bf16, N(0, 1)); per attention layer the queries
  q [B, N, Hq, Da] (bf16, N(0, 1));
* accepted lengths uniform in 1..24 (config 4) and a target-model stand-in
  that agrees with the draft along one root-to-leaf path.
"""
from __future__ import annotations

import torch


def cycle_inputs(cfg, dev, seed: int) -> dict:
    """Device-resident inputs of one cycle of `cfg` (a CycleConfig)."""
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    B, S, V, N = cfg.B, cfg.S, cfg.V, cfg.N
    logits = torch.randn(B, S, V, device=dev, generator=g) * 3.0
    pk = torch.randint(0, V, (B, S), device=dev, generator=g)
    logits.view(-1, V)[torch.arange(B * S, device=dev), pk.view(-1)] += 6.0
    root = torch.randint(0, V, (B,), device=dev, generator=g)
    pre1 = torch.randint(0, V, (B,), device=dev, generator=g)
    x = torch.empty(cfg.layers, B, N, cfg.C, dtype=torch.bfloat16, device=dev)
    for l in range(cfg.layers):        # one layer at a time: no fp32 copy of the whole tensor
        x[l] = torch.randn(B, N, cfg.C, device=dev, generator=g)
    a = torch.randn(cfg.layers, B, N, cfg.Hv, device=dev, generator=g).to(torch.bfloat16)
    b = torch.randn(cfg.layers, B, N, cfg.Hv, device=dev, generator=g).to(torch.bfloat16)
    acc_len = torch.randint(1, 25, (B,), device=dev, generator=g)
    out = dict(logits=logits, root=root, pre1=pre1, x=x, a=a, b=b, acc_len=acc_len, q=None)
    if cfg.attn_layers:
        q = torch.empty(cfg.attn_layers, B, N, cfg.Hq, cfg.Da, dtype=torch.bfloat16, device=dev)
        for j in range(cfg.attn_layers):
            q[j] = torch.randn(B, N, cfg.Hq, cfg.Da, device=dev, generator=g)
        out["q"] = q
    return out


def path_target(tree: dict, acc_len: torch.Tensor) -> torch.Tensor:
    """Target-model stand-in for greedy acceptance: the target's token at node
    u is the draft token of u's child on the root-to-leaf path through the
    deepest node (the first one in node order), while depth(u) + 1 <
    acc_len[b]; elsewhere -1 (no child matches).  The accepted path is that
    path cut at acc_len nodes, so the accepted length is
    min(acc_len[b], deepest depth + 1).  Returns [B, N] int64."""
    depth, parent, tokens = tree["depth"], tree["parent"], tree["tokens"]
    B, N = depth.shape
    dev = depth.device
    leaf = depth.argmax(1)                                              # first deepest node
    on_path = tree["anc"][torch.arange(B, device=dev), leaf] > 0.5       # ancestors-or-self of the leaf
    m = torch.arange(N, device=dev).expand(B, N)
    valid = on_path & (m > 0)
    # next path node of each path node: scatter every non-root path node into its parent's column
    nxt = torch.full((B, N + 1), -1, dtype=torch.int64, device=dev)
    nxt.scatter_(1, torch.where(valid, parent, N), torch.where(valid, m, -1))
    nxt = nxt[:, :N]
    tgt = torch.gather(tokens, 1, nxt.clamp(min=0))
    keep = (nxt >= 0) & (depth + 1 < acc_len[:, None])
    return torch.where(keep, tgt, torch.full_like(tgt, -1))


def expected_path(parent, depth, anc, acc_len: int):
    """Host restatement of the path `path_target` makes greedy acceptance take
    (numpy arrays of one request): node ids, root first."""
    import numpy as np
    leaf = int(np.argmax(depth))
    nodes = sorted((int(m) for m in np.nonzero(np.asarray(anc)[leaf] > 0.5)[0]), key=lambda u: int(depth[u]))
    return nodes[:max(1, min(int(acc_len), len(nodes)))]
