"""`Builder` with the reference's interface (fc1_builder.py:8-54).

Score + build for one request (logits [S, V], as the plugin calls it at
fc1_branch64.py:25) or a batch (logits [B, S, V]).  `run()` is three kernel
launches (score, dense PMI, beam + tree structure) on the current stream and
is captured once into a CUDA graph; `__call__` copies the inputs into the
static buffers and replays it, like the reference.

Environment, as in the reference: FC1_TREE_N (default 32), FC1_CHAIN_FIRST,
FC1_NGRAM_PATH (npz table or cached table file; `ng=` passes an already
loaded NGramGPU).  Added here: FC1_NGRAM_CACHE, a cached-table file that is
loaded instead of the npz when intact and written after a build otherwise.
"""
from __future__ import annotations

import os

import torch

from . import kernels as K
from .ngram_gpu import NGramGPU


class Builder:

    def __init__(self, logits, ngram=True, compile_build=False, ng=None, n=None, graph=True,
                 lam_a=0.3, lam_p=0.6, lmax=99):
        self.n = int(n if n is not None else os.environ.get("FC1_TREE_N", "32"))
        self.batched = logits.dim() == 3
        lg = logits if self.batched else logits.unsqueeze(0)
        self.B, self.slots, self.V = lg.shape
        self.chain_first = os.environ.get("FC1_CHAIN_FIRST", "0") == "1"
        self.lam_a, self.lam_p, self.lmax = lam_a, lam_p, lmax
        dev = logits.device
        self.logits = torch.zeros_like(lg)
        self.root = torch.zeros(self.B, device=dev, dtype=torch.long)
        self.pre1 = torch.zeros_like(self.root)
        if ngram:
            self.ng = ng if ng is not None else NGramGPU(
                os.environ.get("FC1_NGRAM_PATH", "data/ngram_counts.npz"), dev, beta3=60.0,
                cache=os.environ.get("FC1_NGRAM_CACHE") or None)
        else:
            self.ng = None
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        self.ws = K.score_build_workspace(self.B, self.slots, self.V, self.n, use_ngram=ngram, device=dev)
        self.out = K.tree_outputs(self.B, self.slots, self.n, dev)
        self.graph = None
        self.run()
        torch.cuda.synchronize()
        if graph:
            self.graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self.graph):
                self.run()

    def run(self):
        K.score_build(None if self.ng is None else self.ng.table, self.logits, self.root, self.pre1, self.n,
                      self.ws, self.out, lmax=self.lmax, chain_first=self.chain_first, use_ngram=self.ng is not None,
                      lam_a=self.lam_a, lam_p=self.lam_p, status=self.status)

    # reference attribute names (fc1_builder.py:38-47)
    @property
    def tokens(self):
        return self.out["tokens"] if self.batched else self.out["tokens"][0]

    @property
    def parent(self):
        return self.out["parent"] if self.batched else self.out["parent"][0]

    @property
    def depth(self):
        return self.out["depth"] if self.batched else self.out["depth"][0]

    @property
    def anc(self):
        return self.out["anc"] if self.batched else self.out["anc"][0]

    @property
    def cidx(self):
        return self.out["cidx"] if self.batched else self.out["cidx"][0]

    @property
    def nxt(self):
        return self.out["nxt"] if self.batched else self.out["nxt"][0]

    @property
    def sib(self):
        return self.out["sib"] if self.batched else self.out["sib"][0]

    def __call__(self, logits, root, pre1):
        lg = logits if self.batched else logits.unsqueeze(0)
        self.logits.copy_(lg)
        self.root.copy_(root.reshape(self.B))
        self.pre1.copy_(pre1.reshape(self.B))
        if self.graph is not None:
            self.graph.replay()
        else:
            self.run()
        tok = self.out["tokens"] if self.batched else self.out["tokens"][0][None]
        return (tok, self.depth, self.parent, self.anc, self.nxt, self.sib)

    def device_status(self) -> int:
        return int(self.status.item())
