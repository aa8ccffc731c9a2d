"""Running the reference's own builder code -- TEST / BASELINE INFRASTRUCTURE ONLY.

Imported by tests/golden/make_golden.py (golden vectors from the reference
sources) and by bench.py's CPU-baseline / reference legs (the reference's
torch builder timed on host cores, from the installed copy under
baseline/_ref).  Never part of the product path.

The reference modules import one another by bare name (`import tree_ops as
TO`, `from ngram_gpu import NGramGPU`, fc1_builder.py:4-5), so their
directory goes on sys.path.  The one piece the reference does not ship -- the
closure returned by `tree_ops.ngram_path_fn` (tree_ops.py:66 returns an
undefined `fn`) -- is supplied by `reconstructed_fn`, the reconstruction the
oracle (oracle/builder.py `path_scores`) and the CUDA path implement; the
reference's own code computes the PMI tensor T it closes over, the beam
search and the tree structure.
"""
from __future__ import annotations

import sys


def load_reference(ref_dir: str, kernels: bool = True):
    """Import the reference modules from `ref_dir` (its dforktree/ directory).
    kernels=False skips the Triton modules (CPU-only builder use)."""
    if ref_dir not in sys.path:
        sys.path.insert(0, ref_dir)
    import torch  # noqa: F401
    import ngram_gpu  # noqa: F401
    import tree_ops  # noqa: F401
    import fc1_builder  # noqa: F401
    if kernels:
        import tree_kernels  # noqa: F401
        import fc1_block_inverse  # noqa: F401
        import fc1_fused  # noqa: F401
        import fc1_conv  # noqa: F401
    return sys.modules


def reconstructed_fn(T, lp, rest, lam_a, lam_p):
    """Fork-aware closure: x = lp[s] + lam * t with lam = lam_a while every
    ancestor was candidate 0, else lam_p; normalised against the retained
    out-of-list mass rest[s] (oracle/builder.py `path_scores`).  t reads T by
    its order (T is [S-1] + (M,) * order): T[s-1][cand] for order 2,
    T[s-1][pc, cand] for 3, T[s-1][ppc, pc, cand] for 4."""
    import torch
    order = T.dim() - 1

    def fn(s, cand, pc, ppc, al):
        Ts = T[s - 1]
        t = Ts[cand] if order == 2 else (Ts[pc, cand] if order == 3 else Ts[ppc, pc, cand])
        lam = torch.where(al, lam_a, lam_p)[:, None].to(t.dtype)
        x = lp[s][None, :] + lam * t
        r = rest[s].reshape(1, 1).expand(x.shape[0], 1)
        return x - torch.logsumexp(torch.cat((x, r), -1), -1, keepdim=True)

    return fn


def patch_path_fn(mods):
    """Wrap tree_ops.ngram_path_fn: let the reference build T, then return the
    reconstructed closure over it.  Returns a dict that receives the last T."""
    TO = mods["tree_ops"]
    if getattr(TO.ngram_path_fn, "_dft_patched", None) is not None:
        return TO.ngram_path_fn._dft_patched
    original = TO.ngram_path_fn
    captured = {}

    class _Capture:
        def __init__(self, ng):
            self.ng = ng

        def pmi(self, *args):
            out = self.ng.pmi(*args)
            captured["T"] = out.float()
            return out

    def patched(ng, order, ids, lp, rest, pre1, root, lam_a, lam_p):
        TO.fn = None  # the name `fn` that the shipped function returns
        original(_Capture(ng), order, ids, lp, rest, pre1, root, lam_a, lam_p)
        del TO.fn
        return reconstructed_fn(captured["T"], lp, rest, lam_a, lam_p)

    patched._dft_patched = captured
    TO.ngram_path_fn = patched
    return captured


def cpu_builder(mods, ng, S: int, N: int, chain_first: bool = False):
    """A reference fc1_builder.Builder on CPU tensors, without the CUDA graph
    of Builder.__init__ (fc1_builder.py:20-23): set .logits / .root / .pre1
    and call .run() (fc1_builder.py:26-47)."""
    import torch
    FB = mods["fc1_builder"]
    b = FB.Builder.__new__(FB.Builder)
    b.n = N
    b.slots = S
    b.chain_first = chain_first
    b.root = torch.zeros(1, dtype=torch.long)
    b.pre1 = torch.zeros(1, dtype=torch.long)
    b.ng = ng
    return b
