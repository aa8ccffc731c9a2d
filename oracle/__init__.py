"""CPU oracle for the DForkTree draft-tree cycle -- TEST INFRASTRUCTURE ONLY.

This package restates the reference's algorithm (Perseus037/DForkTree,
`dforktree/*.py`) in numpy so that the CUDA path can be checked against it.
Only `tests/`, `__graft_entry__.smoke()` and the `cpu_baseline` / reference
legs of `bench.py` may import it, and only as the checker or the timed CPU
baseline.  The product path (`dforktree_b200`) never imports it and has no
CPU fallback.

Pinning: every function here was checked against golden vectors produced by
the reference code itself (imported from its sources, Triton kernels run under
`TRITON_INTERPRET=1` on CPU), see `tests/golden/make_golden.py` and
`tests/test_oracle_golden.py`.  One exception is parity-unpinned: the
fork-aware scoring closure returned by `tree_ops.ngram_path_fn`
(`dforktree/tree_ops.py:55-66`) is missing from the shipped reference
(`return fn` with `fn` undefined), so `builder.path_scores` restates the
reconstruction documented beside it; the goldens pin everything around it.

Modules:
  ngram    -- NGramGPU lookup and smoothing (ngram_gpu.py:8-70)
  builder  -- score, fork-aware closure, beam_tree, tree_struct, Builder.run
              (fc1_builder.py:26-47, tree_ops.py:7-89)
  gdn      -- tree conv, GDN tree verifier, closed-form commit
              (fc1_conv.py:8-27, tree_kernels.py:17-208,
               fc1_block_inverse.py:10-83, fc1_fused.py:27-49)
"""
