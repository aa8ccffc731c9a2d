"""Generate the tree-attention golden fixtures from flashinfer itself.

The reference plugin verifies the draft tree's attention layers through
flashinfer's paged prefill (a third-party dependency, the version SGLang
0.5.22 pins; installed in this image): fc1_plan.py:16-33 plans it for one
request -- qo_indptr [0, n], kv_indptr [0, prefix + n], page size 1, the
fc1_branch64.py:39 mask [ones(n, prefix) | anc] bit-packed little-endian --
and every attention layer calls `run`.  This script makes exactly those calls
(fa2 backend, bf16) on the inputs of `cases.ATTN_CASES` and stores each
case's output as raw bf16 bits with an input checksum.  It needs a CUDA
device (flashinfer JIT-builds its prefill kernel on first use):

    python tests/golden/make_attn_golden.py [--out DIR]
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from tests.golden import cases  # noqa: E402


def run_case(case, dev):
    import flashinfer
    import torch
    d = cases.attn_inputs(case)
    N, Hq, Hkv, D = case["N"], case["Hq"], case["Hkv"], cases.ATTN_D
    t = lambda x: torch.from_numpy(x).to(dev)
    q = t(d["q"]).to(torch.bfloat16)
    k = t(d["k"]).to(torch.bfloat16).unsqueeze(1)            # [pages, page_size 1, Hkv, D]
    v = t(d["v"]).to(torch.bfloat16).unsqueeze(1)
    ws = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    outs = []
    for b in range(len(case["prefixes"])):
        lo, hi = int(d["kv_indptr"][b]), int(d["kv_indptr"][b + 1])
        L = hi - lo
        mask = torch.cat((torch.ones(N, L - N, dtype=torch.bool, device=dev),
                          t(d["anc"][b]) > 0.5), 1).flatten()         # fc1_branch64.py:39
        w = flashinfer.BatchPrefillWithPagedKVCacheWrapper(ws, "NHD", backend="fa2")
        w.plan(torch.tensor([0, N], dtype=torch.int32, device=dev), torch.tensor([0, L], dtype=torch.int32, device=dev),
               t(d["kv_indices"][lo:hi]), torch.ones(1, dtype=torch.int32, device=dev), Hq, Hkv, D, 1,
               custom_mask=mask, q_data_type=torch.bfloat16, kv_data_type=torch.bfloat16)
        outs.append(w.run(q[b], (k, v)))
    torch.cuda.synchronize()
    o = torch.stack(outs)                                                 # [B, N, Hq, D] bf16
    return o.view(torch.int16).cpu().numpy().view(np.uint16), d


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    import flashinfer
    import torch
    dev = torch.device("cuda", 0)
    for case in cases.ATTN_CASES:
        o_bits, d = run_case(case, dev)
        np.savez_compressed(os.path.join(args.out, case["name"] + ".npz"), o_bf16=o_bits,
                            checksum=cases.checksum(d["q"], d["k"], d["v"], d["kv_indices"], d["anc"]),
                            flashinfer=np.array(flashinfer.__version__))
        print(case["name"], o_bits.shape)


if __name__ == "__main__":
    main()
