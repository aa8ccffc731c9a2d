"""Tree-masked attention verify with the plan / run shape the plugin uses.

The reference verifies the draft tree's gated full-attention layers through
flashinfer's paged prefill wrapper: `fc1_plan.install` (fc1_plan.py:8-33)
replaces its `plan` with a host-length fast path for one request (page size
1, `n` query rows, `HOST_KV_LEN` keys, the custom mask of fc1_branch64.py:39
bit-packed), and every attention layer then calls `run`.  This wrapper keeps
that split: `plan` once per cycle from host-known lengths (no device
readback), `run(q, kv_cache)` per layer on the current stream, backed by
`dft_tree_attn` (tcgen05 kernel, csrc/dft_attn.cu) for a whole batch.

The custom mask is accepted in the plugin's form -- the flattened boolean
[n, prefix + n] rows of each request, prefix columns all visible -- or
directly as the [B, n, n] ancestor matrix.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib as L
from . import kernels as K


class TreeAttentionWrapper:

    def __init__(self, device=None):
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.workspace = None
        self.status = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._plan = None

    def plan(self, kv_indptr, kv_indices, num_qo_heads, num_kv_heads, head_dim, n, anc=None, custom_mask=None,
             kv_lens_host=None, page_size=1, sm_scale=None):
        """kv_indptr [B + 1] / kv_indices: each request's key slots (prefix
        first, then its n tree tokens in node order).  kv_lens_host: host list
        of per-request key counts (the plan's HOST_KV_LEN); read from
        kv_indptr, with a sync, when omitted."""
        if page_size != 1:
            raise L.DFTError("tree attention plans page size 1 (fc1_plan.py:23)")
        B = kv_indptr.numel() - 1
        if kv_lens_host is None:
            p = kv_indptr.to(torch.int64).cpu()
            kv_lens_host = (p[1:] - p[:-1]).tolist()
        kv_lens_host = [int(x) for x in kv_lens_host]
        if len(kv_lens_host) != B or min(kv_lens_host) < n:
            raise L.DFTError("every request needs at least its n tree keys")
        if anc is None:
            if custom_mask is None:
                raise L.DFTError("plan needs anc [B, n, n] or the flattened custom mask")
            rows, off = [], 0
            for Lb in kv_lens_host:
                rows.append(custom_mask[off:off + n * Lb].view(n, Lb)[:, Lb - n:])
                off += n * Lb
            anc = torch.stack(rows)
        self._plan = dict(B=B, n=n, Hq=num_qo_heads, Hkv=num_kv_heads, D=head_dim,
                          kv_indptr=kv_indptr.to(device=self.device, dtype=torch.int32).contiguous(),
                          kv_indices=kv_indices.to(device=self.device, dtype=torch.int32).contiguous(),
                          anc=anc.reshape(B, n, n).to(device=self.device, dtype=torch.float32).contiguous(),
                          max_kv_len=max(kv_lens_host), sm_scale=sm_scale)
        return self

    def run(self, q, kv_cache, out=None):
        """q [B*n, Hq, D] or [B, n, Hq, D] bf16; kv_cache = (k, v) each
        [slots, Hkv, D] (or one [slots, 2, Hkv, D] tensor).  Returns o shaped like q."""
        p = self._plan
        if p is None:
            raise L.DFTError("run before plan")
        k_cache, v_cache = kv_cache if isinstance(kv_cache, (tuple, list)) else (kv_cache[:, 0], kv_cache[:, 1])
        shape = q.shape
        q4 = q.view(p["B"], p["n"], p["Hq"], p["D"])
        o4 = None if out is None else out.view(p["B"], p["n"], p["Hq"], p["D"])
        a, o4, keep = K.tree_attn_args(q4, k_cache, v_cache, p["kv_indptr"], p["kv_indices"], p["anc"],
                                       p["max_kv_len"], p["sm_scale"], o4)
        lib = L.lib()
        need = lib.dft_tree_attn_workspace_bytes(C.byref(a))
        if need < 0:
            raise L.DFTError("tree attention: shape outside the tensor-core path")
        if need > 0 and (self.workspace is None or self.workspace.numel() < need):
            self.workspace = torch.empty(need, dtype=torch.uint8, device=self.device)
        L.check(lib.dft_tree_attn(C.byref(a), None if need == 0 else self.workspace.data_ptr(),
                                  self.status.data_ptr(), L.stream_handle()), "dft_tree_attn")
        del keep
        return o4.view(shape)

    def device_status(self) -> int:
        """Bits raised by runs so far (DFT_DEV_*); reads the device (syncs)."""
        return int(self.status.item())
