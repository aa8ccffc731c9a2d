"""GDN adapter with the reference's interface (fc1_fused.py:1-98).

`Context` / `CTX` hold the per-layer aux buffers (k, vn, G) the verifier saves
for the commit; `snapshots` is the closed-form commit (fc1_fused.py:27-49) as
a function; `make_hooks` returns the two SGLang hooks `fused`
(TritonGDNKernel.target_verify) and `fused_commit`
(commit_mamba_states_after_verify) over the sm_100a kernels; `install()`
patches SGLang exactly where the reference does (needs sglang==0.5.22).
"""
from __future__ import annotations

import os

import torch

from . import kernels as K

NN = int(os.environ.get("FC1_TREE_N", "64"))
BS = int(os.environ.get("FC1_DRAFT_BLOCK", "24"))
CTX = None
NATIVE_REFERENCE = False
_installed = False


class Context:
    """fc1_fused.py:12-20 (layers x heads x NN x 128 aux buffers)."""

    def __init__(self, layers=24, heads=32, nn=None, dim=128, device="cuda"):
        nn = NN if nn is None else nn
        self.anc = torch.eye(nn, device=device, dtype=torch.float32)
        self.keys = torch.empty(layers, heads, nn, dim, device=device)
        self.values = torch.empty_like(self.keys)
        self.gains = torch.empty(layers, heads, nn, device=device)
        self.layers = {}
        self.inter_indices = None
        self.cidx = torch.cat((torch.arange(3, device=device).expand(nn, 3),
                               torch.arange(3, 3 + nn, device=device)[:, None]), 1).long()
        self.current_mixed = None


def snapshots(temporal, keys, values, gains, anc, accept_index, ends, slot, inter_slot, intermediate_ssm):
    """Closed-form commit for one request (fc1_fused.py:27-49).

    temporal [L, slots, H, Dv, Dk]; keys/values [L, H, NN, 128]; gains [L, H, NN];
    anc [NN, NN]; accept_index [1, BS] path nodes (-1 pad); ends [E] end nodes
    (-1 skip); slot / inter_slot: 1-element index tensors; writes
    intermediate_ssm[l, inter_slot, u, h] for every end u >= 0."""
    L_, H = keys.shape[0], keys.shape[1]
    NNn = keys.shape[2]
    path = accept_index.reshape(1, -1)
    e = ends.reshape(1, -1)
    K.gdn_commit(temporal, intermediate_ssm, keys.unsqueeze(1), values.unsqueeze(1), gains.unsqueeze(1),
                 anc.reshape(1, NNn, NNn), path, e, Hk=H, Hv=H, slots_in=slot.reshape(-1)[:1].to(torch.int64),
                 slots_out=inter_slot.reshape(-1)[:1].to(torch.int64), aux_k_per_v=True)


def make_hooks(original_target_verify, original_commit, verify_commit_step_indices):
    """The two hook functions of install() (fc1_fused.py:59-87), given SGLang's
    originals and its `_verify_commit_step_indices`."""

    def fused(self, A_log, dt_bias, q, k, v, a, b, **kw):
        global CTX
        if kw["cache_steps"] != NN:
            return original_target_verify(self, A_log, dt_bias, q, k, v, a, b, **kw)
        if CTX is None:
            CTX = Context()
        key = A_log.data_ptr()
        if key not in CTX.layers:
            CTX.layers[key] = (len(CTX.layers), -A_log.float().exp())
        li, neg = CTX.layers[key]
        if not (li < CTX.keys.shape[0] and q.shape[0] == 1 and q.shape[1] == NN):
            raise ValueError("fused tree verify: unsupported layer count or shape")
        CTX.inter_indices = kw["intermediate_state_indices"]
        pool = kw["ssm_states"]
        from .tree_kernels import tree_gdn_split
        out = tree_gdn_split(CTX.current_mixed, a.reshape(NN, -1), b.reshape(NN, -1), A_log, dt_bias,
                             pool[0].transpose(-1, -2), CTX.anc, q.shape[2], v.shape[2], q.shape[3], v.shape[3],
                             aux=(CTX.keys[li], CTX.values[li], CTX.gains[li]), neg_exp_A=neg,
                             state_indices=kw["cache_indices"], state_slot_stride=pool.stride(0))
        return out.unsqueeze(0)

    def fused_commit(target_worker, batch, accept_lens, accept_index, draft_token_num, prepared_step_indices=None):
        if CTX is not None and draft_token_num == NN and accept_index.numel():
            last, track = verify_commit_step_indices(batch=batch, accept_index=accept_index, accept_lens=accept_lens,
                                                     draft_token_num=draft_token_num)
            if track is None:
                track = torch.full_like(last, -1)
            ends = torch.cat((last, track)).contiguous()
            pool = target_worker.model_runner.req_to_token_pool
            state = pool.get_speculative_mamba2_params_all_layers()
            slots = pool.get_mamba_indices(batch.req_pool_indices)
            snapshots(state.temporal, CTX.keys, CTX.values, CTX.gains, CTX.anc, accept_index, ends, slots,
                      CTX.inter_indices, state.intermediate_ssm)
        return original_commit(target_worker, batch, accept_lens, accept_index, draft_token_num,
                               prepared_step_indices)

    return fused, fused_commit


def install():
    """Patch SGLang's GDN verify / commit / routing (fc1_fused.py:53-97).
    Idempotent: a second call (the reference's register() reaching this module
    through its bare name) keeps the hooks already installed."""
    global _installed
    if _installed:
        return
    from sglang.srt.layers.attention.linear.kernels.gdn_triton import TritonGDNKernel
    from sglang.srt.speculative import eagle_worker_common as common
    from sglang.srt.speculative.spec_utils import _verify_commit_step_indices
    from sglang.srt.layers.attention.linear.gdn_backend import GDNAttnBackend

    fused, fused_commit = make_hooks(TritonGDNKernel.target_verify, common.commit_mamba_states_after_verify,
                                     _verify_commit_step_indices)
    routing = GDNAttnBackend._target_verify_supports_strided_qkv

    def direct_routing(self, **kwargs):
        if not NATIVE_REFERENCE and kwargs["draft_token_num"] == NN:
            return True
        return routing(self, **kwargs)

    GDNAttnBackend._target_verify_supports_strided_qkv = direct_routing
    TritonGDNKernel.target_verify = fused
    common.commit_mamba_states_after_verify = fused_commit
    _installed = True


def set_tree(anc, cidx):
    """The tree hand-off of fc1_branch64.py:26-30 as a call: copy the built
    tree's ancestor matrix [NN, NN] and conv columns [NN, 4] into the hooks'
    context (created on first use, as the hooks do)."""
    global CTX
    if CTX is None:
        CTX = Context(device=anc.device)
    CTX.anc.copy_(anc)
    CTX.cidx.copy_(cidx)
