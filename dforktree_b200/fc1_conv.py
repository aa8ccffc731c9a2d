"""Tree conv hook with the reference's interface (fc1_conv.py:1-46).

`conv` applies the tree causal conv for one request with the plugin's tensors
(x [1, C, NN] channels-first, conv_state [slots, C, 3], weight [C, 4],
conv_state_indices, intermediate_state_indices, intermediate_conv_window
[slots, NN, C, 3]) on dft_tree_conv; `make_hook` / `install` patch SGLang's
causal_conv1d_update like the reference.
"""
from __future__ import annotations

import torch

from . import fc1_fused as F
from . import kernels as K


def conv(conv_state, x, weight, bias, cidx, conv_state_indices, intermediate_state_indices,
         intermediate_conv_window):
    """fc1_conv.py:8-27 for one request; returns y [1, NN, C] (x.dtype)."""
    _, Cn, N = x.shape
    xv = x[0].transpose(0, 1).unsqueeze(0)            # [1, N, C] view, channel stride x.stride(1)
    y = torch.empty(1, N, Cn, dtype=x.dtype, device=x.device)
    K.tree_conv(xv, conv_state, weight, bias, cidx.reshape(1, N, 4), y=y, iw=intermediate_conv_window,
                state_slots=conv_state_indices.reshape(-1)[:1].to(torch.int64),
                iw_slots=intermediate_state_indices.reshape(-1)[:1].to(torch.int64))
    return y


def make_hook(original):
    def call(x, conv_state, weight, bias=None, activation=None, **kw):
        if F.NATIVE_REFERENCE or x.ndim != 3 or x.shape[0] != 1 or x.shape[-1] != F.NN:
            return original(x, conv_state, weight, bias, activation, **kw)
        if weight.shape[-1] != 4 or activation not in ("silu", "swish", True):
            raise ValueError("tree conv: width-4 SiLU conv only")
        if F.CTX is None:
            F.CTX = F.Context(device=x.device)
        out = conv(conv_state, x, weight, bias, F.CTX.cidx, kw["conv_state_indices"],
                   kw["intermediate_state_indices"], kw["intermediate_conv_window"])
        F.CTX.current_mixed = out[0]
        return out.transpose(1, 2)

    return call


_installed = False


def install():
    """Patch SGLang's causal_conv1d_update (fc1_conv.py:29-46); idempotent."""
    global _installed
    if _installed:
        return
    from sglang.srt.layers.attention.linear import gdn_backend as backend
    backend.causal_conv1d_update = make_hook(backend.causal_conv1d_update)
    _installed = True
