"""SGLang plugin entry point with the reference's interface (fc1_plugin.py:22-55).

`register()` installs the sm_100a hooks (GDN verify, commit, tree conv) when
FC1_FUSED=1, exactly where the reference installs its Triton ones.  The
reference's remaining registration (the FC1_DFLASH_TREE speculative
algorithm, its DFlash worker and the flashinfer plan override) is SGLang
serving glue outside the hot path and is not part of this package.  Needs
sglang==0.5.22 (pyproject.toml:11).
"""
from __future__ import annotations

import os

_registered = False


def register():
    global _registered
    if _registered:
        return
    try:
        import sglang  # noqa: F401
    except ImportError as e:
        raise ImportError("dforktree_b200.fc1_plugin.register needs sglang==0.5.22") from e
    if os.environ.get("FC1_FUSED") == "1":
        from .fc1_fused import install
        install()
        from .fc1_conv import install as install_conv
        install_conv()
    _registered = True
