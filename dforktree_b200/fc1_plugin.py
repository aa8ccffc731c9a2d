"""SGLang plugin entry point with the reference's interface (fc1_plugin.py:22-55).

The reference's modules import one another by bare name after putting their
own directory on sys.path (fc1_plugin.py:26): `verify_branch` does
`from fc1_builder import Builder` (fc1_branch64.py:18) and, with FC1_FUSED=1,
`import fc1_fused; fc1_fused.CTX.anc.copy_(anc); fc1_fused.CTX.cidx.copy_(...)`
(fc1_branch64.py:26-30) -- the hand-off of each built tree to the verify and
commit hooks.  `alias_reference_modules()` binds those bare names to this
package's mirrors, so the reference's own call sites build trees with the
sm_100a builder and write this package's hook context, unmodified.

`register()` = alias the modules, then the reference's own registration when
its package is importable (the FC1_DFLASH_TREE algorithm, its worker, the
decode-graph capture override and the flashinfer plan override are SGLang
serving glue outside the hot path; their `from fc1_fused import install` /
`from fc1_conv import install` now resolve to this package), else this
package's hooks alone (FC1_FUSED=1).  Needs sglang==0.5.22 (pyproject.toml:11).
"""
from __future__ import annotations

import importlib
import os
import sys

_registered = False

# bare module names of the reference (dforktree/) that this package mirrors
REFERENCE_MODULES = ("ngram_gpu", "tree_ops", "fc1_builder", "tree_kernels", "fc1_fused", "fc1_conv")


def alias_reference_modules() -> dict:
    """Make `import <name>` of every name in REFERENCE_MODULES return this
    package's module.  Returns the previous sys.modules entries (None where
    there was none) so that a caller can restore them."""
    prev = {}
    for name in REFERENCE_MODULES:
        prev[name] = sys.modules.get(name)
        sys.modules[name] = importlib.import_module(f"{__package__}.{name}")
    return prev


def restore_modules(prev: dict) -> None:
    for name, mod in prev.items():
        if mod is None:
            sys.modules.pop(name, None)
        else:
            sys.modules[name] = mod


def register():
    global _registered
    if _registered:
        return
    try:
        import sglang  # noqa: F401
    except ImportError as e:
        raise ImportError("dforktree_b200.fc1_plugin.register needs sglang==0.5.22") from e
    alias_reference_modules()
    try:
        from dforktree import fc1_plugin as reference_plugin
    except ImportError:
        reference_plugin = None
    if reference_plugin is not None:
        reference_plugin.register()
    elif os.environ.get("FC1_FUSED") == "1":
        from .fc1_fused import install
        install()
        from .fc1_conv import install as install_conv
        install_conv()
    _registered = True
