"""CPU: the reference's bare-name imports (fc1_branch64.py:18, 27) resolve to
this package after fc1_plugin.alias_reference_modules(), and the previous
bindings come back with restore_modules()."""
import sys

from dforktree_b200 import fc1_plugin


def test_alias_and_restore_reference_module_names():
    sentinel = object()
    sys.modules["fc1_fused"] = sentinel
    try:
        prev = fc1_plugin.alias_reference_modules()
        import fc1_builder
        import fc1_fused
        import tree_kernels
        from dforktree_b200 import fc1_fused as ours
        assert fc1_fused is ours
        assert fc1_builder.Builder.__module__ == "dforktree_b200.fc1_builder"
        assert hasattr(tree_kernels, "tree_gdn_split") and hasattr(fc1_fused, "set_tree")
        assert set(prev) == set(fc1_plugin.REFERENCE_MODULES)
        fc1_plugin.restore_modules(prev)
        assert sys.modules["fc1_fused"] is sentinel
        assert "fc1_builder" not in sys.modules or sys.modules["fc1_builder"] is not ours
    finally:
        sys.modules.pop("fc1_fused", None)
