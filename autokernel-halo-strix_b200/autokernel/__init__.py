"""autokernel — swap PyTorch modules for B200 (sm_100a) kernels in place.

    import autokernel
    model = autokernel.optimize(model, training=True)   # apply all patterns
    autokernel.report(model)                             # what was replaced
    autokernel.restore(model)                            # undo
    autokernel.list_patterns()

Same public API as the reference package (autokernel/__init__.py:14-16,
autokernel/_registry.py:64-178).
"""
from autokernel._registry import list_patterns, optimize, report, restore

__all__ = ["optimize", "report", "restore", "list_patterns"]
