"""B200-native MoE feed-forward engine with the reference's public surface.

Lazy exports, as in the reference (src/moe_dispatch/__init__.py:1-23): importing
the package loads nothing; the kernel library is loaded on first GPU use.
"""

from importlib import import_module

__version__ = "0.2.0+b200"
__all__ = ["dispatch", "combine", "PackedTokens", "CudaWorkspace", "MoEBlock", "MoEConfig",
           "MoEWeights", "make_weights", "capture_forward", "get_extension", "HostPipeline"]
_EXPORTS = {
    "dispatch": (".ops", "dispatch"),
    "combine": (".ops", "combine"),
    "PackedTokens": (".ops", "PackedTokens"),
    "CudaWorkspace": (".workspace", "CudaWorkspace"),
    "MoEBlock": (".layer", "MoEBlock"),
    "MoEConfig": (".layer", "MoEConfig"),
    "MoEWeights": (".layer", "MoEWeights"),
    "make_weights": (".layer", "make_weights"),
    "capture_forward": (".graphs", "capture_forward"),
    "get_extension": ("._extension", "get_extension"),
    "HostPipeline": (".host_pipeline", "HostPipeline"),
}


def __getattr__(name):
    if name not in _EXPORTS:
        raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
    module, symbol = _EXPORTS[name]
    value = getattr(import_module(module, __name__), symbol)
    globals()[name] = value
    return value
