"""fxgpu (B200 build): fused gather-linear and the window MLP on sm_100a.

Same public names as the reference package (ml/fxgpu/__init__.py:8-27):
FusedGatherLinear, fused_gather_linear, WindowMLP; exports are lazy.
"""

__all__ = ["FusedGatherLinear", "fused_gather_linear", "WindowMLP"]


def __getattr__(name):
    if name in ("FusedGatherLinear", "fused_gather_linear"):
        from . import fused_linear as _m
        return getattr(_m, name)
    if name == "WindowMLP":
        from .model import WindowMLP
        return WindowMLP
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
