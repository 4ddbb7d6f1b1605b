"""fxb200: runtime plumbing of the B200 build (C-ABI loader, build recipe,
tensor-level kernel helpers, data-parallel gradient sync).

The reference-named operator surface lives in the sibling packages `fxlm`
(GPT ops, FlatAdamW, model) and `fxgpu` (fused gather-linear, WindowMLP).
"""
__all__ = ["build", "load_library"]


def build(force=False):
    from .build import build as _b
    return _b(force=force)


def load_library():
    from ._lib import load
    return load()
