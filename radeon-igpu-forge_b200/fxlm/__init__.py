"""fxlm (B200 build): small-GPT training ops on sm_100a.

Same public names as the reference package (ml/fxlm/__init__.py:13-46):
flash attention (fwd + bwd), fused RMSNorm, fused cross-entropy and
linear-CE, FlatAdamW, GPT/GPTConfig; plus `fused_linear` / `fused_mlp`, the
tensor-core linears the reference ran through rocBLAS. Exports are lazy so
that `fxlm.env` can be imported before torch, as in the reference.
"""

__all__ = [
    "setup_lm_env",
    "require_gpu",
    "flash_attention",
    "flash_attention_qkv",
    "fused_cross_entropy",
    "linear_cross_entropy",
    "rms_norm",
    "fused_linear",
    "fused_mlp",
    "FlatAdamW",
    "GPT",
    "GPTConfig",
    "GraphedStep",
    "GraphedFunction",
]


def __getattr__(name):
    if name in ("setup_lm_env", "require_gpu"):
        from . import env as _m
        return getattr(_m, name)
    if name in ("flash_attention", "flash_attention_qkv"):
        from . import attention as _m
        return getattr(_m, name)
    if name in ("fused_cross_entropy", "linear_cross_entropy"):
        from . import cross_entropy as _m
        return getattr(_m, name)
    if name == "rms_norm":
        from .norm import rms_norm
        return rms_norm
    if name in ("fused_linear", "fused_mlp"):
        from . import linear as _m
        return getattr(_m, name)
    if name == "FlatAdamW":
        from .optim import FlatAdamW
        return FlatAdamW
    if name in ("GraphedStep", "GraphedFunction"):
        from . import graph as _m
        return getattr(_m, name)
    if name in ("GPT", "GPTConfig"):
        from . import model as _m
        return getattr(_m, name)
    raise AttributeError(f"module {__name__!r} has no attribute {name!r}")
