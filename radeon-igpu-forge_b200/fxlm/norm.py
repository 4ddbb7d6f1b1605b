"""fxlm.norm: fused RMSNorm on sm_100a (16-bit or fp32 I/O, fp32 math).

y = x * rsqrt(mean(x^2) + eps) * w, as the reference's rms_norm
(ml/fxlm/norm.py:45-90, kernels norm.hip:33-127). One C-ABI call per
direction: fxb_rmsnorm_fwd saves rstd; fxb_rmsnorm_bwd writes dx and reduces
dw deterministically. When the weight is owned by FlatAdamW its gradient is
accumulated straight into the fp32 flat-gradient slot.
"""
import torch

from fxb200 import _lib
from fxb200.ops import param_grad_sink

_DTYPES = (torch.float16, torch.bfloat16, torch.float32)


def _check(x, w):
    """Validation of ml/fxlm/norm.py:30-42 (dtype widened to bf16/fp16/fp32)."""
    if x.dtype not in _DTYPES or w.dtype != x.dtype:
        raise TypeError(f"x and weight must share a bf16/fp16/fp32 dtype ({x.dtype}, {w.dtype})")
    if not (x.is_cuda and w.is_cuda):
        raise TypeError("x and weight must be cuda tensors")
    D = x.shape[-1]
    if w.shape != (D,):
        raise ValueError(f"weight must be ({D},), got {tuple(w.shape)}")
    if D % 8 != 0 or D > 8192:
        raise ValueError(f"D={D}: need D % 8 == 0 and D <= 8192")
    if not x.is_contiguous() or not w.is_contiguous():
        raise ValueError("x and weight must be contiguous")
    return D


def rmsnorm_fwd(x2, w, eps):
    """(y, rstd) for a (rows, D) contiguous input."""
    N, D = x2.shape
    y = torch.empty_like(x2)
    rstd = torch.empty(N, device=x2.device, dtype=torch.float32)
    _lib.call("fxb_rmsnorm_fwd", _lib.dtype_code(x2.dtype), _lib.ptr(x2), _lib.ptr(w),
              _lib.ptr(y), _lib.ptr(rstd), N, D, float(eps), _lib.stream_ptr(x2.device))
    return y, rstd


def rmsnorm_bwd(x2, w, rstd, dy2, dres=None, need_dw=True):
    """dx (+ dres, the residual-path gradient, in the same pass) and dw.

    dw goes into w's FlatAdamW fp32 slot when it has one (returned as None),
    else it is returned in w's dtype (None when need_dw is False)."""
    N, D = x2.shape
    dx = torch.empty_like(x2)
    lib = _lib.load()
    ws = torch.empty(max(1, lib.fxb_rmsnorm_bwd_workspace(N, D) // 4), device=x2.device,
                     dtype=torch.float32)
    sink = param_grad_sink(w) if need_dw else None
    if sink is not None:
        dw, dw_ret, acc = sink, None, 1
    else:
        dw = torch.empty_like(w)
        dw_ret, acc = (dw if need_dw else None), 0
    _lib.call("fxb_rmsnorm_bwd", _lib.dtype_code(x2.dtype), _lib.ptr(x2), _lib.ptr(w),
              _lib.ptr(rstd), _lib.ptr(dy2), _lib.ptr(dres), _lib.ptr(dx), _lib.ptr(dw),
              _lib.dtype_code(dw.dtype), acc, _lib.ptr(ws), N, D, _lib.stream_ptr(x2.device))
    return dx, dw_ret


class _RMSNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, eps):
        D = _check(x, w)
        N = x.numel() // D
        x2 = x.view(N, D)
        y, rstd = rmsnorm_fwd(x2, w, eps)
        ctx.save_for_backward(x2, w, rstd)
        ctx.oshape = x.shape
        return y.view(x.shape)

    @staticmethod
    def backward(ctx, dy):
        x2, w, rstd = ctx.saved_tensors
        N, D = x2.shape
        dx, dw = rmsnorm_bwd(x2, w, rstd, dy.contiguous().view(N, D),
                             need_dw=ctx.needs_input_grad[1])
        return dx.view(ctx.oshape), dw, None


def rms_norm(x, weight, eps=1e-6):
    """x (..., D), weight (D,) -> y, same dtype (bf16 / fp16 / fp32)."""
    return _RMSNorm.apply(x, weight, float(eps))
