"""fxgpu.fused_linear: FusedGatherLinear on sm_100a.

out = (window of X starting at row idx[b], flattened window-major) @ W^T + bias,
the reference's fused gather + GEMM layer (ml/fxgpu/fused_linear.py:27-101):
Xg[b, w*F + f] = X[idx[b] + w, f]; forward also keeps Xg for the weight
gradient; backward returns dW = g^T Xg and db = g.sum(0) and no gradient for
X (input layer). Here the window rows are copied by fxb_gather_windows (each
window is a contiguous span of row-major X) and the GEMM runs on tcgen05 with
the bias added in its epilogue; db is a column-sum kernel.
"""
import torch

from fxb200 import _lib, ops


def _check(X16, idx32, weight, bias):
    """Validation of ml/fxgpu/fused_linear.py:37-64 (dtype widened to bf16)."""
    F = X16.shape[1]
    K = weight.shape[1]
    if K % F != 0:
        raise ValueError(f"weight.shape[1]={K} is not a multiple of X16.shape[1]={F} "
                         f"(K = window * F)")
    if F % 8 != 0:
        raise ValueError("pad F to a multiple of 8 with zero columns "
                         f"(F={F}; rows must be 16-byte aligned)")
    if X16.dtype not in (torch.float16, torch.bfloat16):
        raise TypeError(f"X16 must be fp16 or bf16, got {X16.dtype}")
    if idx32.dtype != torch.int32:
        raise TypeError(f"idx32 must be int32, got {idx32.dtype}")
    if weight.dtype != X16.dtype or bias.dtype != X16.dtype:
        raise TypeError("weight and bias must match X16's dtype")
    if not (X16.is_cuda and idx32.is_cuda and weight.is_cuda and bias.is_cuda):
        raise TypeError("all tensors must be cuda tensors")
    if not (X16.is_contiguous() and idx32.is_contiguous() and weight.is_contiguous()
            and bias.is_contiguous()):
        raise ValueError("all tensors must be contiguous (call .contiguous())")
    if idx32.dim() != 1:
        raise ValueError(f"idx32 must be (B,), shape={tuple(idx32.shape)}")
    if weight.dim() != 2 or bias.dim() != 1 or bias.shape[0] != weight.shape[0]:
        raise ValueError("weight must be (N,K) and bias (N,)")
    return F, K


def gather_windows(X16, idx32, window):
    """Xg (B, window*F) = the windows of X starting at idx32 rows."""
    B = idx32.numel()
    R, F = X16.shape
    Xg = torch.empty(B, window * F, device=X16.device, dtype=X16.dtype)
    _lib.call("fxb_gather_windows", _lib.dtype_code(X16.dtype), _lib.ptr(X16), R, F,
              _lib.ptr(idx32), B, window, _lib.ptr(Xg), _lib.stream_ptr(X16.device))
    return Xg


def bias_grad(g, bias):
    """db = g.sum(0): into bias's flat fp32 slot (returns None) or as a tensor."""
    sink = ops.param_grad_sink(bias)
    rows, cols = g.shape
    if sink is not None:
        _lib.call("fxb_colsum", _lib.dtype_code(g.dtype), _lib.ptr(g), rows, cols, _lib.ptr(sink),
                  1, _lib.stream_ptr(g.device))
        return None
    out = torch.empty(cols, device=g.device, dtype=torch.float32)
    _lib.call("fxb_colsum", _lib.dtype_code(g.dtype), _lib.ptr(g), rows, cols, _lib.ptr(out),
              0, _lib.stream_ptr(g.device))
    return out.to(bias.dtype)


class FusedGatherLinear(torch.autograd.Function):
    """out[b, n] = sum_k Xg[b, k] * weight[n, k] + bias[n]

    Xg[b, w*F + f] = X[idx[b] + w, f] (window-major).
    X16: (R, F) fp16/bf16 contiguous; idx32: (B,) int32 contiguous;
    weight: (N, K) same dtype, K = W*F; bias: (N,).
    """

    @staticmethod
    def forward(ctx, X16, idx32, weight, bias):
        F, K = _check(X16, idx32, weight, bias)
        Xg = gather_windows(X16, idx32, K // F)
        C = torch.empty(idx32.numel(), weight.shape[0], device=X16.device, dtype=X16.dtype)
        ops.gemm(Xg, weight, C, epilogue=ops.EPI_BIAS, bias=bias)
        if any(ctx.needs_input_grad):
            ctx.save_for_backward(Xg, weight, bias)
        return C

    @staticmethod
    def backward(ctx, g):
        Xg, weight, bias = ctx.saved_tensors
        g = g.contiguous()
        dW = ops.weight_grad(g, Xg, weight) if ctx.needs_input_grad[2] else None
        db = bias_grad(g, bias) if ctx.needs_input_grad[3] else None
        return None, None, dW, db


def fused_gather_linear(X16, idx32, weight, bias):
    """Thin wrapper for FusedGatherLinear.apply."""
    return FusedGatherLinear.apply(X16, idx32, weight, bias)
