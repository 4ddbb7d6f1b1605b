"""fxlm.linear: the GPT block's linears on tcgen05 tensor cores.

The reference runs these through rocBLAS via nn.Linear (ml/fxlm/model.py:48-51,
61, 69-71: qkv, proj + residual, fc -> GELU(tanh) -> fc2 + residual). Here they
are autograd Functions over the tcgen05 GEMM with fused epilogues:
  fused_linear(x, W, residual)  y = x W^T (+ residual)       (qkv, proj)
  fused_mlp(h, W1, W2, residual) y = residual + gelu(h W1^T) W2^T
The MLP keeps the pre-activation Z from the fc epilogue and folds gelu'(Z)
into the epilogue of fc2's dX GEMM. Weight gradients are produced by a split-K
GEMM that accumulates fp32 directly into the FlatAdamW flat-gradient slot when
the weight is managed by FlatAdamW (else they are returned to autograd).
fp32 tensors take the library's fp32 GEMM (the 1e-5 parity mode) through the
same calls and epilogues.
"""
import torch

from fxb200 import ops

_DTYPES = (torch.float16, torch.bfloat16, torch.float32)


def _check(x, W):
    if x.dtype not in _DTYPES or W.dtype != x.dtype:
        raise TypeError(f"x and weight must share bf16, fp16 or fp32 ({x.dtype}, {W.dtype})")
    if not (x.is_cuda and W.is_cuda):
        raise TypeError("x and weight must be cuda tensors")
    if W.dim() != 2 or x.shape[-1] != W.shape[1]:
        raise ValueError(f"shape mismatch: x{tuple(x.shape)} W{tuple(W.shape)}")
    if not W.is_contiguous():
        raise ValueError("weight must be contiguous")


class _Linear(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, W, residual):
        _check(x, W)
        K, N = W.shape[1], W.shape[0]
        x2 = x.reshape(-1, K)
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        res2 = None
        if residual is not None:
            if residual.shape[:-1] != x.shape[:-1] or residual.shape[-1] != N:
                raise ValueError("residual shape mismatch")
            res2 = residual.reshape(-1, N)
            if not res2.is_contiguous():
                res2 = res2.contiguous()
        y = ops.linear_fwd(x2, W, res2)
        ctx.save_for_backward(x2, W)
        ctx.has_res = residual is not None
        ctx.xshape = x.shape
        return y.view(*x.shape[:-1], N)

    @staticmethod
    def backward(ctx, dy):
        x2, W = ctx.saved_tensors
        N = W.shape[0]
        dy2 = dy.reshape(-1, N)
        if not dy2.is_contiguous():
            dy2 = dy2.contiguous()
        dx = ops.linear_dx(dy2, W).view(ctx.xshape) if ctx.needs_input_grad[0] else None
        gw = ops.weight_grad(dy2, x2, W) if ctx.needs_input_grad[1] else None
        dres = dy if ctx.has_res else None
        return dx, gw, dres


class _MLP(torch.autograd.Function):
    @staticmethod
    def forward(ctx, h, W1, W2, residual):
        _check(h, W1)
        D, F = W1.shape[1], W1.shape[0]
        if W2.shape != (D, F) or W2.dtype != W1.dtype:
            raise ValueError(f"fc2 weight must be ({D},{F}), got {tuple(W2.shape)}")
        h2 = h.reshape(-1, D)
        if not h2.is_contiguous():
            h2 = h2.contiguous()
        M = h2.shape[0]
        gz = torch.empty(M, F, device=h.device, dtype=h.dtype)  # gelu'(z), for backward
        a = torch.empty(M, F, device=h.device, dtype=h.dtype)
        ops.gemm(h2, W1, a, epilogue=ops.EPI_GELU_DERIV, Z=gz)
        out = torch.empty(M, D, device=h.device, dtype=h.dtype)
        if residual is not None:
            res2 = residual.reshape(-1, D)
            if not res2.is_contiguous():
                res2 = res2.contiguous()
            ops.gemm(a, W2, out, epilogue=ops.EPI_RESIDUAL, R=res2)
        else:
            ops.gemm(a, W2, out)
        ctx.save_for_backward(h2, gz, a, W1, W2)
        ctx.has_res = residual is not None
        ctx.hshape = h.shape
        return out.view(h.shape)

    @staticmethod
    def backward(ctx, dout):
        h2, gz, a, W1, W2 = ctx.saved_tensors
        D = W1.shape[1]
        d2 = dout.reshape(-1, D)
        if not d2.is_contiguous():
            d2 = d2.contiguous()
        dz = torch.empty_like(gz)
        ops.gemm(d2, W2, dz, b_trans=True, epilogue=ops.EPI_MUL, R=gz)   # dz = (dout W2) * gelu'(z)
        gW2 = ops.weight_grad(d2, a, W2) if ctx.needs_input_grad[2] else None
        dh = ops.linear_dx(dz, W1).view(ctx.hshape) if ctx.needs_input_grad[0] else None
        gW1 = ops.weight_grad(dz, h2, W1) if ctx.needs_input_grad[1] else None
        dres = dout if ctx.has_res else None
        return dh, gW1, gW2, dres


def fused_linear(x, weight, residual=None):
    """y = x @ weight.T (+ residual); x (..., K), weight (N, K)."""
    return _Linear.apply(x, weight, residual)


def fused_mlp(h, w_fc, w_fc2, residual=None):
    """y = residual + gelu_tanh(h @ w_fc.T) @ w_fc2.T."""
    return _MLP.apply(h, w_fc, w_fc2, residual)
