"""fxlm.block: the two halves of a GPT block as single autograd Functions.

The reference block (ml/fxlm/model.py:58-72) is
    x1 = x  + proj(attn(qkv(rmsnorm(x))))
    x2 = x1 + fc2(gelu(fc(rmsnorm(x1))))
built from separate ops, so autograd sums the gradient of x (and x1) arriving
through the RMSNorm with the one arriving through the residual in an extra
elementwise kernel. Here each half is one Function: its backward hands the
residual-path gradient to the RMSNorm backward kernel, which adds it while
writing dx (fxb_rmsnorm_bwd's dres), and the GEMM epilogues carry the residual
add, GELU and GELU' as in fxlm.linear. Numerically identical to composing
rms_norm / fused_linear / flash_attention_qkv / fused_mlp.
"""
import math

import torch

from fxb200 import ops
from .attention import _fwd as _attn_fwd, _bwd as _attn_bwd
from .norm import _check as _norm_check, rmsnorm_fwd, rmsnorm_bwd


class _AttnBlock(torch.autograd.Function):
    """x1 = x + proj(flash_attention_qkv(qkv(rms_norm(x))))"""

    @staticmethod
    def forward(ctx, x, ln_w, Wqkv, Wproj, eps, n_head):
        B, T, D = x.shape
        _norm_check(x, ln_w)
        x2 = x.reshape(B * T, D)
        h, rstd = rmsnorm_fwd(x2, ln_w, eps)
        qkv = ops.linear_fwd(h, Wqkv)                      # (B*T, 3D)
        qkv5 = qkv.view(B, T, 3, n_head, D // n_head)
        scale = 1.0 / math.sqrt(D // n_head)
        o, lse = _attn_fwd(qkv5[:, :, 0], qkv5[:, :, 1], qkv5[:, :, 2], True, scale)
        o2 = o.view(B * T, D)
        x1 = ops.linear_fwd(o2, Wproj, residual=x2)
        ctx.save_for_backward(x2, ln_w, rstd, h, qkv, o, lse, Wqkv, Wproj)
        ctx.meta = (B, T, D, n_head, scale)
        return x1.view(B, T, D)

    @staticmethod
    def backward(ctx, dx1):
        x2, ln_w, rstd, h, qkv, o, lse, Wqkv, Wproj = ctx.saved_tensors
        B, T, D, H, scale = ctx.meta
        dx1 = dx1.reshape(B * T, D)
        if not dx1.is_contiguous():
            dx1 = dx1.contiguous()
        dev = dx1.device
        # the weight gradients run on a side stream beside the dX chain: the
        # fork is taken where their inputs are ready, and each dX GEMM is
        # queued before its dW partner so that the critical path gets the SMs
        side = ops.dw_side_stream(dev)                     # dx1, o ready
        do = ops.linear_dx(dx1, Wproj)                     # d(attn out)
        gWproj = ops.weight_grad(dx1, o.view(B * T, D), Wproj, side) if ctx.needs_input_grad[3] else None
        qkv5 = qkv.view(B, T, 3, H, D // H)
        dqkv = torch.empty_like(qkv)
        d5 = dqkv.view(B, T, 3, H, D // H)
        _attn_bwd(qkv5[:, :, 0], qkv5[:, :, 1], qkv5[:, :, 2], o, lse, do.view(B, T, H, D // H),
                  True, scale, d5[:, :, 0], d5[:, :, 1], d5[:, :, 2])
        if side is not None:
            side = ops.dw_side_stream(dev)                 # dqkv ready
        dh = ops.linear_dx(dqkv, Wqkv)
        gWqkv = ops.weight_grad(dqkv, h, Wqkv, side) if ctx.needs_input_grad[2] else None
        dx, gln = rmsnorm_bwd(x2, ln_w, rstd, dh, dres=dx1, need_dw=ctx.needs_input_grad[1])
        ops.dw_join(side, dev)
        return dx.view(B, T, D), gln, gWqkv, gWproj, None, None


class _MLPBlock(torch.autograd.Function):
    """x2 = x1 + fc2(gelu_tanh(fc(rms_norm(x1))))"""

    @staticmethod
    def forward(ctx, x, ln_w, W1, W2, eps):
        B, T, D = x.shape
        _norm_check(x, ln_w)
        x2 = x.reshape(B * T, D)
        h, rstd = rmsnorm_fwd(x2, ln_w, eps)
        F = W1.shape[0]
        # gz = gelu'(z) is saved instead of the pre-activation z: the forward
        # epilogue gets it from the same tanh as gelu(z), and the backward's
        # dz = (dy W2) * gz becomes a plain multiply in its epilogue
        gz = torch.empty(B * T, F, device=x.device, dtype=x.dtype)
        a = torch.empty(B * T, F, device=x.device, dtype=x.dtype)
        ops.gemm(h, W1, a, epilogue=ops.EPI_GELU_DERIV, Z=gz)
        y = ops.linear_fwd(a, W2, residual=x2)
        ctx.save_for_backward(x2, ln_w, rstd, h, gz, a, W1, W2)
        ctx.shape = (B, T, D)
        return y.view(B, T, D)

    @staticmethod
    def backward(ctx, dy):
        x2, ln_w, rstd, h, gz, a, W1, W2 = ctx.saved_tensors
        B, T, D = ctx.shape
        d2 = dy.reshape(B * T, D)
        if not d2.is_contiguous():
            d2 = d2.contiguous()
        dev = d2.device
        # the weight gradients run on a side stream beside the dX chain (see
        # _AttnBlock.backward)
        side = ops.dw_side_stream(dev)                     # d2, a ready
        dz = torch.empty_like(gz)
        ops.gemm(d2, W2, dz, b_trans=True, epilogue=ops.EPI_MUL, R=gz)   # (dy W2) * gelu'(z)
        gW2 = ops.weight_grad(d2, a, W2, side) if ctx.needs_input_grad[3] else None
        if side is not None:
            side = ops.dw_side_stream(dev)                 # dz ready
        dh = ops.linear_dx(dz, W1)
        gW1 = ops.weight_grad(dz, h, W1, side) if ctx.needs_input_grad[2] else None
        dx, gln = rmsnorm_bwd(x2, ln_w, rstd, dh, dres=d2, need_dw=ctx.needs_input_grad[1])
        ops.dw_join(side, dev)
        return dx.view(B, T, D), gln, gW1, gW2, None


def attn_block(x, ln_w, Wqkv, Wproj, eps, n_head):
    """x + proj(causal_attention(qkv(rms_norm(x, ln_w, eps)))) in one Function."""
    return _AttnBlock.apply(x, ln_w, Wqkv, Wproj, float(eps), int(n_head))


def mlp_block(x, ln_w, W1, W2, eps):
    """x + fc2(gelu_tanh(fc(rms_norm(x, ln_w, eps)))) in one Function."""
    return _MLPBlock.apply(x, ln_w, W1, W2, float(eps))
