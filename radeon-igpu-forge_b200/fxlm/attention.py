"""fxlm.attention: flash attention on tcgen05 tensor cores (sm_100a).

Same surface as the reference (ml/fxlm/attention.py): q, k, v are (B,T,H,Dh)
views with unit stride on Dh and free other strides (so the fused qkv buffer
is used without copies); o is returned (B,T,H,Dh) contiguous and lse (B,H,T)
fp32 is saved for backward. Dh in {64, 128}, forward and backward. dtype:
bf16 or fp16 on the tcgen05 kernels (the reference is fp16 only), or fp32 on
the library's fp32 kernels (the 1e-5 parity mode).
"""
import ctypes
import math

import torch

from fxb200 import _lib


def _check_qkv(q, k, v):
    """Validation of ml/fxlm/attention.py:57-79 (dtype widened to bf16/fp16/fp32)."""
    if q.dim() != 4 or k.shape != q.shape or v.shape != q.shape:
        raise ValueError(f"q, k, v must share one 4-D shape: {tuple(q.shape)} "
                         f"{tuple(k.shape)} {tuple(v.shape)}")
    B, T, H, Dh = q.shape
    if Dh not in (64, 128):
        raise ValueError(f"head_dim {Dh} not supported (64 or 128)")
    if T < 1 or B < 1 or H < 1:
        raise ValueError(f"invalid shape: {tuple(q.shape)}")
    for nm, t in (("q", q), ("k", k), ("v", v)):
        if t.dtype not in (torch.float16, torch.bfloat16, torch.float32) or t.dtype != q.dtype:
            raise TypeError(f"{nm} must be bf16, fp16 or fp32 (and match q), got {t.dtype}")
        if not t.is_cuda:
            raise TypeError(f"{nm} must be a cuda tensor")
        if t.stride(-1) != 1:
            raise ValueError(f"{nm} last axis must be contiguous (stride(-1)={t.stride(-1)})")
    if q.numel() >= 2 ** 31:
        raise ValueError("tensor too large (2^31 element limit)")
    return B, T, H, Dh


def _strides3(t):
    s = t.stride()
    return s[0], s[1], s[2]


def _args(q, k, v, causal, scale):
    B, T, H, Dh = q.shape
    a = _lib.AttnArgs()
    a.dtype = _lib.dtype_code(q.dtype)
    a.B, a.T, a.H, a.D = B, T, H, Dh
    a.scale = float(scale)
    a.causal = int(bool(causal))
    a.q = q.data_ptr(); a.q_sb, a.q_st, a.q_sh = _strides3(q)
    a.k = k.data_ptr(); a.k_sb, a.k_st, a.k_sh = _strides3(k)
    a.v = v.data_ptr(); a.v_sb, a.v_st, a.v_sh = _strides3(v)
    return a


def _fwd(q, k, v, causal, scale):
    B, T, H, Dh = _check_qkv(q, k, v)
    dev = q.device
    o = torch.empty(B, T, H, Dh, device=dev, dtype=q.dtype)
    lse = torch.empty(B, H, T, device=dev, dtype=torch.float32)
    a = _args(q, k, v, causal, scale)
    a.o = o.data_ptr(); a.o_sb, a.o_st, a.o_sh = _strides3(o)
    a.lse = lse.data_ptr()
    _lib.check(_lib.load().fxb_attn_fwd(ctypes.byref(a), _lib.stream_ptr(dev)), "fxb_attn_fwd")
    return o, lse


def _bwd(q, k, v, o, lse, do, causal, scale, dq, dk, dv):
    B, T, H, Dh = q.shape
    do = do.contiguous()
    dev = q.device
    lib = _lib.load()
    ws = torch.empty(lib.fxb_attn_bwd_workspace(B, T, H, Dh) // 4 + 4, device=dev,
                     dtype=torch.float32)
    a = _args(q, k, v, causal, scale)
    a.o = o.data_ptr(); a.o_sb, a.o_st, a.o_sh = _strides3(o)
    a.lse = lse.data_ptr()
    a.dout = do.data_ptr(); a.do_sb, a.do_st, a.do_sh = _strides3(do)
    a.dq = dq.data_ptr(); a.dq_sb, a.dq_st, a.dq_sh = _strides3(dq)
    a.dk = dk.data_ptr(); a.dk_sb, a.dk_st, a.dk_sh = _strides3(dk)
    a.dv = dv.data_ptr(); a.dv_sb, a.dv_st, a.dv_sh = _strides3(dv)
    a.workspace = ws.data_ptr()
    _lib.check(lib.fxb_attn_bwd(ctypes.byref(a), _lib.stream_ptr(dev)), "fxb_attn_bwd")
    return dq, dk, dv


class _FlashAttn(torch.autograd.Function):
    """flash_attention(q,k,v): o (B,T,H,Dh) contiguous."""

    @staticmethod
    def forward(ctx, q, k, v, causal, scale):
        o, lse = _fwd(q, k, v, causal, scale)
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.causal, ctx.scale = causal, scale
        return o

    @staticmethod
    def backward(ctx, do):
        q, k, v, o, lse = ctx.saved_tensors
        dq = torch.empty(q.shape, device=q.device, dtype=q.dtype)
        dk = torch.empty(q.shape, device=q.device, dtype=q.dtype)
        dv = torch.empty(q.shape, device=q.device, dtype=q.dtype)
        _bwd(q, k, v, o, lse, do, ctx.causal, ctx.scale, dq, dk, dv)
        return dq, dk, dv, None, None


class _FlashAttnQKV(torch.autograd.Function):
    """flash_attention_qkv(qkv): qkv (B,T,3,H,Dh) contiguous; one dqkv buffer."""

    @staticmethod
    def forward(ctx, qkv, causal, scale):
        if qkv.dim() != 5 or qkv.shape[2] != 3:
            raise ValueError(f"qkv must be (B,T,3,H,Dh), got {tuple(qkv.shape)}")
        if not qkv.is_contiguous():
            raise ValueError("qkv must be contiguous")
        q, k, v = qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]
        o, lse = _fwd(q, k, v, causal, scale)
        ctx.save_for_backward(qkv, o, lse)
        ctx.causal, ctx.scale = causal, scale
        return o

    @staticmethod
    def backward(ctx, do):
        qkv, o, lse = ctx.saved_tensors
        dqkv = torch.empty_like(qkv)
        _bwd(qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2], o, lse, do, ctx.causal, ctx.scale,
             dqkv[:, :, 0], dqkv[:, :, 1], dqkv[:, :, 2])
        return dqkv, None, None


def flash_attention(q, k, v, causal=True, scale=None):
    """q,k,v (B,T,H,Dh) -> o (B,T,H,Dh)."""
    Dh = q.shape[-1]
    if scale is None:
        scale = 1.0 / math.sqrt(Dh)
    return _FlashAttn.apply(q, k, v, causal, float(scale))


def flash_attention_qkv(qkv, causal=True, scale=None):
    """qkv (B,T,3,H,Dh) contiguous -> o (B,T,H,Dh)."""
    if qkv.dim() != 5:
        raise ValueError(f"qkv must be (B,T,3,H,Dh), got {tuple(qkv.shape)}")
    Dh = qkv.shape[-1]
    if scale is None:
        scale = 1.0 / math.sqrt(Dh)
    return _FlashAttnQKV.apply(qkv, causal, float(scale))
