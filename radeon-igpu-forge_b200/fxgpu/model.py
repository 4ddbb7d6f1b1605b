"""fxgpu.model: WindowMLP — 3-layer MLP over window inputs (B200 build).

Same structure, parameters, init scales and methods as the reference
(ml/fxgpu/model.py:15-57): L1 = gathered-window linear K -> hidden, act,
hidden -> hidden2, act, hidden2 -> 1; master=True keeps fp32 parameters and
computes in the 16-bit dtype; forward_dense is the unfused twin used for
parity. Additions: `act` ("silu" as the reference, or "gelu" as BASELINE
config 5) and `dtype` (fp16 as the reference, or bf16).

The training forward is one autograd Function over the sm_100a kernels:
gather -> GEMM(+bias, +act, pre-activation kept) -> GEMM(+bias, +act) ->
GEMM(+bias); backward folds each activation derivative into the epilogue of
the next dX GEMM, and weight / bias gradients go straight into FlatAdamW's
flat fp32 buffer when the parameters are managed by it.
"""
import torch
from torch import nn
import torch.nn.functional as Fn

from fxb200 import ops
from .fused_linear import FusedGatherLinear, gather_windows, bias_grad

_EPI_ACT = {"silu": ops.EPI_BIAS_SILU, "gelu": ops.EPI_BIAS_GELU}
_EPI_DACT = {"silu": ops.EPI_DSILU, "gelu": ops.EPI_DGELU}


class _PadCache:
    """Persistent zero-padded copies for the 1-output head: the GEMM wants
    N % 8 == 0, so W3 / b3 are written into row 0 of 8-row buffers and dy into
    column 0 of a (B, 8) buffer; rows / columns 1..7 stay zero. The buffers
    are allocated once per shape and refreshed in place each call (no
    per-step allocation or zero fill, and stable addresses under CUDA-graph
    capture)."""

    def __init__(self):
        self.bufs = {}

    def get(self, name, shape, like):
        key = (name, tuple(shape), like.dtype, like.device)
        t = self.bufs.get(key)
        if t is None:
            t = torch.zeros(shape, device=like.device, dtype=like.dtype)
            self.bufs[key] = t
        return t

    def pad_rows(self, W, b, rows=8):
        Wp = self.get("W", (rows, W.shape[1]), W)
        bp = self.get("b", (rows,), b)
        Wp[:W.shape[0]].copy_(W)
        bp[:b.shape[0]].copy_(b)
        return Wp, bp

    def pad_cols(self, dy, dtype, cols=8):
        d8 = self.get("dy", (dy.shape[0], cols), torch.empty((), device=dy.device, dtype=dtype))
        d8[:, :dy.shape[1]].copy_(dy)
        return d8


class _WindowMLPFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, X16, idx32, W1, b1, W2, b2, W3, b3, act, window, pads):
        B = idx32.numel()
        dev, dt = X16.device, X16.dtype
        Xg = gather_windows(X16, idx32, window)
        H1, H2 = W1.shape[0], W2.shape[0]
        z1 = torch.empty(B, H1, device=dev, dtype=dt)
        a1 = torch.empty(B, H1, device=dev, dtype=dt)
        ops.gemm(Xg, W1, a1, epilogue=_EPI_ACT[act], Z=z1, bias=b1)
        z2 = torch.empty(B, H2, device=dev, dtype=dt)
        a2 = torch.empty(B, H2, device=dev, dtype=dt)
        ops.gemm(a1, W2, a2, epilogue=_EPI_ACT[act], Z=z2, bias=b2)
        W3p, b3p = pads.pad_rows(W3, b3)
        y8 = torch.empty(B, W3p.shape[0], device=dev, dtype=dt)
        ops.gemm(a2, W3p, y8, epilogue=ops.EPI_BIAS, bias=b3p)
        ctx.save_for_backward(Xg, z1, a1, z2, a2, W1, b1, W2, b2, W3, b3, W3p)
        ctx.act = act
        ctx.pads = pads
        return y8[:, :W3.shape[0]].contiguous()

    @staticmethod
    def backward(ctx, dy):
        Xg, z1, a1, z2, a2, W1, b1, W2, b2, W3, b3, W3p = ctx.saved_tensors
        act = ctx.act
        dy8 = ctx.pads.pad_cols(dy, z1.dtype, W3p.shape[0])
        # layer 3
        dz2 = torch.empty_like(z2)
        ops.gemm(dy8, W3p, dz2, b_trans=True, epilogue=_EPI_DACT[act], R=z2)
        sink3 = ops.param_grad_sink(W3)
        if sink3 is not None:
            dW3p = ctx.pads.get("dW3", W3p.shape, torch.empty((), device=dy.device, dtype=torch.float32))
            dW3p.zero_()
            ops.linear_dw_into(dy8, a2, dW3p)
            sink3.add_(dW3p[:W3.shape[0]])
            gW3 = None
        else:
            gW3 = ops.weight_grad(dy8, a2, W3p)[:W3.shape[0]].contiguous()
        gb3 = bias_grad(dy.contiguous().to(z1.dtype), b3)  # (B, 1): no copy in the usual case
        # layer 2
        dz1 = torch.empty_like(z1)
        ops.gemm(dz2, W2, dz1, b_trans=True, epilogue=_EPI_DACT[act], R=z1)
        gW2 = ops.weight_grad(dz2, a1, W2)
        gb2 = bias_grad(dz2, b2)
        # layer 1 (input layer: no gradient for X)
        gW1 = ops.weight_grad(dz1, Xg, W1)
        gb1 = bias_grad(dz1, b1)
        ctx.pads = None
        return None, None, gW1, gb1, gW2, gb2, gW3, gb3, None, None, None


class WindowMLP(nn.Module):
    def __init__(self, n_feat, window, hidden=256, hidden2=128, master=True, dropout=0.0,
                 act="silu", dtype=torch.float16):
        super().__init__()
        if act not in _EPI_ACT:
            raise ValueError(f"act must be one of {sorted(_EPI_ACT)}")
        self.n_feat = n_feat
        self.window = window
        self.master = master
        self.dropout = dropout
        self.act = act
        self.cdtype = dtype
        pdtype = torch.float32 if master else dtype
        K = window * n_feat
        self.W1 = nn.Parameter(torch.randn(hidden, K, dtype=pdtype) * 0.03)
        self.b1 = nn.Parameter(torch.zeros(hidden, dtype=pdtype))
        self.W2 = nn.Parameter(torch.randn(hidden2, hidden, dtype=pdtype) * 0.06)
        self.b2 = nn.Parameter(torch.zeros(hidden2, dtype=pdtype))
        self.W3 = nn.Parameter(torch.randn(1, hidden2, dtype=pdtype) * 0.1)
        self.b3 = nn.Parameter(torch.zeros(1, dtype=pdtype))
        self._pads = _PadCache()

    def _half_params(self):
        ps = (self.W1, self.b1, self.W2, self.b2, self.W3, self.b3)
        return [p if p.dtype == self.cdtype else p.to(self.cdtype) for p in ps]

    def _act(self, h):
        return Fn.silu(h) if self.act == "silu" else Fn.gelu(h, approximate="tanh")

    def _trunk(self, h1, W2, b2, W3, b3):
        h = self._act(h1)
        if self.dropout > 0 and self.training:
            h = Fn.dropout(h, p=self.dropout)
        h = self._act(Fn.linear(h, W2, b2))
        return Fn.linear(h, W3, b3)

    def forward(self, X16, idx32):
        """X16 (R,F) + idx32 (B,) -> (B,1) logit in the compute dtype."""
        W1, b1, W2, b2, W3, b3 = self._half_params()
        if self.dropout > 0 and self.training:
            h1 = FusedGatherLinear.apply(X16, idx32, W1, b1)
            return self._trunk(h1, W2, b2, W3, b3)
        return _WindowMLPFn.apply(X16, idx32, W1, b1, W2, b2, W3, b3, self.act, self.window,
                                  self._pads)

    def forward_dense(self, xb16):
        """Same computation from a pre-gathered (B,K) batch (parity twin)."""
        W1, b1, W2, b2, W3, b3 = self._half_params()
        h1 = Fn.linear(xb16, W1, b1)
        return self._trunk(h1, W2, b2, W3, b3)
