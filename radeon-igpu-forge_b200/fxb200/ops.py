"""Thin tensor-level helpers over the C ABI (GEMM, embedding, axpy).

These are the building blocks the reference-named ops (fxlm.*, fxgpu.*) call.
Every function launches on torch's current stream, allocates outputs with
torch (the library never allocates) and raises RuntimeError on failure.
"""
import ctypes
import os

import torch

from . import _lib
from ._lib import (EPI_STORE, EPI_RESIDUAL, EPI_GELU, EPI_DGELU, EPI_BIAS,  # noqa: F401
                   EPI_BIAS_GELU, EPI_BIAS_SILU, EPI_ACCUM_F32, EPI_DSILU,
                   EPI_GELU_DERIV, EPI_MUL)

_TC_DTYPES = (torch.bfloat16, torch.float16)
_GEMM_DTYPES = _TC_DTYPES + (torch.float32,)  # fp32: the library's fp32 parity-mode GEMM

# Optional per-launch timing of the GEMM (bench.py's live roofline): when a
# list is installed here, every gemm() appends (flops, start, end) with CUDA
# events recorded on the launching stream around the C-ABI call.
_GEMM_TIMING = None


def set_gemm_timing(records):
    """Install a list to collect (flops, start_event, end_event) per GEMM, or None."""
    global _GEMM_TIMING
    _GEMM_TIMING = records


# GEMM workspace (tail split, see fxb_gemm_args.workspace): one buffer per
# (device, stream) for eager launches, allocated on first use and kept. A
# captured CUDA graph gets workspaces of its own (see `graph_workspaces`), so
# two graphs, or a graph and eager launches, never share arrival counters.
# The first 4096 bytes are arrival counters that must be zero before a GEMM
# starts; GEMMs reset them themselves, except after an expired wait (device
# error word bit 1), when `_reset_workspaces` zeroes them.
_GEMM_WS = {}
_CAPTURE_WS = None  # dict of the graph being captured, or None


def _gemm_workspace(device):
    st = torch.cuda.current_stream(device)
    key = (device.index, st.cuda_stream)
    table = _CAPTURE_WS if _CAPTURE_WS is not None else _GEMM_WS
    ws = table.get(key)
    if ws is None:
        n = int(_lib.load().fxb_gemm_workspace_size())
        ws = torch.empty(n, device=device, dtype=torch.uint8)
        ws[:4096].zero_()  # the arrival counters (inside a capture: a memset node of the graph)
        table[key] = ws
    return ws


class graph_workspaces:
    """Context manager used around a CUDA-graph capture: GEMMs captured inside
    it use workspaces stored in `table` (owned by the graph object, alive as
    long as the graph), whose counters are zeroed by a memset node at the
    start of every replay's first GEMM on that stream."""

    def __init__(self, table):
        self.table = table

    def __enter__(self):
        global _CAPTURE_WS
        self.prev, _CAPTURE_WS = _CAPTURE_WS, self.table
        return self.table

    def __exit__(self, *exc):
        global _CAPTURE_WS
        _CAPTURE_WS = self.prev
        return False


def _reset_workspaces(code):
    """After an expired GEMM wait the owner of a tail tile may have left its
    counter non-zero: zero the counters of every eager workspace (graph
    workspaces are zeroed at the start of each replay)."""
    if code & _lib.DERR_GEMM_WAIT:
        for ws in _GEMM_WS.values():
            ws[:4096].zero_()


_lib._ON_DEVICE_ERROR.append(_reset_workspaces)


def _rowmajor(t, name):
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError(f"{name} must be a 2-D row-major view (stride(1) == 1)")
    return t.stride(0)


def gemm(A, B, out, *, a_trans=False, b_trans=False, epilogue=EPI_STORE, alpha=1.0,
         R=None, Z=None, bias=None):
    """out[M,N] = epilogue(opA(A) @ opB(B)^T) on tcgen05 tensor cores.

    opA(A) = A (M,K) or, with a_trans, A stored (K,M); opB(B) = B (N,K) or,
    with b_trans, B stored (K,N). A and B share one dtype (bf16 / fp16 on the
    tensor cores, or fp32: the fp32 parity-mode kernel, then every other
    tensor is fp32 too); `out`, R, Z and bias share out's dtype (fp32 out is
    required for EPI_ACCUM_F32).
    """
    if A.dtype not in _GEMM_DTYPES or B.dtype != A.dtype:
        raise TypeError(f"gemm operands must share bf16, fp16 or fp32 ({A.dtype}, {B.dtype})")
    if not (A.is_cuda and B.is_cuda and out.is_cuda):
        raise TypeError("gemm operands must be cuda tensors")
    lda = _rowmajor(A, "A")
    ldb = _rowmajor(B, "B")
    ldc = _rowmajor(out, "out")
    M = A.shape[1] if a_trans else A.shape[0]
    K = A.shape[0] if a_trans else A.shape[1]
    N = B.shape[1] if b_trans else B.shape[0]
    Kb = B.shape[0] if b_trans else B.shape[1]
    if Kb != K or tuple(out.shape) != (M, N):
        raise ValueError(f"gemm shape mismatch: A{tuple(A.shape)} B{tuple(B.shape)} "
                         f"out{tuple(out.shape)} a_trans={a_trans} b_trans={b_trans}")
    a = _lib.GemmArgs()
    a.dtype = _lib.dtype_code(A.dtype)
    a.M, a.N, a.K = M, N, K
    a.A, a.lda, a.a_trans = A.data_ptr(), lda, int(a_trans)
    a.B, a.ldb, a.b_trans = B.data_ptr(), ldb, int(b_trans)
    a.C, a.ldc, a.c_dtype = out.data_ptr(), ldc, _lib.dtype_code(out.dtype)
    a.epilogue = epilogue
    a.alpha = float(alpha)
    if R is not None:
        a.R, a.ldr = R.data_ptr(), _rowmajor(R, "R")
    if Z is not None:
        a.Z, a.ldz = Z.data_ptr(), _rowmajor(Z, "Z")
    if bias is not None:
        a.bias = bias.data_ptr()
    ws = _gemm_workspace(A.device)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    if _GEMM_TIMING is not None:
        st = torch.cuda.current_stream(A.device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(st)
        _lib.check(_lib.load().fxb_gemm(ctypes.byref(a), _lib.stream_ptr(A.device)), "fxb_gemm")
        e1.record(st)
        _GEMM_TIMING.append((2.0 * M * N * K, e0, e1))
        return out
    _lib.check(_lib.load().fxb_gemm(ctypes.byref(a), _lib.stream_ptr(A.device)), "fxb_gemm")
    return out


def linear_fwd(x2d, W, residual=None):
    """y = x W^T (+ residual)."""
    y = torch.empty(x2d.shape[0], W.shape[0], device=x2d.device, dtype=x2d.dtype)
    if residual is None:
        return gemm(x2d, W, y)
    return gemm(x2d, W, y, epilogue=EPI_RESIDUAL, R=residual)


def linear_dx(dy, W, out=None):
    """dx = dy W   (dy (M,N), W (N,K) -> (M,K))."""
    if out is None:
        out = torch.empty(dy.shape[0], W.shape[1], device=dy.device, dtype=dy.dtype)
    return gemm(dy, W, out, b_trans=True)


def linear_dw_into(dy, x, dw32, alpha=1.0):
    """dw32 (fp32, (N,K)) += alpha * dy^T x   (dy (M,N), x (M,K)); split-K red.add."""
    return gemm(dy, x, dw32, a_trans=True, b_trans=True, epilogue=EPI_ACCUM_F32, alpha=alpha)


def param_grad_sink(p):
    """fp32 flat-gradient view of a parameter managed by FlatAdamW, or None."""
    g = getattr(p, "_fxb_grad", None)
    if g is not None:
        owner = getattr(p, "_fxb_owner", None)
        if owner is not None:
            owner._grad_dirty = True
    return g


# Weight-gradient GEMMs on a side stream. A block's backward has dX GEMMs on
# its critical path and dW GEMMs that nothing in the block waits for; each
# persistent GEMM leaves SMs idle in its first and last waves. Forking the
# dW GEMMs onto a per-device side stream (when their inputs are ready) and
# joining it at the end of the block's backward lets them fill those SMs.
# The join happens while every input is still referenced, so the caching
# allocator never reuses memory a side-stream GEMM still reads; the gradient
# hooks of data parallelism and the optimizer run after the join. Inside a
# CUDA-graph capture the fork and join become graph edges.
# FXB_DW_STREAM=0 keeps everything on the current stream.
_DW_STREAMS = {}


def dw_side_stream(device):
    """The side stream for weight-gradient GEMMs on `device`, made to wait
    for all work queued so far on the current stream; None when disabled."""
    if os.environ.get("FXB_DW_STREAM", "1") == "0" or device.type != "cuda":
        return None
    side = _DW_STREAMS.get(device.index)
    if side is None:
        side = torch.cuda.Stream(device=device)
        _DW_STREAMS[device.index] = side
    side.wait_stream(torch.cuda.current_stream(device))
    return side


def dw_join(side, device):
    """The current stream waits for everything queued on `side`."""
    if side is not None:
        torch.cuda.current_stream(device).wait_stream(side)


def weight_grad(dy, x, W, side=None):
    """dW for y = x W^T: accumulated into W's flat fp32 slot when W belongs to
    a FlatAdamW (returns None), else returned as a tensor of W's dtype. With
    `side` (from dw_side_stream), the accumulation is queued on that stream;
    the caller joins it (dw_join) before the inputs can be freed."""
    sink = param_grad_sink(W)
    if sink is not None:
        if side is not None:
            with torch.cuda.stream(side):
                linear_dw_into(dy, x, sink.view(W.shape[0], W.shape[1]))
        else:
            linear_dw_into(dy, x, sink.view(W.shape[0], W.shape[1]))
        return None
    tmp = torch.zeros(W.shape[0], W.shape[1], device=W.device, dtype=torch.float32)
    linear_dw_into(dy, x, tmp)
    return tmp.to(W.dtype)


def axpy(dst, src, scale=None, accumulate=True):
    """dst (+)= src * (*scale)  elementwise over numel (scale: 0-dim fp32 cuda tensor)."""
    if dst.numel() != src.numel():
        raise ValueError("axpy: size mismatch")
    if not (dst.is_contiguous() and src.is_contiguous()):
        raise ValueError("axpy: tensors must be contiguous")
    _lib.call("fxb_axpy", _lib.dtype_code(dst.dtype), _lib.ptr(dst), _lib.dtype_code(src.dtype),
              _lib.ptr(src), _lib.ptr(scale), 1 if accumulate else 0, dst.numel(),
              _lib.stream_ptr(dst.device))
    return dst
