"""fxlm.cross_entropy: fused CE and linear-CE on sm_100a.

Semantics of the reference (ml/fxlm/cross_entropy.py): `fused_cross_entropy`
writes the gradient (softmax - onehot) * scale / n_valid in the forward pass
(:77-99); `linear_cross_entropy` computes loss = CE(x W^T) chunk by chunk,
producing dx and an fp32 dW already in forward and only rescaling them in
backward (:107-149); with grad disabled it takes a loss-only path (:170-199).
B200 changes: the logits GEMM, dx GEMM and split-K dW GEMM run on the tcgen05
kernel; the CE kernel overwrites the logits chunk with its gradient in place;
the default chunk is bounded by memory, not by the iGPU's ~50 GFLOP budget:
all rows while their 16-bit logits fit in 1 GiB, else 1 GiB chunks. On B200
fewer, larger chunks are faster because the dx GEMM of a chunk (chunk x D
output) only fills the 148 SMs at a few thousand rows: at the config-4 head
(8192 x 768 x 32768) one 537 MB chunk takes 1.49 ms forward + backward,
2048-row chunks (134 MB) 1.66 ms and the reference's 768-row chunks (50 MB)
2.12 ms.
"""
import torch

from fxb200 import _lib
from fxb200 import ops

_DTYPES = (torch.float16, torch.bfloat16, torch.float32)


def _inv_nvalid(target, ignore_index):
    """1/n_valid as a device tensor (0 when n_valid == 0); no host sync.
    Follows ml/fxlm/cross_entropy.py:41-45."""
    nv = (target != ignore_index).sum(dtype=torch.float32)
    return torch.where(nv > 0, nv.reciprocal(), nv)


def _ce_rows(logits, target, grad, row_loss, mul, ignore_index):
    """One launch: row_loss[r] = CE of row r (0 if ignored); grad (may alias
    logits) written. The caller sums row_loss in a fixed order."""
    N, V = logits.shape
    _lib.call("fxb_ce_fwd_grad", _lib.dtype_code(logits.dtype), _lib.ptr(logits),
              logits.stride(0), _lib.ptr(target), _lib.ptr(grad), _lib.ptr(row_loss),
              _lib.ptr(mul), N, V, int(ignore_index), _lib.stream_ptr(logits.device))


def _check_logits(logits, target):
    """Validation of ml/fxlm/cross_entropy.py:62-74 (dtype widened)."""
    if logits.dtype not in _DTYPES:
        raise TypeError(f"logits must be bf16/fp16/fp32, got {logits.dtype}")
    if not (logits.is_cuda and target.is_cuda):
        raise TypeError("logits and target must be cuda tensors")
    if not logits.is_contiguous() or not target.is_contiguous():
        raise ValueError("logits and target must be contiguous")
    if target.dtype != torch.int64:
        raise TypeError(f"target must be int64, got {target.dtype}")
    if logits.dim() != 2 or target.dim() != 1 or target.shape[0] != logits.shape[0]:
        raise ValueError(f"expected logits (N,V) and target (N,): "
                         f"{tuple(logits.shape)} vs {tuple(target.shape)}")


class _FusedCE(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, target, ignore_index):
        _check_logits(logits, target)
        N, V = logits.shape
        dev = logits.device
        inv_n = _inv_nvalid(target, ignore_index)
        row_loss = torch.empty(N, device=dev, dtype=torch.float32)
        grad = torch.empty(N, V, device=dev, dtype=logits.dtype)
        _ce_rows(logits, target, grad, row_loss, inv_n, ignore_index)
        ctx.save_for_backward(grad)
        return row_loss.sum() * inv_n

    @staticmethod
    def backward(ctx, g):
        (grad,) = ctx.saved_tensors
        out = torch.empty_like(grad)
        ops.axpy(out, grad, scale=g.float().reshape(()).contiguous(), accumulate=False)
        return out, None, None


def fused_cross_entropy(logits, target, ignore_index=-100):
    """logits (N,V), target (N,) int64 -> fp32 scalar mean loss over valid rows."""
    return _FusedCE.apply(logits, target, int(ignore_index))


def _auto_chunk(N, D, V):
    """Rows per chunk: all rows while the (rows, V) 16-bit logits stay within
    1 GiB, else a multiple of 128 rows that does."""
    cap = max(128, ((1 << 30) // (2 * V)) // 128 * 128)
    return N if N <= cap else cap


def _check_lin(x, weight, target):
    """Validation of ml/fxlm/cross_entropy.py:152-167 (bf16, fp16 or fp32)."""
    if x.dtype not in _DTYPES or weight.dtype != x.dtype:
        raise TypeError(f"x and weight must share bf16, fp16 or fp32 ({x.dtype}, {weight.dtype})")
    if not (x.is_cuda and weight.is_cuda and target.is_cuda):
        raise TypeError("all tensors must be cuda tensors")
    if not (x.is_contiguous() and weight.is_contiguous() and target.is_contiguous()):
        raise ValueError("x, weight, target must be contiguous")
    if target.dtype != torch.int64:
        raise TypeError("target must be int64")
    N, D = x.shape
    V, Dw = weight.shape
    if Dw != D or target.shape != (N,):
        raise ValueError(f"shape mismatch: x{tuple(x.shape)} W{tuple(weight.shape)} "
                         f"t{tuple(target.shape)}")
    return N, D, V


class _LinearCE(torch.autograd.Function):
    """loss = CE(x @ W.T, target) with the logits materialised one chunk at a
    time (at most 1 GiB of them, see _auto_chunk); dx and dW are produced in
    forward like the reference."""

    @staticmethod
    def forward(ctx, x, weight, target, grad_scale, ignore_index, chunk_rows):
        N, D, V = _check_lin(x, weight, target)
        dev = x.device
        if chunk_rows is None:
            chunk_rows = _auto_chunk(N, D, V)
        inv_n = _inv_nvalid(target, ignore_index)
        gs_t = (grad_scale if torch.is_tensor(grad_scale)
                else torch.tensor(float(grad_scale), device=dev, dtype=torch.float32))
        mul = inv_n * gs_t.float()
        row_loss = torch.empty(N, device=dev, dtype=torch.float32)
        dx = torch.empty(N, D, device=dev, dtype=x.dtype)
        dW = torch.zeros(V, D, device=dev, dtype=torch.float32)
        dl_buf = torch.empty(min(chunk_rows, N), V, device=dev, dtype=x.dtype)
        for r0 in range(0, N, chunk_rows):
            r1 = min(r0 + chunk_rows, N)
            xc = x[r0:r1]
            dl = dl_buf[:r1 - r0]
            ops.gemm(xc, weight, dl)                          # logits chunk
            _ce_rows(dl, target[r0:r1], dl, row_loss[r0:r1], mul, ignore_index)  # in place
            # dx and dW only read dl: dW runs on the weight-gradient side
            # stream beside dx, joined before the next chunk overwrites dl
            side = ops.dw_side_stream(dev)
            ops.gemm(dl, weight, dx[r0:r1], b_trans=True)     # dx chunk
            if side is not None:
                with torch.cuda.stream(side):
                    ops.linear_dw_into(dl, xc, dW)            # dW += dl^T x (fp32)
                ops.dw_join(side, dev)
            else:
                ops.linear_dw_into(dl, xc, dW)
        ctx.save_for_backward(dx, dW)
        ctx.grad_scale = grad_scale
        ctx.weight = weight
        return row_loss.sum() * inv_n

    @staticmethod
    def backward(ctx, g):
        dx, dW = ctx.saved_tensors
        gs = ctx.grad_scale
        inv = torch.reciprocal(gs.float()) if torch.is_tensor(gs) else 1.0 / float(gs)
        s = (g.float() * inv).reshape(()).contiguous()
        gx = torch.empty_like(dx)
        ops.axpy(gx, dx, scale=s, accumulate=False)
        weight = ctx.weight
        gw = None
        if ctx.needs_input_grad[1]:
            sink = ops.param_grad_sink(weight)
            if sink is not None:
                ops.axpy(sink, dW, scale=s, accumulate=True)
            else:
                gw = torch.empty(dW.shape, device=dW.device, dtype=weight.dtype)
                ops.axpy(gw, dW, scale=s, accumulate=False)
        ctx.weight = None
        return gx, gw, None, None, None, None


def _linear_ce_loss_only(x, weight, target, ignore_index, chunk_rows):
    """Grad-disabled path: no dx/dW/dlogits buffers (ml/fxlm/cross_entropy.py:170-183).

    16-bit inputs take fxb_linear_ce_loss: the logits never leave the chip
    (the GEMM epilogue reduces each tile to per-row softmax statistics in
    tensor memory and registers; chunk_rows does not apply). fp32 inputs keep
    the chunk loop on the fp32 kernels."""
    N, D, V = _check_lin(x, weight, target)
    dev = x.device
    inv_n = _inv_nvalid(target, ignore_index)
    row_loss = torch.empty(N, device=dev, dtype=torch.float32)
    if x.dtype != torch.float32 and D % 8 == 0 and V % 8 == 0:
        lib = _lib.load()
        ws = torch.empty(max(16, int(lib.fxb_linear_ce_loss_workspace(N, V))), device=dev,
                         dtype=torch.uint8)
        _lib.call("fxb_linear_ce_loss", _lib.dtype_code(x.dtype), _lib.ptr(x), x.stride(0),
                  _lib.ptr(weight), weight.stride(0), _lib.ptr(target), _lib.ptr(row_loss),
                  _lib.ptr(ws), N, D, V, int(ignore_index), _lib.stream_ptr(dev))
        return row_loss.sum() * inv_n
    if chunk_rows is None:
        chunk_rows = _auto_chunk(N, D, V)
    buf = torch.empty(min(chunk_rows, N), V, device=dev, dtype=x.dtype)
    for r0 in range(0, N, chunk_rows):
        r1 = min(r0 + chunk_rows, N)
        lg = buf[:r1 - r0]
        ops.gemm(x[r0:r1], weight, lg)
        _ce_rows(lg, target[r0:r1], None, row_loss[r0:r1], inv_n, ignore_index)
    return row_loss.sum() * inv_n


def linear_cross_entropy(x, weight, target, grad_scale=1.0, ignore_index=-100,
                         chunk_rows=None):
    """x (N,D), weight (V,D) bf16/fp16, target (N,) int64 -> fp32 loss.

    grad_scale: python float or 0-dim fp32 cuda tensor (loss scale).
    chunk_rows: None -> all rows while their logits fit in 1 GiB, else 1 GiB
    chunks (a multiple of 128 rows).
    Without grad the loss-only path is used (no dx/dW allocation).
    """
    if not (torch.is_grad_enabled() and (x.requires_grad or weight.requires_grad)):
        return _linear_ce_loss_only(x, weight, target, ignore_index, chunk_rows)
    return _LinearCE.apply(x, weight, target, grad_scale, int(ignore_index), chunk_rows)
