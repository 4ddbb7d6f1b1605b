"""fxb_rmsnorm_bwd_static (no allocation, file-scope device scratch) against
fxb_rmsnorm_bwd (caller workspace), through the C ABI, and on its own against
fp32 PyTorch autograd.

Two calls of the static entry in a row on different shapes and inputs (the
second one reuses the scratch the first one left behind), each compared with
the workspace entry on the same inputs and with F.rms_norm's fp32 gradients;
then the size limit.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda")


def _inputs(dev, rows, D, dtype, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    x = (torch.randn(rows, D, generator=g) * 2).to(dtype).to(dev)
    w = (torch.randn(D, generator=g) * 0.5 + 1).to(dtype).to(dev)
    dy = torch.randn(rows, D, generator=g).to(dtype).to(dev)
    dres = torch.randn(rows, D, generator=g).to(dtype).to(dev)
    rstd = torch.rsqrt(x.float().pow(2).mean(-1) + 1e-6).contiguous()
    dw0 = torch.randn(D, generator=g).to(dev)  # fp32 slot the accumulate case adds to
    return x, w, dy, dres, rstd, dw0


def _bwd(lib_call, static, x, w, rstd, dy, dres, dw, acc):
    from fxb200 import _lib
    rows, D = x.shape
    dx = torch.empty_like(x)
    common = (_lib.dtype_code(x.dtype), _lib.ptr(x), _lib.ptr(w), _lib.ptr(rstd), _lib.ptr(dy),
              _lib.ptr(dres), _lib.ptr(dx), _lib.ptr(dw), _lib.dtype_code(dw.dtype), acc)
    if static:
        lib_call("fxb_rmsnorm_bwd_static", *common, rows, D, _lib.stream_ptr(x.device))
    else:
        nbytes = _lib.load().fxb_rmsnorm_bwd_workspace(rows, D)
        ws = torch.empty(max(1, nbytes // 4), device=x.device, dtype=torch.float32)
        lib_call("fxb_rmsnorm_bwd", *common, _lib.ptr(ws), rows, D, _lib.stream_ptr(x.device))
    torch.cuda.synchronize()
    return dx


def test_static_scratch_matches_workspace_entry_twice(dev):
    from fxb200 import _lib
    cases = [
        # rows, D, dtype, seed, with dres, accumulate into dw
        (8192, 768, torch.bfloat16, 11, False, 0),
        (1000, 512, torch.float16, 12, True, 1),
    ]
    for rows, D, dtype, seed, with_res, acc in cases:
        x, w, dy, dres, rstd, dw0 = _inputs(dev, rows, D, dtype, seed)
        res = dres if with_res else None
        dw_ref, dw_new = dw0.clone(), dw0.clone()
        dx_ref = _bwd(_lib.call, False, x, w, rstd, dy, res, dw_ref, acc)
        dx_new = _bwd(_lib.call, True, x, w, rstd, dy, res, dw_new, acc)
        # same kernels with the same block count: equal up to a tolerance of
        # 1e-6 relative (they are expected to agree exactly)
        torch.testing.assert_close(dx_new.float(), dx_ref.float(), rtol=1e-6, atol=1e-6)
        torch.testing.assert_close(dw_new, dw_ref, rtol=1e-6, atol=1e-6)
        # and on its own against fp32 autograd through F.rms_norm on the same
        # rounded inputs, with the reference's tolerance rule (2 x the error
        # of torch's own low-precision backward, + 1e-3)
        gx32, gw32 = _torch_grads(x, w, dy, torch.float32)
        gx16, gw16 = _torch_grads(x, w, dy, dtype)
        if with_res:
            gx32 = gx32 + dres.float()
            gx16 = (gx16.float() + dres.float()).to(dtype)
        if acc:
            gw32 = gw32 + dw0
            gw16 = gw16.float() + dw0
        for ours, r32, lp, nm in ((dx_new, gx32, gx16, "dx"), (dw_new, gw32, gw16, "dw")):
            e_our = (ours.float() - r32).abs().max().item()
            e_lp = (lp.float() - r32).abs().max().item()
            assert e_our <= 2 * e_lp + 1e-3, f"{nm} ({rows}x{D}): err {e_our:.3e} vs torch-lowp {e_lp:.3e}"
    assert _lib.device_error(clear=True) == 0


def _torch_grads(x, w, dy, dtype):
    """d(rms_norm(x, w)) / dx and / dw contracted with dy, by PyTorch autograd
    in `dtype` (eps 1e-6, as the rstd the test passes)."""
    import torch.nn.functional as F
    xr = x.detach().to(dtype).requires_grad_()
    wr = w.detach().to(dtype).requires_grad_()
    F.rms_norm(xr, (x.shape[1],), wr, 1e-6).backward(dy.to(dtype))
    return xr.grad, wr.grad.float()


def test_static_scratch_rejects_oversize(dev):
    from fxb200 import _lib
    lib = _lib.load()
    cap = lib.fxb_rmsnorm_bwd_static_max_bytes()
    assert cap == 4 << 20
    rows, D = 1 << 20, 8192  # partials for this shape exceed the static array
    assert lib.fxb_rmsnorm_bwd_workspace(rows, D) > cap
    x = torch.empty(16, D, device=dev, dtype=torch.bfloat16)  # never read: rejected first
    w = torch.ones(D, device=dev, dtype=torch.bfloat16)
    dw = torch.zeros(D, device=dev)
    rc = lib.fxb_rmsnorm_bwd_static(_lib.dtype_code(x.dtype), _lib.ptr(x), _lib.ptr(w), None,
                                    _lib.ptr(x), None, _lib.ptr(x), _lib.ptr(dw),
                                    _lib.dtype_code(dw.dtype), 0, rows, D,
                                    _lib.stream_ptr(dev))
    assert rc == -1
    assert b"static array holds" in lib.fxb_last_error()
