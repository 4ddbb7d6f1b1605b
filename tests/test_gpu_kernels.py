"""GPU parity tests of the sm_100a kernels through the C ABI (ctypes).

Each op is compared with an fp32 PyTorch computation on the same rounded
inputs, with the reference's own tolerance rule (ml/fxlm/selftest.py:49-53):
max|ours - fp32| <= 2 * max|torch_lowp - fp32| + 1e-3, where torch_lowp is the
same op run by PyTorch in the low-precision dtype.
"""
import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

DTYPES = [torch.bfloat16, torch.float16]


def rule(ours, ref32, lowp):
    e_our = (ours.float() - ref32).abs().max().item()
    e_lp = (lowp.float() - ref32).abs().max().item()
    return e_our <= 2 * e_lp + 1e-3, e_our, e_lp


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda")


@pytest.fixture(autouse=True)
def _no_expired_waits(dev):
    """Every test must leave the device error word (expired bounded waits) at 0."""
    yield
    from fxb200 import _lib
    code = _lib.device_error(clear=True)
    assert code == 0, f"a kernel's bounded wait expired (device error word {code})"


# ------------------------------------------------------------------ RMSNorm
@pytest.mark.parametrize("dtype", DTYPES + [torch.float32])
@pytest.mark.parametrize("N,D", [(4, 8), (37, 64), (129, 768), (1000, 512), (8192, 768), (33, 2048),
                                 (5, 1032), (300, 1536), (33, 4096), (17, 8192), (1000, 8192)])
def test_rms_norm(dev, dtype, N, D):
    from fxlm.norm import rms_norm
    torch.manual_seed(N * 1000 + D)
    x = (torch.randn(N, D, device=dev) * 3).to(dtype)
    w = (torch.randn(D, device=dev) * 0.5 + 1).to(dtype)
    g = torch.randn(N, D, device=dev).to(dtype)
    xq, wq = x.detach().clone().requires_grad_(), w.detach().clone().requires_grad_()
    xr, wr = x.detach().float().clone().requires_grad_(), w.detach().float().clone().requires_grad_()
    xt, wt = x.detach().clone().requires_grad_(), w.detach().clone().requires_grad_()
    y = rms_norm(xq, wq, 1e-6)
    yr = F.rms_norm(xr, (D,), wr, 1e-6)
    yt = F.rms_norm(xt, (D,), wt, 1e-6)
    y.backward(g); yr.backward(g.float()); yt.backward(g)
    for ours, ref, lp, nm in ((y, yr, yt, "y"), (xq.grad, xr.grad, xt.grad, "dx"),
                              (wq.grad, wr.grad, wt.grad, "dw")):
        ok, e, b = rule(ours, ref.detach(), lp)
        if dtype == torch.float32:
            ok = e <= 1e-5 * max(1.0, ref.abs().max().item())
        assert ok, f"{nm}: err {e:.3e} vs torch-lowp {b:.3e}"


# ------------------------------------------------------------------ fused CE
@pytest.mark.parametrize("dtype", DTYPES + [torch.float32])
@pytest.mark.parametrize("N,V", [(5, 32), (100, 512), (301, 8192), (64, 32768), (7, 50), (3, 40000)])
def test_fused_ce(dev, dtype, N, V):
    from fxlm.cross_entropy import fused_cross_entropy
    torch.manual_seed(N + V)
    lg = (torch.randn(N, V, device=dev) * 4).to(dtype)
    tg = torch.randint(0, V, (N,), device=dev)
    tg[::7] = -100
    l32 = F.cross_entropy(lg.float(), tg, ignore_index=-100)
    l16 = F.cross_entropy(lg, tg, ignore_index=-100)
    lq = fused_cross_entropy(lg, tg, -100)
    ok1, e1, b1 = rule(lq, l32, l16)
    lg2 = lg.detach().clone().requires_grad_()
    lg3 = lg.detach().float().clone().requires_grad_()
    lg4 = lg.detach().clone().requires_grad_()
    fused_cross_entropy(lg2, tg, -100).backward()
    F.cross_entropy(lg3, tg, ignore_index=-100).backward()
    F.cross_entropy(lg4, tg, ignore_index=-100).backward()
    ok2, e2, b2 = rule(lg2.grad, lg3.grad, lg4.grad)
    if dtype == torch.float32:
        ok1 = e1 <= 1e-5 * max(1.0, l32.abs().item())
        ok2 = e2 <= 1e-6
    assert ok1, f"loss err {e1} vs {b1}"
    assert ok2, f"grad err {e2} vs {b2}"


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("N,V", [(1000, 32768), (445, 24576)])
def test_ce_rows_in_shared_memory(dev, dtype, N, V):
    """Rows of 48-72 KB go through shared memory (one bulk copy in, one out):
    gradient written over the logits (in place, as the linear-CE chunk loop
    does), ignored and out-of-range targets, masked (-inf) columns, leading
    -inf vectors, loss-only calls; per-row losses against fp32 torch."""
    from fxb200 import _lib
    torch.manual_seed(N)
    lg = (torch.randn(N, V, device=dev) * 4).to(dtype)
    lg[:, :40] = float("-inf")          # a thread's first vectors all masked
    lg[3, 1000:2000] = float("-inf")
    tg = torch.randint(40, V, (N,), device=dev)
    tg[::9] = -100
    tg[5] = V + 3                       # out of range: treated as ignored
    tg[3] = 3000                        # outside row 3's masked columns
    valid = (tg >= 0) & (tg < V)
    ref32 = torch.where(valid, F.cross_entropy(lg.float(), tg.clamp(0, V - 1), reduction="none"),
                        torch.zeros((), device=dev))
    p = torch.softmax(lg.float(), dim=1)
    p[valid.nonzero().squeeze(1), tg[valid]] -= 1.0
    gref = p * (valid.float() / N)[:, None]
    st = _lib.stream_ptr(dev)
    mul = torch.full((), 1.0 / N, device=dev)
    loss = torch.empty(N, device=dev)
    loss2 = torch.empty(N, device=dev)
    _lib.call("fxb_ce_fwd_grad", _lib.dtype_code(dtype), _lib.ptr(lg), V, _lib.ptr(tg), None,
              _lib.ptr(loss2), _lib.ptr(mul), N, V, -100, st)
    buf = lg.clone()
    _lib.call("fxb_ce_fwd_grad", _lib.dtype_code(dtype), _lib.ptr(buf), V, _lib.ptr(tg), _lib.ptr(buf),
              _lib.ptr(loss), _lib.ptr(mul), N, V, -100, st)
    torch.cuda.synchronize()
    assert torch.equal(loss, loss2)
    assert (loss - ref32).abs().max().item() <= 1e-4 * max(1.0, ref32.abs().max().item())
    err = (buf.float() - gref).abs().max().item()
    assert err <= 2e-2 * gref.abs().max().item(), err
    assert not torch.isnan(buf.float()).any()


# ------------------------------------------------------------------ GEMM
@pytest.fixture(params=["1sm", "2sm"])
def gemm_mode(request, monkeypatch):
    """Run each GEMM case through the 1-SM and the 2-SM (cta_group::2) kernel."""
    monkeypatch.setenv("FXB_GEMM_FORCE", request.param)
    return request.param


def _gemm_ref(A, B, a_trans, b_trans):
    Af = A.float().t() if a_trans else A.float()
    Bf = B.float().t() if b_trans else B.float()
    return Af @ Bf.t()


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("a_trans,b_trans", [(False, False), (False, True), (True, True), (True, False)])
@pytest.mark.parametrize("M,N,K", [(128, 128, 64), (256, 512, 256), (200, 136, 72),
                                   (1000, 768, 768), (8192, 2304, 768), (64, 3072, 8192)])
def test_gemm_store(dev, gemm_mode, dtype, a_trans, b_trans, M, N, K):
    from fxb200 import ops
    torch.manual_seed(M + N + K)
    A = (torch.randn(K, M, device=dev) if a_trans else torch.randn(M, K, device=dev)).to(dtype)
    B = (torch.randn(K, N, device=dev) if b_trans else torch.randn(N, K, device=dev)).to(dtype)
    C = torch.empty(M, N, device=dev, dtype=dtype)
    ops.gemm(A, B, C, a_trans=a_trans, b_trans=b_trans)
    ref = _gemm_ref(A, B, a_trans, b_trans)
    err = (C.float() - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-2, f"rel err {err:.3e}"


@pytest.mark.parametrize("epi", ["store", "residual", "dgelu"])
@pytest.mark.parametrize("M,N,K,b_trans", [(8192, 768, 3072, False), (8192, 768, 2304, True),
                                           (512, 1024, 4096, False), (2000, 520, 1032, True)])
def test_gemm_tail_split(dev, gemm_mode, epi, M, N, K, b_trans):
    """Tail split: the tiles left over after the full waves are cut along K
    and their fp32 partial tiles reduced through the workspace. Same result
    as the reference within the tolerance, bitwise equal on a second call
    (fixed reduction order, counters reset) and equal to the call without a
    workspace (no split) to fp32 rounding."""
    import ctypes
    from fxb200 import _lib, ops
    dtype = torch.bfloat16
    pair, bn, sp = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
    code = {"store": ops.EPI_STORE, "residual": ops.EPI_RESIDUAL, "dgelu": ops.EPI_DGELU}[epi]
    _lib.call("fxb_gemm_plan", M, N, K, code, ctypes.byref(pair), ctypes.byref(bn), ctypes.byref(sp))
    torch.manual_seed(M + K)
    A = (torch.randn(M, K, device=dev) / math.sqrt(K)).to(dtype)
    B = (torch.randn(K, N, device=dev) if b_trans else torch.randn(N, K, device=dev)).to(dtype)
    R = torch.randn(M, N, device=dev).to(dtype)
    kw = {} if epi == "store" else dict(epilogue=code, R=R)
    C1 = torch.empty(M, N, device=dev, dtype=dtype)
    C2 = torch.empty_like(C1)
    ops.gemm(A, B, C1, b_trans=b_trans, **kw)
    ops.gemm(A, B, C2, b_trans=b_trans, **kw)
    acc = _gemm_ref(A, B, False, b_trans)
    if epi == "residual":
        ref = acc + R.float()
    elif epi == "dgelu":
        x = R.float()
        t = torch.tanh(0.7978845608028654 * (x + 0.044715 * x ** 3))
        ref = acc * (0.5 * (1 + t) + 0.5 * x * (1 - t * t) * 0.7978845608028654 * (1 + 3 * 0.044715 * x * x))
    else:
        ref = acc
    err = (C1.float() - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-2, f"rel err {err:.3e}"
    assert torch.equal(C1, C2), "second call differs (counters not reset or order not fixed)"
    # the same GEMM without a workspace (no tail split)
    a = _lib.GemmArgs()
    a.dtype, a.M, a.N, a.K = _lib.dtype_code(dtype), M, N, K
    a.A, a.lda, a.a_trans = A.data_ptr(), K, 0
    a.B, a.ldb, a.b_trans = B.data_ptr(), (N if b_trans else K), int(b_trans)
    C3 = torch.empty_like(C1)
    a.C, a.ldc, a.c_dtype = C3.data_ptr(), N, _lib.dtype_code(dtype)
    a.epilogue, a.alpha = code, 1.0
    if epi != "store":
        a.R, a.ldr = R.data_ptr(), N
    _lib.check(_lib.load().fxb_gemm(ctypes.byref(a), _lib.stream_ptr(dev)), "fxb_gemm")
    torch.cuda.synchronize()
    d = (C1.float() - C3.float()).abs().max().item()
    assert d <= 2e-2 * max(1.0, C3.float().abs().max().item()), d
    if gemm_mode == "2sm" and (M, N, K) == (8192, 768, 3072):
        assert sp.value > 1, "tail split expected for this shape"


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("M,N,K", [(300, 264, 136), (4096, 3072, 768)])
def test_gemm_epilogues(dev, gemm_mode, dtype, M, N, K):
    from fxb200 import ops
    torch.manual_seed(7)
    A = (torch.randn(M, K, device=dev) / math.sqrt(K)).to(dtype)
    B = torch.randn(N, K, device=dev).to(dtype)
    acc = A.float() @ B.float().t()
    tol = 1e-2 * acc.abs().max().item()
    # residual (in place)
    R = torch.randn(M, N, device=dev).to(dtype)
    C = R.clone()
    ops.gemm(A, B, C, epilogue=ops.EPI_RESIDUAL, R=C)
    assert (C.float() - (acc + R.float())).abs().max().item() < tol + 1e-2
    # gelu with pre-activation
    Z = torch.empty(M, N, device=dev, dtype=dtype)
    C = torch.empty(M, N, device=dev, dtype=dtype)
    ops.gemm(A, B, C, epilogue=ops.EPI_GELU, Z=Z)
    assert (Z.float() - acc).abs().max().item() < tol
    assert (C.float() - F.gelu(Z.float(), approximate="tanh")).abs().max().item() < 2e-2
    # dgelu
    zz = torch.randn(M, N, device=dev).to(dtype)
    ops.gemm(A, B, C, epilogue=ops.EPI_DGELU, R=zz)
    zr = zz.float().requires_grad_()
    F.gelu(zr, approximate="tanh").backward(acc)
    assert (C.float() - zr.grad).abs().max().item() < 2e-2 * zr.grad.abs().max().item() + 1e-2
    # bias + gelu / bias + silu
    bias = torch.randn(N, device=dev).to(dtype)
    ops.gemm(A, B, C, epilogue=ops.EPI_BIAS_GELU, Z=Z, bias=bias)
    assert (Z.float() - (acc + bias.float())).abs().max().item() < tol + 2e-2
    ops.gemm(A, B, C, epilogue=ops.EPI_BIAS_SILU, Z=Z, bias=bias)
    assert (C.float() - F.silu(Z.float())).abs().max().item() < 2e-2
    ops.gemm(A, B, C, epilogue=ops.EPI_BIAS, bias=bias)
    assert (C.float() - (acc + bias.float())).abs().max().item() < tol + 2e-2
    # gelu + its derivative (both from the rounded pre-activation), then the
    # backward as a multiply by that derivative
    G = torch.empty(M, N, device=dev, dtype=dtype)
    ops.gemm(A, B, C, epilogue=ops.EPI_GELU_DERIV, Z=G)
    zq = acc.to(dtype).float().requires_grad_()
    gref = F.gelu(zq, approximate="tanh")
    gref.backward(torch.ones_like(gref))
    # (the kernel rounds its own fp32 accumulator: a pre-activation may land
    # one 16-bit ulp away from torch's, hence the magnitude-relative bound)
    assert (C.float() - gref.detach()).abs().max().item() < 1e-2 * gref.abs().max().item() + 2e-2
    assert (G.float() - zq.grad).abs().max().item() < 2e-2
    ops.gemm(A, B, C, epilogue=ops.EPI_MUL, R=G, alpha=0.5)
    assert (C.float() - 0.5 * acc * G.float()).abs().max().item() < 2e-2 * (acc * G.float()).abs().max().item() + 1e-2


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("M,N,K", [(333, 200, 96), (1024, 1032, 256)])
def test_gemm_output_layouts(dev, gemm_mode, dtype, M, N, K):
    """Outputs written through strided views (column slices of wider buffers),
    fp32 C with alpha, and ragged M / N tails; cells outside the view stay
    untouched."""
    from fxb200 import ops
    torch.manual_seed(M * 7 + N)
    A = (torch.randn(M, K, device=dev) / math.sqrt(K)).to(dtype)
    B = torch.randn(N, K, device=dev).to(dtype)
    acc = A.float() @ B.float().t()
    tol = 1e-2 * acc.abs().max().item()
    wide = torch.full((M, N + 72), 7.0, device=dev, dtype=dtype)
    zwide = torch.full((M, N + 24), 7.0, device=dev, dtype=dtype)
    C, Z = wide[:, 8:8 + N], zwide[:, 16:16 + N]
    ops.gemm(A, B, C, epilogue=ops.EPI_GELU, Z=Z)
    assert (Z.float() - acc).abs().max().item() < tol
    assert (C.float() - F.gelu(Z.float(), approximate="tanh")).abs().max().item() < 2e-2
    assert (wide[:, :8] == 7).all() and (wide[:, 8 + N:] == 7).all()
    assert (zwide[:, :16] == 7).all() and (zwide[:, 16 + N:] == 7).all()
    R = torch.randn(M, N, device=dev).to(dtype)
    ops.gemm(A, B, C, epilogue=ops.EPI_RESIDUAL, R=R)
    assert (C.float() - (acc + R.float())).abs().max().item() < tol + 1e-2
    assert (wide[:, :8] == 7).all() and (wide[:, 8 + N:] == 7).all()
    C32w = torch.full((M, N + 4), 7.0, device=dev)
    C32 = C32w[:, :N]
    ops.gemm(A, B, C32, alpha=0.25)
    assert (C32 - 0.25 * acc).abs().max().item() < 1e-3 * acc.abs().max().item()
    assert (C32w[:, N:] == 7).all()


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("Mtok,N,K", [(8192, 768, 768), (8192, 3072, 768), (1000, 264, 72)])
def test_gemm_dw_accum(dev, gemm_mode, dtype, Mtok, N, K):
    """dW (fp32) += dy^T x via split-K red.add, accumulating twice."""
    from fxb200 import ops
    torch.manual_seed(11)
    dy = torch.randn(Mtok, N, device=dev).to(dtype)
    x = torch.randn(Mtok, K, device=dev).to(dtype)
    dW = torch.zeros(N, K, device=dev, dtype=torch.float32)
    ops.linear_dw_into(dy, x, dW)
    ops.linear_dw_into(dy, x, dW, alpha=0.5)
    ref = 1.5 * (dy.float().t() @ x.float())
    err = (dW - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-4, f"rel err {err:.3e}"


# ------------------------------------------------------------------ attention
def _ref_attn(q, k, v, causal, scale):
    qt, kt, vt = (t.float().permute(0, 2, 1, 3) for t in (q, k, v))
    s = qt @ kt.transpose(-1, -2) * scale
    if causal:
        T = q.shape[1]
        mask = torch.ones(T, T, device=q.device, dtype=torch.bool).triu(1)
        s = s.masked_fill(mask, float("-inf"))
    return (torch.softmax(s, -1) @ vt).permute(0, 2, 1, 3)


def _sdpa(q, k, v, causal, scale):
    o = F.scaled_dot_product_attention(q.permute(0, 2, 1, 3), k.permute(0, 2, 1, 3),
                                       v.permute(0, 2, 1, 3), is_causal=causal, scale=scale)
    return o.permute(0, 2, 1, 3)


ATTN_CASES = [(1, 1, 1, 64), (1, 17, 1, 64), (2, 64, 2, 64), (1, 100, 8, 64), (3, 256, 8, 64),
              (2, 513, 2, 64), (1, 130, 4, 128), (2, 200, 8, 128), (1, 33, 1, 128),
              (2, 1024, 12, 64), (1, 1, 1, 128), (2, 257, 3, 128), (1, 1024, 4, 128)]


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("B,T,H,Dh", ATTN_CASES)
def test_attention(dev, dtype, causal, B, T, H, Dh):
    from fxlm.attention import flash_attention
    torch.manual_seed(B * 7 + T * 13 + Dh)
    scale = 1.0 / math.sqrt(Dh)
    qkv = torch.randn(B, T, 3, H, Dh, device=dev).to(dtype)
    q, k, v = (qkv[:, :, i].requires_grad_() for i in range(3))
    o = flash_attention(q, k, v, causal=causal, scale=scale)
    oref = _ref_attn(q.detach(), k.detach(), v.detach(), causal, scale)
    o16 = _sdpa(q.detach(), k.detach(), v.detach(), causal, scale)
    ok, e, b = rule(o, oref, o16)
    assert ok, f"fwd err {e} vs {b}"
    g = torch.randn_like(o)
    o.backward(g)
    qr, kr, vr = (t.detach().float().requires_grad_() for t in (q, k, v))
    _ref_attn(qr, kr, vr, causal, scale).backward(g.float())
    qt, kt, vt = (t.detach().clone().requires_grad_() for t in (q, k, v))
    _sdpa(qt, kt, vt, causal, scale).backward(g)
    for ours, ref, lp, nm in ((q.grad, qr.grad, qt.grad, "dq"), (k.grad, kr.grad, kt.grad, "dk"),
                              (v.grad, vr.grad, vt.grad, "dv")):
        ok, e, b = rule(ours, ref, lp)
        assert ok, f"{nm}: err {e} vs {b}"


@pytest.mark.parametrize("causal", [True, False])
def test_attention_qkv_and_lse(dev, causal):
    from fxlm.attention import flash_attention_qkv, _fwd
    torch.manual_seed(5)
    B, T, H, Dh = 2, 100, 4, 64
    qkv = torch.randn(B, T, 3, H, Dh, device=dev).to(torch.bfloat16).requires_grad_()
    o = flash_attention_qkv(qkv, causal=causal)
    q, k, v = qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]
    scale = 1.0 / math.sqrt(Dh)
    oref = _ref_attn(q.detach(), k.detach(), v.detach(), causal, scale)
    o16 = _sdpa(q.detach(), k.detach(), v.detach(), causal, scale)
    assert rule(o, oref, o16)[0]
    g = torch.randn_like(o)
    o.backward(g)
    qr, kr, vr = (t.detach().float().requires_grad_() for t in (q, k, v))
    _ref_attn(qr, kr, vr, causal, scale).backward(g.float())
    qt, kt, vt = (t.detach().clone().requires_grad_() for t in (q, k, v))
    _sdpa(qt, kt, vt, causal, scale).backward(g)
    for i, (rg, tg) in enumerate(((qr, qt), (kr, kt), (vr, vt))):
        assert rule(qkv.grad[:, :, i], rg.grad, tg.grad)[0], f"grad {i}"
    # logsumexp of the scaled scores, natural log
    _o, lse = _fwd(q.detach(), k.detach(), v.detach(), causal, scale)
    s = (q.detach().float().permute(0, 2, 1, 3) @ k.detach().float().permute(0, 2, 3, 1)) * scale
    if causal:
        s = s.masked_fill(torch.ones(T, T, device=dev, dtype=torch.bool).triu(1), float("-inf"))
    assert (lse - torch.logsumexp(s, -1)).abs().max().item() < 1e-2


# ------------------------------------------------------------------ embedding / axpy
def test_embedding(dev):
    from fxlm.model import _Embedding
    torch.manual_seed(3)
    V, D, B, T = 300, 64, 4, 50
    tok = torch.randn(V, D, device=dev).to(torch.bfloat16).requires_grad_()
    pos = torch.randn(T + 6, D, device=dev).to(torch.bfloat16).requires_grad_()
    idx = torch.randint(0, V, (B, T), device=dev)
    out = _Embedding.apply(idx, tok, pos)
    ref = tok.detach().float()[idx] + pos.detach().float()[:T]
    assert (out.float() - ref).abs().max().item() < 2e-2
    g = torch.randn(B, T, D, device=dev).to(torch.bfloat16)
    out.backward(g)
    gt = torch.zeros(V, D, device=dev).index_add_(0, idx.reshape(-1), g.float().reshape(-1, D))
    gp = torch.zeros(T + 6, D, device=dev)
    gp[:T] = g.float().sum(0)
    assert (tok.grad.float() - gt).abs().max().item() < 3e-2 * max(1.0, gt.abs().max().item())
    assert (pos.grad.float() - gp).abs().max().item() < 3e-2 * max(1.0, gp.abs().max().item())


@pytest.mark.parametrize("n", [8, 1000, 110_906_112 // 4 + 8])
def test_adamw_sumsq_deterministic(dev, n):
    """fxb_adamw_sumsq_det: the sum of squares (fp64 reference, fp32 rounding
    bound) and the non-finite flag of fxb_adamw_sumsq, bitwise identical on
    every call, with the workspace's ticket counter reset."""
    from fxb200 import _lib
    P, st = _lib.ptr, _lib.stream_ptr(dev)
    torch.manual_seed(11)
    g = torch.randn(n, device=dev) * 3.0
    ws = torch.zeros((int(_lib.load().fxb_adamw_sumsq_ws_bytes()) + 3) // 4, device=dev,
                     dtype=torch.int32)
    ref = float((g.double() ** 2).sum())
    outs = []
    for _ in range(3):
        sc = torch.zeros(2, device=dev)
        fl = torch.zeros((), device=dev, dtype=torch.int32)
        _lib.call("fxb_adamw_sumsq_det", 0, P(g), n, P(sc), P(fl), P(ws), st)
        torch.cuda.synchronize()
        outs.append(sc[0].item())
        assert int(fl) == 0
        assert int(ws[-1]) == 0  # the ticket counter (last word) is reset
    assert outs[0] == outs[1] == outs[2]
    assert abs(outs[0] - ref) <= 1e-5 * ref
    sc = torch.zeros(2, device=dev)
    fl = torch.zeros((), device=dev, dtype=torch.int32)
    _lib.call("fxb_adamw_sumsq", 0, P(g), n, P(sc), P(fl), st)
    torch.cuda.synchronize()
    assert abs(sc[0].item() - ref) <= 1e-5 * ref
    g[n // 2] = float("nan")
    sc.zero_()
    _lib.call("fxb_adamw_sumsq_det", 0, P(g), n, P(sc), P(fl), P(ws), st)
    torch.cuda.synchronize()
    assert int(fl) == 1


def test_device_error_word_clear(dev):
    from fxb200 import _lib
    torch.cuda.synchronize()
    assert _lib.device_error(clear=True) == 0


# ------------------------------------------------------------------ config 3 at full size
# RMSNorm over [65536, 768], the LM-head GEMM
# [65536, 768] x [32768, 768]^T and cross-entropy over [65536, 32768] logits,
# bf16, each with the plan the library picks for that shape (GEMM tile, split
# and tail split; CE row path). Checked against fp32 torch on every row where
# that is cheap and on seeded row samples where the fp32 reference would be
# tens of GB.
C3_N, C3_D, C3_V = 65536, 768, 32768


def test_config3_rms_norm_full_shape(dev):
    from fxlm.norm import rms_norm
    torch.manual_seed(31)
    x = (torch.randn(C3_N, C3_D, device=dev) * 3).to(torch.bfloat16)
    w = (torch.randn(C3_D, device=dev) * 0.5 + 1).to(torch.bfloat16)
    g = torch.randn(C3_N, C3_D, device=dev).to(torch.bfloat16)
    xq, wq = x.clone().requires_grad_(), w.clone().requires_grad_()
    xr, wr = x.float().requires_grad_(), w.float().requires_grad_()
    xt, wt = x.clone().requires_grad_(), w.clone().requires_grad_()
    y = rms_norm(xq, wq, 1e-6)
    yr = F.rms_norm(xr, (C3_D,), wr, 1e-6)
    yt = F.rms_norm(xt, (C3_D,), wt, 1e-6)
    y.backward(g); yr.backward(g.float()); yt.backward(g)
    for ours, ref, lp, nm in ((y, yr, yt, "y"), (xq.grad, xr.grad, xt.grad, "dx"),
                              (wq.grad, wr.grad, wt.grad, "dw")):
        ok, e, b = rule(ours, ref.detach(), lp)
        assert ok, f"{nm}: err {e:.3e} vs torch-lowp {b:.3e}"


def test_config3_head_gemms_full_shape(dev):
    """logits = x W^T, dx = dlogits W and dW += dlogits^T x at the config-3
    shapes through the head's own calls (fxb200.ops.linear_fwd / linear_dx /
    linear_dw_into); 512 sampled logits rows and dx rows, 256 sampled dW rows
    against fp32 matmuls of the same bf16 inputs."""
    import ctypes
    from fxb200 import _lib, ops
    plans = []
    for M, N, K, epi in ((C3_N, C3_V, C3_D, ops.EPI_STORE), (C3_N, C3_D, C3_V, ops.EPI_STORE),
                         (C3_V, C3_D, C3_N, ops.EPI_ACCUM_F32)):
        pair, bn, sp = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
        _lib.call("fxb_gemm_plan", M, N, K, epi, ctypes.byref(pair), ctypes.byref(bn), ctypes.byref(sp))
        plans.append((pair.value, bn.value, sp.value))
    torch.manual_seed(32)
    x = (torch.randn(C3_N, C3_D, device=dev)).to(torch.bfloat16)
    W = (torch.randn(C3_V, C3_D, device=dev) * 0.02).to(torch.bfloat16)
    logits = ops.linear_fwd(x, W)
    rows = torch.randint(0, C3_N, (512,), device=dev, generator=torch.Generator(dev).manual_seed(7))
    ref = x[rows].float() @ W.float().t()
    err = (logits[rows].float() - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-2, f"logits rel err {err:.3e} (plan {plans[0]})"
    del logits, ref
    dl = (torch.randn(C3_N, C3_V, device=dev) * 1e-3).to(torch.bfloat16)
    dx = ops.linear_dx(dl, W)
    ref = dl[rows].float() @ W.float()
    err = (dx[rows].float() - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-2, f"dx rel err {err:.3e} (plan {plans[1]})"
    del dx, ref
    dw = torch.zeros(C3_V, C3_D, device=dev, dtype=torch.float32)
    ops.linear_dw_into(dl, x, dw)
    vrows = torch.randint(0, C3_V, (256,), device=dev, generator=torch.Generator(dev).manual_seed(8))
    ref = dl[:, vrows].float().t() @ x.float()
    err = (dw[vrows] - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-3, f"dW rel err {err:.3e} (plan {plans[2]})"


def test_config3_cross_entropy_full_shape(dev):
    """Per-row losses of all 65536 rows against fp32 torch (in 4096-row
    chunks), and the in-place gradient (softmax - onehot) / N on 256 sampled
    rows, with ignored targets."""
    from fxb200 import _lib
    torch.manual_seed(33)
    N, V = C3_N, C3_V
    lg = (torch.randn(N, V, device=dev) * 4).to(torch.bfloat16)
    tg = torch.randint(0, V, (N,), device=dev)
    tg[::11] = -100
    valid = tg >= 0
    st = _lib.stream_ptr(dev)
    mul = torch.full((), 1.0 / N, device=dev)
    loss = torch.empty(N, device=dev)
    buf = lg.clone()
    _lib.call("fxb_ce_fwd_grad", _lib.dtype_code(torch.bfloat16), _lib.ptr(buf), V, _lib.ptr(tg),
              _lib.ptr(buf), _lib.ptr(loss), _lib.ptr(mul), N, V, -100, st)
    torch.cuda.synchronize()
    worst = 0.0
    for r0 in range(0, N, 4096):
        sl = slice(r0, r0 + 4096)
        ref = F.cross_entropy(lg[sl].float(), tg[sl].clamp(min=0), reduction="none")
        ref = torch.where(valid[sl], ref, torch.zeros((), device=dev))
        worst = max(worst, (loss[sl] - ref).abs().max().item())
    assert worst <= 1e-4 * 20, f"per-row loss err {worst}"
    rows = torch.randint(0, N, (256,), device=dev, generator=torch.Generator(dev).manual_seed(9))
    p = torch.softmax(lg[rows].float(), dim=1)
    vr = valid[rows]
    p[vr.nonzero().squeeze(1), tg[rows][vr]] -= 1.0
    gref = p * (vr.float() / N)[:, None]
    err = (buf[rows].float() - gref).abs().max().item()
    assert err <= 2e-2 * gref.abs().max().item(), err
    assert not torch.isnan(buf[rows].float()).any()
