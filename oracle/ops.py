"""CPU oracle for the per-op math of the reference hot path (numpy, float64).

TEST INFRASTRUCTURE ONLY. This module restates, in plain numpy, what the
reference's kernels compute so that tests can check the sm_100a kernels
against it. Nothing in the product path imports it; only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg may.

Each function cites the reference code it restates (paths relative to the
reference repository). Arithmetic is carried out in float64 so the oracle is
a tighter reference than either fp32 or 16-bit device math.

Parity pin: tests/test_oracle.py checks these functions against golden
vectors produced by the reference's own PyTorch code paths
(tests/golden/make_golden.py).
"""
import numpy as np

F64 = np.float64


def _f(a):
    return np.asarray(a, dtype=F64)


# ---------------------------------------------------------------- RMSNorm
def rms_norm_fwd(x, w, eps):
    """y = x * rsqrt(mean(x^2) + eps) * w, rstd per row.
    ml/fxlm/kernels/norm.hip:33-59 (rms_norm_fwd)."""
    x = _f(x)
    rstd = 1.0 / np.sqrt((x * x).mean(-1, keepdims=True) + eps)
    return x * rstd * _f(w), rstd[..., 0]


def rms_norm_bwd(x, w, rstd, dy):
    """dx = rstd*w*dy - x * rstd^3 * sum(x*w*dy) / D ; dw = sum_rows x*rstd*dy.
    ml/fxlm/kernels/norm.hip:64-95 (dx) and :102-127 (dw partials) summed as
    ml/fxlm/norm.py:82."""
    x, w, dy = _f(x), _f(w), _f(dy)
    r = _f(rstd)[..., None]
    D = x.shape[-1]
    t = (x * w * dy).sum(-1, keepdims=True)
    dx = r * w * dy - x * (r ** 3) * t / D
    dw = (x * r * dy).reshape(-1, D).sum(0)
    return dx, dw


# ---------------------------------------------------------------- cross entropy
def ce_fwd_grad(logits, target, mul, ignore_index=-100):
    """Row-wise CE with the gradient written in the same pass.
    loss_sum = sum over valid rows of (logsumexp(row) - row[t]);
    grad = (softmax(row) - onehot(t)) * mul, zero for rows whose target is
    ignore_index or outside [0, V).  ml/fxlm/kernels/ce.hip:32-116."""
    lg = _f(logits)
    N, V = lg.shape
    t = np.asarray(target, dtype=np.int64)
    valid = (t != ignore_index) & (t >= 0) & (t < V)
    m = lg.max(-1, keepdims=True)
    e = np.exp(lg - m)
    Z = e.sum(-1, keepdims=True)
    lse = (m + np.log(Z))[:, 0]
    tt = np.where(valid, t, 0)
    xt = lg[np.arange(N), tt]
    loss_sum = float(np.sum(np.where(valid, lse - xt, 0.0)))
    p = e / Z
    p[np.arange(N), tt] -= 1.0
    grad = np.where(valid[:, None], p * mul, 0.0)
    return loss_sum, grad


def inv_nvalid(target, ignore_index=-100):
    """1 / n_valid (0 if none).  ml/fxlm/cross_entropy.py:41-45."""
    nv = int((np.asarray(target) != ignore_index).sum())
    return 1.0 / nv if nv > 0 else 0.0


def fused_cross_entropy(logits, target, ignore_index=-100):
    """Mean CE over valid rows and its gradient wrt logits.
    ml/fxlm/cross_entropy.py:77-99."""
    inv = inv_nvalid(target, ignore_index)
    loss_sum, grad = ce_fwd_grad(logits, target, inv, ignore_index)
    return loss_sum * inv, grad


def linear_cross_entropy(x, W, target, ignore_index=-100):
    """loss = CE(x W^T) mean over valid rows; returns (loss, dx, dW) of the
    unscaled loss. ml/fxlm/cross_entropy.py:107-149 (the chunking and the
    grad_scale round trip cancel out: gx = dx * g / grad_scale)."""
    x, W = _f(x), _f(W)
    logits = x @ W.T
    loss, dl = fused_cross_entropy(logits, target, ignore_index)
    return loss, dl @ W, dl.T @ x


# ---------------------------------------------------------------- attention
def attention_fwd(q, k, v, causal, scale):
    """o = softmax(q k^T * scale) v with the causal mask key <= query;
    lse = logsumexp of the scaled scores (natural log), shape (B,H,T).
    ml/fxlm/kernels/attention.hip:104-224; q,k,v,o are (B,T,H,D)."""
    q, k, v = _f(q), _f(k), _f(v)
    qt, kt, vt = (a.transpose(0, 2, 1, 3) for a in (q, k, v))  # (B,H,T,D)
    s = qt @ kt.transpose(0, 1, 3, 2) * scale
    T = q.shape[1]
    if causal:
        s = np.where(np.triu(np.ones((T, T), dtype=bool), 1), -np.inf, s)
    m = s.max(-1, keepdims=True)
    e = np.exp(s - m)
    Z = e.sum(-1, keepdims=True)
    p = e / Z
    o = (p @ vt).transpose(0, 2, 1, 3)
    lse = (m + np.log(Z))[..., 0]
    return o, lse


def attention_bwd(q, k, v, o, lse, do, causal, scale):
    """delta = rowsum(dO*O) (attention.hip:229-251); P = exp(s*scale - lse);
    dP = dO V^T; dS = P*(dP - delta); dQ = dS K * scale; dK = dS^T Q * scale;
    dV = P^T dO  (attention.hip:256-534)."""
    q, k, v, o, do = _f(q), _f(k), _f(v), _f(o), _f(do)
    qt, kt, vt, ot, dot = (a.transpose(0, 2, 1, 3) for a in (q, k, v, o, do))
    T = q.shape[1]
    s = qt @ kt.transpose(0, 1, 3, 2) * scale
    p = np.exp(s - _f(lse)[..., None])
    if causal:
        p = np.where(np.triu(np.ones((T, T), dtype=bool), 1), 0.0, p)
    delta = (dot * ot).sum(-1, keepdims=True)
    dp = dot @ vt.transpose(0, 1, 3, 2)
    ds = p * (dp - delta)
    dq = ds @ kt * scale
    dk = ds.transpose(0, 1, 3, 2) @ qt * scale
    dv = p.transpose(0, 1, 3, 2) @ dot
    back = lambda a: a.transpose(0, 2, 1, 3)  # noqa: E731
    return back(dq), back(dk), back(dv), delta[..., 0]


# ---------------------------------------------------------------- GELU / linears
def gelu_tanh(x):
    """torch.nn.functional.gelu(approximate="tanh"), used at ml/fxlm/model.py:71."""
    x = _f(x)
    return 0.5 * x * (1.0 + np.tanh(np.sqrt(2.0 / np.pi) * (x + 0.044715 * x ** 3)))


def gelu_tanh_grad(x):
    x = _f(x)
    u = np.sqrt(2.0 / np.pi) * (x + 0.044715 * x ** 3)
    t = np.tanh(u)
    du = np.sqrt(2.0 / np.pi) * (1.0 + 3 * 0.044715 * x * x)
    return 0.5 * (1.0 + t) + 0.5 * x * (1.0 - t * t) * du


def silu(x):
    x = _f(x)
    return x / (1.0 + np.exp(-x))


# ---------------------------------------------------------------- FlatAdamW
def adamw_sumsq(grad):
    """(sum g^2, any non-finite).  ml/fxlm/kernels/optim.hip:26-75."""
    g = _f(grad)
    return float((g * g).sum()), bool(~np.isfinite(g).all())


def adamw_final(sumsq, bad, scale, max_norm, step):
    """found_inf, norm, clip coefficient and the step counter.
    ml/fxlm/kernels/optim.hip:77-93."""
    bad = bad or not np.isfinite(sumsq)
    norm = np.sqrt(sumsq) / scale
    clip = 0.0 if bad else min(1.0, max_norm / (norm + 1e-6))
    return bad, norm, clip, (step if bad else step + 1)


def adamw_update(master, m, v, grad, wd_mask, clip, scale, step, lr, b1, b2, eps, wd):
    """Decoupled-weight-decay AdamW on flat arrays (no-op when found_inf is
    handled by the caller). ml/fxlm/kernels/optim.hip:96-162."""
    master, m, v, g = _f(master).copy(), _f(m).copy(), _f(v).copy(), _f(grad) * (clip / scale)
    bc1 = 1.0 - b1 ** step
    bc2 = 1.0 - b2 ** step
    master = np.where(wd_mask, master - lr * wd * master, master)
    m = m * b1 + (1.0 - b1) * g
    v = v * b2 + (1.0 - b2) * g * g
    master = master - lr * (m / bc1) / (np.sqrt(v / bc2) + eps)
    return master, m, v


def amp_update_scale(scale, growth, found_inf, growth_factor=2.0, backoff=0.5, interval=1000):
    """torch._amp_update_scale_ as called at ml/fxlm/optim.py:170-171."""
    if found_inf:
        return scale * backoff, 0
    growth += 1
    if growth == interval:
        return scale * growth_factor, 0
    return scale, growth


# ---------------------------------------------------------------- fxgpu gather-linear
def gather_window(X, idx, window):
    """Xg[b, w*F + f] = X[idx[b] + w, f] (window-major flattening).
    ml/fxgpu/fused_linear.py:28-33; ml/fxgpu/selftest.py:36-40."""
    X = _f(X)
    idx = np.asarray(idx, dtype=np.int64)
    rows = idx[:, None] + np.arange(window)[None, :]
    return X[rows].reshape(len(idx), -1)


def gather_linear_fwd(X, idx, W, bias):
    """out = Xg W^T + bias.  ml/fxgpu/gather_gemm.hip:17-180."""
    K = W.shape[1]
    F = X.shape[1]
    Xg = gather_window(X, idx, K // F)
    return Xg @ _f(W).T + _f(bias), Xg
