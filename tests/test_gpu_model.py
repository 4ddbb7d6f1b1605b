"""GPU parity tests at model level, against the oracle and the golden fixtures.

Cases follow the reference's selftest (ml/fxlm/selftest.py): linear-CE with a
tensor grad_scale, ignored targets and a chunk size that does not divide N
(:99-134), FlatAdamW grad-injection parity, inf skip, scale growth and grad
accumulation (:219-298), a GPT whose loss and every gradient match the fp32
reference (:301-333) and a 20-step run whose loss must fall (:335-352). The
bar of the B200 build (bf16): per-op outputs and gradients within 2e-2
relative, first-step loss within 1e-3 relative, 200-step loss curve within
2% of the reference.
"""
import json
import math
import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu
GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CFG1 = dict(vocab_size=256, seq_len=256, n_layer=4, n_head=4, d_model=256)


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda")


@pytest.fixture(autouse=True)
def _no_expired_waits(dev):
    yield
    from fxb200 import _lib
    assert _lib.device_error(clear=True) == 0


def rel(a, b):
    a, b = a.double().cpu(), b.double().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-30)).item()


@pytest.fixture(scope="module")
def golden_ops():
    return np.load(os.path.join(GOLD, "ops.npz"))


# ------------------------------------------------------------------ golden op vectors
def test_golden_rmsnorm(dev, golden_ops):
    from fxlm.norm import rms_norm
    g = golden_ops
    for k in ("rms_37x64", "rms_129x768"):
        x = torch.tensor(g[k + "_x"], device=dev).bfloat16().requires_grad_()
        w = torch.tensor(g[k + "_w"], device=dev).bfloat16().requires_grad_()
        y = rms_norm(x, w, 1e-6)
        y.backward(torch.tensor(g[k + "_dy"], device=dev).bfloat16())
        assert rel(y.float(), torch.tensor(g[k + "_y"])) < 2e-2
        assert rel(x.grad.float(), torch.tensor(g[k + "_dx"])) < 2e-2
        assert rel(w.grad.float(), torch.tensor(g[k + "_dw"])) < 2e-2


def test_golden_ce_and_linear_ce(dev, golden_ops):
    from fxlm.cross_entropy import fused_cross_entropy, linear_cross_entropy
    g = golden_ops
    for k in ("ce_100x512", "ce_33x8192"):
        lg = torch.tensor(g[k + "_logits"], device=dev).bfloat16().requires_grad_()
        tg = torch.tensor(g[k + "_target"], device=dev)
        loss = fused_cross_entropy(lg, tg, -100)
        loss.backward()
        assert abs(loss.item() - float(g[k + "_loss"])) <= 1e-3 * abs(float(g[k + "_loss"]))
        assert rel(lg.grad.float(), torch.tensor(g[k + "_grad"])) < 2e-2
    x = torch.tensor(g["lce_x"], device=dev).bfloat16().requires_grad_()
    W = torch.tensor(g["lce_W"], device=dev).bfloat16().requires_grad_()
    tg = torch.tensor(g["lce_target"], device=dev)
    loss = linear_cross_entropy(x, W, tg, grad_scale=1.0, chunk_rows=128)
    loss.backward()
    assert abs(loss.item() - float(g["lce_loss"])) <= 1e-3 * abs(float(g["lce_loss"]))
    assert rel(x.grad.float(), torch.tensor(g["lce_dx"])) < 2e-2
    assert rel(W.grad.float(), torch.tensor(g["lce_dW"])) < 2e-2


def test_golden_attention(dev, golden_ops):
    from fxlm.attention import flash_attention
    g = golden_ops
    for causal in (True, False):
        k = f"attn_c{int(causal)}"
        qkv = torch.tensor(g[k + "_qkv"], device=dev).bfloat16()
        q, kk, v = (qkv[:, :, i].clone().requires_grad_() for i in range(3))
        o = flash_attention(q, kk, v, causal=causal)
        o.backward(torch.tensor(g[k + "_do"], device=dev).bfloat16())
        assert rel(o.float(), torch.tensor(g[k + "_o"])) < 2e-2
        for t, nm in ((q, "_dq"), (kk, "_dk"), (v, "_dv")):
            assert rel(t.grad.float(), torch.tensor(g[k + nm])) < 2e-2, nm


# ------------------------------------------------------------------ linear-CE (selftest cases)
@pytest.mark.parametrize("N,D,V,gs", [(50, 64, 128, 1.0), (301, 256, 8192, 1.0), (1027, 512, 4096, None)])
def test_linear_ce_selftest_cases(dev, N, D, V, gs):
    from fxlm.cross_entropy import linear_cross_entropy
    torch.manual_seed(N + D + V)
    x = torch.randn(N, D, device=dev).bfloat16()
    W = (torch.randn(V, D, device=dev) * 0.02).bfloat16()
    tg = torch.randint(0, V, (N,), device=dev)
    tg[::11] = -100
    grad_scale = torch.tensor(65536.0, device=dev) if gs is None else gs
    xq, Wq = x.clone().requires_grad_(), W.clone().requires_grad_()
    xr, Wr = x.float().requires_grad_(), W.float().requires_grad_()
    lq = linear_cross_entropy(xq, Wq, tg, grad_scale=grad_scale, chunk_rows=128)
    lr = F.cross_entropy(xr @ Wr.t(), tg, ignore_index=-100)
    assert abs(lq.item() - lr.item()) <= 1e-3 * abs(lr.item())
    lq.backward(); lr.backward()
    assert rel(xq.grad.float(), xr.grad) < 2e-2
    assert rel(Wq.grad.float(), Wr.grad) < 2e-2


def test_linear_ce_no_grad_path(dev):
    """The loss-only path (logits kept on chip, fp32 logits) and the training
    path (bf16 logits) give the same loss within the bf16 rounding of the
    logits, and the loss-only result carries no graph."""
    from fxlm.cross_entropy import linear_cross_entropy
    torch.manual_seed(7)
    x = torch.randn(200, 128, device=dev).bfloat16()
    W = (torch.randn(512, 128, device=dev) * 0.02).bfloat16()
    tg = torch.randint(0, 512, (200,), device=dev)
    lg = linear_cross_entropy(x, W, tg, grad_scale=1.0)
    with torch.no_grad():
        ln = linear_cross_entropy(x, W, tg)
    assert ln.grad_fn is None and abs(float(ln) - float(lg)) < 1e-3 * abs(float(lg))


@pytest.mark.parametrize("N,D,V", [(1, 64, 8), (200, 128, 136), (1000, 64, 512), (777, 256, 4104),
                                   (4096, 768, 32768)])
def test_linear_ce_loss_on_chip(dev, N, D, V):
    """fxb_linear_ce_loss (logits reduced to per-row softmax statistics in the
    GEMM epilogue, never written) against fp32 PyTorch on the same 16-bit
    inputs: mean loss within 1e-3 relative, every row's loss within 2e-3 of
    its reference (ignored and out-of-range targets give 0), for vocabularies
    that end inside a tile and a single-row batch."""
    from fxb200 import _lib
    torch.manual_seed(N + D + V)
    for dt in (torch.bfloat16, torch.float16):
        x = torch.randn(N, D, device=dev).to(dt)
        W = (torch.randn(V, D, device=dev) * (2.0 / math.sqrt(D))).to(dt)
        tg = torch.randint(0, V, (N,), device=dev)
        tg[::7] = -100
        if N > 3:
            tg[3] = V + 5  # out of range: no loss, like an ignored row
        row = torch.empty(N, device=dev)
        lib = _lib.load()
        ws = torch.empty(int(lib.fxb_linear_ce_loss_workspace(N, V)), device=dev, dtype=torch.uint8)
        _lib.call("fxb_linear_ce_loss", _lib.dtype_code(dt), _lib.ptr(x), D, _lib.ptr(W), D, _lib.ptr(tg),
                  _lib.ptr(row), _lib.ptr(ws), N, D, V, -100, _lib.stream_ptr(dev))
        logits = x.float() @ W.float().t()
        valid = (tg != -100) & (tg >= 0) & (tg < V)
        ref = torch.zeros(N, device=dev)
        ref[valid] = torch.logsumexp(logits[valid], -1) - logits[valid].gather(1, tg[valid, None])[:, 0]
        assert (row - ref).abs().max().item() < 2e-3, (dt, (row - ref).abs().max().item())
        assert abs(row.sum().item() - ref.sum().item()) <= 1e-3 * abs(ref.sum().item()) + 1e-4


# ------------------------------------------------------------------ FlatAdamW
def test_flat_adamw_golden(dev, golden_ops):
    """Grad injection vs the reference selftest's torch AdamW + clip oracle
    (golden masters), master rel-err < 1e-5 and flat copy == master.half()."""
    from fxlm.optim import FlatAdamW
    g = golden_ops
    model = torch.nn.Sequential(torch.nn.Linear(64, 32, bias=False), torch.nn.LayerNorm(32),
                                torch.nn.Linear(32, 16, bias=False)).to(dev)
    with torch.no_grad():
        for i, p in enumerate(model.parameters()):
            p.copy_(torch.tensor(g[f"adamw_init_{i}"]))
    opt = FlatAdamW(model, lr=1e-3, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1,
                    max_grad_norm=0.5, init_scale=float(g["adamw_scale"]), growth_interval=1000,
                    param_dtype=torch.float16)
    ps = list(model.parameters())
    for st in range(6):
        for i, p in enumerate(ps):
            p.grad = torch.tensor(g[f"adamw_grads_{i}"][st], device=dev).half()
        opt.step(lr=1e-3)
        for i, (nm, p, off, n, _w) in enumerate(opt._info):
            ref = torch.tensor(g[f"adamw_master_{i}"][st])
            ours = opt.master[off:off + n].view(p.shape).cpu()
            err = (ours - ref).abs().max().item() / ref.abs().max().clamp(min=1e-6).item()
            assert err < 1e-5, f"step {st} param {nm}: rel err {err:.2e}"
        assert all(torch.equal(p, opt.master[o:o + ne].view(p.shape).half())
                   for _n, p, o, ne, _w in opt._info)


def test_flat_adamw_inf_skip_growth_accum(dev):
    from fxlm.optim import FlatAdamW
    torch.manual_seed(0)
    model = torch.nn.Sequential(torch.nn.Linear(256, 512, bias=False), torch.nn.LayerNorm(512),
                                torch.nn.Linear(512, 128, bias=False)).to(dev)
    opt = FlatAdamW(model, lr=1e-3, max_grad_norm=0.5, init_scale=8.0, growth_interval=4,
                    param_dtype=torch.float16)
    ps = list(model.parameters())
    for p in ps:
        p.grad = (torch.randn(p.shape, device=dev) * 0.1).half()
    opt.step(lr=1e-3)
    # inf: step skipped, scale halved, step counter unchanged
    sc0, st0 = float(opt.scale), int(opt._step_ctr)
    m0, mm0, vv0 = opt.master.clone(), opt.m.clone(), opt.v.clone()
    for p in ps:
        p.grad = torch.zeros(p.shape, device=dev).half()
    ps[0].grad.view(-1)[0] = float("inf")
    stats = opt.step(lr=1e-3)
    assert bool(stats["found_inf"]) and float(stats["scale"]) == sc0 * 0.5
    assert int(opt._step_ctr) == st0
    assert torch.equal(m0, opt.master) and torch.equal(mm0, opt.m) and torch.equal(vv0, opt.v)
    assert float(opt.grad.abs().max()) == 0.0  # gradient consumed even when skipped
    opt.zero_grad()
    # growth after growth_interval clean steps
    sc0 = float(opt.scale)
    for _ in range(opt.growth_interval):
        for p in ps:
            p.grad = torch.zeros(p.shape, device=dev).half()
        opt.step(lr=1e-3)
    assert float(opt.scale) == sc0 * 2.0
    # grad accumulation into p.grad
    g1 = torch.randn(ps[0].shape, device=dev).half()
    ps[0].grad = g1.clone()
    ps[0].grad.add_(g1)
    assert torch.equal(ps[0].grad, (g1.float() * 2).half())
    opt.zero_grad()


# ------------------------------------------------------------------ GPT
def _our_gpt(cfg, eps, seed, dev):
    from fxlm import GPT, GPTConfig
    torch.manual_seed(seed)
    return GPT(GPTConfig(**cfg, eps=eps)).to(dev)


def test_gpt_tiny_vs_oracle(dev):
    """Config 1 on the bf16 path: loss within 1e-3 rel and every gradient
    within 2e-2 rel of the fp32 oracle (pinned to the reference by
    tests/test_oracle.py); then one FlatAdamW step. From the same gradients
    the fp32 master update matches the oracle optimizer to 1e-5 per
    parameter, and the bf16 parameters are the masters rounded. From each
    side's own gradients the updated parameters agree within 1e-2 over the
    flat vector: a first AdamW step moves each element by about lr * sign(g),
    so the elements whose bf16 gradient lies near zero may move the other
    way. (fp32 mode holds the whole step to 1e-5: tests/test_gpu_fp32.py.)"""
    from fxlm import FlatAdamW
    from oracle import gpt as og
    cfg = CFG1
    state = og.init_state(cfg, 0)
    x, y = og.zipf_tokens(256, 32, 256, seed=0)
    ref_loss, ref_grads = og.loss_and_grads(state, {**cfg, "eps": 1e-5}, x, y)
    m = _our_gpt(cfg, 1e-5, 0, dev)
    m.load_state_dict(state)
    opt = FlatAdamW(m, lr=3e-4, init_scale=1.0)
    loss = m(x.to(dev), y.to(dev), grad_scale=opt.scale)
    opt.backward(loss)
    assert abs(loss.item() - ref_loss.item()) <= 1e-3 * abs(ref_loss.item())
    our_grads = {}
    for name, p, off, n, _w in opt._info:
        ours = opt.grad[off:off + n].view(p.shape)
        r = rel(ours, ref_grads[name])
        assert r < 2e-2, f"{name}: grad rel err {r:.3e}"
        our_grads[name] = ours.detach().cpu().clone()
    ref_opt = og.OracleFlatAdamW(list(state.items()), lr=3e-4, init_scale=1.0)
    ref_opt.step(ref_grads)
    same_g = og.OracleFlatAdamW(list(state.items()), lr=3e-4, init_scale=1.0)
    same_g.step(our_grads)
    opt.step()
    torch.cuda.synchronize()
    ours_flat, ref_flat = [], []
    for name, p, off, n, _w in opt._info:
        w = opt.master[off:off + n].view(p.shape)
        r = rel(w, same_g.master[name])
        assert r < 1e-5, f"{name}: FlatAdamW update rel err {r:.3e} (same gradients)"
        assert torch.equal(p.detach(), w.to(p.dtype)), f"{name}: bf16 parameter is not the rounded master"
        ours_flat.append(w.reshape(-1).double().cpu())
        ref_flat.append(ref_opt.master[name].reshape(-1).double())
    whole = rel(torch.cat(ours_flat), torch.cat(ref_flat))
    assert whole < 1e-2, f"updated parameters: rel err {whole:.3e} over the flat vector"
    print(f"\nbf16 config-1 step: updated params rel {whole:.2e} (flat) against the fp32 oracle")


def test_gpt_fused_vs_torch_paths(dev):
    """The fused model and its own torch paths on the same bf16 weights both
    track the fp32 reference (selftest.py:301-333)."""
    from fxlm import GPT, GPTConfig
    torch.manual_seed(0)
    c = dict(vocab_size=256, seq_len=64, n_layer=2, n_head=2, d_model=128)
    mf = GPT(GPTConfig(**c)).to(dev)
    mt = GPT(GPTConfig(**c, attn_impl="sdpa", norm_impl="torch", ce_impl="torch", linear_impl="torch")).to(dev)
    mt.load_state_dict(mf.state_dict())
    mr = GPT(GPTConfig(**c, attn_impl="sdpa", norm_impl="torch", ce_impl="torch", linear_impl="torch")).to(dev)
    mr.load_state_dict(mf.state_dict())
    mf.bfloat16(); mt.bfloat16()
    idx = torch.randint(0, 256, (8, 64), device=dev)
    tgt = torch.randint(0, 256, (8, 64), device=dev)
    lf, lt, lr_ = mf(idx, tgt), mt(idx, tgt), mr(idx, tgt)
    assert abs(lf.item() - lr_.item()) <= 2 * abs(lt.item() - lr_.item()) + 1e-3
    lf.backward(); lt.backward(); lr_.backward()
    pt, pr = dict(mt.named_parameters()), dict(mr.named_parameters())
    for nm, p in mf.named_parameters():
        e_our = (p.grad.float() - pr[nm].grad).abs().max().item()
        e_t = (pt[nm].grad.float() - pr[nm].grad).abs().max().item()
        assert e_our <= 2 * e_t + 1e-3, f"{nm}: {e_our} vs torch-bf16 {e_t}"


def test_gpt_20_step_learn(dev):
    from fxlm import GPT, GPTConfig, FlatAdamW
    torch.manual_seed(0)
    m = GPT(GPTConfig(vocab_size=256, seq_len=64, n_layer=2, n_head=2, d_model=128)).to(dev)
    opt = FlatAdamW(m, lr=3e-3, betas=(0.9, 0.95), weight_decay=0.1, max_grad_norm=1.0,
                    init_scale=8.0, growth_interval=1000)
    idx = torch.randint(0, 256, (8, 64), device=dev)
    tgt = torch.randint(0, 256, (8, 64), device=dev)
    losses, skips = [], 0
    for _ in range(20):
        loss = m(idx, tgt, grad_scale=opt.scale)
        opt.backward(loss)
        stats = opt.step(lr=3e-3)
        opt.zero_grad()
        skips += int(bool(stats["found_inf"]))
        losses.append(float(loss.detach()))
    assert losses[-1] < losses[0] * 0.9 and skips == 0, losses


def _curve(dev, steps, seed_of_step):
    from fxlm import FlatAdamW
    from oracle import gpt as og
    m = _our_gpt(CFG1, 1e-5, 0, dev)
    m.load_state_dict(og.init_state(CFG1, 0))
    opt = FlatAdamW(m, lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1,
                    max_grad_norm=1.0, init_scale=1.0)
    losses = []
    for s in range(steps):
        x, y = og.zipf_tokens(256, 32, 256, seed=seed_of_step(s))
        loss = m(x.to(dev), y.to(dev), grad_scale=opt.scale)
        opt.backward(loss)
        opt.step()
        opt.zero_grad()
        losses.append(loss.detach())
    return [float(v) for v in losses]


def test_loss_curve_200_steps(dev):
    """Config 1, 200 FlatAdamW steps, a fresh Zipf batch every step: every
    step's loss within 2% of the reference curve (golden curve_tiny.json).
    The fixed-batch (memorisation) curve is reported: its fast-falling phase
    amplifies bf16 rounding, so it is a diagnostic, not the criterion."""
    with open(os.path.join(GOLD, "curve_tiny.json")) as f:
        gold = json.load(f)
    ref = gold["losses_stream"]
    ours = _curve(dev, len(ref), lambda s: 1000 + s)
    dev_rel = [abs(a - b) / abs(b) for a, b in zip(ours, ref)]
    fixed_ref = gold["losses"]
    fixed = _curve(dev, len(fixed_ref), lambda s: 0)
    fdev = [abs(a - b) / abs(b) for a, b in zip(fixed, fixed_ref)]
    print(f"\nstream curve: max rel dev {max(dev_rel):.4f}, final {ours[-1]:.4f} vs {ref[-1]:.4f}; "
          f"fixed-batch curve: max rel dev {max(fdev):.4f} (step {int(np.argmax(fdev))}), "
          f"final {fixed[-1]:.4f} vs {fixed_ref[-1]:.4f}")
    assert max(dev_rel) < 0.02, f"max rel deviation {max(dev_rel):.4f} at step {int(np.argmax(dev_rel))}"


def test_gpt_d768_first_step_loss(dev):
    """Config 4 (d768 x 12L, V32768, B8 T1024): first-step loss within 1e-3
    relative and gradient norm within 2e-2 of the reference (golden)."""
    from fxlm import FlatAdamW
    from fxb200.data import zipf_tokens
    with open(os.path.join(GOLD, "gpt_d768.json")) as f:
        ref = json.load(f)
    cfg = dict(vocab_size=32768, seq_len=1024, n_layer=12, n_head=12, d_model=768)
    m = _our_gpt(cfg, 1e-6, 3, dev)
    opt = FlatAdamW(m, init_scale=1.0)
    x, y = zipf_tokens(32768, 8, 1024, seed=3)
    loss = m(x.to(dev), y.to(dev), grad_scale=opt.scale)
    opt.backward(loss)
    gn = opt.grad.double().norm().item()
    assert abs(loss.item() - ref["loss"]) <= 1e-3 * ref["loss"], (loss.item(), ref["loss"])
    assert abs(gn - ref["grad_norm"]) <= 2e-2 * ref["grad_norm"], (gn, ref["grad_norm"])


def _cfg4_losses(dev, steps, batch_of_step, param_dtype, torch_path=False):
    """Losses and gradient norms of `steps` config-4 training steps from the
    reference init (seed 3) with FlatAdamW (lr 6e-4, betas (0.9, 0.95), wd 0.1,
    clip 1.0); torch_path runs the reference's own PyTorch path of the model
    (sdpa, torch RMSNorm / CE / linears) instead of the fused kernels."""
    from fxlm import GPT, GPTConfig, FlatAdamW
    cfg = dict(vocab_size=32768, seq_len=1024, n_layer=12, n_head=12, d_model=768, eps=1e-6)
    if torch_path:
        cfg.update(attn_impl="sdpa", norm_impl="torch", ce_impl="torch", linear_impl="torch")
    torch.manual_seed(3)
    m = GPT(GPTConfig(**cfg)).to(dev)
    opt = FlatAdamW(m, lr=6e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1, max_grad_norm=1.0,
                    init_scale=1.0, param_dtype=param_dtype)
    L, N = torch.zeros(steps, device=dev), torch.zeros(steps, device=dev)
    for s in range(steps):
        x, y = batch_of_step(s)
        loss = m(x.to(dev), y.to(dev), grad_scale=opt.scale)
        opt.backward(loss)
        st = opt.step(6e-4)
        opt.zero_grad()
        L[s], N[s] = loss.detach(), st["grad_norm"]
    out = L.cpu().tolist(), N.cpu().tolist()
    del m, opt
    torch.cuda.empty_cache()
    return out


def test_config4_spike_fp32_matches_torch_path(dev):
    """Config 4 on its fixed batch spikes at step 3 (loss 14.0); past the
    spike the trajectory depends on fp32 summation order, so the reference's
    CPU curve cannot be tracked there by any implementation (the reference's
    own PyTorch path in fp32 on this GPU lands at 13.57 at step 4, the CPU run
    at 8.11). Through the spike, the fused kernels in fp32 mode follow that
    PyTorch path on the same device: losses within 1e-4 and gradient norms
    within 1e-3 for the first 5 steps, and the first 4 losses within 1e-4 of
    the reference's CPU curve."""
    from fxb200.data import zipf_tokens
    torch.backends.cuda.matmul.allow_tf32 = False
    x, y = zipf_tokens(32768, 8, 1024, seed=3)
    fixed = lambda s: (x, y)  # noqa: E731
    lf, nf = _cfg4_losses(dev, 5, fixed, torch.float32)
    lt, nt = _cfg4_losses(dev, 5, fixed, torch.float32, torch_path=True)
    for s in range(5):
        assert abs(lf[s] - lt[s]) <= 1e-4 * lt[s], (s, lf, lt)
        assert abs(nf[s] - nt[s]) <= 1e-3 * nt[s], (s, nf, nt)
    with open(os.path.join(GOLD, "curve_d768.json")) as f:
        ref = json.load(f)["acc1"]["losses"]
    for s in range(4):
        assert abs(lf[s] - ref[s]) <= 1e-4 * ref[s], (s, lf[:4], ref[:4])


def test_config4_curve_200_steps(dev):
    """Config 4 (d768 x 12L, V32768, bf16 + fp32-master FlatAdamW), 200 steps
    on a fresh Zipf batch every step: every step's loss within 2% of the
    reference's own fp32 CPU curve on the same batches (golden
    curve_d768.json "acc1_stream", from tests/golden/make_golden.py)."""
    from fxb200.data import zipf_tokens
    with open(os.path.join(GOLD, "curve_d768.json")) as f:
        gold = json.load(f).get("acc1_stream")
    if not gold:
        pytest.skip("no acc1_stream curve in tests/golden/curve_d768.json")
    ref = gold["losses"]
    ours, _ = _cfg4_losses(dev, len(ref), lambda s: zipf_tokens(32768, 8, 1024, seed=1000 * (s + 1)),
                           torch.bfloat16)
    dev_rel = [abs(a - b) / abs(b) for a, b in zip(ours, ref)]
    print(f"\nconfig-4 curve: {len(ref)} steps, max rel dev {max(dev_rel):.4f} "
          f"(step {int(np.argmax(dev_rel))}), final {ours[-1]:.4f} vs {ref[-1]:.4f}")
    assert max(dev_rel) < 0.02, f"max rel deviation {max(dev_rel):.4f} at step {int(np.argmax(dev_rel))}"


def test_graphed_step_matches_eager(dev):
    """fxlm.GraphedStep (one captured training step, replayed) follows the
    eager step: same losses over a fresh batch per step and the same master
    weights, including a learning-rate change between replays."""
    from fxlm import FlatAdamW, GraphedStep
    from oracle import gpt as og
    batches = [og.zipf_tokens(256, 32, 256, seed=500 + s) for s in range(6)]
    lrs = [3e-4, 3e-4, 3e-4, 1e-4, 1e-4, 5e-5]

    def fresh():
        m = _our_gpt(CFG1, 1e-5, 0, dev)
        m.load_state_dict(og.init_state(CFG1, 0))
        return m, FlatAdamW(m, lr=3e-4, init_scale=1.0)

    me, oe = fresh()
    eager = []
    for (x, y), lr in zip(batches, lrs):
        loss = me(x.to(dev), y.to(dev), grad_scale=oe.scale)
        oe.backward(loss)
        oe.step(lr=lr)
        oe.zero_grad()
        eager.append(float(loss.detach()))

    mg, og_ = fresh()
    x0, y0 = batches[0]
    g = GraphedStep(mg, og_, x0.to(dev), y0.to(dev), warmup=1)  # step 0 runs eagerly here
    assert g.launches_per_step > 0
    graphed = []
    for (x, y), lr in zip(batches[1:], lrs[1:]):
        graphed.append(float(g(x.to(dev), y.to(dev), lr=lr)))
    for a, b in zip(graphed, eager[1:]):
        assert abs(a - b) <= 1e-3 * abs(b), (graphed, eager[1:])
    r = rel(og_.master, oe.master)
    assert r < 1e-2, f"master rel diff {r:.3e}"


def test_prepare_train_resume_sample(dev, tmp_path):
    """The reference's workflow end to end (ml/fxlm/prepare_bytes.py ->
    train_lm.py -> sample.py): byte tokens of this package's sources, a small
    run with eval and checkpoint, a resumed run, and generation from the
    checkpoint. The fused bf16 model's last-position logits at several
    prompt lengths track the fp32 model within twice the error of the same
    weights on the bf16 torch path."""
    from fxlm import prepare_bytes, train_lm, sample
    from fxlm.model import GPT, GPTConfig
    pkg = os.path.join(os.path.dirname(GOLD), "..", "radeon-igpu-forge_b200", "fxlm")
    data = str(tmp_path / "data" / "src")
    meta = prepare_bytes.main([os.path.join(pkg, "*.py"), "--out", data])
    assert meta["vocab_size"] == 256 and meta["n_val"] > 200
    out = str(tmp_path / "run")
    common = ["--data", data + "_train.bin", "--out", out, "--seq-len", "64", "--layers", "2",
              "--heads", "2", "--dim", "128", "--batch", "8", "--warmup", "5",
              "--eval-every", "30", "--eval-batches", "2", "--log-every", "10"]
    train_lm.main(common + ["--steps", "30"])
    ckpt = os.path.join(out, "ckpt_last.pt")
    sd = torch.load(ckpt, map_location="cpu", weights_only=False)
    assert sd["step"] == 30 and sd["meta"]["tokenizer"] == "bytes"
    with pytest.raises(SystemExit, match="exists"):
        train_lm.main(common + ["--steps", "31"])
    train_lm.main(common + ["--steps", "40", "--resume", ckpt])
    sd2 = torch.load(ckpt, map_location="cpu", weights_only=False)
    assert sd2["step"] == 40
    assert any(not torch.equal(sd["model"][k], sd2["model"][k]) for k in sd["model"])

    mf, meta, missing = sample.load_checkpoint(ckpt, dev)
    assert not missing and mf.tok_emb.weight.dtype == torch.bfloat16
    torch_cfg = dict(sd2["config"], attn_impl="sdpa", norm_impl="torch", ce_impl="torch",
                     linear_impl="torch")
    mt = GPT(GPTConfig(**torch_cfg)).to(dev)
    mt.load_state_dict({k: v for k, v in sd2["model"].items()})
    mr = GPT(GPTConfig(**torch_cfg)).to(dev).eval()
    mr.load_state_dict(mt.state_dict())
    mt = mt.bfloat16().eval()
    g = torch.Generator().manual_seed(5)
    with torch.inference_mode():
        for T in (1, 4, 37, 64):
            idx = torch.randint(0, 256, (1, T), generator=g).to(dev)
            lf = mf(idx)[:, -1].float()
            lt = mt(idx)[:, -1].float()
            lr_ = mr(idx)[:, -1]
            e_our, e_t = (lf - lr_).abs().max().item(), (lt - lr_).abs().max().item()
            assert e_our <= 2 * e_t + 2e-2, (T, e_our, e_t)

    args = ["--ckpt", ckpt, "--prompt", "def ", "--max-new", "48", "--seed", "3"]
    a, b = sample.main(args), sample.main(args)
    assert isinstance(a, str) and a == b and len(a.encode("utf-8", "replace")) >= 1
