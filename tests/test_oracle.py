"""CPU: pin the oracle to the reference's own outputs (golden fixtures).

tests/golden/*.npz|json were produced by running the reference's PyTorch code
(tests/golden/make_golden.py). These tests check that oracle/ops.py (numpy)
and oracle/gpt.py (PyTorch CPU) reproduce them, and that the B200 package
builds bit-identical initial weights and synthetic tokens.
"""
import json
import os

import numpy as np
import pytest
import torch

from oracle import ops as O
from oracle import gpt as og

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
CFG1 = dict(vocab_size=256, seq_len=256, n_layer=4, n_head=4, d_model=256)


@pytest.fixture(scope="module")
def g():
    return np.load(os.path.join(GOLD, "ops.npz"))


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def test_rmsnorm_oracle(g):
    for k in ("rms_37x64", "rms_129x768"):
        y, rstd = O.rms_norm_fwd(g[k + "_x"], g[k + "_w"], 1e-6)
        dx, dw = O.rms_norm_bwd(g[k + "_x"], g[k + "_w"], rstd, g[k + "_dy"])
        assert rel(y, g[k + "_y"]) < 1e-6
        assert rel(dx, g[k + "_dx"]) < 1e-5
        assert rel(dw, g[k + "_dw"]) < 1e-5


def test_ce_oracle(g):
    for k in ("ce_100x512", "ce_33x8192"):
        loss, grad = O.fused_cross_entropy(g[k + "_logits"], g[k + "_target"], -100)
        assert abs(loss - float(g[k + "_loss"])) < 1e-5 * abs(float(g[k + "_loss"]))
        assert rel(grad, g[k + "_grad"]) < 1e-5
    loss, dx, dW = O.linear_cross_entropy(g["lce_x"], g["lce_W"], g["lce_target"], -100)
    assert abs(loss - float(g["lce_loss"])) < 1e-5 * abs(float(g["lce_loss"]))
    assert rel(dx, g["lce_dx"]) < 1e-5
    assert rel(dW, g["lce_dW"]) < 1e-5


def test_ce_edge_cases():
    # all rows ignored: zero loss, zero grad, inv_nvalid 0 (cross_entropy.py:41-45)
    lg = np.random.default_rng(0).standard_normal((4, 10))
    tg = np.full(4, -100)
    loss, grad = O.fused_cross_entropy(lg, tg)
    assert loss == 0.0 and not grad.any()
    # out-of-range target counts as invalid row in the kernel (ce.hip:43)
    s, gr = O.ce_fwd_grad(lg, np.array([0, 10, -5, 3]), 1.0)
    assert not gr[1].any() and not gr[2].any() and gr[0].any()


def test_attention_oracle(g):
    import math
    for causal in (True, False):
        k = f"attn_c{int(causal)}"
        qkv = g[k + "_qkv"]
        q, kk, v = qkv[:, :, 0], qkv[:, :, 1], qkv[:, :, 2]
        scale = 1 / math.sqrt(q.shape[-1])
        o, lse = O.attention_fwd(q, kk, v, causal, scale)
        assert rel(o, g[k + "_o"]) < 1e-5
        dq, dk, dv, _ = O.attention_bwd(q, kk, v, o, lse, g[k + "_do"], causal, scale)
        assert rel(dq, g[k + "_dq"]) < 1e-5
        assert rel(dk, g[k + "_dk"]) < 1e-5
        assert rel(dv, g[k + "_dv"]) < 1e-5


def test_attention_oracle_single_token():
    # T = 1: causal and non-causal attention both return v, lse = q.k*scale
    rng = np.random.default_rng(1)
    q, k, v = (rng.standard_normal((1, 1, 2, 64)) for _ in range(3))
    for causal in (True, False):
        o, lse = O.attention_fwd(q, k, v, causal, 0.125)
        assert np.allclose(o, v)
        assert np.allclose(lse[0, :, 0], (q * k).sum(-1)[0, 0] * 0.125)


def test_gelu_oracle(g):
    assert rel(O.gelu_tanh(g["gelu_z"]), g["gelu_a"]) < 1e-6
    assert rel(O.gelu_tanh_grad(g["gelu_z"]), g["gelu_da"]) < 1e-5


def test_adamw_oracle(g):
    """The flat-kernel restatement reproduces the reference selftest's torch
    AdamW + clip procedure (golden masters) within 1e-5."""
    n = sum(1 for k in g.files if k.startswith("adamw_init_"))
    shapes = [g[f"adamw_init_{i}"].shape for i in range(n)]
    flat = lambda arrs: np.concatenate([np.asarray(a, np.float64).reshape(-1) for a in arrs])  # noqa: E731
    master = flat([g[f"adamw_init_{i}"] for i in range(n)])
    m = np.zeros_like(master)
    v = np.zeros_like(master)
    wd_mask = flat([np.full(s, len(s) >= 2, dtype=np.float64) for s in shapes]).astype(bool)
    scale, step = float(g["adamw_scale"]), 0
    for st in range(6):
        grad = flat([g[f"adamw_grads_{i}"][st] for i in range(n)])
        ss, bad = O.adamw_sumsq(grad)
        bad, norm, clip, step = O.adamw_final(ss, bad, scale, 0.5, step)
        master, m, v = O.adamw_update(master, m, v, grad, wd_mask, clip, scale, step,
                                      1e-3, 0.9, 0.95, 1e-8, 0.1)
        ref = flat([g[f"adamw_master_{i}"][st] for i in range(n)])
        assert np.abs(master - ref).max() / np.abs(ref).max() < 1e-5


def test_amp_scale_semantics():
    s, gr = O.amp_update_scale(8.0, 3, True)
    assert (s, gr) == (4.0, 0)
    s, gr = O.amp_update_scale(8.0, 3, False, interval=4)
    assert (s, gr) == (16.0, 0)


def test_gather_linear_oracle(g):
    idx = g["wmlp_idx"]
    W1, b1 = g["wmlp_W1"], g["wmlp_b1"]
    h1, Xg = O.gather_linear_fwd(g["wmlp_X"], idx, W1, b1)
    assert np.array_equal(Xg.astype(np.float32), g["wmlp_xb"])
    assert rel(h1, g["wmlp_h1"]) < 1e-6
    h = O.silu(h1)
    h = O.silu(h @ np.asarray(g["wmlp_W2"], np.float64).T + g["wmlp_b2"])
    y = h @ np.asarray(g["wmlp_W3"], np.float64).T + g["wmlp_b3"]
    assert rel(y, g["wmlp_y"]) < 1e-5


# ------------------------------------------------------------------ model oracle
@pytest.fixture(scope="module")
def gt():
    return np.load(os.path.join(GOLD, "gpt_tiny.npz"))


def _check_init(state, gt):
    for n, t in state.items():
        flat = t.reshape(-1).double()
        assert abs(flat.sum().item() - float(gt[f"init_sum:{n}"])) <= 1e-6 * max(1.0, abs(float(gt[f"init_sq:{n}"])))
        sel = torch.from_numpy(gt[f"init_sel:{n}"])
        assert torch.equal(t.reshape(-1)[sel].float(), torch.from_numpy(gt[f"init_val:{n}"]))


def test_oracle_init_matches_reference(gt):
    _check_init(og.init_state(CFG1, 0), gt)


def test_package_init_matches_reference(gt):
    """fxlm.model.GPT (B200 package) builds the reference's initial weights."""
    from fxlm import GPT, GPTConfig
    torch.manual_seed(0)
    m = GPT(GPTConfig(**CFG1, eps=1e-5))
    _check_init(m.state_dict(), gt)


def test_tokens_match_reference(gt):
    from fxb200.data import zipf_tokens
    x, y = og.zipf_tokens(256, 32, 256, seed=0)
    assert np.array_equal(x.numpy(), gt["x"]) and np.array_equal(y.numpy(), gt["y"])
    x2, y2 = zipf_tokens(256, 32, 256, seed=0)
    assert torch.equal(x, x2) and torch.equal(y, y2)


def test_oracle_gpt_loss_and_grads(gt):
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    state = og.init_state(CFG1, 0)
    x, y = og.zipf_tokens(256, 32, 256, seed=0)
    loss, grads = og.loss_and_grads(state, {**CFG1, "eps": 1e-5}, x, y)
    assert abs(loss.item() - float(gt["loss"])) < 1e-5 * float(gt["loss"])
    for n, gr in grads.items():
        assert abs(gr.double().norm().item() - float(gt[f"grad_norm:{n}"])) <= 1e-4 * float(gt[f"grad_norm:{n}"]) + 1e-12
        sel = torch.from_numpy(gt[f"init_sel:{n}"])
        ref = torch.from_numpy(gt[f"grad_val:{n}"]).double()
        got = gr.reshape(-1)[sel].double()
        assert (got - ref).abs().max().item() <= 1e-4 * max(ref.abs().max().item(), 1e-12)


def test_oracle_optimizer_tracks_reference_curve():
    """OracleFlatAdamW reproduces the first steps of the reference curve
    (torch AdamW + clip, the selftest's FlatAdamW oracle)."""
    with open(os.path.join(GOLD, "curve_tiny.json")) as f:
        ref = json.load(f)["losses"]
    losses = og.train_curve(CFG1 | {"eps": 1e-5}, steps=4, B=32, T=256, data_seed=0,
                            threads=os.cpu_count())
    for a, b in zip(losses, ref[:4]):
        assert abs(a - b) < 1e-4 * abs(b)
