"""CPU oracle for the reference GPT training step (PyTorch on CPU, fp32).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py, never by the product path.

RefGPT restates the reference model (ml/fxlm/model.py:22-130) with its own
PyTorch path only (attn_impl="sdpa", norm_impl="torch", ce_impl="torch",
model.py:31-33,53-56,65-68,102-105,128-130): same parameter names, module
construction order and initialisation (N(0,0.02), proj/fc2 at 0.02/sqrt(2L),
pos_emb zeros, model.py:83,88-100), so under the same torch.manual_seed it
produces the reference's initial weights. OracleFlatAdamW restates the
FlatAdamW step (ml/fxlm/optim.py:136-173 and kernels/optim.hip) on CPU fp32
tensors. zipf_tokens is the synthetic-data definition used by every config.

Parity pin: tests/test_oracle.py compares RefGPT's loss and gradients and the
optimizer step against golden vectors that tests/golden/make_golden.py
produced by running the reference's own ml/fxlm/model.py here.
"""
import math

import numpy as np
import torch
from torch import nn
import torch.nn.functional as F


# ---------------------------------------------------------------- data
def zipf_tokens(V, B, T, seed, s=1.1):
    """Token ids i.i.d. with p_k ∝ (k+1)^-s, k in [0, V), shape (B, T+1);
    returns (x, y) = (seq[:, :-1], seq[:, 1:]) like ml/fxlm/train_lm.py:148-152."""
    k = np.arange(V, dtype=np.float64)
    p = (k + 1.0) ** (-s)
    p /= p.sum()
    seq = np.random.default_rng(seed).choice(V, size=(B, T + 1), p=p)
    seq = torch.from_numpy(seq.astype(np.int64))
    return seq[:, :-1].contiguous(), seq[:, 1:].contiguous()


# ---------------------------------------------------------------- model
class RefBlock(nn.Module):
    """ml/fxlm/model.py:37-72 with the torch paths."""

    def __init__(self, D, H, mlp_ratio, eps):
        super().__init__()
        self.n_head, self.head_dim, self.eps = H, D // H, eps
        self.ln1_w = nn.Parameter(torch.ones(D))
        self.ln2_w = nn.Parameter(torch.ones(D))
        self.qkv = nn.Linear(D, 3 * D, bias=False)
        self.proj = nn.Linear(D, D, bias=False)
        self.fc = nn.Linear(D, mlp_ratio * D, bias=False)
        self.fc2 = nn.Linear(mlp_ratio * D, D, bias=False)

    def forward(self, x):
        B, T, D = x.shape
        h = F.rms_norm(x, (D,), self.ln1_w, self.eps)
        qkv = self.qkv(h).view(B, T, 3, self.n_head, self.head_dim)
        q, k, v = (qkv[:, :, i].transpose(1, 2) for i in range(3))
        y = F.scaled_dot_product_attention(q, k, v, is_causal=True)
        x = x + self.proj(y.transpose(1, 2).reshape(B, T, D))
        h = F.rms_norm(x, (D,), self.ln2_w, self.eps)
        return x + self.fc2(F.gelu(self.fc(h), approximate="tanh"))


class RefGPT(nn.Module):
    """ml/fxlm/model.py:75-130, tied embeddings, torch CE path."""

    def __init__(self, vocab_size, seq_len, n_layer, n_head, d_model, mlp_ratio=4, eps=1e-6):
        super().__init__()
        D = d_model
        self.eps = eps
        self.tok_emb = nn.Embedding(vocab_size, D)
        self.pos_emb = nn.Parameter(torch.zeros(seq_len, D))
        self.blocks = nn.ModuleList(RefBlock(D, n_head, mlp_ratio, eps) for _ in range(n_layer))
        self.lnf_w = nn.Parameter(torch.ones(D))
        self.apply(self._init)
        s = 0.02 / math.sqrt(2 * n_layer)
        for b in self.blocks:
            nn.init.normal_(b.proj.weight, std=s)
            nn.init.normal_(b.fc2.weight, std=s)

    @staticmethod
    def _init(m):
        if isinstance(m, (nn.Linear, nn.Embedding)):
            nn.init.normal_(m.weight, std=0.02)

    def forward(self, idx, targets):
        B, T = idx.shape
        x = self.tok_emb(idx) + self.pos_emb[:T]
        for blk in self.blocks:
            x = blk(x)
        x = F.rms_norm(x, (x.shape[-1],), self.lnf_w, self.eps)
        logits = F.linear(x, self.tok_emb.weight)
        return F.cross_entropy(logits.float().view(-1, logits.shape[-1]), targets.reshape(-1))


def init_state(cfg, seed=0):
    """Reference initial weights (fp32 state dict) for cfg = dict(vocab_size,
    seq_len, n_layer, n_head, d_model[, mlp_ratio, eps]) under manual_seed(seed)."""
    torch.manual_seed(seed)
    return RefGPT(**cfg).state_dict()


def loss_and_grads(state, cfg, idx, targets):
    """fp32 CPU loss and parameter gradients of the reference model."""
    m = RefGPT(**cfg)
    m.load_state_dict(state)
    loss = m(idx, targets)
    loss.backward()
    return loss.detach(), {n: p.grad.detach().clone() for n, p in m.named_parameters()}


# ---------------------------------------------------------------- optimizer
class OracleFlatAdamW:
    """FlatAdamW semantics on CPU fp32 (ml/fxlm/optim.py:136-173,
    ml/fxlm/kernels/optim.hip:26-162): step() takes gradients of the *scaled*
    loss (loss * scale), detects non-finite values, clips the unscaled global
    norm to max_grad_norm, applies decoupled weight decay on ndim >= 2 params
    and updates the dynamic loss scale."""

    def __init__(self, named_params, lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1,
                 max_grad_norm=1.0, init_scale=2.0 ** 16, growth_interval=1000):
        self.names = [n for n, _ in named_params]
        self.master = {n: p.detach().float().clone() for n, p in named_params}
        self.wd_on = {n: (p.dim() >= 2 and weight_decay != 0) for n, p in named_params}
        self.m = {n: torch.zeros_like(t) for n, t in self.master.items()}
        self.v = {n: torch.zeros_like(t) for n, t in self.master.items()}
        self.lr, self.betas, self.eps, self.wd = lr, betas, eps, weight_decay
        self.max_grad_norm = max_grad_norm
        self.scale, self.growth, self.growth_interval = float(init_scale), 0, int(growth_interval)
        self.step_ctr = 0

    def step(self, scaled_grads, lr=None):
        lr = self.lr if lr is None else lr
        b1, b2 = self.betas
        sumsq = sum(float((g.double() ** 2).sum()) for g in scaled_grads.values())
        bad = any(not torch.isfinite(g).all() for g in scaled_grads.values()) or not math.isfinite(sumsq)
        norm = math.sqrt(sumsq) / self.scale if math.isfinite(sumsq) else float("inf")
        if not bad:
            clip = min(1.0, self.max_grad_norm / (norm + 1e-6))
            self.step_ctr += 1
            bc1 = 1.0 - b1 ** self.step_ctr
            bc2 = 1.0 - b2 ** self.step_ctr
            inv = clip / self.scale
            for n in self.names:
                g = scaled_grads[n].float() * inv
                w = self.master[n]
                if self.wd_on[n]:
                    w -= lr * self.wd * w
                self.m[n].mul_(b1).add_((1 - b1) * g)
                self.v[n].mul_(b2).add_((1 - b2) * g * g)
                w -= lr * (self.m[n] / bc1) / (torch.sqrt(self.v[n] / bc2) + self.eps)
        if bad:
            self.scale *= 0.5
            self.growth = 0
        else:
            self.growth += 1
            if self.growth == self.growth_interval:
                self.scale *= 2.0
                self.growth = 0
        return {"grad_norm": norm, "found_inf": bad, "scale": self.scale}


def train_curve(cfg, steps, B, T, data_seed, init_seed=0, lr=3e-4, wd=0.1, max_grad_norm=1.0,
                init_scale=1.0, threads=None):
    """Loss of each step of `steps` FlatAdamW steps of the reference model on
    a fixed Zipf batch (CPU fp32). Used for the loss-curve parity check."""
    if threads:
        torch.set_num_threads(threads)
    state = init_state(cfg, init_seed)
    m = RefGPT(**cfg)
    m.load_state_dict(state)
    opt = OracleFlatAdamW(list(m.named_parameters()), lr=lr, weight_decay=wd,
                          max_grad_norm=max_grad_norm, init_scale=init_scale)
    x, y = zipf_tokens(cfg["vocab_size"], B, T, data_seed)
    losses = []
    for _ in range(steps):
        with torch.no_grad():
            for n, p in m.named_parameters():
                p.copy_(opt.master[n])
        m.zero_grad(set_to_none=True)
        loss = m(x, y)
        (loss * opt.scale).backward()
        opt.step({n: p.grad for n, p in m.named_parameters()})
        losses.append(float(loss))
    return losses
