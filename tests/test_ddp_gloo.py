"""CPU, 2 processes over gloo: the data-parallel bucketing of fxb200.ddp.

A tiny model whose linear layers follow the fused-op contract (the weight
gradient is written straight into the optimizer's flat fp32 buffer inside
backward, nothing in p.grad) runs on two ranks with different batches. After
the optimizer's pre-step hook the flat gradient on every rank must equal the
mean of the per-rank gradients, i.e. what a single process computes with
gradient accumulation over both batches (the reference's ACC path,
ml/fxlm/train_lm.py:199-203). A second test makes one rank fail on the host
before its collectives; the survivor must get an error from the process
group timeout instead of hanging.
"""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
import torch.nn as nn


class _FlatLinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w):
        ctx.save_for_backward(x, w)
        return x @ w.t()

    @staticmethod
    def backward(ctx, g):
        x, w = ctx.saved_tensors
        w._fxb_grad.add_(g.reshape(-1, g.shape[-1]).t() @ x.reshape(-1, x.shape[-1]))
        return g @ w, None


class _Block(nn.Module):
    def __init__(self, d):
        super().__init__()
        self.w = nn.Parameter(torch.randn(d, d) * 0.1)

    def forward(self, x):
        return torch.tanh(_FlatLinearFn.apply(x, self.w)) + x


class _Model(nn.Module):
    def __init__(self, d=16, L=3):
        super().__init__()
        self.emb = nn.Parameter(torch.randn(d) * 0.1)
        self.blocks = nn.ModuleList(_Block(d) for _ in range(L))

    def forward(self, x):
        x = x + self.emb
        for b in self.blocks:
            x = b(x)
        return (x ** 2).mean()


class _FlatOpt:
    """Host stand-in with FlatAdamW's bookkeeping (flat grad, offsets, hooks)."""

    def __init__(self, model):
        self._info, off = [], 0
        for n, p in model.named_parameters():
            self._info.append((n, p, off, p.numel(), int(p.dim() >= 2)))
            off += (p.numel() + 7) & ~7
        self.numel = off
        self.grad = torch.zeros(off)
        for n, p, o, k, _ in self._info:
            p._fxb_grad = self.grad[o:o + k].view(p.shape)
        self.pre_step_hooks = []

    def fold(self):
        for n, p, o, k, _ in self._info:
            if p.grad is not None:
                self.grad[o:o + k].add_(p.grad.reshape(-1))
                p.grad = None

    def step(self):
        self.fold()
        for h in self.pre_step_hooks:
            h(self)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _grads_single(batches):
    torch.manual_seed(0)
    m = _Model()
    opt = _FlatOpt(m)
    for xb in batches:
        (m(xb) / len(batches)).backward()
    opt.fold()
    return opt.grad.clone()


def _worker(rank, world, port, batches, out_q, fail_rank):
    import sys
    here = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(here, "radeon-igpu-forge_b200"))
    from fxb200.ddp import DataParallel
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    try:
        torch.manual_seed(0)
        m = _Model()
        opt = _FlatOpt(m)
        DataParallel(m, opt)
        if rank == fail_rank:
            raise RuntimeError("simulated rank failure before backward")
        m(batches[rank]).backward()
        opt.step()
        out_q.put((rank, "ok", opt.grad.clone()))
    except Exception as e:  # report, then leave without further collectives
        out_q.put((rank, "error", repr(e)))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, fail_rank=-1):
    torch.manual_seed(123)
    batches = [torch.randn(4, 5, 16) for _ in range(world)]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, batches, q, fail_rank))
             for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, status, payload = q.get(timeout=120)
        res[r] = (status, payload)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return batches, res


def test_dp_buckets_equal_accumulation():
    batches, res = _run(2)
    ref = _grads_single(batches)
    for r in range(2):
        status, g = res[r]
        assert status == "ok", g
        assert torch.allclose(g, ref, atol=1e-6, rtol=1e-5), (g - ref).abs().max()


def test_dp_rank_failure_surfaces_as_error():
    _batches, res = _run(2, fail_rank=1)
    assert res[1][0] == "error" and "simulated" in res[1][1]
    status, msg = res[0]
    assert status == "error", "survivor should see a collective error, not hang"


# ------------------------------------------------------------------ config 5 (window MLP)
class _WindowMLPLike(nn.Module):
    """The window model's parameter layout (W1, b1, W2, b2, W3, b3) and
    gradient contract: weight gradients written into the flat buffer inside
    backward, bias gradients arriving in p.grad (folded at step). It has no
    `blocks`, so data parallelism reduces the whole flat gradient from the
    optimizer's pre-step hook."""

    def __init__(self, K=24, H1=16, H2=8):
        super().__init__()
        self.W1 = nn.Parameter(torch.randn(H1, K) * 0.1)
        self.b1 = nn.Parameter(torch.randn(H1) * 0.1)
        self.W2 = nn.Parameter(torch.randn(H2, H1) * 0.1)
        self.b2 = nn.Parameter(torch.randn(H2) * 0.1)
        self.W3 = nn.Parameter(torch.randn(1, H2) * 0.1)
        self.b3 = nn.Parameter(torch.zeros(1))

    def forward(self, xb, tgt):
        h = torch.nn.functional.gelu(_FlatLinearFn.apply(xb, self.W1) + self.b1, approximate="tanh")
        h = torch.nn.functional.gelu(_FlatLinearFn.apply(h, self.W2) + self.b2, approximate="tanh")
        y = _FlatLinearFn.apply(h, self.W3) + self.b3
        return ((y - tgt) ** 2).mean()


def _wmlp_worker(rank, world, port, batches, out_q, zero):
    import sys
    here = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(here, "radeon-igpu-forge_b200"))
    from fxb200.ddp import DataParallel
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=20))
    try:
        torch.manual_seed(0)
        m = _WindowMLPLike()
        opt = _FlatOpt(m)
        dp = DataParallel(m, opt)
        assert not dp.buckets and dp._rest == [(0, opt.numel)]  # one pre-step range
        m(*batches[rank]).backward()
        opt.step()
        out_q.put((rank, "ok", opt.grad.clone()))
    except Exception as e:
        out_q.put((rank, "error", repr(e)))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_window_mlp_dp_equals_accumulation():
    """Config 5 data parallelism: two gloo ranks with different batches of the
    window model end with the mean gradient, i.e. the single-process
    accumulation over both batches."""
    world = 2
    torch.manual_seed(5)
    batches = [(torch.randn(32, 24), torch.randn(32, 1)) for _ in range(world)]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_wmlp_worker, args=(r, world, port, batches, q, False))
             for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, status, payload = q.get(timeout=120)
        res[r] = (status, payload)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    torch.manual_seed(0)
    m = _WindowMLPLike()
    opt = _FlatOpt(m)
    for xb, tb in batches:
        (m(xb, tb) / world).backward()
    opt.fold()
    for r in range(world):
        status, g = res[r]
        assert status == "ok", g
        assert torch.allclose(g, opt.grad, atol=1e-6, rtol=1e-5), (g - opt.grad).abs().max()


def _bf16_worker(rank, world, port, batches, out_q):
    import sys
    here = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(here, "radeon-igpu-forge_b200"))
    from fxb200.ddp import DataParallel
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=20))
    try:
        torch.manual_seed(0)
        m = _Model()
        opt = _FlatOpt(m)
        DataParallel(m, opt, comm_dtype=torch.bfloat16)
        m(batches[rank]).backward()
        opt.step()
        out_q.put((rank, "ok", opt.grad.clone()))
    except Exception as e:
        out_q.put((rank, "error", repr(e)))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_dp_bf16_wire_matches_accumulation():
    """comm_dtype=bfloat16: buckets cross the wire as bf16 and come back as
    fp32; the result equals the single-process mean within bf16 rounding."""
    world = 2
    torch.manual_seed(123)
    batches = [torch.randn(4, 5, 16) for _ in range(world)]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_bf16_worker, args=(r, world, port, batches, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(world):
        r, status, payload = q.get(timeout=120)
        res[r] = (status, payload)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    ref = _grads_single(batches)
    for r in range(world):
        status, g = res[r]
        assert status == "ok", g
        assert torch.allclose(g, ref, atol=1e-3, rtol=1e-2), (g - ref).abs().max()
        assert torch.equal(res[0][1], g)
