"""GPU, 2 processes over NCCL: data parallelism of the config-1 GPT, and its
optimizer-sharded (ZeRO-1) variant against it.

Two ranks train on different batches (seed 700 + rank). Each rank runs two
copies of the same model: one stepping eagerly, one captured with its bucket
all-reduces inside a CUDA graph (fxlm.GraphedStep + fxb200.ddp.DataParallel)
and replayed. Checks: the two copies stay together (same losses, same master
weights), every rank ends with the same master weights, and the first step's
averaged gradient equals what one process gets by accumulating both batches
(the reference's ACC path, ml/fxlm/train_lm.py:199-203). Skipped with fewer
than two GPUs.
"""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CFG1 = dict(vocab_size=256, seq_len=256, n_layer=4, n_head=4, d_model=256)
WORLD = 2


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _fresh(dev):
    from fxlm import GPT, GPTConfig, FlatAdamW
    from oracle import gpt as og
    torch.manual_seed(0)
    m = GPT(GPTConfig(**CFG1, eps=1e-5)).to(dev)
    m.load_state_dict(og.init_state(CFG1, 0))
    return m, FlatAdamW(m, lr=3e-4, init_scale=1.0)


def _worker(rank, port, out_q):
    import sys
    for p in (os.path.join(ROOT, "radeon-igpu-forge_b200"), ROOT):
        sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    graphed = None
    try:
        from fxb200.ddp import DataParallel
        from fxlm import GraphedStep
        from oracle import gpt as og
        batches = [og.zipf_tokens(256, 8, 256, seed=700 + 10 * s + rank) for s in range(4)]
        batches = [(x.to(dev), y.to(dev)) for x, y in batches]

        # first-step gradient: DP mean of both ranks' batches
        mg, og_ = _fresh(dev)
        DataParallel(mg, og_)
        x, y = batches[0]
        loss = mg(x, y, grad_scale=og_.scale)
        og_.backward(loss)
        og_._fold_param_grads()  # what step() does before its pre-step hooks
        for h in og_.pre_step_hooks:
            h(og_)
        torch.cuda.synchronize()
        dp_grad = og_.grad.detach().cpu().clone()
        og_.zero_grad()
        del mg, og_

        me, oe = _fresh(dev)
        DataParallel(me, oe)
        mc, oc = _fresh(dev)
        DataParallel(mc, oc)
        eager = []
        for x, y in batches:
            loss = me(x, y, grad_scale=oe.scale)
            oe.backward(loss)
            oe.step(lr=3e-4)
            oe.zero_grad()
            eager.append(float(loss.detach()))
        graphed = GraphedStep(mc, oc, batches[0][0], batches[0][1], warmup=1)
        replayed = [float(graphed(x, y)) for x, y in batches[1:]]
        torch.cuda.synchronize()
        out_q.put((rank, "ok", dict(dp_grad=dp_grad, eager=eager, replayed=replayed,
                                     master_e=oe.master.detach().cpu(),
                                     master_g=oc.master.detach().cpu())))
    except Exception as e:  # report, then leave
        out_q.put((rank, "error", repr(e)))
    finally:
        if graphed is not None:
            graphed.release()
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(target):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(WORLD):
        r, status, payload = q.get(timeout=600)
        res[r] = (status, payload)
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    for r in range(WORLD):
        assert res[r][0] == "ok", res[r][1]
    return [res[r][1] for r in range(WORLD)]


def _zero_worker(rank, port, out_q):
    import sys
    for p in (os.path.join(ROOT, "radeon-igpu-forge_b200"), ROOT):
        sys.path.insert(0, p)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=WORLD, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    graphed = None
    try:
        from fxb200.ddp import DataParallel
        from fxb200.zero import ShardedDataParallel
        from fxlm import GraphedStep
        from oracle import gpt as og
        batches = [og.zipf_tokens(256, 8, 256, seed=900 + 10 * s + rank) for s in range(4)]
        batches = [(x.to(dev), y.to(dev)) for x, y in batches]

        def run(m, o):
            out = []
            for x, y in batches:
                loss = m(x, y, grad_scale=o.scale)
                o.backward(loss)
                st = o.step(lr=3e-4)
                o.zero_grad()
                out.append((float(loss.detach()), float(st["grad_norm"])))
            return out

        md, od = _fresh(dev)
        DataParallel(md, od)
        dp = run(md, od)
        mz, oz = _fresh(dev)
        sz = ShardedDataParallel(mz, oz)
        zr = run(mz, oz)
        sz.finish_gather()  # the last update's parameters (gathered lazily otherwise)
        flat_z = oz.flat16.detach().float().cpu()
        sz.consolidate()
        mg, og2 = _fresh(dev)
        sg = ShardedDataParallel(mg, og2)
        graphed = GraphedStep(mg, og2, batches[0][0], batches[0][1], warmup=1)
        replayed = [float(graphed(x, y)) for x, y in batches[1:]]
        torch.cuda.synchronize()
        sg.consolidate()
        out_q.put((rank, "ok", dict(
            dp=dp, zero=zr, replayed=replayed, shard=oz.shard,
            flat_dp=od.flat16.detach().float().cpu(), flat_z=flat_z,
            master_dp=od.master.detach().cpu(), master_z=oz.master.detach().cpu(),
            master_g=og2.master.detach().cpu(), m_z=oz.m.detach().cpu())))
    except Exception as e:  # report, then leave
        out_q.put((rank, "error", repr(e)))
    finally:
        if graphed is not None:
            graphed.release()
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def test_zero1_sharded_update_matches_dp():
    """ZeRO-1 (fxb200.zero): each rank updates half of FlatAdamW's buffers
    and gathers the bf16 parameters. With two ranks the reduced gradient is
    the same sum as DP's all-reduce; the norm is summed from two shard
    partials instead of one pass, so losses and weights agree with DP to
    rounding. Eager and graph-captured runs agree; ranks end bitwise equal."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    o = _run(_zero_worker)
    assert [x["shard"][0] for x in o] == [0, o[0]["shard"][1]]
    for r in range(WORLD):
        for (ld, nd), (lz, nz) in zip(o[r]["dp"], o[r]["zero"]):
            assert abs(lz - ld) <= 1e-4 * abs(ld), (o[r]["dp"], o[r]["zero"])
            assert abs(nz - nd) <= 1e-4 * abs(nd), (o[r]["dp"], o[r]["zero"])
        for a, (b, _n) in zip(o[r]["replayed"], o[r]["zero"][1:]):
            assert abs(a - b) <= 1e-3 * abs(b), (o[r]["replayed"], o[r]["zero"])
        d = ((o[r]["master_z"] - o[r]["master_dp"]).norm() / o[r]["master_dp"].norm()).item()
        assert d < 1e-4, f"rank {r}: zero vs dp master rel {d:.3e}"
        d = ((o[r]["master_g"] - o[r]["master_z"]).norm() / o[r]["master_z"].norm()).item()
        assert d < 1e-2, f"rank {r}: graphed vs eager zero master rel {d:.3e}"
        d = ((o[r]["flat_z"] - o[r]["flat_dp"]).norm() / o[r]["flat_dp"].norm()).item()
        assert d < 1e-3, f"rank {r}: zero vs dp bf16 params rel {d:.3e}"
    for key in ("flat_z", "master_z", "m_z", "master_g"):
        assert torch.equal(o[0][key], o[1][key]), key


def test_dp_nccl_graph_matches_eager_and_accumulation():
    if not torch.cuda.is_available() or torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(WORLD):
        r, status, payload = q.get(timeout=600)
        res[r] = (status, payload)
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    for r in range(WORLD):
        assert res[r][0] == "ok", res[r][1]
    o = [res[r][1] for r in range(WORLD)]

    # accumulation over both ranks' first batches, one process (cuda:0)
    from oracle import gpt as og
    dev = torch.device("cuda", 0)
    m, opt = _fresh(dev)
    for r in range(WORLD):
        x, y = og.zipf_tokens(256, 8, 256, seed=700 + r)
        loss = m(x.to(dev), y.to(dev), grad_scale=opt.scale)
        opt.backward(loss / WORLD)
    opt._fold_param_grads()
    acc = opt.grad.detach().cpu()
    opt.zero_grad()
    for r in range(WORLD):
        g = o[r]["dp_grad"]
        rel = ((g.double() - acc.double()).norm() / acc.double().norm()).item()
        assert rel < 1e-3, f"rank {r}: DP grad vs accumulation rel {rel:.3e}"

    for r in range(WORLD):
        for a, b in zip(o[r]["replayed"], o[r]["eager"][1:]):
            assert abs(a - b) <= 1e-3 * abs(b), (o[r]["replayed"], o[r]["eager"])
        d = ((o[r]["master_g"] - o[r]["master_e"]).norm() / o[r]["master_e"].norm()).item()
        assert d < 1e-2, f"rank {r}: graphed vs eager master rel {d:.3e}"
    # identical reduced gradients -> identical weights on every rank
    assert torch.equal(o[0]["master_e"], o[1]["master_e"])
    assert torch.equal(o[0]["master_g"], o[1]["master_g"])
