"""CPU tests of the optimizer-sharding host logic (fxb200.zero).

Shard arithmetic (cover, alignment, equal padded sizes), bucket pieces cut at
shard boundaries, the weight-decay segments of a shard, and the collective
hooks of ShardedDataParallel run as three gloo ranks against a stand-in for
FlatAdamW's buffers (the real optimizer needs a GPU): each rank ends with the
mean gradient of its own shard, the summed norm partials and flags, the
gathered parameters, a zeroed gradient outside its shard, and after
consolidate() the same master / m / v as every other rank. The reference has
no multi-GPU path; the oracle is the single-process mean.
"""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fxb200.zero import shard_ranges, split_by_shard
from fxlm.optim import shard_segments


@pytest.mark.parametrize("numel", [0, 8, 16, 24, 72, 8000, 110_906_112])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_ranges_cover_and_align(numel, world):
    shards, size = shard_ranges(numel, world)
    assert len(shards) == world and size % 8 == 0
    assert size * world >= numel and size * world - numel < 8 * world + size
    cur = 0
    for lo, hi in shards:
        assert lo == cur and lo <= hi and lo % 8 == 0 and hi % 8 == 0
        assert hi - lo <= size
        cur = hi
    assert cur == numel


def test_split_by_shard():
    shards, _ = shard_ranges(72, 3)          # [(0,24), (24,48), (48,72)]
    assert shards == [(0, 24), (24, 48), (48, 72)]
    assert split_by_shard(16, 40, shards) == [(0, 16, 24), (1, 24, 40)]
    assert split_by_shard(0, 72, shards) == [(0, 0, 24), (1, 24, 48), (2, 48, 72)]
    assert split_by_shard(24, 48, shards) == [(1, 24, 48)]
    assert split_by_shard(30, 30, shards) == []


def test_shard_segments():
    ends, wds = [16, 40, 48, 96], [1, 0, 1, 1]
    assert shard_segments(ends, wds, 0, 96) == (ends, wds)
    assert shard_segments(ends, wds, 24, 64) == ([16, 24, 40], [0, 1, 1])
    assert shard_segments(ends, wds, 40, 48) == ([8], [1])
    assert shard_segments(ends, wds, 48, 48) == ([], [])


class _Model(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.blocks = torch.nn.ModuleList([torch.nn.Linear(5, 3, bias=False), torch.nn.Linear(7, 2)])
        self.emb = torch.nn.Parameter(torch.zeros(10, 3))
        self.extra = torch.nn.Parameter(torch.zeros(5))

    def forward(self):
        # touches every block, so that forward pre-hooks run as in a GPT
        self.blocks[0](torch.zeros(1, 5, dtype=torch.bfloat16))
        self.blocks[1](torch.zeros(1, 7, dtype=torch.bfloat16))


class _FlatStandIn:
    """The buffers and hook lists of FlatAdamW that the sharding touches."""

    def __init__(self, model):
        self._info, off = [], 0
        for name, p in model.named_parameters():
            self._info.append((name, p, off, p.numel(), int(p.dim() >= 2)))
            off += (p.numel() + 7) & ~7
        self.numel = off
        self.grad = torch.zeros(off)
        self.master, self.m, self.v = torch.zeros(off), torch.zeros(off), torch.zeros(off)
        self.flat16 = torch.zeros(off, dtype=torch.bfloat16)
        for _nm, p, o, n, _w in self._info:       # parameters are views, as in FlatAdamW
            p.data = self.flat16[o:o + n].view(p.shape)
        self.scratch = torch.zeros(2)
        self._flags = torch.zeros((), dtype=torch.int32)
        self.pre_step_hooks, self.norm_hooks, self.post_step_hooks = [], [], []
        self.shard = None

    def set_shard(self, lo, hi):
        self.shard = (lo, hi)


def _worker(rank, world, port, q, defer=False):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        from fxb200.zero import ShardedDataParallel
        model = _Model()
        opt = _FlatStandIn(model)
        sdp = ShardedDataParallel(model, opt, defer_gather=defer)
        lo, hi = opt.shard
        n = opt.numel
        base = torch.arange(n, dtype=torch.float32) + 1
        opt.grad.copy_(base * (rank + 1))
        for h in opt.pre_step_hooks:              # bucket reduces to the owners
            h(opt)
        res = {"shard": (lo, hi), "numel": n, "buckets": [(s, e) for _n, s, e in sdp.buckets],
               "grad_shard": opt.grad[lo:hi].clone()}
        opt.scratch[0] = float(rank + 1)          # this shard's sum of squares
        opt._flags.fill_(1 if rank == 1 else 0)
        for h in opt.norm_hooks:
            h(opt)
        res["norm"] = (float(opt.scratch[0]), int(opt._flags))
        s = sdp.shard_size
        sdp.flat16_padded[rank * s:(rank + 1) * s] = float(rank + 1)   # "updated" shard
        opt.grad[lo:hi].zero_()                   # what the shard update leaves
        for h in opt.post_step_hooks:
            h(opt)
        if defer:
            # the gather waits for the next forward: only this rank's shard is new
            res["flat16_before"] = opt.flat16.float().clone()
            model()
            sdp.finish_gather()                   # nothing left to do
        res["flat16"] = opt.flat16.float().clone()
        res["grad_after"] = opt.grad.clone()
        for t, k in ((opt.master, 1.0), (opt.m, 2.0), (opt.v, 3.0)):
            t[lo:hi] = k * (rank + 1)
        sdp.consolidate()
        res["state"] = torch.stack([opt.master, opt.m, opt.v]).clone()
        res["param_is_view"] = all(p.data_ptr() == opt.flat16[off:].data_ptr()
                                   for _nm, p, off, _n, _w in opt._info)
        q.put((rank, "ok", res))
    except Exception as e:  # report, then leave
        q.put((rank, "error", repr(e)))
    finally:
        dist.destroy_process_group()


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


@pytest.mark.parametrize("defer", [False, True])
def test_sharded_hooks_three_gloo_ranks(defer):
    """defer=True: the parameter gather runs in the next forward's pre-hook
    (per-range broadcasts from the owners, the GPU path's order) instead of
    right after the update."""
    world = 3
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, defer)) for r in range(world)]
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
    for r in range(world):
        assert res[r][0] == "ok", res[r][1]
    o = [res[r][1] for r in range(world)]
    n = o[0]["numel"]
    # flat layout: emb [0, 30), extra [32, 37), blocks.0 [40, 55), blocks.1
    # [56, 70) + bias [72, 74): 80 elements, shards of 32 (padded to 96, so
    # the parameters are re-homed); the remainder range [0, 40) straddles the
    # first shard boundary, block 1's bucket [56, 80) the second
    assert n == 80 and [x["shard"] for x in o] == [(0, 32), (32, 64), (64, 80)]
    assert o[0]["buckets"] == [(40, 56), (56, 80)]
    mean = (torch.arange(n, dtype=torch.float32) + 1) * 2.0      # (1 + 2 + 3) / 3
    expect_flat = torch.cat([torch.full((32,), float(r + 1)) for r in range(world)])[:n]
    for r in range(world):
        lo, hi = o[r]["shard"]
        assert torch.equal(o[r]["grad_shard"], mean[lo:hi]), r
        assert o[r]["norm"] == (6.0, 1)
        assert torch.equal(o[r]["flat16"], expect_flat)
        if defer:
            lo, hi = o[r]["shard"]
            before = o[r]["flat16_before"]
            assert torch.equal(before[lo:hi], expect_flat[lo:hi])
            assert torch.count_nonzero(torch.cat([before[:lo], before[hi:]])) == 0
        assert torch.count_nonzero(o[r]["grad_after"]) == 0
        assert o[r]["param_is_view"]
        assert torch.equal(o[r]["state"], o[0]["state"])
    assert torch.equal(o[0]["state"][1], 2.0 * expect_flat)
