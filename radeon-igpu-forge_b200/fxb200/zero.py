"""Optimizer-state sharding (ZeRO stage 1) for FlatAdamW over data parallelism.

The reference trains on one GPU (ml/fxlm/train_lm.py) and has no sharding;
this is the data-parallel variant in which each of the W ranks updates only
its own contiguous shard of FlatAdamW's flat buffers:

  - backward: the same gradient buckets as fxb200.ddp.DataParallel (one per
    transformer block, launched as soon as the block's gradients are final,
    on a side stream), but each bucket is reduced (mean) only to the rank(s)
    owning it, split at shard boundaries: every rank sends its whole
    gradient once and receives its shard, instead of receiving everything;
  - step: the sum of squares covers the rank's shard; the partial sums (and
    the non-finite flags) are summed over the ranks before finalize, so every
    rank derives the same norm, clip coefficient, found_inf and loss scale;
    the AdamW update (the HBM-bound pass over 38 bytes per parameter) runs
    over the shard only;
  - after the update the gradient outside the shard is zeroed for the next
    backward, and the low-precision parameters are gathered in place: one
    all-gather into a flat buffer padded to W equal shards. With
    defer_gather=True the gather moves to the start of the next forward and
    overlaps it instead: every parameter range is broadcast from the rank
    owning it, on the side stream, in the order the forward uses them
    (embeddings and the final norm first, then the blocks), and each block's
    forward waits only for its own range (finish_gather() completes a
    pending gather for readers outside a forward). Measured at 2 GPUs on the
    config-4 step it was 0.8% slower than the single all-gather (about
    twenty broadcasts against one collective), so it is off by default.

The fp32 master, m and v outside a rank's shard are not maintained there;
`consolidate()` broadcasts every shard so that `opt.state_dict()` is whole
(call it before saving a checkpoint). Shards are multiples of 8 elements,
as FlatAdamW's parameter offsets are.

Every hook only enqueues work (events, NCCL calls on the side stream, stream
waits, device ops), so the step can be captured in a CUDA graph
(fxlm.GraphedStep), like DataParallel's.
"""
import os

import torch
import torch.distributed as dist

from .ddp import DataParallel


def shard_ranges(numel, world):
    """([(lo, hi)] per rank, shard size S): S = ceil(numel / world) rounded
    up to a multiple of 8; rank r owns [r*S, (r+1)*S) clipped to numel (the
    last shards may be short or empty)."""
    if world < 1 or numel < 0:
        raise ValueError(f"bad numel={numel} world={world}")
    size = ((-(-numel // world)) + 7) & ~7
    return [(min(r * size, numel), min((r + 1) * size, numel)) for r in range(world)], size


def split_by_shard(start, end, shards):
    """Pieces (rank, a, b) of [start, end) cut at the shard boundaries, in
    rank order."""
    out = []
    for r, (lo, hi) in enumerate(shards):
        a, b = max(start, lo), min(end, hi)
        if a < b:
            out.append((r, a, b))
    return out


class ShardedDataParallel(DataParallel):
    """DataParallel with FlatAdamW's update sharded over the ranks.

    sdp = ShardedDataParallel(model, opt)    # after FlatAdamW(model, ...)
    loss = model(x, y, grad_scale=opt.scale); opt.backward(loss); opt.step(lr)
    sdp.consolidate(); torch.save(opt.state_dict(), ...)
    """

    def __init__(self, model, opt, process_group=None, block_attr="blocks", comm_dtype=None,
                 defer_gather=None):
        super().__init__(model, opt, process_group=process_group, block_attr=block_attr,
                         comm_dtype=comm_dtype)
        self.rank = dist.get_rank(process_group)
        self.shards, self.shard_size = shard_ranges(opt.numel, self.world)
        self._global = [dist.get_global_rank(process_group, r) if process_group is not None else r
                        for r in range(self.world)]
        padded = self.world * self.shard_size
        if opt.flat16.numel() != padded:
            # re-home the parameters in a buffer of W equal shards, so that
            # the all-gather after the update can run in place
            buf = torch.zeros(padded, dtype=opt.flat16.dtype, device=opt.flat16.device)
            buf[:opt.numel].copy_(opt.flat16)
            for _nm, p, off, n, _wd in opt._info:
                p.data = buf[off:off + n].view(p.shape)
            opt.flat16 = buf[:opt.numel]
            self.flat16_padded = buf
        else:
            self.flat16_padded = opt.flat16
        lo, hi = self.shards[self.rank]
        opt.set_shard(lo, hi)
        opt.norm_hooks.append(self._sum_norm)
        opt.post_step_hooks.append(self._gather)
        # deferred gather (optional): parameter ranges in forward
        # order, group 0 = everything outside the blocks, group 1 + i = block i
        # (FXB_ZERO_DEFER=1 turns it on when the argument is not given)
        if defer_gather is None:
            defer_gather = os.environ.get("FXB_ZERO_DEFER", "0") == "1"
        self.defer_gather = bool(defer_gather)
        self._gather_pending = False
        self._gather_groups = [list(self._rest)] + [[(s, e)] for _n, s, e in self.buckets]
        self._gather_events = None  # per group, recorded by the forward that gathered
        if self.defer_gather:
            model.register_forward_pre_hook(self._pre_forward)
            blocks = getattr(model, block_attr, None)
            if blocks is not None:
                for i, blk in enumerate(blocks):
                    if i in self._block_bucket:
                        blk.register_forward_pre_hook(self._make_wait_hook(1 + self._block_bucket[i]))

    # -- backward: each bucket piece to its owner ---------------------------
    def _reduce_range(self, start, end):
        grad = self.opt.grad
        pieces = split_by_shard(start, end, self.shards)
        out = []
        wire_all = self._wire
        if self.stream is None:
            # CPU / gloo (tests): SUM, then the owner divides after the wait
            for r, a, b in pieces:
                view = grad[a:b]
                if wire_all is not None:
                    wire = wire_all[a:b]
                    wire.copy_(view)
                    w = dist.reduce(wire, dst=self._global[r], op=dist.ReduceOp.SUM, group=self.pg,
                                    async_op=True)
                    out.append((w, view, r == self.rank, wire) if r == self.rank else (w, view, False))
                    continue
                w = dist.reduce(view, dst=self._global[r], op=dist.ReduceOp.SUM, group=self.pg,
                                async_op=True)
                out.append((w, view, r == self.rank))
            return out
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(grad.device))
        with torch.cuda.stream(self.stream):
            self.stream.wait_event(ev)
            for r, a, b in pieces:
                view = grad[a:b]
                if wire_all is not None:
                    # the bucket crosses NVLink as bf16; the owner widens its
                    # reduced piece back into the fp32 gradient (stream-ordered)
                    wire = wire_all[a:b]
                    wire.copy_(view)
                    w = dist.reduce(wire, dst=self._global[r], op=dist.ReduceOp.AVG, group=self.pg,
                                    async_op=True)
                    if r == self.rank:
                        w.wait()  # the side stream waits for NCCL's stream (no host sync)
                        view.copy_(wire)
                    out.append((w, view, False))
                    continue
                w = dist.reduce(view, dst=self._global[r], op=dist.ReduceOp.AVG, group=self.pg,
                                async_op=True)
                out.append((w, view, False))
        return out

    # -- step: global norm from the shards' partial sums ---------------------
    def _sum_norm(self, opt):
        # scratch[0] holds this shard's sum of squares; scratch[1] is free
        # until finalize writes the clip coefficient, so the flags ride along
        # and both are summed in one all-reduce
        pair = opt.scratch[:2]
        opt.scratch[1:2].copy_(opt._flags.view(1))
        if self.stream is None:
            dist.all_reduce(pair, op=dist.ReduceOp.SUM, group=self.pg)
        else:
            cur = torch.cuda.current_stream(pair.device)
            self.stream.wait_stream(cur)
            with torch.cuda.stream(self.stream):
                dist.all_reduce(pair, op=dist.ReduceOp.SUM, group=self.pg)
            cur.wait_stream(self.stream)
        opt._flags.copy_(opt.scratch[1])

    # -- after the update: everyone's parameters, a clean gradient -----------
    def _gather(self, opt):
        if self.defer_gather:
            lo, hi = opt.shard
            opt.grad[:lo].zero_()
            opt.grad[hi:].zero_()
            self._gather_pending = True
            return
        self._gather_all()
        lo, hi = opt.shard
        opt.grad[:lo].zero_()
        opt.grad[hi:].zero_()

    def _gather_all(self):
        """All-gather every rank's shard of the low-precision parameters."""
        s = self.shard_size
        mine = self.flat16_padded[self.rank * s:(self.rank + 1) * s]
        if self.stream is None:
            dist.all_gather_into_tensor(self.flat16_padded, mine, group=self.pg)
        else:
            cur = torch.cuda.current_stream(mine.device)
            self.stream.wait_stream(cur)
            with torch.cuda.stream(self.stream):
                dist.all_gather_into_tensor(self.flat16_padded, mine, group=self.pg)
            cur.wait_stream(self.stream)

    def finish_gather(self):
        """Complete a deferred parameter gather now (before reading the
        parameters outside a forward: checkpoints, replica checks)."""
        if self._gather_pending:
            self._gather_all()
            self._gather_pending = False

    # -- deferred gather: broadcasts overlapping the next forward -------------
    def _broadcast_ranges(self, ranges):
        works = []
        for start, end in ranges:
            for r, a, b in split_by_shard(start, end, self.shards):
                works.append(dist.broadcast(self.flat16_padded[a:b], src=self._global[r],
                                            group=self.pg, async_op=True))
        return works

    def _pre_forward(self, _module, _args):
        capturing = self.stream is not None and torch.cuda.is_current_stream_capturing()
        if not (self._gather_pending or capturing):
            self._gather_events = None
            return
        # a captured step always starts with the gather: its replays follow
        # each other, every one gathering the update of the one before
        self._gather_pending = False
        if self.stream is None:
            for grp in self._gather_groups:
                for w in self._broadcast_ranges(grp):
                    w.wait()
            self._gather_events = None
            return
        cur = torch.cuda.current_stream(self.flat16_padded.device)
        self.stream.wait_stream(cur)  # the update has written this rank's shard
        events = []
        with torch.cuda.stream(self.stream):
            for grp in self._gather_groups:
                for w in self._broadcast_ranges(grp):
                    w.wait()  # the side stream waits for NCCL's stream (no host sync)
                ev = torch.cuda.Event()
                ev.record(self.stream)
                events.append(ev)
        self._gather_events = events
        cur.wait_event(events[0])  # embeddings and the final norm; each block
        # waits for its own group in its forward pre-hook (every group is
        # some block's, so a captured step joins all of them)

    def _make_wait_hook(self, gidx):
        def hook(_module, _args):
            ev = self._gather_events
            if ev is not None:
                torch.cuda.current_stream(self.flat16_padded.device).wait_event(ev[gidx])
        return hook

    def consolidate(self):
        """Broadcast every rank's shard of master, m and v, so that each rank
        holds the whole optimizer state (before opt.state_dict()); a deferred
        parameter gather is completed first."""
        self.finish_gather()
        opt = self.opt
        for r, (lo, hi) in enumerate(self.shards):
            if hi > lo:
                for t in (opt.master, opt.m, opt.v):
                    dist.broadcast(t[lo:hi], src=self._global[r], group=self.pg)
