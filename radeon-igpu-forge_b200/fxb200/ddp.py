"""Data-parallel gradient synchronisation for FlatAdamW (one process per GPU).

The reference is single-GPU (ml/fxgpu/env.py:12, ml/fxlm/env.py:46). This
module adds the one exchange step of data parallelism: the mean all-reduce of
FlatAdamW's flat fp32 gradient. The flat buffer is split into buckets that
follow parameter groups (one transformer block per bucket, the embeddings
last); each bucket is all-reduced with NCCL (AVG) on a side stream as soon as
its gradients are final, overlapping the rest of backward:

  - a block's gradients are final when the gradient with respect to that
    block's input has been produced (all of the block's backward launches
    precede it on the compute stream): a tensor hook registered in a forward
    pre-hook records an event there and enqueues the bucket's all-reduce on the
    communication stream after that event;
  - whatever no hook covered (embeddings, parameters outside blocks) is
    reduced from FlatAdamW's pre-step hook, after which the compute stream
    waits for every reduction before the optimizer kernels read the buffer.

Every rank runs the same buckets in the same order, so all ranks apply the
identical reduced gradient and keep identical found_inf / loss-scale state.
"""
import torch
import torch.distributed as dist


class DataParallel:
    """Attach bucketed gradient all-reduce to (model, FlatAdamW).

    dp = DataParallel(model, opt)          # after FlatAdamW(model, ...)
    loss = model(x, y, grad_scale=opt.scale); opt.backward(loss); opt.step(lr)
    """

    def __init__(self, model, opt, process_group=None, block_attr="blocks", bucket_mb=None,
                 comm_dtype=None):
        if not dist.is_available() or not dist.is_initialized():
            raise RuntimeError("torch.distributed must be initialised before DataParallel")
        self.model, self.opt = model, opt
        self.pg = process_group
        self.world = dist.get_world_size(process_group)
        dev = opt.grad.device
        # comm_dtype=torch.bfloat16: buckets cross NVLink as bf16 (half the bytes
        # of the fp32 gradient; NCCL sums in bf16) and are widened back to fp32
        # after the reduction; None keeps the fp32 gradient on the wire
        if comm_dtype not in (None, torch.float32, torch.bfloat16):
            raise ValueError(f"comm_dtype must be None, float32 or bfloat16, got {comm_dtype}")
        self.comm_dtype = None if comm_dtype in (None, torch.float32) else comm_dtype
        self._wire = (torch.empty(opt.grad.numel(), device=dev, dtype=self.comm_dtype)
                      if self.comm_dtype is not None else None)
        self.stream = torch.cuda.Stream(device=dev) if dev.type == "cuda" else None
        # the hooks only enqueue work (events, NCCL on a side stream, stream
        # waits) and never read results on the host, so a step that runs
        # them can be captured in a CUDA graph (fxlm.GraphedStep)
        self.graph_capturable = self.stream is not None
        self._pending = []      # (work, bucket) launched this backward
        self._done = set()
        # bucket = contiguous range of the flat gradient: one per block
        offs = {name: (off, n) for name, _p, off, n, _w in opt._info}
        blocks = getattr(model, block_attr, None)
        self.buckets = []       # (name, start, end)
        self._block_bucket = {}
        if blocks is not None:
            for i, _blk in enumerate(blocks):
                prefix = f"{block_attr}.{i}."
                rng = [(o, o + ((n + 7) & ~7)) for nm, (o, n) in offs.items() if nm.startswith(prefix)]
                if rng:
                    b = (f"block{i}", min(r[0] for r in rng), max(r[1] for r in rng))
                    self._block_bucket[i] = len(self.buckets)
                    self.buckets.append(b)
        covered = sorted((s, e) for _n, s, e in self.buckets)
        # remainder ranges (embeddings, final norm, ...): reduced at pre-step
        self._rest = []
        cur = 0
        for s, e in covered:
            if s > cur:
                self._rest.append((cur, s))
            cur = max(cur, e)
        if cur < opt.numel:
            self._rest.append((cur, opt.numel))
        if blocks is not None:
            for i, blk in enumerate(blocks):
                if i in self._block_bucket:
                    blk.register_forward_pre_hook(self._make_pre_hook(self._block_bucket[i]))
        opt.pre_step_hooks.append(self._finish)

    # -- hooks ---------------------------------------------------------------
    def _make_pre_hook(self, bidx):
        def pre_hook(_module, args):
            x = args[0]
            if torch.is_grad_enabled() and isinstance(x, torch.Tensor) and x.requires_grad:
                x.register_hook(lambda g, b=bidx: self._launch(b))
        return pre_hook

    def _reduce_range(self, start, end):
        """Enqueue the mean all-reduce of grad[start:end]; returns a list of
        (work, view, needs_div)."""
        view = self.opt.grad[start:end]
        if self.stream is None:
            # CPU / gloo (tests): gloo has no AVG, so SUM then divide after wait
            if self._wire is not None:
                wire = self._wire[start:end]
                wire.copy_(view)
                w = dist.all_reduce(wire, op=dist.ReduceOp.SUM, group=self.pg, async_op=True)
                return [(w, view, True, wire)]
            return [(dist.all_reduce(view, op=dist.ReduceOp.SUM, group=self.pg, async_op=True), view, True)]
        ev = torch.cuda.Event()
        ev.record(torch.cuda.current_stream(view.device))
        with torch.cuda.stream(self.stream):
            self.stream.wait_event(ev)
            if self._wire is not None:
                wire = self._wire[start:end]
                wire.copy_(view)
                w = dist.all_reduce(wire, op=dist.ReduceOp.AVG, group=self.pg, async_op=True)
                w.wait()          # the side stream waits for NCCL's stream (no host sync)
                view.copy_(wire)  # then widens the reduced bucket back to fp32
                return [(w, view, False)]
            return [(dist.all_reduce(view, op=dist.ReduceOp.AVG, group=self.pg, async_op=True), view, False)]

    def _launch(self, bidx):
        if bidx in self._done:
            return
        self._done.add(bidx)
        _n, s, e = self.buckets[bidx]
        self._pending.extend(self._reduce_range(s, e))

    def _finish(self, _opt):
        # buckets whose hook did not fire (e.g. no grad path) are reduced here,
        # in bucket order, so every rank issues the same collective sequence
        for b in range(len(self.buckets) - 1, -1, -1):
            if b not in self._done:
                self._launch(b)
        for s, e in self._rest:
            self._pending.extend(self._reduce_range(s, e))
        for item in self._pending:
            w, view, needs_div = item[:3]
            w.wait()
            if len(item) > 3:  # CPU path with a narrower wire dtype
                view.copy_(item[3])
            if needs_div:
                view.div_(self.world)
        if self.stream is not None:
            torch.cuda.current_stream(self.opt.grad.device).wait_stream(self.stream)
        self._pending = []
        self._done = set()
