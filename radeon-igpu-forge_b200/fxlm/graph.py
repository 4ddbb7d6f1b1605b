"""fxlm.graph: one whole training step (forward, backward, FlatAdamW update)
captured in a CUDA graph and replayed.

The reference runs its step eagerly from Python (ml/fxlm/train_lm.py training
loop; no compiler on its hot path). A step of the B200 build is ~300 kernel
launches, each a ctypes call; at B200 speeds the host then becomes the
bound. Capturing the step once and replaying it removes the per-launch host
work without changing a single kernel or its arguments.

    step = GraphedStep(model, opt, x_example, y_example)   # runs `warmup` real steps, then captures
    loss = step(x, y, lr=3e-4)    # copies the batch into the static inputs, replays; loss stays on device

Conditions (checked where cheap): fixed batch shape; the optimizer is a
FlatAdamW whose gradient buffer is consumed by its update (so no zeroing op
is needed between replays); the learning rate is read from `opt.lr_dev`, a
device scalar written before each replay; optimizer hooks (pre-step, norm,
post-step) only if their owner declares `graph_capturable`
(fxb200.ddp.DataParallel and fxb200.zero.ShardedDataParallel do: their
collectives are NCCL calls on a side stream forked from the capturing
stream, so they are recorded into the graph and replayed with it). The
warm-up steps before capture are real training steps (they also trigger every
lazy initialisation: library load, tensor-map encoders, shared-memory
attributes, NCCL communicators). A graph that holds NCCL calls must be
released (`release()`) before the process group is destroyed.
"""
import torch

from fxb200 import _lib, ops


class GraphedStep:
    def __init__(self, model, opt, x_example, y_example, warmup=3):
        for kind in ("pre_step_hooks", "norm_hooks", "post_step_hooks"):
            for h in getattr(opt, kind, None) or ():
                if not getattr(getattr(h, "__self__", None), "graph_capturable", False):
                    raise ValueError(f"GraphedStep: optimizer has a {kind[:-1].replace('_', '-')} "
                                     "that cannot be captured; run the step eagerly")
        if warmup < 1:
            raise ValueError("GraphedStep: warmup >= 1 (lazy initialisation must happen "
                             "before capture)")
        self.model, self.opt = model, opt
        dev = opt.grad.device
        self.x = torch.empty_like(x_example, device=dev)
        self.y = torch.empty_like(y_example, device=dev)
        self.x.copy_(x_example)
        self.y.copy_(y_example)
        if opt.lr_dev is None:
            opt.lr_dev = torch.full((), float(opt.lr), device=dev, dtype=torch.float32)
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                self._step()
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        _lib.raise_on_device_error("during GraphedStep warm-up")
        self.graph = torch.cuda.CUDAGraph()
        self._ws = {}  # GEMM workspaces of this graph
        n0 = _lib.launch_count()
        with ops.graph_workspaces(self._ws), torch.cuda.graph(self.graph):
            self.loss = self._step()
        # kernels of this library inside one replay
        self.launches_per_step = _lib.launch_count() - n0

    def _step(self):
        loss = self.model(self.x, self.y, grad_scale=self.opt.scale)
        self.opt.backward(loss)
        self.opt.step()
        self.opt.zero_grad()
        return loss.detach()

    def __call__(self, x=None, y=None, lr=None):
        """Copy (x, y) into the static inputs (when given), set the learning
        rate (when given) and replay; returns the step's loss (device)."""
        for name, dst, src in (("x", self.x, x), ("y", self.y, y)):
            if src is None:
                continue
            if tuple(src.shape) != tuple(dst.shape) or src.dtype != dst.dtype:
                raise ValueError(f"GraphedStep: {name} is {tuple(src.shape)} {src.dtype}, "
                                 f"captured with {tuple(dst.shape)} {dst.dtype}")
            dst.copy_(src, non_blocking=True)
        if lr is not None:
            self.opt.lr_dev.fill_(float(lr))
        self.graph.replay()
        return self.loss

    def check(self):
        """Synchronise and raise RuntimeError if a kernel's bounded wait expired
        in a replay since the last check (call it where the loop reads the
        loss anyway, e.g. at log steps)."""
        _lib.raise_on_device_error("in a GraphedStep replay")

    def release(self):
        """Free the captured graph (required before destroy_process_group when
        the step holds NCCL collectives)."""
        if self.graph is not None:
            torch.cuda.synchronize()
            self.graph.reset()
            self.graph = None


class GraphedFunction:
    """Any training step as a replayed CUDA graph: `fn(*static_args)` is run
    `warmup` times on a side stream (real steps: lazy initialisation happens
    there), then captured once; each call copies its arguments into the
    static device buffers (None keeps the previous contents), replays, and
    returns the captured output (device tensors, overwritten by the next
    call).

        def train_step(idx, tgt):
            loss = ((model(X16, idx).float() - tgt) ** 2).mean()
            opt.backward(loss); opt.step(); opt.zero_grad()
            return loss.detach()
        step = GraphedFunction(train_step, idx_example, tgt_example)
        loss = step(idx, tgt)

    The same conditions as GraphedStep hold for what `fn` does: fixed shapes,
    no host synchronisation, and a FlatAdamW learning rate that changes
    between replays read from `opt.lr_dev` (set it before constructing).
    Tensors the closure reads but that are not arguments are captured by
    address: update them in place.
    """

    def __init__(self, fn, *example_args, warmup=3):
        if warmup < 1:
            raise ValueError("GraphedFunction: warmup >= 1 (lazy initialisation must happen "
                             "before capture)")
        if not example_args or not all(isinstance(a, torch.Tensor) and a.is_cuda
                                       for a in example_args):
            raise TypeError("GraphedFunction: example arguments must be cuda tensors")
        self.fn = fn
        dev = example_args[0].device
        self.args = [a.detach().clone() for a in example_args]
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for _ in range(warmup):
                fn(*self.args)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        _lib.raise_on_device_error("during GraphedFunction warm-up")
        self.graph = torch.cuda.CUDAGraph()
        self._ws = {}  # GEMM workspaces of this graph
        n0 = _lib.launch_count()
        with ops.graph_workspaces(self._ws), torch.cuda.graph(self.graph):
            self.out = fn(*self.args)
        self.launches_per_call = _lib.launch_count() - n0

    def __call__(self, *args):
        if len(args) > len(self.args):
            raise TypeError(f"GraphedFunction: {len(args)} arguments, captured with {len(self.args)}")
        for i, (dst, src) in enumerate(zip(self.args, args)):
            if src is None:
                continue
            # copy_ would broadcast or cast silently: a wrong shape or dtype is an error here
            if tuple(src.shape) != tuple(dst.shape):
                raise ValueError(f"GraphedFunction: argument {i} has shape {tuple(src.shape)}, "
                                 f"captured with {tuple(dst.shape)}")
            if src.dtype != dst.dtype:
                raise TypeError(f"GraphedFunction: argument {i} has dtype {src.dtype}, "
                                f"captured with {dst.dtype}")
            dst.copy_(src, non_blocking=True)
        self.graph.replay()
        return self.out

    def check(self):
        """Synchronise and raise RuntimeError if a kernel's bounded wait expired
        in a replay since the last check."""
        _lib.raise_on_device_error("in a GraphedFunction replay")

    def release(self):
        """Free the captured graph (before destroy_process_group when the
        step holds NCCL collectives)."""
        if self.graph is not None:
            torch.cuda.synchronize()
            self.graph.reset()
            self.graph = None
