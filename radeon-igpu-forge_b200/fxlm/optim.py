"""fxlm.optim: FlatAdamW on sm_100a — fp32 master/m/v + low-precision params.

API and semantics of the reference (ml/fxlm/optim.py:50-196): parameters are
copied into one flat fp32 master (8-element aligned offsets, :82-90), every
model parameter becomes a view of one flat low-precision buffer (:94), and
step() runs sum-of-squares + non-finite check -> finalize (found_inf, global
norm, clip coefficient, step counter) -> decoupled-weight-decay AdamW (wd only
on ndim >= 2 params, :82-84) -> torch._amp_update_scale_ (:170-171), with no
host synchronisation.

B200 changes:
  - the gradient is one flat fp32 buffer with the master's offsets. Fused ops
    (fxlm.linear, fxlm.norm, the embedding and linear-CE) accumulate into it
    directly through each parameter's `_fxb_grad` view; gradients that arrive
    the ordinary way in `p.grad` (any other module) are folded in at step();
  - each kernel is one pass over the flat buffers (the reference walks
    64-tensor lists); the update consumes (zeroes) the gradient;
  - the low-precision dtype is bf16 by default (param_dtype), fp16 and fp32
    are accepted.
"""
import torch

from fxb200 import _lib


def _align8(n):
    return (n + 7) & ~7


def shard_segments(ends, wds, lo, hi):
    """Weight-decay segments of flat[lo:hi): `ends` are the parameters'
    exclusive aligned end offsets (ascending), `wds` their flags. Returns
    (ends relative to lo, flags) of the segments that overlap the range, the
    last end clipped to hi - lo."""
    rel_end, rel_wd = [], []
    start = 0
    for e, wd in zip(ends, wds):
        if e > lo and start < hi:
            rel_end.append(min(e, hi) - lo)
            rel_wd.append(int(wd))
        start = e
    return rel_end, rel_wd


class FlatAdamW:
    """fp32 master + low-precision params + dynamic loss scale + global clip.

    opt = FlatAdamW(model, lr=3e-4, betas=(0.9,0.95), eps=1e-8,
                    weight_decay=0.1, max_grad_norm=1.0,
                    init_scale=2.**16, growth_interval=1000, param_dtype=torch.bfloat16)
    opt.backward(loss)              # (loss * opt.scale).backward()
    stats = opt.step(lr=...)        # {grad_norm, found_inf, scale} 0-dim cuda
    opt.zero_grad()
    """

    def __init__(self, model, lr=3e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1,
                 max_grad_norm=1.0, init_scale=2.0 ** 16, growth_interval=1000,
                 param_dtype=torch.bfloat16):
        params = [p for p in model.parameters() if p.requires_grad]
        names = [n for n, p in model.named_parameters() if p.requires_grad]
        if not params:
            raise ValueError("model has no parameters with requires_grad")
        dev = params[0].device
        if dev.type != "cuda":
            raise TypeError("parameters must be on a cuda device")
        if any(p.dtype != torch.float32 for p in params):
            raise TypeError("FlatAdamW expects fp32 parameters "
                            "(it converts them to the flat low-precision buffer)")
        if param_dtype not in (torch.bfloat16, torch.float16, torch.float32):
            raise TypeError(f"param_dtype {param_dtype} not supported")
        self.lr, self.betas, self.eps = lr, betas, eps
        self.weight_decay, self.max_grad_norm = weight_decay, max_grad_norm
        self.growth_interval = int(growth_interval)
        self.param_dtype = param_dtype

        self._info = []  # (name, p, off, numel, wd_flag)
        total = 0
        for name, p in zip(names, params):
            self._info.append((name, p, total, p.numel(),
                               1 if (p.dim() >= 2 and weight_decay != 0) else 0))
            total += _align8(p.numel())
        self.numel = total
        self.master = torch.zeros(total, device=dev, dtype=torch.float32)
        self.m = torch.zeros(total, device=dev, dtype=torch.float32)
        self.v = torch.zeros(total, device=dev, dtype=torch.float32)
        self.flat16 = torch.empty(total, device=dev, dtype=param_dtype)
        self.grad = torch.zeros(total, device=dev, dtype=torch.float32)
        for name, p, off, n, _wd in self._info:
            self.master[off:off + n] = p.data.reshape(-1)
        self.flat16.copy_(self.master)
        for name, p, off, n, _wd in self._info:
            p.data = self.flat16[off:off + n].view(p.shape)
            p._fxb_grad = self.grad[off:off + n].view(p.shape)
            p._fxb_owner = self
        # segment table for the per-parameter weight-decay flag
        ends = [off + _align8(n) for _nm, _p, off, n, _w in self._info]
        wds = [wd for _nm, _p, _o, _n, wd in self._info]
        self._seg_end = torch.tensor(ends, device=dev, dtype=torch.int64)
        self._seg_wd = torch.tensor(wds, device=dev, dtype=torch.int32)
        if len(ends) > 1024:
            raise ValueError(f"{len(ends)} parameters > 1024 segments supported")

        self.scratch = torch.zeros(2, device=dev, dtype=torch.float32)
        # per-block partial sums of the gradient norm, added in a fixed order
        # (bitwise identical norms on data-parallel ranks); kept zeroed by the kernel
        ws_words = (int(_lib.load().fxb_adamw_sumsq_ws_bytes()) + 3) // 4
        self._sumsq_ws = torch.zeros(ws_words, device=dev, dtype=torch.int32)
        self._flags = torch.zeros((), device=dev, dtype=torch.int32)
        self._step_ctr = torch.zeros((), device=dev, dtype=torch.int32)
        self._found_inf = torch.zeros((), device=dev, dtype=torch.float32)
        self._norm = torch.zeros((), device=dev, dtype=torch.float32)
        self.scale = torch.full((), float(init_scale), device=dev, dtype=torch.float32)
        self._growth = torch.zeros((), device=dev, dtype=torch.int32)
        # optional fp32 device scalar holding the learning rate; when set, the
        # update reads it instead of the `lr` argument (a captured CUDA graph
        # follows a schedule by writing this scalar between replays)
        self.lr_dev = None
        self._grad_dirty = False
        # hooks run after the gradient is complete and before the update
        # (data-parallel reduction of self.grad registers one here)
        self.pre_step_hooks = []
        # optimizer sharding (fxb200.zero): the sum of squares and the update
        # cover only [lo, hi) of the flat buffers; norm hooks run between the
        # sum of squares and finalize (cross-rank sum of the partial norms),
        # post-step hooks after the update (gather of the updated parameters)
        self.shard = None
        self.norm_hooks = []
        self.post_step_hooks = []

    # -- helpers -----------------------------------------------------------

    def _fold_param_grads(self):
        """Add gradients that arrived in p.grad (non-fused modules) into the flat buffer."""
        for name, p, off, n, _wd in self._info:
            g = p.grad
            if g is None:
                continue
            if g.dtype not in (torch.float16, torch.bfloat16, torch.float32):
                raise TypeError(f"{name}: unsupported grad dtype {g.dtype}")
            self.grad[off:off + n].add_(g.reshape(-1))
            p.grad = None
            self._grad_dirty = True

    def set_shard(self, lo, hi):
        """Restrict the sum of squares and the update to flat[lo:hi) (lo, hi
        multiples of 8, 0 <= lo <= hi <= numel); set_shard(None, None)
        restores the whole buffer. The caller owns the rest: reducing the norm across shards
        (norm_hooks), refreshing the other parameters and zeroing the
        gradient outside the shard (post_step_hooks)."""
        if lo is None:
            self.shard = None
            return
        lo, hi = int(lo), int(hi)
        if lo % 8 or hi % 8 or not 0 <= lo <= hi <= self.numel:
            raise ValueError(f"bad shard [{lo}, {hi}) of {self.numel}")
        ends = [off + _align8(n) for _nm, _p, off, n, _w in self._info]
        wds = [wd for _nm, _p, _o, _n, wd in self._info]
        rel_end, rel_wd = shard_segments(ends, wds, lo, hi)
        dev = self.grad.device
        self.shard = (lo, hi)
        self._shard_end = torch.tensor(rel_end or [0], device=dev, dtype=torch.int64)
        self._shard_wd = torch.tensor(rel_wd or [0], device=dev, dtype=torch.int32)
        self._shard_nseg = len(rel_end)

    # -- API -----------------------------------------------------------------

    def backward(self, loss):
        self._grad_dirty = True
        (loss * self.scale).backward()

    def step(self, lr=None):
        lr_v = self.lr if lr is None else float(lr)
        self._fold_param_grads()
        for hook in self.pre_step_hooks:
            hook(self)
        st = _lib.stream_ptr(self.grad.device)
        P = _lib.ptr
        if self.shard is None:
            lo, n = 0, self.numel
            seg_end, seg_wd, nseg = self._seg_end, self._seg_wd, len(self._info)
        else:
            lo, n = self.shard[0], self.shard[1] - self.shard[0]
            seg_end, seg_wd, nseg = self._shard_end, self._shard_wd, self._shard_nseg
        if n:
            _lib.call("fxb_adamw_sumsq_det", 0, P(self.grad[lo:]), n, P(self.scratch),
                      P(self._flags), P(self._sumsq_ws), st)
        for hook in self.norm_hooks:
            hook(self)
        _lib.call("fxb_adamw_final", P(self.scratch), P(self._flags), P(self._step_ctr),
                  P(self._found_inf), P(self._norm), P(self.scale),
                  float(self.max_grad_norm), st)
        if n:
            _lib.call("fxb_adamw_update", 0, _lib.dtype_code(self.param_dtype), P(self.grad[lo:]),
                      P(self.master[lo:]), P(self.m[lo:]), P(self.v[lo:]), P(self.flat16[lo:]), n,
                      P(seg_end), P(seg_wd), nseg, P(self.scratch),
                      P(self._found_inf), P(self.scale), P(self._step_ctr), lr_v,
                      P(self.lr_dev) if self.lr_dev is not None else None,
                      float(self.betas[0]), float(self.betas[1]), float(self.eps),
                      float(self.weight_decay), st)
        torch._amp_update_scale_(self.scale, self._growth, self._found_inf, 2.0, 0.5,
                                 self.growth_interval)
        for hook in self.post_step_hooks:
            hook(self)
        # the update consumed (zeroed) the flat gradient; with a shard, a
        # post-step hook zeroes the rest
        self._grad_dirty = False
        return {"grad_norm": self._norm, "found_inf": self._found_inf, "scale": self.scale}

    def zero_grad(self):
        for _n, p, _o, _el, _w in self._info:
            p.grad = None
        if self._grad_dirty:
            self.grad.zero_()
            self._grad_dirty = False

    # -- state ----------------------------------------------------------------

    def state_dict(self):
        return {"master": self.master, "m": self.m, "v": self.v,
                "step": self._step_ctr, "scale": self.scale,
                "growth": self._growth,
                "offsets": [(n_, o, el) for n_, _p, o, el, _w in self._info]}

    def load_state_dict(self, sd):
        self.master.copy_(sd["master"]); self.m.copy_(sd["m"])
        self.v.copy_(sd["v"]); self._step_ctr.copy_(sd["step"])
        self.scale.copy_(sd["scale"]); self._growth.copy_(sd["growth"])
        self.flat16.copy_(self.master)

    def master_state_dict(self):
        """fp32 master weights keyed like model.state_dict()."""
        return {name: self.master[off:off + n].view(p.shape)
                for name, p, off, n, _w in self._info}
