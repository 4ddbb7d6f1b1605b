"""fxlm.train_lm: GPT training driver on B200 (one process per GPU).

Same command line, data format and checkpoint layout as the reference's
ml/fxlm/train_lm.py:24-231: uint16 token .bin (+ .json meta with vocab_size),
device-side random batches (:148-152), linear warmup + cosine LR (:154-160),
gradient accumulation (:199-205), host sync only at log points (:208-222),
atomic checkpoints `ckpt_<tag>.tmp` -> `ckpt_<tag>.pt` holding fp32 master
weights by parameter name, the FlatAdamW state, config, step, meta and args
(:162-174), `--resume` (:134-139) and refusal to overwrite an existing run
(:140-142). Additions: `--synthetic V` trains on Zipf(1.1) tokens instead of
a file; under torchrun the batch is data-parallel over the ranks (NCCL,
bucketed all-reduce; `--zero` shards the optimizer update instead) and only
rank 0 logs and writes checkpoints.

    python -m fxlm.train_lm --data data/demo_train.bin --out runs/demo
    torchrun --nproc-per-node 8 -m fxlm.train_lm --synthetic 32768 --out runs/dp8 ...
"""
import argparse
import datetime
import json
import math
import os
import time


def _parse(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--data", default=None, help="uint16 token .bin (prepare_bytes.py output)")
    ap.add_argument("--synthetic", type=int, default=0,
                    help="vocab size of synthetic Zipf(1.1) tokens (instead of --data)")
    ap.add_argument("--val", default=None)
    ap.add_argument("--seq-len", type=int, default=256)
    ap.add_argument("--layers", type=int, default=8)
    ap.add_argument("--heads", type=int, default=8)
    ap.add_argument("--dim", type=int, default=512)
    ap.add_argument("--batch", type=int, default=16)
    ap.add_argument("--accum", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--lr", type=float, default=6e-4)
    ap.add_argument("--min-lr-frac", type=float, default=0.1)
    ap.add_argument("--warmup", type=int, default=100)
    ap.add_argument("--wd", type=float, default=0.1)
    ap.add_argument("--clip", type=float, default=1.0)
    ap.add_argument("--init-scale", type=float, default=None,
                    help="initial loss scale (default: 2^16 for fp16 as in the reference, "
                         "1 for bf16)")
    ap.add_argument("--eval-every", type=int, default=200)
    ap.add_argument("--eval-batches", type=int, default=20)
    ap.add_argument("--log-every", type=int, default=20)
    ap.add_argument("--out", default=None, help="checkpoint directory (required)")
    ap.add_argument("--resume", default=None, help="checkpoint file")
    ap.add_argument("--attn", choices=["flash", "sdpa"], default="flash")
    ap.add_argument("--norm", choices=["fused", "torch"], default="fused")
    ap.add_argument("--ce", choices=["fused", "torch"], default="fused")
    ap.add_argument("--dtype", choices=["bf16", "fp16"], default="bf16")
    ap.add_argument("--tunable", action="store_true",
                    help="accepted for command-line compatibility (no runtime tuning here)")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--zero", action="store_true",
                    help="under torchrun: shard FlatAdamW's update over the ranks (ZeRO-1)")
    args = ap.parse_args(argv)
    if args.init_scale is None:
        args.init_scale = 2.0 ** 16 if args.dtype == "fp16" else 1.0
    return args


def lr_at(step, args):
    """Linear warmup then cosine to min_lr_frac (ml/fxlm/train_lm.py:154-160)."""
    if step < args.warmup:
        return args.lr * (step + 1) / args.warmup
    t = (step - args.warmup) / max(1, args.steps - args.warmup)
    c = 0.5 * (1.0 + math.cos(math.pi * min(1.0, t)))
    return args.lr * (args.min_lr_frac + (1.0 - args.min_lr_frac) * c)


def main(argv=None):
    args = _parse(argv)
    if args.out is None:
        raise SystemExit("--out <checkpoint dir> is required")
    if args.data is None and not args.synthetic:
        raise SystemExit("give --data <tokens.bin> or --synthetic <vocab>")

    import numpy as np
    import torch
    import torch.distributed as dist
    from fxb200 import _lib
    from fxlm.model import GPT, GPTConfig
    from fxlm.optim import FlatAdamW

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=device)
    torch.manual_seed(args.seed)

    meta = {}
    if args.data:
        prefix = args.data[:-len("_train.bin")] if args.data.endswith("_train.bin") \
            else os.path.splitext(args.data)[0]
        if os.path.exists(prefix + ".json"):
            with open(prefix + ".json", "r", encoding="utf-8") as f:
                meta = json.load(f)
        vocab = int(meta.get("vocab_size", 65536))
        tokens = torch.from_numpy(np.fromfile(args.data, dtype=np.uint16).astype(np.int32)).to(device)
        vt = None
        vpath = args.val or (prefix + "_val.bin" if meta.get("n_val") else None)
        if vpath and os.path.exists(vpath):
            vt = torch.from_numpy(np.fromfile(vpath, dtype=np.uint16).astype(np.int32)).to(device)
    else:
        from fxb200.data import zipf_tokens
        vocab = args.synthetic
        meta = {"vocab_size": vocab, "tokenizer": "synthetic-zipf-1.1"}
        n = max(args.seq_len + 2, 1 << 22)
        tokens = zipf_tokens(vocab, 1, n, seed=args.seed + 1000 * rank)[0].reshape(-1).int().to(device)
        vt = zipf_tokens(vocab, 1, 1 << 18, seed=args.seed + 777)[0].reshape(-1).int().to(device)

    cfg = GPTConfig(vocab_size=vocab, seq_len=args.seq_len, n_layer=args.layers, n_head=args.heads,
                    d_model=args.dim, attn_impl=args.attn, norm_impl=args.norm, ce_impl=args.ce)
    model = GPT(cfg).to(device)
    pdt = torch.bfloat16 if args.dtype == "bf16" else torch.float16
    opt = FlatAdamW(model, lr=args.lr, weight_decay=args.wd, max_grad_norm=args.clip,
                    init_scale=args.init_scale, param_dtype=pdt)
    sharded = None
    if world > 1 and args.zero:
        from fxb200.zero import ShardedDataParallel
        sharded = ShardedDataParallel(model, opt)
    elif world > 1:
        from fxb200.ddp import DataParallel
        DataParallel(model, opt)
    if rank == 0:
        print(f"GPT params: {model.num_params():,} | ranks {world} | vocab {vocab}", flush=True)

    ckpt_path = os.path.join(args.out, "ckpt_last.pt")
    start = 0
    if args.resume:
        sd = torch.load(args.resume, map_location=device, weights_only=False)
        opt.load_state_dict(sd["opt"])
        start = sd["step"]
    elif os.path.exists(ckpt_path):
        raise SystemExit(f"{ckpt_path} exists: choose another --out or use --resume")
    if rank == 0:
        os.makedirs(args.out, exist_ok=True)

    T, B, ACC = args.seq_len, args.batch, args.accum
    ar = torch.arange(T + 1, device=device)
    gen = torch.Generator(device=device)
    gen.manual_seed(args.seed + 17 * rank)

    def get_batch(src):
        offs = torch.randint(0, src.numel() - T - 1, (B,), device=device, generator=gen)
        seq = src[(offs[:, None] + ar[None, :])].long()
        return seq[:, :-1], seq[:, 1:]

    def save_ckpt(step, tag="last"):
        if sharded is not None:
            sharded.consolidate()  # collective: every rank, before rank 0 writes
        if rank != 0:
            return
        sd = {"model": {k: v.detach().to("cpu", torch.float32) for k, v in opt.master_state_dict().items()},
              "opt": {k: (v.detach().cpu() if torch.is_tensor(v) else v) for k, v in opt.state_dict().items()},
              "config": cfg.__dict__, "step": step, "meta": meta, "args": vars(args)}
        tmp = os.path.join(args.out, f"ckpt_{tag}.tmp")
        torch.save(sd, tmp)
        os.replace(tmp, os.path.join(args.out, f"ckpt_{tag}.pt"))

    @torch.no_grad()
    def evaluate():
        tot = torch.zeros((), device=device)
        for _ in range(args.eval_batches):
            x, y = get_batch(vt)
            tot += model(x, y)
        return float(tot) / args.eval_batches

    loss_acc = torch.zeros((), device=device)
    nb, t0, gstep = 0, None, start
    while gstep < args.steps:
        if t0 is None:
            torch.cuda.synchronize()
            t0 = time.perf_counter()
        lr = lr_at(gstep, args)
        for _ in range(ACC):
            x, y = get_batch(tokens)
            loss = model(x, y, grad_scale=opt.scale)
            opt.backward(loss / ACC)
            loss_acc += loss.detach() / ACC
            nb += 1
        stats = opt.step(lr=lr)
        opt.zero_grad()
        gstep += 1
        if gstep % args.log_every == 0 or gstep == 1:
            if world > 1:
                dist.all_reduce(loss_acc, op=dist.ReduceOp.SUM)
                loss_acc /= world
            torch.cuda.synchronize()
            dt = time.perf_counter() - t0
            # a kernel whose bounded wait expired returned early: stop before
            # its results reach the weights of another step or a checkpoint
            _lib.raise_on_device_error(f"before step {gstep}")
            if rank == 0:
                print(f"step {gstep:5d} | loss {float(loss_acc) / nb:.4f} | lr {lr:.2e} | "
                      f"{nb * B * T * world / dt:,.0f} tok/s | gnorm {float(stats['grad_norm']):.3f} | "
                      f"scale {float(stats['scale']):.0f} | skip {int(bool(stats['found_inf']))}", flush=True)
            loss_acc = torch.zeros((), device=device)
            nb, t0 = 0, None
        if vt is not None and (gstep % args.eval_every == 0 or gstep == args.steps):
            vl = evaluate()
            if rank == 0:
                print(f"  eval @ {gstep}: val_loss {vl:.4f}", flush=True)
            save_ckpt(gstep)
    save_ckpt(gstep)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
