"""Generate the golden fixtures of tests/golden/ from the reference itself.

Runs the reference's own PyTorch code (ml/fxlm/model.py with its torch paths,
ml/fxlm/selftest.py's fp32 references, ml/fxgpu/model.py's dense trunk) on
CPU in fp32 and stores small inputs/outputs. The reference package imports
fxgpu.hip_kernel at module level, which loads Windows HIP DLLs; a stub module
is put in sys.modules first (its compile/launch functions are never called on
these paths). Inputs are rounded through bf16 so the GPU tests can feed the
exact same values to the bf16 kernels.

    python tests/golden/make_golden.py --ref /path/to/reference [--skip-curve] [--skip-d768]
    python tests/golden/make_golden.py --ref /path/to/reference --d768-curve ACC --steps 200

Outputs (committed): ops.npz, gpt_tiny.npz, curve_tiny.json, gpt_d768.json,
curve_d768.json (config-4 loss curve, --d768-curve), prepare_bytes.json (the reference's ml/fxlm/prepare_bytes.py run as a script on
the tree of prepare_bytes_tree.py: meta and SHA-256 of the token files).
"""
import argparse
import hashlib
import json
import math
import os
import subprocess
import sys
import tempfile
import time
import types
import zlib

import numpy as np
import torch
import torch.nn as nn
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))


def _import_reference(ref_root):
    ml = os.path.join(ref_root, "ml")
    stub = types.ModuleType("fxgpu.hip_kernel")

    def _unavailable(*a, **k):
        raise RuntimeError("HIP kernels are not available in the golden generator")
    stub.compile_kernel = stub.compile_module = stub.launch = _unavailable
    sys.modules["fxgpu.hip_kernel"] = stub
    sys.path.insert(0, ml)
    import fxlm.model as ref_model  # noqa: E402
    import fxgpu.model as ref_fxgpu_model  # noqa: E402
    import fxlm.selftest as ref_selftest  # noqa: E402  (torch refs _ref_attn, rule)
    return ref_model, ref_fxgpu_model, ref_selftest


def bf16r(t):
    """Round to the nearest bf16 value, keep fp32 storage."""
    return t.to(torch.bfloat16).float()


def np32(t):
    return t.detach().float().cpu().numpy().copy()


def zipf(V, B, T, seed, s=1.1):
    # definition shared with oracle/gpt.py:zipf_tokens (restated here so the
    # generator does not depend on the oracle it pins)
    k = np.arange(V, dtype=np.float64)
    p = (k + 1.0) ** (-s)
    p /= p.sum()
    seq = np.random.default_rng(seed).choice(V, size=(B, T + 1), p=p)
    seq = torch.from_numpy(seq.astype(np.int64))
    return seq[:, :-1].contiguous(), seq[:, 1:].contiguous()


def make_ops(ref_model, ref_fxgpu_model, ref_selftest):
    out = {}
    g = torch.Generator().manual_seed(1234)

    def rn(*shape, scale=1.0):
        return bf16r(torch.randn(*shape, generator=g) * scale)

    # RMSNorm: the reference model's torch path (Fn.rms_norm, model.py:56)
    for (N, D) in [(37, 64), (129, 768)]:
        x = rn(N, D, scale=3.0).requires_grad_()
        w = bf16r(torch.randn(D, generator=g) * 0.5 + 1).requires_grad_()
        dy = rn(N, D)
        y = F.rms_norm(x, (D,), w, 1e-6)
        y.backward(dy)
        k = f"rms_{N}x{D}"
        out.update({k + "_x": np32(x), k + "_w": np32(w), k + "_dy": np32(dy), k + "_y": np32(y),
                    k + "_dx": np32(x.grad), k + "_dw": np32(w.grad)})
    # fused CE: the selftest's fp32 reference F.cross_entropy (selftest.py:83,92)
    for (N, V) in [(100, 512), (33, 8192)]:
        lg = rn(N, V, scale=4.0).requires_grad_()
        tg = torch.randint(0, V, (N,), generator=g)
        tg[::7] = -100
        loss = F.cross_entropy(lg, tg, ignore_index=-100)
        loss.backward()
        k = f"ce_{N}x{V}"
        out.update({k + "_logits": np32(lg), k + "_target": tg.numpy(), k + "_loss": np.float32(loss.item()),
                    k + "_grad": np32(lg.grad)})
    # linear-CE: selftest.py:114 reference
    N, D, V = 301, 128, 1024
    x = rn(N, D).requires_grad_()
    W = rn(V, D, scale=0.02).requires_grad_()
    tg = torch.randint(0, V, (N,), generator=g)
    tg[::11] = -100
    loss = F.cross_entropy(x @ W.t(), tg, ignore_index=-100)
    loss.backward()
    out.update({"lce_x": np32(x), "lce_W": np32(W), "lce_target": tg.numpy(),
                "lce_loss": np.float32(loss.item()), "lce_dx": np32(x.grad), "lce_dW": np32(W.grad)})
    # attention: selftest.py:137-146 _ref_attn (fp32), grads by autograd
    for causal in (True, False):
        B, T, H, Dh = 2, 65, 2, 64
        qkv = rn(B, T, 3, H, Dh)
        q, k_, v = (qkv[:, :, i].clone().requires_grad_() for i in range(3))
        scale = 1.0 / math.sqrt(Dh)
        o = ref_selftest._ref_attn(q, k_, v, causal, scale)
        do = rn(*o.shape)
        o.backward(do)
        kk = f"attn_c{int(causal)}"
        out.update({kk + "_qkv": np32(qkv), kk + "_do": np32(do), kk + "_o": np32(o),
                    kk + "_dq": np32(q.grad), kk + "_dk": np32(k_.grad), kk + "_dv": np32(v.grad)})
    # GELU(tanh) (model.py:71)
    z = rn(4096, scale=3.0).requires_grad_()
    a = F.gelu(z, approximate="tanh")
    a.backward(torch.ones_like(a))
    out.update({"gelu_z": np32(z), "gelu_a": np32(a), "gelu_da": np32(z.grad)})
    # FlatAdamW: the selftest's own oracle, torch AdamW + clip on unscaled
    # grads, wd only on ndim >= 2 (selftest.py:219-261), 6 steps
    torch.manual_seed(0)
    model = nn.Sequential(nn.Linear(64, 32, bias=False), nn.LayerNorm(32), nn.Linear(32, 16, bias=False))
    ps = [p for p in model.parameters()]
    ref = [nn.Parameter(bf16r(p.detach().clone())) for p in ps]
    init = [np32(r) for r in ref]
    ropt = torch.optim.AdamW([{"params": [r for r in ref if r.dim() >= 2], "weight_decay": 0.1},
                              {"params": [r for r in ref if r.dim() < 2], "weight_decay": 0.0}],
                             lr=1e-3, betas=(0.9, 0.95), eps=1e-8)
    scale = 8.0
    grads_all, masters = [], []
    for st in range(6):
        grads = [bf16r(torch.randn(p.shape, generator=g) * 0.1) for p in ps]
        for r, gg in zip(ref, grads):
            r.grad = gg / scale
        torch.nn.utils.clip_grad_norm_(ref, 0.5)
        ropt.step()
        grads_all.append([np32(x) for x in grads])
        masters.append([np32(r) for r in ref])
    for i in range(len(ps)):
        out[f"adamw_init_{i}"] = init[i]
        out[f"adamw_grads_{i}"] = np.stack([ga[i] for ga in grads_all])
        out[f"adamw_master_{i}"] = np.stack([m[i] for m in masters])
    out["adamw_scale"] = np.float32(scale)
    # fxgpu gather-linear + trunk: selftest.py:36-40 unfold reference and the
    # reference WindowMLP's own _trunk (ml/fxgpu/model.py:37-42)
    R, Fe, Wn, HID, H2, Bsz = 200, 16, 4, 32, 16, 50
    X = rn(R, Fe)
    idx = torch.randint(0, R - Wn + 1, (Bsz,), generator=g, dtype=torch.int64)
    torch.manual_seed(4)
    m = ref_fxgpu_model.WindowMLP(Fe, Wn, hidden=HID, hidden2=H2, master=True)
    with torch.no_grad():
        for p in m.parameters():
            p.copy_(bf16r(p))
        m.b1.copy_(bf16r(torch.randn(HID, generator=g) * 0.1))
    xb = X.unfold(0, Wn, 1)[idx].transpose(1, 2).reshape(Bsz, Wn * Fe)
    h1 = F.linear(xb, m.W1, m.b1)
    yout = m._trunk(h1, m.W2, m.b2, m.W3, m.b3)
    out.update({"wmlp_X": np32(X), "wmlp_idx": idx.numpy(), "wmlp_xb": np32(xb), "wmlp_h1": np32(h1),
                "wmlp_y": np32(yout)})
    for nm in ("W1", "b1", "W2", "b2", "W3", "b3"):
        out[f"wmlp_{nm}"] = np32(getattr(m, nm))
    np.savez_compressed(os.path.join(HERE, "ops.npz"), **out)
    print("ops.npz:", len(out), "arrays")


def _cfg_tiny():
    return dict(vocab_size=256, seq_len=256, n_layer=4, n_head=4, d_model=256)


def _ref_gpt(ref_model, cfg, eps):
    c = ref_model.GPTConfig(**cfg, attn_impl="sdpa", norm_impl="torch", ce_impl="torch", eps=eps)
    return ref_model.GPT(c)


def _sample_idx(n, k, seed):
    return np.random.default_rng(seed).choice(n, size=min(k, n), replace=False)


def make_gpt_tiny(ref_model):
    """Config 1: V256 L4 D256 H4 (eps 1e-5), B32 T256, Zipf seed 0, init seed 0."""
    cfg = _cfg_tiny()
    torch.manual_seed(0)
    m = _ref_gpt(ref_model, cfg, 1e-5)
    x, y = zipf(256, 32, 256, seed=0)
    loss = m(x, y)
    loss.backward()
    out = {"loss": np.float32(loss.item()), "x": x.numpy().astype(np.int16), "y": y.numpy().astype(np.int16)}
    for n, p in m.named_parameters():
        flat = p.detach().reshape(-1)
        gflat = p.grad.reshape(-1)
        sel = _sample_idx(flat.numel(), 256, zlib.crc32(n.encode()))
        out[f"init_sum:{n}"] = np.float64(flat.double().sum().item())
        out[f"init_sq:{n}"] = np.float64((flat.double() ** 2).sum().item())
        out[f"init_sel:{n}"] = sel.astype(np.int64)
        out[f"init_val:{n}"] = np32(flat[sel])
        out[f"grad_norm:{n}"] = np.float64(gflat.double().norm().item())
        out[f"grad_val:{n}"] = np32(gflat[sel])
    np.savez_compressed(os.path.join(HERE, "gpt_tiny.npz"), **out)
    print("gpt_tiny.npz: loss", loss.item())


def _curve(ref_model, steps, batch_seed):
    """Loss per step of config 1 with the selftest's FlatAdamW oracle (torch
    AdamW, wd on ndim >= 2, clip 1.0, selftest.py:228-250), lr 3e-4.
    batch_seed(s) -> Zipf seed of step s's batch."""
    cfg = _cfg_tiny()
    torch.manual_seed(0)
    m = _ref_gpt(ref_model, cfg, 1e-5)
    opt = torch.optim.AdamW([{"params": [p for p in m.parameters() if p.dim() >= 2], "weight_decay": 0.1},
                             {"params": [p for p in m.parameters() if p.dim() < 2], "weight_decay": 0.0}],
                            lr=3e-4, betas=(0.9, 0.95), eps=1e-8)
    losses = []
    t0 = time.time()
    for s in range(steps):
        x, y = zipf(256, 32, 256, seed=batch_seed(s))
        opt.zero_grad(set_to_none=True)
        loss = m(x, y)
        loss.backward()
        torch.nn.utils.clip_grad_norm_(list(m.parameters()), 1.0)
        opt.step()
        losses.append(float(loss.detach()))
        if s % 40 == 0:
            print(f"  curve step {s} loss {losses[-1]:.4f} ({time.time() - t0:.0f}s)", flush=True)
    return losses


def make_curve_tiny(ref_model, steps):
    fixed = _curve(ref_model, steps, lambda s: 0)
    stream = _curve(ref_model, steps, lambda s: 1000 + s)
    with open(os.path.join(HERE, "curve_tiny.json"), "w") as f:
        json.dump({"config": "V256 L4 D256 H4 eps1e-5, B32 T256, init seed 0, AdamW lr3e-4 "
                             "b(0.9,0.95) wd0.1 clip1.0",
                   "losses": fixed, "fixed_batch": "zipf seed 0 every step",
                   "losses_stream": stream, "stream": "step s uses zipf seed 1000+s"}, f)


def make_d768(ref_model):
    """Config 4 first-step loss: V32768 L12 D768 H12, B8 T1024, Zipf seed 3, init seed 3."""
    cfg = dict(vocab_size=32768, seq_len=1024, n_layer=12, n_head=12, d_model=768)
    torch.manual_seed(3)
    m = _ref_gpt(ref_model, cfg, 1e-6)
    x, y = zipf(32768, 8, 1024, seed=3)
    t0 = time.time()
    loss = m(x, y)
    loss.backward()
    gn = math.sqrt(sum(float(p.grad.double().pow(2).sum()) for p in m.parameters()))
    res = {"config": "V32768 L12 D768 H12 eps1e-6, B8 T1024, zipf seed 3, init seed 3",
           "loss": float(loss), "grad_norm": gn, "num_params": sum(p.numel() for p in m.parameters()),
           "cpu_seconds": time.time() - t0, "threads": torch.get_num_threads()}
    with open(os.path.join(HERE, "gpt_d768.json"), "w") as f:
        json.dump(res, f, indent=1)
    print("gpt_d768:", res)


def make_curve_d768(ref_model, steps, acc, path, stream=False):
    """Config 4 loss curve: the reference model (torch path, fp32) trained for
    `steps` steps on fixed Zipf batches, the selftest's FlatAdamW oracle
    (torch AdamW lr 6e-4, betas (0.9, 0.95), wd 0.1 on ndim >= 2, clip 1.0).
    acc micro-batches of 8 x 1024 per step (seeds 3 .. 3 + acc - 1, each loss
    divided by acc, as ml/fxlm/train_lm.py:199-205 accumulates) are what
    acc data-parallel ranks of bench.py train on (rank r: seed 3 + r). The
    file is rewritten every 5 steps so a partial run is usable."""
    cfg = dict(vocab_size=32768, seq_len=1024, n_layer=12, n_head=12, d_model=768)
    torch.manual_seed(3)
    m = _ref_gpt(ref_model, cfg, 1e-6)
    opt = torch.optim.AdamW([{"params": [p for p in m.parameters() if p.dim() >= 2], "weight_decay": 0.1},
                             {"params": [p for p in m.parameters() if p.dim() < 2], "weight_decay": 0.0}],
                            lr=6e-4, betas=(0.9, 0.95), eps=1e-8)
    batches = [zipf(32768, 8, 1024, seed=3 + r) for r in range(acc)]
    rec = json.load(open(path)) if os.path.exists(path) else {}
    key = f"acc{acc}" + ("_stream" if stream else "")
    losses, norms = [], []
    t0 = time.time()
    for s in range(steps):
        opt.zero_grad(set_to_none=True)
        tot = 0.0
        if stream:  # a fresh batch every step: micro-batch r of step s has seed 1000 * (s + 1) + r
            batches = [zipf(32768, 8, 1024, seed=1000 * (s + 1) + r) for r in range(acc)]
        for x, y in batches:
            loss = m(x, y)
            (loss / acc).backward()
            tot += float(loss.detach()) / acc
        gn = torch.nn.utils.clip_grad_norm_(list(m.parameters()), 1.0)
        opt.step()
        losses.append(tot)
        norms.append(float(gn))
        if s % 5 == 4 or s == steps - 1:
            data = (f"zipf seeds 1000*(s+1)+r, r < {acc}, a fresh batch every step" if stream else
                    f"zipf seeds 3..{2 + acc} fixed every step")
            rec[key] = {"config": "V32768 L12 D768 H12 eps1e-6, init seed 3, micro-batches 8x1024 "
                                  f"{data}, loss/acc, AdamW lr6e-4 "
                                  "b(0.9,0.95) wd0.1 (ndim>=2) clip1.0, fp32 CPU",
                        "losses": losses, "grad_norms": norms, "steps_done": len(losses),
                        "cpu_seconds": time.time() - t0, "threads": torch.get_num_threads()}
            with open(path + ".tmp", "w") as f:
                json.dump(rec, f)
            os.replace(path + ".tmp", path)
            print(f"  d768 acc{acc} step {s} loss {tot:.4f} norm {norms[-1]:.3f} "
                  f"({time.time() - t0:.0f}s)", flush=True)


def make_prepare_bytes(ref_root):
    sys.path.insert(0, HERE)
    from prepare_bytes_tree import build_tree, CASES
    script = os.path.join(ref_root, "ml", "fxlm", "prepare_bytes.py")
    out = {}
    with tempfile.TemporaryDirectory() as tmp:
        root = os.path.join(tmp, "tree")
        build_tree(root)
        for name, inputs, opts in CASES:
            prefix = os.path.join(tmp, "out", name)
            subprocess.run([sys.executable, script, *[os.path.join(root, i) for i in inputs],
                            "--out", prefix, *opts], check=True, capture_output=True)
            rec = {"meta": json.load(open(prefix + ".json", encoding="utf-8"))}
            for part in ("train", "val"):
                with open(f"{prefix}_{part}.bin", "rb") as f:
                    rec["sha256_" + part] = hashlib.sha256(f.read()).hexdigest()
            out[name] = rec
    with open(os.path.join(HERE, "prepare_bytes.json"), "w") as f:
        json.dump(out, f, indent=1)
    print("prepare_bytes.json:", {k: v["meta"] for k, v in out.items()})


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="root of the reference repository")
    ap.add_argument("--skip-curve", action="store_true")
    ap.add_argument("--skip-d768", action="store_true")
    ap.add_argument("--only-prepare-bytes", action="store_true")
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--d768-curve", type=int, default=0, metavar="ACC",
                    help="only the config-4 loss curve with ACC micro-batches per step")
    ap.add_argument("--stream", action="store_true",
                    help="--d768-curve: a fresh batch every step instead of fixed micro-batches")
    ap.add_argument("--threads", type=int, default=os.cpu_count())
    args = ap.parse_args()
    torch.set_num_threads(args.threads)
    if args.d768_curve:
        ref_model, _, _ = _import_reference(args.ref)
        make_curve_d768(ref_model, args.steps, args.d768_curve, os.path.join(HERE, "curve_d768.json"),
                        stream=args.stream)
        return
    make_prepare_bytes(args.ref)
    if args.only_prepare_bytes:
        return
    ref_model, ref_fxgpu_model, ref_selftest = _import_reference(args.ref)
    make_ops(ref_model, ref_fxgpu_model, ref_selftest)
    make_gpt_tiny(ref_model)
    if not args.skip_d768:
        make_d768(ref_model)
    if not args.skip_curve:
        make_curve_tiny(ref_model, args.steps)


if __name__ == "__main__":
    main()
