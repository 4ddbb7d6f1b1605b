#!/usr/bin/env python
"""Benchmark: GPT d768x12L training step on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step = forward + backward + FlatAdamW update of the reference GPT
architecture (V32768, L12, D768, H12, T1024) on a per-GPU micro-batch of 8
sequences of Zipf(1.1) tokens (seed 3 + rank), bf16 compute with fp32 master
weights. The step is captured once in a CUDA graph (fxlm.GraphedStep, after
the warm-up steps) and replayed; `--no-graph` runs it eagerly. For N > 1 the
driver launches this under torchrun (one rank per GPU, NCCL); gradient
buckets are reduced to the rank owning each shard of FlatAdamW while backward
runs, each rank updates its shard and the bf16 parameters are all-gathered
(fxb200.zero; `--no-zero`: all-reduce and a full update on every rank), and
those NCCL calls are part of the captured graph.

Printed (rank 0, one JSON line): `value` = tokens/s of the whole job with the
token batch already in HBM, timed on the device with CUDA events (max over
ranks); `e2e` = the same loop through the public API with the batch copied
from pinned host memory and the loss read back every step (both asynchronous
and overlapped with the neighbouring steps, as a training loop runs them); `roofline` for the
dominant kernel (the tcgen05 GEMM: summed algorithmic FLOPs / summed event
time of its launches over a second pass of the same steps, run after the timed
region so that its events do not perturb it, against the measured sustained
bf16 peak); `cpu_baseline` = the reference's PyTorch path restated in oracle/gpt.py
on the host cores (bounded sample); `clocks` sampled with nvidia-smi during
the timed region; `gpu_launches` = kernels of libfxb200 in the timed region
(for a replayed graph: the library kernels captured in one step x steps). `--impl reference` times only that CPU path (the reference arm).
"""
import argparse
import datetime
import gc
import json
import os
import re
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "radeon-igpu-forge_b200")
for _p in (PKG, ROOT):
    if _p not in sys.path:
        sys.path.insert(0, _p)

CFG4 = dict(vocab_size=32768, seq_len=1024, n_layer=12, n_head=12, d_model=768)
MB, SEQ = 8, 1024  # per-GPU micro-batch
WORKLOAD = "gpt_d768x12L_v32768: per-GPU micro-batch 8 x seq 1024, bf16 + fp32-master FlatAdamW"


def _metric():
    try:
        with open(os.path.join(ROOT, "BASELINE.json")) as f:
            return json.load(f)["metric"]
    except Exception:
        return "GPT d768x12L train tokens/s"


def _peaks(clocks=None):
    """bf16 tensor peak for the roofline. The burst figure applies unless the
    clock record of the timed region shows the SM clock held below its
    maximum (power capping over a long run), when the sustained one does."""
    capped = False
    if clocks and clocks.get("sm_mhz") and clocks.get("sm_max_mhz"):
        capped = clocks["sm_mhz"] < 0.97 * clocks["sm_max_mhz"]
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        if capped:
            return float(d["bf16_tflops_sustained"]), \
                "MEASURED_PEAKS.json bf16_tflops_sustained (of measured; SM clock below max in the timed region)"
        return float(d["bf16_tflops"]), \
            "MEASURED_PEAKS.json bf16_tflops burst (of measured; SM clock at max in the timed region)"
    except Exception:
        return (1400.0, "fallback 1.4 PFLOP/s sustained (of fallback)") if capped else \
            (1590.0, "fallback 1.59 PFLOP/s burst (of fallback)")


def _hbm_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "MEASURED_PEAKS.json hbm_gbs (of measured)"
    except Exception:
        return 6650.0, "fallback 6.65 TB/s (of fallback)"


def _gemm_traffic():
    """Average DRAM bytes per GEMM launch of one step, from the committed ncu summary."""
    p = os.path.join(ROOT, "profiles", "gemm_tc_gpt_d768_layer.md")
    try:
        with open(p) as f:
            m = re.search(r"avg_dram_bytes_per_launch:\s*([0-9.eE+]+)", f.read())
        return float(m.group(1)) if m else None
    except Exception:
        return None


# ---------------------------------------------------------------- clocks
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.rows = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        self.t = threading.Thread(target=self._read, daemon=True)
        self.t.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                self.rows.append(parts)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.t.join(timeout=2)
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows)}


# ---------------------------------------------------------------- CPU baseline
def _reference_fxlm():
    """The reference's own ml/fxlm package when its source tree is given
    (FXB_REFERENCE_ROOT, or baseline/_ref holding ml/fxlm), loaded under a
    private name with its HIP loader stubbed, so that its PyTorch paths run
    on the CPU; None when no tree is given."""
    import importlib.util
    import types
    for root in (os.environ.get("FXB_REFERENCE_ROOT"), os.path.join(ROOT, "baseline", "_ref")):
        pkg = os.path.join(root, "ml", "fxlm") if root else None
        if not pkg or not os.path.isfile(os.path.join(pkg, "model.py")):
            continue
        if "fxgpu.hip_kernel" not in sys.modules:
            def _no_hip(*_a, **_k):
                raise RuntimeError("HIP kernels are not available on this host")
            parent = types.ModuleType("fxgpu")
            parent.__path__ = []
            stub = types.ModuleType("fxgpu.hip_kernel")
            stub.compile_kernel = stub.compile_module = stub.launch = _no_hip
            sys.modules.setdefault("fxgpu", parent)
            sys.modules["fxgpu.hip_kernel"] = stub
        spec = importlib.util.spec_from_file_location("ref_fxlm", os.path.join(pkg, "__init__.py"),
                                                      submodule_search_locations=[pkg])
        mod = importlib.util.module_from_spec(spec)
        sys.modules["ref_fxlm"] = mod
        spec.loader.exec_module(mod)
        import importlib
        return importlib.import_module("ref_fxlm.model")
    return None


def cpu_baseline(steps=3, warmup=1):
    """The reference's PyTorch path in fp32 on the host cores: one 1024-token
    sequence per step, forward + backward + FlatAdamW step. The model is the
    reference's own ml/fxlm/model.py (torch attention, norm and CE paths) when
    its source tree is given (see _reference_fxlm), else its restatement in
    oracle/gpt.py. The optimizer step is oracle/gpt.py's FlatAdamW restatement
    in both cases: the reference's FlatAdamW runs HIP kernels only."""
    import torch
    from oracle import gpt as og
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    torch.manual_seed(3)
    ref = _reference_fxlm()
    if ref is not None:
        m = ref.GPT(ref.GPTConfig(**CFG4, attn_impl="sdpa", norm_impl="torch", ce_impl="torch"))
        kind, what = "reference", "the reference's ml/fxlm/model.py (torch paths)"
    else:
        m = og.RefGPT(**CFG4)
        kind, what = "port", "oracle/gpt.py restating ml/fxlm/model.py torch path"
    opt = og.OracleFlatAdamW(list(m.named_parameters()), lr=6e-4, weight_decay=0.1,
                             max_grad_norm=1.0, init_scale=1.0)
    x, y = og.zipf_tokens(CFG4["vocab_size"], 1, SEQ, seed=3)
    times = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        m.zero_grad(set_to_none=True)
        loss = m(x, y)
        (loss * opt.scale).backward()
        opt.step({n: p.grad for n, p in m.named_parameters()})
        with torch.no_grad():
            for n, p in m.named_parameters():
                p.copy_(opt.master[n])
        if i >= warmup:
            times.append(time.perf_counter() - t0)
    tps = SEQ / statistics.mean(times)
    return {"value": tps, "unit": "tokens/s", "cores": threads, "kind": kind,
            "sample": f"1 x {SEQ} tokens per step, {steps} timed steps after {warmup} warm-up "
                      f"(fp32, {what} + FlatAdamW)"}


def run_reference(args, rank, world):
    if rank != 0:
        return
    if args.workload == "wmlp":
        base = cpu_baseline_wmlp(steps=max(1, args.steps), warmup=max(1, args.warmup))
        line = {"metric": "fxgpu window MLP train samples/s (BASELINE config 5)", "value": base["value"],
                "unit": "samples/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": 4096 / base["value"] * 1e3, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic N(0,1) (seed 4)",
                "impl": "reference",
                "config": {"workload": WMLP_WORKLOAD, "global_batch": 4096, "parallelism": "cpu",
                           "sample": base["sample"]},
                "cpu_baseline": base,
                "e2e": {"value": base["value"], "unit": "samples/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    base = cpu_baseline(steps=max(1, args.steps), warmup=max(1, args.warmup))
    line = {"metric": _metric(), "value": base["value"], "unit": "tokens/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": SEQ / base["value"] * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic Zipf(1.1) tokens (seed 3)", "impl": "reference",
            "config": {"workload": WORKLOAD, "global_batch": 1, "seq_len": SEQ,
                       "parallelism": "cpu", "sample": base["sample"]},
            "cpu_baseline": base,
            "e2e": {"value": base["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- attention microbench
def attn_tflops(dev, iters=10):
    """Config 2: causal flash attention fwd+bwd, B16 H12 S1024 D64 bf16.

    Forward and backward are each launched `iters` times back to back between
    two events (the library entry points, no autograd), so the times are the
    kernels' own and not the host's call overhead."""
    import math
    import torch
    from fxlm.attention import _fwd, _bwd
    B, H, S, D = 16, 12, 1024, 64
    scale = 1.0 / math.sqrt(D)
    g = torch.Generator(device=dev).manual_seed(1)
    q, k, v, do = (torch.randn(B, S, H, D, device=dev, generator=g).mul_(1 / math.sqrt(D))
                   .to(torch.bfloat16) for _ in range(4))
    dq, dk, dv = (torch.empty_like(q) for _ in range(3))
    fwd_flops = 2 * B * H * S * S * D  # causal: half of 4*B*H*S^2*D
    for _ in range(3):
        o, lse = _fwd(q, k, v, True, scale)
        _bwd(q, k, v, o, lse, do, True, scale, dq, dk, dv)
    torch.cuda.synchronize()
    e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    e0.record()
    for _ in range(iters):
        o, lse = _fwd(q, k, v, True, scale)
    e1.record()
    for _ in range(iters):
        _bwd(q, k, v, o, lse, do, True, scale, dq, dk, dv)
    e2.record()
    torch.cuda.synchronize()
    tf, tb = e0.elapsed_time(e1) / iters, e1.elapsed_time(e2) / iters
    out = {"fwd_tflops": fwd_flops / tf / 1e9, "fwd_bwd_tflops": 3 * fwd_flops / (tf + tb) / 1e9,
           "fwd_ms": tf, "bwd_ms": tb, "shape": "B16 H12 S1024 D64 causal bf16"}
    out["library"] = _sdpa_library_tflops(q, k, v, do, fwd_flops, iters)
    return out


def _sdpa_library_tflops(q, k, v, do, fwd_flops, iters):
    """The same attention through torch's scaled_dot_product_attention, one
    backend at a time (cuDNN, flash), on (B, H, S, D) views of the same
    tensors: library kernels beside this build's, for context. A backend that
    does not run on this GPU reports its error instead."""
    import torch
    from torch.nn.attention import SDPBackend, sdpa_kernel
    F = torch.nn.functional
    res = {}
    qt, kt, vt, dot = (t.transpose(1, 2) for t in (q, k, v, do))
    for name, be in (("cudnn", SDPBackend.CUDNN_ATTENTION), ("flash", SDPBackend.FLASH_ATTENTION)):
        try:
            with sdpa_kernel([be]):
                qg, kg, vg = (t.detach().requires_grad_(True) for t in (qt, kt, vt))
                tf = _time_ms(lambda: F.scaled_dot_product_attention(qt, kt, vt, is_causal=True), iters)
                o = F.scaled_dot_product_attention(qg, kg, vg, is_causal=True)
                tfb = _time_ms(lambda: torch.autograd.grad(o, (qg, kg, vg), dot, retain_graph=True), iters)
            res[name] = {"fwd_tflops": fwd_flops / tf / 1e9, "fwd_ms": tf, "bwd_ms": tfb,
                         "fwd_bwd_tflops": 3 * fwd_flops / (tf + tfb) / 1e9}
        except Exception as e:  # backend unavailable for this GPU / dtype / layout
            res[name] = {"unavailable": f"{type(e).__name__}: {str(e).splitlines()[0][:160]}"}
    return res


# ---------------------------------------------------------------- per-kernel microbenchmarks
def _time_ms(fn, iters, warmup=3):
    import torch
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters


def run_micro(args):
    """One JSON line per kernel (see micro_results)."""
    import torch
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    for o in micro_results(args.micro, args.iters, args.only):
        print(json.dumps(o), flush=True)


def micro_results(micro, iters, only=None):
    """Per-kernel measurements: BASELINE configs 2 and 3 shapes, the block
    GEMMs of config 4 and the AdamW pass over config 4's parameters. Inputs
    are larger than L2 (126 MB) except where noted. Returns a list of dicts."""
    import math
    import torch
    from fxb200 import _lib, ops
    dev = torch.device("cuda", torch.cuda.current_device())
    _lib.load()
    hbm = None
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            pk = json.load(f)
        hbm, tc = float(pk["hbm_gbs"]), float(pk["bf16_tflops"])
    except Exception:
        hbm, tc = 6650.0, 1590.0
    out = []
    which = micro.split(",")
    it = iters
    bf = torch.bfloat16
    if "gemm" in which or "gemm_fc" in which or "all" in which:
        cases = [(8192, 3072, 768, ops.EPI_GELU, "fc+gelu"), (8192, 2304, 768, ops.EPI_STORE, "qkv"),
                 (8192, 768, 3072, ops.EPI_RESIDUAL, "fc2+residual"),
                 (65536, 32768, 768, ops.EPI_STORE, "lm_head cfg3")]
        if "gemm_fc" in which:
            cases = cases[:1]
        for (M, N, K, epi, nm) in cases:
            A = torch.randn(M, K, device=dev).to(bf)
            B = (torch.randn(N, K, device=dev) / math.sqrt(K)).to(bf)
            C = torch.empty(M, N, device=dev, dtype=bf)
            Z = torch.empty(M, N, device=dev, dtype=bf) if epi == ops.EPI_GELU else None
            R = torch.randn(M, N, device=dev).to(bf) if epi == ops.EPI_RESIDUAL else None
            ms = _time_ms(lambda: ops.gemm(A, B, C, epilogue=epi, Z=Z, R=R), it)
            tf = 2.0 * M * N * K / ms / 1e9
            # same plain product through cuBLAS (sanity reference only)
            ms_cb = _time_ms(lambda: torch.matmul(A, B.t(), out=C), it)
            out.append({"kernel": "gemm_tc", "case": f"{nm} M{M} N{N} K{K}", "ms": ms, "tflops": tf,
                        "frac_of_measured_burst": tf / tc,
                        "cublas_plain_tflops": 2.0 * M * N * K / ms_cb / 1e9})
        for (Mt, N, K, nm) in ([] if "gemm_fc" in which else
                               [(8192, 3072, 768, "dW fc"), (8192, 768, 768, "dW proj")]):
            dy = torch.randn(Mt, N, device=dev).to(bf)
            x = torch.randn(Mt, K, device=dev).to(bf)
            dW = torch.zeros(N, K, device=dev)
            ms = _time_ms(lambda: ops.linear_dw_into(dy, x, dW), it)
            tf = 2.0 * Mt * N * K / ms / 1e9
            out.append({"kernel": "gemm_tc (split-K, fp32 red.add)", "case": f"{nm} tokens{Mt} N{N} K{K}",
                        "ms": ms, "tflops": tf, "frac_of_measured_burst": tf / tc})
    if "gemm_layer" in which or "all" in which:
        # the 12 GEMMs of one config-4 transformer layer (M tokens = 8192), each
        # with the planner's tile choice and a plain cuBLAS reference
        T_, D, F_ = 8192, 768, 3072
        shapes = [  # name, M, N, K, a_trans, b_trans, epilogue
            ("fwd qkv", T_, 3 * D, D, False, False, ops.EPI_STORE),
            ("fwd proj+res", T_, D, D, False, False, ops.EPI_RESIDUAL),
            ("fwd fc+gelu(+gelu')", T_, F_, D, False, False, ops.EPI_GELU_DERIV),
            ("fwd fc2+res", T_, D, F_, False, False, ops.EPI_RESIDUAL),
            ("bwd dz=dout.W2*gelu'", T_, F_, D, False, True, ops.EPI_MUL),
            ("bwd dh=dz.W1", T_, D, F_, False, True, ops.EPI_STORE),
            ("bwd dy=dx.Wproj", T_, D, D, False, True, ops.EPI_STORE),
            ("bwd dh=dqkv.Wqkv", T_, D, 3 * D, False, True, ops.EPI_STORE),
            ("bwd dW2", D, F_, T_, True, True, ops.EPI_ACCUM_F32),
            ("bwd dW1", F_, D, T_, True, True, ops.EPI_ACCUM_F32),
            ("bwd dWproj", D, D, T_, True, True, ops.EPI_ACCUM_F32),
            ("bwd dWqkv", 3 * D, D, T_, True, True, ops.EPI_ACCUM_F32),
        ]
        if only:
            keep = only.split(",")
            shapes = [s for s in shapes if any(k in s[0] for k in keep)]
        tot_f, tot_ms = 0.0, 0.0
        for nm, M, N, K, at, bt, epi in shapes:
            A = (torch.randn(K, M, device=dev) if at else torch.randn(M, K, device=dev)).to(bf)
            B = ((torch.randn(K, N, device=dev) if bt else torch.randn(N, K, device=dev)) / math.sqrt(K)).to(bf)
            acc = epi == ops.EPI_ACCUM_F32
            C = torch.zeros(M, N, device=dev, dtype=torch.float32 if acc else bf)
            R = torch.randn(M, N, device=dev).to(bf) if epi in (ops.EPI_RESIDUAL, ops.EPI_MUL) else None
            Z = torch.empty(M, N, device=dev, dtype=bf) if epi == ops.EPI_GELU_DERIV else None
            ms = _time_ms(lambda: ops.gemm(A, B, C, a_trans=at, b_trans=bt, epilogue=epi, R=R, Z=Z), it)
            Ar = A.t() if at else A
            Br = B if bt else B.t()
            Cc = torch.empty(M, N, device=dev, dtype=bf)
            ms_cb = _time_ms(lambda: torch.matmul(Ar, Br, out=Cc), it)
            fl = 2.0 * M * N * K
            tot_f += fl
            tot_ms += ms
            pair, bn, sp = _lib.gemm_plan(M, N, K, epi)
            out.append({"kernel": "gemm_tc" + ("2" if pair else ""), "case": f"layer {nm} M{M} N{N} K{K}",
                        "tile": f"{'256' if pair else '128'}x{bn} splitK{sp}", "ms": ms,
                        "tflops": fl / ms / 1e9, "cublas_plain_tflops": fl / ms_cb / 1e9})
        out.append({"kernel": "gemm_tc (one layer, 12 GEMMs)", "ms": tot_ms, "tflops": tot_f / tot_ms / 1e9,
                    "frac_of_measured_burst": tot_f / tot_ms / 1e9 / tc})
    if "gemm_big" in which:
        M, N, K = 16384, 16384, 768
        A = torch.randn(M, K, device=dev).to(bf)
        B = (torch.randn(N, K, device=dev) / math.sqrt(K)).to(bf)
        C = torch.empty(M, N, device=dev, dtype=bf)
        ms = _time_ms(lambda: ops.gemm(A, B, C), it)
        out.append({"kernel": "gemm_tc", "case": f"big M{M} N{N} K{K}", "ms": ms,
                    "tflops": 2.0 * M * N * K / ms / 1e9})
    if "attn" in which or "all" in which:
        a = attn_tflops(dev, iters=it)
        a.update({"kernel": "attn_fwd + attn_bwd", "case": "BASELINE config 2",
                  "frac_of_measured_burst_fwd_bwd": a["fwd_bwd_tflops"] / tc})
        out.append(a)
    if "rmsnorm" in which or "all" in which:
        from fxlm.norm import _RMSNorm  # noqa: F401
        Nr, D = 65536, 768
        g = torch.Generator(device=dev).manual_seed(2)
        x = torch.randn(Nr, D, device=dev, generator=g).to(bf)
        w = (1 + 0.02 * torch.randn(D, device=dev, generator=g)).to(bf)
        y = torch.empty_like(x)
        rstd = torch.empty(Nr, device=dev)
        st = _lib.stream_ptr(dev)
        f = lambda: _lib.call("fxb_rmsnorm_fwd", 2, _lib.ptr(x), _lib.ptr(w), _lib.ptr(y), _lib.ptr(rstd),  # noqa: E731
                              Nr, D, 1e-6, st)
        ms = _time_ms(f, it)
        byt = 2 * Nr * D * 2 + Nr * 4
        out.append({"kernel": "rmsnorm_fwd", "case": f"config 3 [{Nr},{D}] bf16", "ms": ms,
                    "gbs": byt / ms / 1e6, "frac_of_measured_hbm": byt / ms / 1e6 / hbm})
        dy = torch.randn(Nr, D, device=dev, generator=g).to(bf)
        dx = torch.empty_like(x)
        dw = torch.zeros(D, device=dev)
        ws = torch.empty(_lib.load().fxb_rmsnorm_bwd_workspace(Nr, D) // 4 + 1, device=dev)
        fb = lambda: _lib.call("fxb_rmsnorm_bwd", 2, _lib.ptr(x), _lib.ptr(w), _lib.ptr(rstd), _lib.ptr(dy),  # noqa: E731
                               None, _lib.ptr(dx), _lib.ptr(dw), 0, 0, _lib.ptr(ws), Nr, D, st)
        ms = _time_ms(fb, it)
        byt = 3 * Nr * D * 2 + Nr * 4
        out.append({"kernel": "rmsnorm_bwd", "case": f"config 3 [{Nr},{D}] bf16", "ms": ms,
                    "gbs": byt / ms / 1e6, "frac_of_measured_hbm": byt / ms / 1e6 / hbm})
        # the config-4 step's shape: [8192, 768] with the residual gradient added
        Ns = 8192
        xs, dys, dres = x[:Ns], dy[:Ns], torch.randn(Ns, D, device=dev, generator=g).to(bf)
        ys, dxs = y[:Ns], dx[:Ns]
        fs = lambda: _lib.call("fxb_rmsnorm_fwd", 2, _lib.ptr(xs), _lib.ptr(w), _lib.ptr(ys),  # noqa: E731
                               _lib.ptr(rstd), Ns, D, 1e-6, st)
        ms = _time_ms(fs, it)
        byt = 2 * Ns * D * 2 + Ns * 4
        out.append({"kernel": "rmsnorm_fwd", "case": f"config 4 step [{Ns},{D}] bf16", "ms": ms,
                    "gbs": byt / ms / 1e6, "frac_of_measured_hbm": byt / ms / 1e6 / hbm})
        fbs = lambda: _lib.call("fxb_rmsnorm_bwd", 2, _lib.ptr(xs), _lib.ptr(w), _lib.ptr(rstd),  # noqa: E731
                                _lib.ptr(dys), _lib.ptr(dres), _lib.ptr(dxs), _lib.ptr(dw), 0, 0,
                                _lib.ptr(ws), Ns, D, st)
        ms = _time_ms(fbs, it)
        byt = 4 * Ns * D * 2 + Ns * 4
        out.append({"kernel": "rmsnorm_bwd (+dres, + dw reduce)", "case": f"config 4 step [{Ns},{D}] bf16",
                    "ms": ms, "gbs": byt / ms / 1e6, "frac_of_measured_hbm": byt / ms / 1e6 / hbm})
    if "ce4" in which:
        # the config-4 step's cross entropy: 8192 rows of V 32768 (537 MB of
        # logits, in place as in the linear-CE chunk), small enough to profile
        Nr, V = 8192, 32768
        g = torch.Generator(device=dev).manual_seed(3)
        lg = torch.randn(Nr, V, device=dev, generator=g, dtype=bf)
        tg = torch.randint(0, V, (Nr,), device=dev, generator=g)
        loss = torch.zeros(Nr, device=dev)
        mul = torch.full((), 1.0 / Nr, device=dev)
        st = _lib.stream_ptr(dev)
        f = lambda: _lib.call("fxb_ce_fwd_grad", 2, _lib.ptr(lg), V, _lib.ptr(tg), _lib.ptr(lg),  # noqa: E731
                              _lib.ptr(loss), _lib.ptr(mul), Nr, V, -100, st)
        ms = _time_ms(f, it)
        byt = 2 * Nr * V * 2
        out.append({"kernel": "ce_fwd_grad", "case": f"config 4 step [{Nr},{V}] bf16, gradient in place",
                    "ms": ms, "gbs": byt / ms / 1e6, "frac_of_measured_hbm": byt / ms / 1e6 / hbm})
        del lg
    if ("ce" in which and "ce4" not in which) or "all" in which:
        Nr, V = 65536, 32768
        g = torch.Generator(device=dev).manual_seed(2)
        lg = torch.randn(Nr, V, device=dev, generator=g, dtype=bf)
        tg = torch.randint(0, V, (Nr,), device=dev, generator=g)
        grad = torch.empty_like(lg)
        loss = torch.zeros(Nr, device=dev)  # per-row losses
        mul = torch.full((), 1.0 / Nr, device=dev)
        st = _lib.stream_ptr(dev)
        f = lambda: _lib.call("fxb_ce_fwd_grad", 2, _lib.ptr(lg), V, _lib.ptr(tg), _lib.ptr(grad),  # noqa: E731
                              _lib.ptr(loss), _lib.ptr(mul), Nr, V, -100, st)
        ms = _time_ms(f, it)
        byt = 2 * Nr * V * 2
        out.append({"kernel": "ce_fwd_grad", "case": f"config 3 [{Nr},{V}] bf16 (read logits + write dlogits)",
                    "ms": ms, "gbs": byt / ms / 1e6, "frac_of_measured_hbm": byt / ms / 1e6 / hbm})
        del lg, grad
    if "adamw" in which or "all" in which:
        n = 110_906_112 + 8 * 80
        n -= n % 8
        grad = torch.randn(n, device=dev) * 1e-3
        master, m, v = torch.randn(n, device=dev) * 0.02, torch.zeros(n, device=dev), torch.zeros(n, device=dev)
        p16 = torch.empty(n, device=dev, dtype=bf)
        seg_end = torch.tensor([n], device=dev, dtype=torch.int64)
        seg_wd = torch.tensor([1], device=dev, dtype=torch.int32)
        scratch = torch.zeros(2, device=dev); flags = torch.zeros((), device=dev, dtype=torch.int32)
        step = torch.zeros((), device=dev, dtype=torch.int32); fi = torch.zeros((), device=dev)
        norm = torch.zeros((), device=dev); scale = torch.ones((), device=dev)
        st = _lib.stream_ptr(dev)
        P = _lib.ptr

        def f():
            _lib.call("fxb_adamw_sumsq", 0, P(grad), n, P(scratch), P(flags), st)
            _lib.call("fxb_adamw_final", P(scratch), P(flags), P(step), P(fi), P(norm), P(scale), 1.0, st)
            _lib.call("fxb_adamw_update", 0, 2, P(grad), P(master), P(m), P(v), P(p16), n, P(seg_end),
                      P(seg_wd), 1, P(scratch), P(fi), P(scale), P(step), 6e-4, None, 0.9, 0.95, 1e-8, 0.1, st)
        ms = _time_ms(f, it)
        byt = n * (4 + 4 + 4 + 24 + 2)
        out.append({"kernel": "adamw_sumsq + adamw_final + adamw_update", "case": f"{n} params fp32 grad",
                    "ms": ms, "gbs": byt / ms / 1e6, "frac_of_measured_hbm": byt / ms / 1e6 / hbm,
                    "bytes_per_param": 38})
    if "head" in which:
        # the config-4 LM head: linear_cross_entropy over 8192 rows (D 768,
        # V 32768) forward + backward, at several logits-chunk sizes
        from fxlm.cross_entropy import linear_cross_entropy
        Nr, D, V = 8192, 768, 32768
        g = torch.Generator(device=dev).manual_seed(3)
        x = torch.randn(Nr, D, device=dev, generator=g).to(bf).requires_grad_()
        W = (torch.randn(V, D, device=dev, generator=g) * 0.02).to(bf).requires_grad_()
        tg = torch.randint(0, V, (Nr,), device=dev, generator=g)
        for ch in (8192, 4096, 2048, 1024, 768):
            def f():
                loss = linear_cross_entropy(x, W, tg, chunk_rows=ch)
                loss.backward()
            ms = _time_ms(f, it)
            out.append({"kernel": "linear_cross_entropy fwd+bwd (3 GEMMs + CE per chunk)",
                        "case": f"N{Nr} D{D} V{V} chunk_rows {ch} (logits chunk {ch * V * 2 / 1e6:.0f} MB)",
                        "ms": ms, "tflops": 3 * 2.0 * Nr * D * V / ms / 1e9})
        # loss only: logits reduced on chip (fxb_linear_ce_loss) against the
        # logits GEMM + CE kernel over a materialised logits buffer
        from fxlm.cross_entropy import _ce_rows, _inv_nvalid
        xd, Wd = x.detach(), W.detach()

        def fused():
            with torch.no_grad():
                return linear_cross_entropy(xd, Wd, tg)
        lg_buf = torch.empty(Nr, V, device=dev, dtype=bf)
        rl = torch.empty(Nr, device=dev)

        def unfused():
            ops.gemm(xd, Wd, lg_buf)
            _ce_rows(lg_buf, tg, None, rl, _inv_nvalid(tg, -100), -100)
            return rl.sum()
        for nm, fn in (("loss only, logits kept on chip (fxb_linear_ce_loss)", fused),
                       ("loss only, logits GEMM + CE kernel over 537 MB of logits", unfused)):
            ms = _time_ms(fn, it)
            out.append({"kernel": "linear cross entropy " + nm, "case": f"N{Nr} D{D} V{V} bf16",
                        "ms": ms, "tflops": 2.0 * Nr * D * V / ms / 1e9})
    if "wmlp" in which or "all" in which:
        # the fxgpu window MLP training step (gather-linear
        # 1024 -> 512 + bias + GELU, 512 -> 256 + GELU, 256 -> 1, MSE, FlatAdamW)
        from fxgpu import WindowMLP
        from fxlm.optim import FlatAdamW
        R, Fe, Wn, Bsz = 500_000, 16, 64, 32768
        g = torch.Generator(device=dev).manual_seed(4)
        X16 = torch.randn(R, Fe, device=dev, generator=g).half()
        idx32 = torch.randint(0, R - Wn + 1, (Bsz,), device=dev, generator=g, dtype=torch.int32)
        tgt = torch.randn(Bsz, 1, device=dev, generator=g)
        torch.manual_seed(4)
        m = WindowMLP(Fe, Wn, hidden=512, hidden2=256, master=True, act="gelu",
                      dtype=torch.float16).to(dev)
        opt = FlatAdamW(m, lr=1e-3, init_scale=1024.0, param_dtype=torch.float16)

        def step():
            loss = ((m(X16, idx32).float() - tgt) ** 2).mean()
            opt.backward(loss)
            opt.step()
            opt.zero_grad()
        ms = _time_ms(step, it)
        flop = 94.6e9  # L1 fwd + dW, L2 and L3 fwd + dX + dW (no dX for L1)
        case = f"config 5: R={R} F={Fe} window={Wn} B={Bsz} 1024-512-256-1 GELU fp16"
        out.append({"kernel": "WindowMLP train step (gather, 3 GEMMs fwd, 5 bwd, FlatAdamW)",
                    "case": case + ", eager", "ms": ms, "tflops": flop / ms / 1e9,
                    "frac_of_measured_burst": flop / ms / 1e9 / tc, "samples_per_s": Bsz / ms * 1e3})
        # the same step captured once in a CUDA graph and replayed (the eager
        # loop is bound by host launch overhead at this size)
        try:
            from fxlm import GraphedFunction

            def train_step(ix, t):
                loss = ((m(X16, ix).float() - t) ** 2).mean()
                opt.backward(loss)
                opt.step()
                opt.zero_grad()
                return loss.detach()
            graphed = GraphedFunction(train_step, idx32, tgt)
            ms_g = _time_ms(lambda: graphed(idx32, tgt), it)
            out.append({"kernel": "WindowMLP train step (gather, 3 GEMMs fwd, 5 bwd, FlatAdamW)",
                        "case": case + ", CUDA graph replay (fxlm.GraphedFunction, batch copied in)",
                        "ms": ms_g, "tflops": flop / ms_g / 1e9,
                        "frac_of_measured_burst": flop / ms_g / 1e9 / tc, "samples_per_s": Bsz / ms_g * 1e3,
                        "library_launches_per_step": graphed.launches_per_call})
            graphed.release()
        except Exception as e:  # report the eager number regardless
            out.append({"kernel": "WindowMLP train step, CUDA graph replay", "case": case,
                        "error": repr(e)[:300]})
    return out


def kernel_rooflines(iters=30):
    """Roofline entries for the non-GEMM kernels of the north star, event-timed
    in this run (1 GPU): attention forward and forward + backward at config 2
    against the bf16 tensor peak; RMSNorm forward / backward (config 3 and the
    step's shape), cross entropy (config 3) and the FlatAdamW pass (config 4's
    parameters) against the measured HBM copy bandwidth."""
    hbm, hbm_src = _hbm_peak()
    tc, tc_src = _peaks({"sm_mhz": 1.0, "sm_max_mhz": 1.0})  # kernels timed alone: burst
    res = []
    for o in micro_results("attn,rmsnorm,ce,adamw", iters):
        k = o.get("kernel", "")
        if k.startswith("attn"):
            for what, key, ms in (("attn_fwd2_kernel", "fwd_tflops", o["fwd_ms"]),
                                  ("attn_fwd2_kernel + attn_bwd_kernel (+ prep, post)", "fwd_bwd_tflops",
                                   o["fwd_ms"] + o["bwd_ms"])):
                a = o[key]
                res.append({"kernel": what, "case": "BASELINE config 2: " + o["shape"], "bound": "tensor",
                            "achieved": a, "peak": tc, "unit": "TFLOP/s", "frac": a / tc, "ms": ms,
                            "peak_source": tc_src})
        elif "gbs" in o:
            res.append({"kernel": k, "case": o["case"], "bound": "hbm", "achieved": o["gbs"], "peak": hbm,
                        "unit": "GB/s", "frac": o["gbs"] / hbm, "ms": o["ms"], "peak_source": hbm_src})
    return res


def attach_dp(args, world, model, opt):
    """N > 1: the data-parallel gradient exchange the run uses (ZeRO-1 or
    all-reduce; fp32 or bf16 on the wire)."""
    import torch
    if world <= 1:
        return None
    cd = torch.bfloat16 if args.grad_bf16 else None
    if args.zero:
        from fxb200.zero import ShardedDataParallel
        return ShardedDataParallel(model, opt, comm_dtype=cd)
    from fxb200.ddp import DataParallel
    return DataParallel(model, opt, comm_dtype=cd)


# ---------------------------------------------------------------- loss-curve and data-parallel checks
def _gpt_and_opt(dev):
    """Config-4 model from the reference init (seed 3) and its FlatAdamW."""
    import torch
    from fxlm import GPT, GPTConfig, FlatAdamW
    torch.manual_seed(3)
    model = GPT(GPTConfig(**CFG4, eps=1e-6)).to(dev)
    opt = FlatAdamW(model, lr=6e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1,
                    max_grad_norm=1.0, init_scale=1.0, param_dtype=torch.bfloat16)
    return model, opt


def _golden_curve(acc):
    try:
        with open(os.path.join(ROOT, "tests", "golden", "curve_d768.json")) as f:
            return json.load(f).get(f"acc{acc}_stream")
    except Exception:
        return None


def curve_check(args, rank, world, local_rank, dev):
    """Config-4 loss curve of `steps` training steps from the reference init,
    outside the timed region, on a fresh Zipf batch every step (micro-batch r
    of step s: seed 1000 * (s + 1) + r; rank r trains micro-batch r).

    N = 1: every step's loss against the reference's own fp32 CPU curve on the
    same batches (tests/golden/curve_d768.json "acc1_stream", produced by
    tests/golden/make_golden.py from ml/fxlm/model.py), within 2%.
    N > 1: the data-parallel run (the bench's collectives: ZeRO-1 or
    all-reduce) against a single-process gradient accumulation of the same N
    micro-batches on rank 0 (loss / N per micro-batch, the reference's
    accumulation path, ml/fxlm/train_lm.py:199-205), which is what data
    parallelism must equal, and against the reference's CPU curve when one was
    generated for that accumulation count. Every rank's parameters must end
    bitwise equal.

    A fixed-batch curve is not used as the criterion: at this learning rate
    the memorisation run spikes at step 3, and past the spike the trajectory
    depends on the order of fp32 summation (the reference's own PyTorch path
    in fp32 on the GPU and on the CPU part there), so no implementation tracks
    the CPU curve within 2% beyond it."""
    import torch
    import torch.distributed as dist
    from fxb200.data import zipf_tokens
    steps = args.curve_steps if args.curve_steps is not None else (200 if world == 1 else 100)
    if steps <= 0:
        return None
    gold = _golden_curve(world)
    V = CFG4["vocab_size"]

    def batch(s, r):
        x, y = zipf_tokens(V, MB, SEQ, seed=1000 * (s + 1) + r)
        return x.pin_memory(), y.pin_memory()

    model, opt = _gpt_and_opt(dev)
    dp = attach_dp(args, world, model, opt)
    losses = torch.zeros(steps, device=dev)
    norms = torch.zeros(steps, device=dev)
    for s in range(steps):
        xh, yh = batch(s, rank)
        x, y = xh.to(dev, non_blocking=True), yh.to(dev, non_blocking=True)
        loss = model(x, y, grad_scale=opt.scale)
        opt.backward(loss)
        st = opt.step(6e-4)
        opt.zero_grad()
        losses[s] = loss.detach()
        norms[s] = st["grad_norm"]
    torch.cuda.synchronize()
    out = {"steps": steps, "data": "a fresh Zipf batch every step (seed 1000*(step+1) + rank), "
                                   "reference init (seed 3)"}
    if world > 1:
        dist.all_reduce(losses, op=dist.ReduceOp.SUM)
        losses /= world
        if hasattr(dp, "finish_gather"):
            dp.finish_gather()  # ZeRO-1 gathers the last update's parameters lazily
        # bitwise identity of the replicas: a position-weighted checksum of the
        # bf16 parameters, gathered from every rank
        bits = opt.flat16.view(torch.int16).to(torch.int64)
        w = torch.arange(bits.numel(), device=dev, dtype=torch.int64) % 65521 + 1
        h = torch.stack([(bits * w).sum(), bits.sum()])
        hs = [torch.zeros_like(h) for _ in range(world)]
        dist.all_gather(hs, h)
        out["ranks_bitwise_equal"] = all(torch.equal(hs[0], t) for t in hs)
    ours = losses.cpu().tolist()
    our_norms = norms.cpu().tolist()
    del model, opt
    gc.collect()
    torch.cuda.empty_cache()
    ref, kind = None, None
    if world == 1:
        if gold:
            ref, kind = gold["losses"], "reference fp32 CPU curve (tests/golden/curve_d768.json acc1_stream)"
    elif rank == 0:
        # single-process accumulation of the N micro-batches (rank 0 alone)
        m1, o1 = _gpt_and_opt(dev)
        acc_l = torch.zeros(steps, device=dev)
        acc_n = torch.zeros(steps, device=dev)
        for s in range(steps):
            tot = torch.zeros((), device=dev)
            for r in range(world):
                xh, yh = batch(s, r)
                lb = m1(xh.to(dev, non_blocking=True), yh.to(dev, non_blocking=True), grad_scale=o1.scale)
                o1.backward(lb / world)
                tot += lb.detach() / world
            st = o1.step(6e-4)
            o1.zero_grad()
            acc_l[s] = tot
            acc_n[s] = st["grad_norm"]
        torch.cuda.synchronize()
        ref = acc_l.cpu().tolist()
        kind = f"single-process accumulation of the {world} micro-batches (rank 0, same kernels)"
        nref = acc_n.cpu().tolist()
        out["grad_norm_step1"] = {"dp": our_norms[0], "accumulation": nref[0],
                                  "rel": abs(our_norms[0] - nref[0]) / max(abs(nref[0]), 1e-30)}
        del m1, o1
        gc.collect()
        torch.cuda.empty_cache()
        if gold:
            g = gold["losses"][:steps]
            out["vs_reference_cpu"] = {"steps": len(g), "max_rel_dev": max(
                abs(a - b) / abs(b) for a, b in zip(ours, g))}
    if world > 1:
        dist.barrier(device_ids=[local_rank])
    if ref is not None:
        n = min(len(ref), len(ours))
        dev_rel = [abs(a - b) / abs(b) for a, b in zip(ours[:n], ref[:n])]
        out.update({"against": kind, "steps_compared": n, "max_rel_dev": max(dev_rel),
                    "at_step": int(max(range(n), key=lambda i: dev_rel[i])),
                    "first_loss": ours[0], "ref_first_loss": ref[0], "final_loss": ours[n - 1],
                    "ref_final_loss": ref[n - 1], "tolerance": 0.02, "within_tolerance": max(dev_rel) < 0.02})
    elif rank == 0:
        out["against"] = "none (no golden curve for this accumulation count)"
    return out


# ---------------------------------------------------------------- config 5: window MLP
WMLP = dict(R=500_000, F=16, window=64, B=32768, hidden=512, hidden2=256)
WMLP_WORKLOAD = ("fxgpu window MLP (BASELINE config 5): per-GPU batch 32768, window 64 x 16 features -> "
                 "1024 -> 512 (+bias, GELU) -> 256 (GELU) -> 1, MSE, fp16 + fp32-master FlatAdamW lr 1e-3")
WMLP_FLOP = 94.6e9  # per 32768-sample step: L1 fwd + dW, L2 / L3 fwd + dX + dW


def cpu_baseline_wmlp(steps=3, warmup=1, rows=4096):
    """The reference window model's dense path (forward_dense, fp32) with
    autograd and an AdamW step on the host cores, on `rows` samples per step."""
    import torch
    from fxgpu.model import WindowMLP
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(4)
    xb = torch.randn(rows, WMLP["window"] * WMLP["F"], generator=g)
    tgt = torch.randn(rows, 1, generator=g)
    torch.manual_seed(4)
    m = WindowMLP(WMLP["F"], WMLP["window"], hidden=WMLP["hidden"], hidden2=WMLP["hidden2"],
                  master=True, act="gelu", dtype=torch.float32)
    opt = torch.optim.AdamW(m.parameters(), lr=1e-3, betas=(0.9, 0.95), weight_decay=0.1)
    times = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        opt.zero_grad(set_to_none=True)
        loss = ((m.forward_dense(xb) - tgt) ** 2).mean()
        loss.backward()
        opt.step()
        if i >= warmup:
            times.append(time.perf_counter() - t0)
    v = rows / statistics.mean(times)
    return {"value": v, "unit": "samples/s", "cores": threads, "kind": "port",
            "sample": f"{rows} samples per step, {steps} timed steps after {warmup} warm-up (fp32 dense "
                      f"trunk of the reference WindowMLP, ml/fxgpu/model.py forward_dense, + torch AdamW)"}


def run_wmlp(args, rank, world, local_rank):
    """Config 5 at N GPUs: each rank trains on its own 32768-sample batch
    (index seed 4 + rank) of one shared 500K x 16 fp16 series; the flat fp32
    gradient is reduced by fxb200.ddp.DataParallel (the model has no blocks:
    one reduction from the optimizer's pre-step hook) or ZeRO-1; the whole step
    (gather, 3 GEMMs forward, 5 backward, reduction, FlatAdamW) is one
    replayed CUDA graph."""
    import torch
    import torch.distributed as dist
    from fxb200 import _lib
    from fxgpu import WindowMLP
    from fxlm import FlatAdamW, GraphedFunction

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    _lib.load()
    R, Fe, Wn, Bsz = WMLP["R"], WMLP["F"], WMLP["window"], WMLP["B"]
    g = torch.Generator(device=dev).manual_seed(4)
    X16 = torch.randn(R, Fe, device=dev, generator=g).half()
    gi = torch.Generator().manual_seed(4 + rank)
    idx_host = torch.randint(0, R - Wn + 1, (Bsz,), generator=gi, dtype=torch.int32).pin_memory()
    tgt_host = torch.randn(Bsz, 1, generator=gi).pin_memory()
    idx, tgt = idx_host.to(dev), tgt_host.to(dev)
    torch.manual_seed(4)
    m = WindowMLP(Fe, Wn, hidden=WMLP["hidden"], hidden2=WMLP["hidden2"], master=True, act="gelu",
                  dtype=torch.float16).to(dev)
    opt = FlatAdamW(m, lr=1e-3, init_scale=1024.0, param_dtype=torch.float16)
    opt.lr_dev = torch.full((), 1e-3, device=dev)
    attach_dp(args, world, m, opt)

    def train_step(ix, t):
        loss = ((m(X16, ix).float() - t) ** 2).mean()
        opt.backward(loss)
        opt.step()
        opt.zero_grad()
        return loss.detach()

    graphed = GraphedFunction(train_step, idx, tgt, warmup=max(3, args.warmup))

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    torch.cuda.synchronize()
    barrier()
    clk = ClockSampler(local_rank)
    clk.start()
    time.sleep(0.3)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        loss = graphed(None, None)
    e1.record()
    torch.cuda.synchronize()
    clocks = clk.stop()
    barrier()
    t_ms = max_over_ranks(e0.elapsed_time(e1))
    samples = world * Bsz * args.steps
    value = samples / (t_ms / 1e3)
    # end to end: the batch (indices, targets) from pinned host memory every
    # step, the loss read back every step (synchronously: a 4-byte copy)
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    last = None
    for _ in range(args.steps):
        loss = graphed(idx_host.to(dev, non_blocking=True), tgt_host.to(dev, non_blocking=True))
        last = float(loss)
    f1.record()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(f0.elapsed_time(f1))
    graphed.check()
    launches = graphed.launches_per_call * args.steps
    graphed.release()
    if rank == 0:
        peak, peak_src = _peaks(clocks)
        achieved = WMLP_FLOP * world * args.steps / (t_ms / 1e3) / 1e12 / world
        line = {"metric": "fxgpu window MLP train samples/s (BASELINE config 5)", "value": value,
                "unit": "samples/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": t_ms / args.steps, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "fp16", "data": "synthetic N(0,1) series and targets (seed 4)",
                "config": {"workload": WMLP_WORKLOAD, "global_batch": Bsz * world,
                           "parallelism": f"dp{world}" + ("-zero1" if args.zero and world > 1 else ""),
                           "step": "CUDA graph replay (fxlm.GraphedFunction)",
                           "l2": "no flush: a step moves ~1 GB (> 126 MB L2)"},
                "e2e": {"value": samples / (e2e_ms / 1e3), "unit": "samples/s",
                        "h2d_bytes_per_step": Bsz * 4 + Bsz * 4, "d2h_bytes_per_step": 4,
                        "last_loss": last},
                "gpu_launches": launches,
                "roofline": {"bound": "tensor", "kernel": "whole step (3 GEMMs fwd, 5 bwd, gather, FlatAdamW)",
                             "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
                             "traffic": None, "peak_source": peak_src,
                             "flops_per_step": WMLP_FLOP},
                "clocks": clocks, "final_loss": last}
        if world == 1 and not args.no_cpu:
            line["cpu_baseline"] = cpu_baseline_wmlp()
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()


# ---------------------------------------------------------------- our arm
def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from fxb200 import _lib, ops
    from fxb200.data import zipf_tokens
    from fxlm import GPT, GPTConfig, FlatAdamW

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    _lib.load()

    torch.manual_seed(3)
    model = GPT(GPTConfig(**CFG4, eps=1e-6)).to(dev)
    opt = FlatAdamW(model, lr=6e-4, betas=(0.9, 0.95), eps=1e-8, weight_decay=0.1,
                    max_grad_norm=1.0, init_scale=1.0, param_dtype=torch.bfloat16)
    attach_dp(args, world, model, opt)
    x_cpu, y_cpu = zipf_tokens(CFG4["vocab_size"], MB, SEQ, seed=3 + rank)
    x_host, y_host = x_cpu.pin_memory(), y_cpu.pin_memory()
    x_dev, y_dev = x_cpu.to(dev), y_cpu.to(dev)

    def eager_step(x, y):
        loss = model(x, y, grad_scale=opt.scale)
        opt.backward(loss)
        opt.step(6e-4)
        opt.zero_grad()
        return loss

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # one process per GPU: the step is captured in a CUDA graph (fxlm.GraphedStep,
    # warm-up steps run before capture); with N > 1 the graph includes the
    # bucketed NCCL gradient all-reduces
    graphed = None
    if not args.no_graph:
        from fxlm import GraphedStep
        graphed = GraphedStep(model, opt, x_dev, y_dev, warmup=args.warmup)

        def step(x, y):
            return graphed()  # x, y already are the graph's static inputs
    else:
        step = eager_step
        for _ in range(args.warmup):
            step(x_dev, y_dev)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()

    # ---- device-timed steps, inputs resident in HBM
    clk = ClockSampler(local_rank)
    clk.start()
    time.sleep(0.3)
    n0 = _lib.launch_count()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(args.steps):
        loss = step(x_dev, y_dev)
    ev1.record()
    torch.cuda.synchronize()
    launches = (graphed.launches_per_step * args.steps if graphed is not None
                else _lib.launch_count() - n0)
    clocks = clk.stop()
    barrier()
    t_ms = max_over_ranks(ev0.elapsed_time(ev1))
    tokens = world * MB * SEQ * args.steps
    value = tokens / (t_ms / 1e3)
    final_loss = float(loss.item())

    # ---- GEMM roofline: the same steps again with an event pair around every
    # GEMM launch (kept out of the timed region above)
    # (weight-gradient GEMMs stay on the launching stream here, so that no two
    # timed GEMMs overlap)
    records = []
    dw_env = os.environ.get("FXB_DW_STREAM")
    os.environ["FXB_DW_STREAM"] = "0"
    ops.set_gemm_timing(records)
    for _ in range(args.steps):
        eager_step(x_dev, y_dev)
    torch.cuda.synchronize()
    ops.set_gemm_timing(None)
    if dw_env is None:
        del os.environ["FXB_DW_STREAM"]
    else:
        os.environ["FXB_DW_STREAM"] = dw_env
    barrier()
    g_flops = sum(r[0] for r in records)
    g_ms = sum(r[1].elapsed_time(r[2]) for r in records)
    n_gemm = len(records)
    achieved = g_flops / (g_ms / 1e3) / 1e12 if g_ms > 0 else None

    # ---- end to end through the public API: H2D batch + D2H loss each step,
    # pipelined as a training loop would run them: step k+1's batch is copied
    # from pinned host memory on a side stream while step k runs (two device
    # staging buffers; the step's own inputs are filled by a device copy), and
    # each step's loss is copied to pinned host memory asynchronously and read
    # once the next step has been queued; the last loss is read before the end
    # event
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    xin, yin = (graphed.x, graphed.y) if graphed is not None else (x_dev, y_dev)
    cstream = torch.cuda.Stream(device=dev)
    comp = torch.cuda.current_stream(dev)
    stage = [(torch.empty_like(xin), torch.empty_like(yin)) for _ in range(2)]
    loss_host = [torch.empty((), dtype=torch.float32, pin_memory=True) for _ in range(2)]
    ev_in = [torch.cuda.Event() for _ in range(2)]    # batch landed in stage[i]
    ev_used = [torch.cuda.Event() for _ in range(2)]  # stage[i] copied into the step's inputs
    ev_loss = [torch.cuda.Event() for _ in range(2)]  # loss of the step reached loss_host[i]

    def fetch(i):
        with torch.cuda.stream(cstream):
            cstream.wait_event(ev_used[i])
            stage[i][0].copy_(x_host, non_blocking=True)
            stage[i][1].copy_(y_host, non_blocking=True)
            ev_in[i].record(cstream)

    for i in range(2):
        ev_used[i].record(comp)
    e0.record()
    fetch(0)
    last = None
    for k in range(args.steps):
        cur = k & 1
        if k + 1 < args.steps:
            fetch(1 - cur)
        comp.wait_event(ev_in[cur])
        xin.copy_(stage[cur][0], non_blocking=True)
        yin.copy_(stage[cur][1], non_blocking=True)
        ev_used[cur].record(comp)
        loss = step(xin, yin)
        loss_host[cur].copy_(loss.detach().float(), non_blocking=True)
        ev_loss[cur].record(comp)
        if k > 0:
            ev_loss[1 - cur].synchronize()
            last = float(loss_host[1 - cur])
    ev_loss[(args.steps - 1) & 1].synchronize()
    last = float(loss_host[(args.steps - 1) & 1])
    e1.record()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    e2e = {"value": tokens / (e2e_ms / 1e3), "unit": "tokens/s",
           "h2d_bytes_per_step": x_host.numel() * 8 + y_host.numel() * 8, "d2h_bytes_per_step": 4,
           "copies": "pipelined (next batch H2D on a side stream, loss D2H read one step later)",
           "last_loss": last}

    attn = attn_tflops(dev) if (rank == 0 and not args.no_attn) else None
    barrier()
    derr = _lib.device_error(clear=True)

    # ---- loss curve (N = 1: against the reference; N > 1: against gradient
    # accumulation) and replica identity, on a fresh model after the timed work
    step_mode = "CUDA graph replay (fxlm.GraphedStep)" if graphed is not None else "eager"
    if graphed is not None:
        graphed.release()
        graphed = None
    del model, opt
    gc.collect()
    torch.cuda.empty_cache()
    curve = curve_check(args, rank, world, local_rank, dev)
    derr |= _lib.device_error(clear=True)

    if rank == 0:
        peak, peak_src = _peaks(clocks)
        traffic = _gemm_traffic()
        line = {
            "metric": _metric(), "value": value, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": t_ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic Zipf(1.1) tokens, seed 3 + rank; reference init (seed 3)",
            "config": {"workload": WORKLOAD, "global_batch": MB * world, "seq_len": SEQ,
                       "parallelism": f"dp{world}" + ("-zero1" if args.zero and world > 1 else "")
                                      + ("-bf16grad" if args.grad_bf16 and world > 1 else ""),
                       "model": "GPT d768x12L tied, V32768",
                       "step": step_mode,
                       "l2": "no flush: one step moves several GB (> 126 MB L2)"},
            "e2e": e2e,
            "gpu_launches": launches,
            "roofline": {"bound": "tensor", "kernel": "gemm_tc_kernel (all GEMM launches of the step)",
                         "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": (achieved / peak) if achieved else None,
                         "traffic": traffic, "peak_source": peak_src,
                         "gemm_launches": n_gemm, "gemm_flops_per_step": g_flops / args.steps,
                         "gemm_ms_per_step": g_ms / args.steps,
                         "gemm_timing": "an event pair around every GEMM launch in a separate eager "
                                        "pass of the same steps (host gaps before a launch count "
                                        "toward its time)"},
            "model_tflops": value * 717e6 / 1e12,  # 717 MFLOP/token (6 x 110.1M matmul params + attention)
            "clocks": clocks,
            "final_loss": final_loss,
            "device_error_word": derr,
        }
        if attn is not None:
            line["attn"] = attn
        if curve is not None:
            line["curve_check"] = curve
        if world == 1 and not args.no_kernels:
            line["kernels"] = kernel_rooflines()
        if world == 1 and not args.no_cpu:
            line["cpu_baseline"] = cpu_baseline()
        print(json.dumps(line), flush=True)
    if graphed is not None:
        graphed.release()  # a graph holding NCCL calls must go before the process group
    if world > 1:
        dist.barrier(device_ids=[local_rank])
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["gpt", "wmlp"], default="gpt",
                    help="gpt: BASELINE config 4 (default); wmlp: config 5, the window MLP")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-attn", action="store_true", help="skip the attention microbench")
    ap.add_argument("--no-kernels", action="store_true",
                    help="skip the per-kernel roofline entries (N = 1)")
    ap.add_argument("--no-graph", action="store_true",
                    help="run the step eagerly instead of replaying a captured CUDA graph")
    ap.add_argument("--no-zero", dest="zero", action="store_false", default=None,
                    help="N > 1: plain data parallelism (all-reduce, every rank updates every "
                         "parameter) instead of the sharded update (fxb200.zero, the default "
                         "for the gpt workload)")
    ap.add_argument("--grad-bf16", action="store_true",
                    help="N > 1: gradient buckets cross NVLink as bf16 (half the bytes) instead of fp32")
    ap.add_argument("--zero", dest="zero", action="store_true",
                    help="N > 1: the sharded update (default for gpt; the window MLP's 0.66 M "
                         "parameters are cheaper to all-reduce than to shard)")
    ap.add_argument("--micro", default=None,
                    help="per-kernel microbenchmarks instead of the step: all or a comma list "
                         "of gemm,attn,rmsnorm,ce,adamw,wmlp")
    ap.add_argument("--iters", type=int, default=20, help="iterations per microbenchmark")
    ap.add_argument("--curve-steps", type=int, default=None,
                    help="loss-curve check length after the timed run (default 200 at N = 1, "
                         "100 at N > 1; 0 skips it)")
    ap.add_argument("--only", default=None,
                    help="gemm_layer: comma-separated substrings selecting shapes (profiling)")
    args = ap.parse_args()
    if args.zero is None:
        args.zero = args.workload == "gpt"
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.micro:
        return run_micro(args)
    if args.impl == "reference":
        return run_reference(args, rank, world)
    if args.workload == "wmlp":
        return run_wmlp(args, rank, world, local_rank)
    return run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
