"""fxlm.sample: text generation from a `fxlm.train_lm` checkpoint.

Same command line and decoding loop as the reference's ml/fxlm/sample.py:22-77:
the fp32 master weights are loaded by parameter name into a GPT built from
the checkpoint's config and cast to the inference dtype; each new token
re-runs the forward on the last `seq_len` tokens (no KV cache), divides the
last position's fp32 logits by max(temperature, 1e-5), keeps the top-k
(ties with the k-th value kept), and draws from the softmax. Byte-level
checkpoints (`meta.tokenizer == "bytes"`) encode the prompt as UTF-8 bytes
(an empty prompt starts from "\\n") and decode the output with replacement.
Additions: `--dtype` (default: the dtype the checkpoint was trained in, fp16
when it does not say, as the reference's `model.half()`), `--seed`, and for
other tokenizers `--prompt-ids` / token ids printed on stdout.

    python -m fxlm.sample --ckpt runs/demo/ckpt_last.pt --prompt "def " \\
        --max-new 200 --temperature 0.8 --top-k 50
"""
import argparse
import sys

_DTYPES = {"bf16": "bfloat16", "fp16": "float16", "fp32": "float32"}


def load_checkpoint(path, device, dtype=None):
    """(model, meta, missing) from a train_lm checkpoint; `dtype` None picks
    the training dtype recorded in the checkpoint's args, else fp16."""
    import torch
    from fxlm.model import GPT, GPTConfig

    sd = torch.load(path, map_location="cpu", weights_only=False)
    cfg = GPTConfig(**sd["config"])
    if dtype is None:
        dtype = getattr(torch, _DTYPES[(sd.get("args") or {}).get("dtype", "fp16")])
    model = GPT(cfg)
    missing = []
    with torch.no_grad():
        for name, p in model.named_parameters():
            if name in sd["model"]:
                p.copy_(sd["model"][name].to(p.dtype))
            else:
                missing.append(name)
    model = model.to(device=device, dtype=dtype).eval()
    return model, sd.get("meta", {}), missing


def generate(model, ids, max_new, temperature=0.8, top_k=50, generator=None):
    """Append `max_new` sampled tokens to `ids` (1-D or (1, n) int64) and
    return the (1, n + max_new) sequence (ml/fxlm/sample.py:63-73)."""
    import torch

    x = ids.view(1, -1)
    seq_len = model.cfg.seq_len
    for _ in range(max_new):
        with torch.inference_mode():
            logits = model(x[:, -seq_len:])[:, -1, :].float()
        logits = logits / max(temperature, 1e-5)
        if top_k > 0:
            kth = torch.topk(logits, min(top_k, logits.shape[-1])).values[:, -1:]
            logits = logits.masked_fill(logits < kth, float("-inf"))
        probs = torch.softmax(logits, dim=-1)
        nxt = torch.multinomial(probs, 1, generator=generator)
        x = torch.cat([x, nxt], dim=1)
    return x


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--ckpt", required=True)
    ap.add_argument("--prompt", default="")
    ap.add_argument("--prompt-ids", default=None,
                    help="comma-separated token ids (tokenizers other than bytes)")
    ap.add_argument("--max-new", type=int, default=200)
    ap.add_argument("--temperature", type=float, default=0.8)
    ap.add_argument("--top-k", type=int, default=50)
    ap.add_argument("--dtype", choices=sorted(_DTYPES), default=None)
    ap.add_argument("--seed", type=int, default=None)
    args = ap.parse_args(argv)

    from fxlm.env import setup_lm_env
    setup_lm_env(tunable=False)
    import torch
    from fxlm.env import require_gpu

    device = require_gpu()
    dtype = getattr(torch, _DTYPES[args.dtype]) if args.dtype else None
    model, meta, missing = load_checkpoint(args.ckpt, device, dtype)
    if missing:
        print("missing parameters:", missing, file=sys.stderr)
    gen = None
    if args.seed is not None:
        gen = torch.Generator(device=device)
        gen.manual_seed(args.seed)

    tok = meta.get("tokenizer", "bytes")
    if tok == "bytes":
        raw = list(args.prompt.encode("utf-8")) or [10]
        def decode(t):
            return bytes(t.tolist()).decode("utf-8", errors="replace")
    elif args.prompt_ids:
        raw = [int(s) for s in args.prompt_ids.split(",") if s.strip()]
        def decode(t):
            return " ".join(str(v) for v in t.tolist())
    else:
        raise SystemExit(f"tokenizer '{tok}' has no text encoding: give --prompt-ids")
    ids = torch.tensor(raw, dtype=torch.long, device=device)
    out = generate(model, ids, args.max_new, args.temperature, args.top_k, gen)[0, ids.numel():]
    text = decode(out)
    sys.stdout.write(text + "\n")
    sys.stdout.flush()
    return text


if __name__ == "__main__":
    main()
