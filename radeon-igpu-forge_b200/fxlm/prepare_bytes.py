"""fxlm.prepare_bytes: text files -> byte-level uint16 token files.

Writes the token format `fxlm.train_lm` reads, the same as the reference's
ml/fxlm/prepare_bytes.py:18-99: every byte of the input text is one token
(vocabulary 256), stored as little-endian uint16 in `<out>_train.bin` and
`<out>_val.bin` (the last `val_frac` of the bytes, at least one token), with
`<out>.json` = {vocab_size: 256, tokenizer: "bytes", n_train, n_val,
n_files}. Inputs are files, directories (walked, filtered by extension) or
glob patterns; a file whose first 8 KB hold a NUL byte is skipped as binary;
`max_bytes` truncates the concatenation.

    python -m fxlm.prepare_bytes --out data/demo "src/**/*.py" docs/
"""
import argparse
import glob
import json
import os

import numpy as np

_SNIFF_BYTES = 8192


def collect_files(inputs, exts=(".txt", ".md", ".py")):
    """Expand directories (by extension) and globs; a pattern without glob
    hits is kept as a path (ml/fxlm/prepare_bytes.py:35-45)."""
    exts = tuple(e.lower() for e in exts)
    out = []
    for item in inputs:
        if os.path.isdir(item):
            for root, _dirs, names in os.walk(item):
                out.extend(os.path.join(root, n) for n in names if n.lower().endswith(exts))
            continue
        hits = sorted(glob.glob(item))
        out.extend(hits or [item])
    return [f for f in out if os.path.isfile(f)]


def is_text(path):
    """False for unreadable files and for files with a NUL byte in the first
    8 KB (ml/fxlm/prepare_bytes.py:49-60)."""
    try:
        with open(path, "rb") as fh:
            return b"\x00" not in fh.read(_SNIFF_BYTES)
    except OSError:
        return False


def read_corpus(files, max_bytes=0):
    """Concatenated bytes of `files` in order, cut at `max_bytes` (0: no
    limit), as in ml/fxlm/prepare_bytes.py:67-80."""
    parts, total = [], 0
    for f in files:
        try:
            with open(f, "rb") as fh:
                data = fh.read()
        except OSError:
            continue
        if max_bytes:
            data = data[:max_bytes - total]
        parts.append(data)
        total += len(data)
        if max_bytes and total >= max_bytes:
            break
    return b"".join(parts)


def write_tokens(raw, out, val_frac=0.01, n_files=0):
    """Split bytes into train / val uint16 token files plus the .json meta
    (ml/fxlm/prepare_bytes.py:81-97). Returns the meta dict."""
    toks = np.frombuffer(raw, dtype=np.uint8).astype("<u2")
    n = int(toks.size)
    n_val = max(1, int(n * val_frac))
    n_train = n - n_val
    os.makedirs(os.path.dirname(os.path.abspath(out)), exist_ok=True)
    toks[:n_train].tofile(out + "_train.bin")
    toks[n_train:].tofile(out + "_val.bin")
    meta = {"vocab_size": 256, "tokenizer": "bytes", "n_train": n_train, "n_val": n_val,
            "n_files": int(n_files)}
    with open(out + ".json", "w", encoding="utf-8") as f:
        json.dump(meta, f, indent=2)
    return meta


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("inputs", nargs="+", help="text files, directories or globs")
    ap.add_argument("--out", required=True, help="output prefix: <out>_train.bin + <out>.json")
    ap.add_argument("--val-frac", type=float, default=0.01)
    ap.add_argument("--max-bytes", type=int, default=0, help="0: no limit")
    ap.add_argument("--ext", default=".txt,.md,.py",
                    help="extensions taken when walking a directory (comma separated)")
    args = ap.parse_args(argv)

    exts = tuple(e.strip() for e in args.ext.split(",") if e.strip())
    files = collect_files(args.inputs, exts)
    if not files:
        raise SystemExit("no input files found: " + " ".join(args.inputs))
    text = [f for f in files if is_text(f)]
    if len(text) < len(files):
        print(f"skipped {len(files) - len(text)} binary files")
    if not text:
        raise SystemExit("no text files left after the binary filter")
    print(f"reading {len(text)} files...")
    meta = write_tokens(read_corpus(text, args.max_bytes), args.out, args.val_frac, len(text))
    print(f"wrote {args.out}_train.bin ({meta['n_train']:,} tokens) | "
          f"{args.out}_val.bin ({meta['n_val']:,}) | {args.out}.json")
    return meta


if __name__ == "__main__":
    main()
