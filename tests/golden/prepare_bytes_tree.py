"""Deterministic input tree and cases for the prepare_bytes golden fixture.

Shared by tests/golden/make_golden.py (which runs the reference's
ml/fxlm/prepare_bytes.py on it and records the outputs' SHA-256) and
tests/test_host_tools.py (which runs fxlm.prepare_bytes on the same tree).
Every directory holds at most one matching file so that the walk order does
not depend on the file system.
"""
import os

import numpy as np

_ALPHABET = ("abcdefghijklmnopqrstuvwxyz ABCDEFGHIJ0123456789\n\t()[]{}:=+-*/#'\"._,"
             "çğıöşüÇĞİÖŞÜ€")


def _text(seed, n_chars):
    rng = np.random.default_rng(seed)
    chars = rng.choice(list(_ALPHABET), size=n_chars)
    return "".join(chars).encode("utf-8")


def build_tree(root):
    """Write the input files under `root` and return nothing."""
    files = {
        "a.py": _text(1, 3000),
        "b.md": _text(2, 1500),
        "c.txt": _text(3, 800),
        "blob.py": b"text first" + b"\x00" + _text(4, 100),   # binary: NUL in the first 8 KB
        "late_nul.txt": _text(5, 9000) + b"\x00tail",         # NUL after 8 KB: kept as text
        os.path.join("dir", "d.py"): _text(6, 700),
        os.path.join("dir", "skip.rst"): _text(7, 200),
        os.path.join("dir", "sub", "e.txt"): _text(8, 400),
    }
    for rel, data in files.items():
        path = os.path.join(root, rel)
        os.makedirs(os.path.dirname(path), exist_ok=True)
        with open(path, "wb") as f:
            f.write(data)


# (name, positional inputs relative to the tree root, options)
CASES = [
    ("files", ["a.py", "blob.py", "b.md", "late_nul.txt"], []),
    ("glob_maxbytes", ["*.txt", "a.py"], ["--max-bytes", "5000", "--val-frac", "0.05"]),
    ("dir_ext", ["dir", "c.txt"], ["--ext", ".py,.txt", "--val-frac", "0.2"]),
]
