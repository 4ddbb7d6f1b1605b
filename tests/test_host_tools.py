"""CPU tests of the host-side tools around the training step.

`fxlm.prepare_bytes` (the reference's ml/fxlm/prepare_bytes.py:18-99): file
collection from directories / globs / paths, the NUL-byte binary filter, the
max-bytes cut, the train / val split and the uint16 + json format that
`fxlm.train_lm` reads. `fxlm.sample` (ml/fxlm/sample.py:22-77): checkpoint
loading by parameter name and the decoding loop (context crop to seq_len,
temperature, top-k with ties kept, seeded draws), run on the model's own
PyTorch path on CPU or on a stub model with fixed logits.
"""
import json
import os

import numpy as np
import pytest
import torch

from fxlm import prepare_bytes as pb
from fxlm import sample as smp


def _write(path, data):
    os.makedirs(os.path.dirname(path), exist_ok=True)
    with open(path, "wb") as f:
        f.write(data)


@pytest.fixture
def corpus(tmp_path):
    d = tmp_path / "src"
    _write(str(d / "a.py"), b"print('hi')\n")
    _write(str(d / "b.md"), "# türkçe\n".encode("utf-8"))
    _write(str(d / "sub" / "c.txt"), b"x" * 300)
    _write(str(d / "skip.rst"), b"not taken by extension\n")
    _write(str(d / "bin.py"), b"abc\x00def")
    return d


def test_collect_files_dirs_globs_and_paths(corpus, tmp_path):
    got = pb.collect_files([str(corpus)], (".py", ".md", ".txt"))
    names = sorted(os.path.relpath(f, corpus) for f in got)
    assert names == ["a.py", "b.md", "bin.py", os.path.join("sub", "c.txt")]
    # a glob is sorted and not filtered by extension
    got = pb.collect_files([str(corpus / "*.rst"), str(corpus / "*.py")], (".txt",))
    assert [os.path.basename(f) for f in got] == ["skip.rst", "a.py", "bin.py"]
    # a path without glob hits is kept only when it is a file
    assert pb.collect_files([str(tmp_path / "nope.txt")]) == []


def test_binary_filter_and_corpus_order(corpus):
    files = pb.collect_files([str(corpus / "a.py"), str(corpus / "bin.py"), str(corpus / "b.md")])
    text = [f for f in files if pb.is_text(f)]
    assert [os.path.basename(f) for f in text] == ["a.py", "b.md"]
    raw = pb.read_corpus(text)
    assert raw == b"print('hi')\n" + "# türkçe\n".encode("utf-8")
    # max_bytes cuts inside a file and stops reading
    assert pb.read_corpus(text, max_bytes=5) == b"print"
    assert pb.read_corpus(text, max_bytes=14) == raw[:14]


def test_main_writes_train_val_and_meta(corpus, tmp_path):
    out = str(tmp_path / "data" / "demo")
    meta = pb.main([str(corpus), "--out", out, "--val-frac", "0.1"])
    raw = b"".join(open(f, "rb").read() for f in
                   sorted(pb.collect_files([str(corpus)])) if pb.is_text(f))
    tr = np.fromfile(out + "_train.bin", dtype="<u2")
    va = np.fromfile(out + "_val.bin", dtype="<u2")
    n = len(raw)
    assert meta["n_val"] == max(1, int(n * 0.1)) and meta["n_train"] == n - meta["n_val"]
    assert tr.size == meta["n_train"] and va.size == meta["n_val"]
    assert int(np.concatenate([tr, va]).max()) < 256
    with open(out + ".json", encoding="utf-8") as f:
        on_disk = json.load(f)
    assert on_disk == {"vocab_size": 256, "tokenizer": "bytes", "n_train": meta["n_train"],
                       "n_val": meta["n_val"], "n_files": 3}
    # the walk order of os.walk is not sorted: compare as multisets of files
    got = bytes(np.concatenate([tr, va]).astype(np.uint8))
    assert sorted(got) == sorted(raw)


def test_main_tiny_input_keeps_one_val_token(tmp_path):
    _write(str(tmp_path / "one.txt"), b"ab")
    meta = pb.main([str(tmp_path / "one.txt"), "--out", str(tmp_path / "o")])
    assert (meta["n_train"], meta["n_val"]) == (1, 1)
    assert np.fromfile(str(tmp_path / "o_val.bin"), dtype="<u2").tolist() == [ord("b")]


def test_main_errors(tmp_path):
    with pytest.raises(SystemExit, match="no input files"):
        pb.main([str(tmp_path / "missing*.txt"), "--out", str(tmp_path / "o")])
    _write(str(tmp_path / "z.txt"), b"\x00\x01")
    with pytest.raises(SystemExit, match="no text files"):
        pb.main([str(tmp_path / "z.txt"), "--out", str(tmp_path / "o")])


# ------------------------------------------------------------------ sample
CFG = dict(vocab_size=256, seq_len=16, n_layer=2, n_head=2, d_model=64,
           attn_impl="sdpa", norm_impl="torch", ce_impl="torch", linear_impl="torch")


def _torch_model():
    from fxlm.model import GPT, GPTConfig
    torch.manual_seed(0)
    return GPT(GPTConfig(**CFG)).eval()


def test_generate_top1_is_greedy_and_crops_context():
    m = _torch_model()
    prompt = torch.arange(20, dtype=torch.long) % 256        # longer than seq_len
    out = smp.generate(m, prompt, 6, temperature=1.0, top_k=1)
    assert out.shape == (1, 26) and torch.equal(out[0, :20], prompt)
    x = prompt.view(1, -1)
    for _ in range(6):
        with torch.no_grad():
            nxt = m(x[:, -16:])[:, -1, :].argmax(-1, keepdim=True)
        x = torch.cat([x, nxt], 1)
    assert torch.equal(out, x)


def test_generate_seeded_draws_repeat():
    m = _torch_model()
    p = torch.tensor([10], dtype=torch.long)
    a = smp.generate(m, p, 8, 0.8, 50, torch.Generator().manual_seed(3))
    b = smp.generate(m, p, 8, 0.8, 50, torch.Generator().manual_seed(3))
    assert torch.equal(a, b)


class _FixedLogits(torch.nn.Module):
    """Stub with the GPT call shape: logits (1, T, V) from a fixed row."""

    def __init__(self, row, seq_len=8):
        super().__init__()
        self.row = row
        self.cfg = type("C", (), {"seq_len": seq_len})()
        self.seen = []

    def forward(self, x):
        self.seen.append(x.shape[1])
        return self.row.view(1, 1, -1).expand(1, x.shape[1], -1).clone()


def test_generate_top_k_keeps_ties_and_temperature_floor():
    row = torch.tensor([0.0, 5.0, 3.0, 5.0, 1.0, 3.0])
    m = _FixedLogits(row)
    g = torch.Generator().manual_seed(0)
    out = smp.generate(m, torch.tensor([0]), 400, temperature=1.0, top_k=3, generator=g)[0, 1:]
    # the 3rd largest value is 3.0: both 3.0 entries are kept with both 5.0s
    assert set(out.tolist()) <= {1, 2, 3, 5} and {1, 3} <= set(out.tolist())
    assert max(m.seen) == 8                                   # context cropped to seq_len
    # temperature 0 is floored at 1e-5: sampling becomes argmax among the maxima
    out = smp.generate(_FixedLogits(row), torch.tensor([0]), 50, temperature=0.0, top_k=0,
                       generator=torch.Generator().manual_seed(1))[0, 1:]
    assert set(out.tolist()) <= {1, 3}


def test_load_checkpoint_by_name(tmp_path):
    m = _torch_model()
    sd = {"model": {k: v.detach().float().clone() for k, v in m.state_dict().items()},
          "config": dict(CFG, eps=1e-6, mlp_ratio=4, tie_embeddings=True),
          "meta": {"vocab_size": 256, "tokenizer": "bytes"}, "args": {"dtype": "bf16"}, "step": 7}
    del sd["model"]["lnf_w"]
    path = str(tmp_path / "ckpt.pt")
    torch.save(sd, path)
    got, meta, missing = smp.load_checkpoint(path, "cpu")
    assert missing == ["lnf_w"] and meta["tokenizer"] == "bytes"
    assert got.tok_emb.weight.dtype == torch.bfloat16 and not got.training
    assert torch.equal(got.tok_emb.weight, m.tok_emb.weight.bfloat16())
    assert torch.equal(got.blocks[1].fc2.weight, m.blocks[1].fc2.weight.bfloat16())
    got32, _, _ = smp.load_checkpoint(path, "cpu", torch.float32)
    assert torch.equal(got32.blocks[0].qkv.weight, m.blocks[0].qkv.weight)
    del sd["args"]                                            # no recorded dtype: fp16
    torch.save(sd, path)
    assert smp.load_checkpoint(path, "cpu")[0].pos_emb.dtype == torch.float16


def test_prepare_bytes_matches_reference_outputs(tmp_path):
    """Same token files and meta as the reference's own script on the same
    tree (tests/golden/prepare_bytes.json, made by make_golden.py)."""
    import hashlib
    import sys
    gold_dir = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
    sys.path.insert(0, gold_dir)
    try:
        from prepare_bytes_tree import build_tree, CASES
    finally:
        sys.path.remove(gold_dir)
    with open(os.path.join(gold_dir, "prepare_bytes.json")) as f:
        gold = json.load(f)
    root = str(tmp_path / "tree")
    build_tree(root)
    assert sorted(gold) == sorted(c[0] for c in CASES)
    for name, inputs, opts in CASES:
        prefix = str(tmp_path / "out" / name)
        meta = pb.main([os.path.join(root, i) for i in inputs] + ["--out", prefix] + opts)
        assert meta == gold[name]["meta"], name
        for part in ("train", "val"):
            with open(f"{prefix}_{part}.bin", "rb") as f:
                assert hashlib.sha256(f.read()).hexdigest() == gold[name]["sha256_" + part], (name, part)


# ------------------------------------------------------------------ train_lm
def test_train_lm_cli_defaults_and_lr_schedule():
    """Defaults of the reference's command line (ml/fxlm/train_lm.py:26-51)
    and its warmup + cosine schedule (:154-160), restated here."""
    import math
    from fxlm import train_lm
    a = train_lm._parse(["--data", "x_train.bin", "--out", "o", "--tunable"])
    assert (a.seq_len, a.layers, a.heads, a.dim, a.batch, a.accum, a.steps) == (256, 8, 8, 512, 16, 1, 2000)
    assert (a.lr, a.min_lr_frac, a.warmup, a.wd, a.clip) == (6e-4, 0.1, 100, 0.1, 1.0)
    assert (a.eval_every, a.eval_batches, a.log_every, a.seed) == (200, 20, 20, 0)
    assert a.init_scale == 1.0 and a.dtype == "bf16"
    assert train_lm._parse(["--out", "o", "--dtype", "fp16"]).init_scale == 2.0 ** 16
    assert train_lm._parse(["--out", "o", "--init-scale", "8"]).init_scale == 8.0

    def ref(step, lr, warm, steps, mf):
        if step < warm:
            return lr * (step + 1) / warm
        t = (step - warm) / max(1, steps - warm)
        return lr * (mf + (1.0 - mf) * 0.5 * (1.0 + math.cos(math.pi * min(1.0, t))))
    for steps, warm in ((2000, 100), (10, 0), (5, 5), (1, 1)):
        a = train_lm._parse(["--out", "o", "--steps", str(steps), "--warmup", str(warm)])
        for s in list(range(0, steps + 3)):
            assert train_lm.lr_at(s, a) == pytest.approx(ref(s, a.lr, warm, steps, a.min_lr_frac), rel=1e-12)
    a = train_lm._parse(["--out", "o"])
    assert train_lm.lr_at(99, a) == pytest.approx(6e-4) and train_lm.lr_at(100, a) == pytest.approx(6e-4)
    assert train_lm.lr_at(2000, a) == pytest.approx(6e-5) and train_lm.lr_at(5000, a) == pytest.approx(6e-5)


def test_graphed_function_argument_checks():
    """Host-side checks of fxlm.GraphedFunction (capture itself needs a GPU)."""
    from fxlm import GraphedFunction
    with pytest.raises(TypeError, match="cuda tensors"):
        GraphedFunction(lambda a: a, torch.zeros(4))
    with pytest.raises(TypeError, match="cuda tensors"):
        GraphedFunction(lambda: None)
    with pytest.raises(ValueError, match="warmup"):
        GraphedFunction(lambda a: a, torch.zeros(4), warmup=0)
