"""Synthetic token data used by the benchmarks and the training driver.

Zipf(s) token ids: p_k ∝ (k+1)^-s for k in [0, V), drawn i.i.d. with
numpy.random.default_rng(seed).choice, shape (B, T+1); inputs/targets are the
sequence and its shift by one, like the reference's get_batch
(ml/fxlm/train_lm.py:148-152). The same definition is restated independently
in the oracle and in the golden-fixture generator.
"""
import numpy as np
import torch


def zipf_tokens(V, B, T, seed, s=1.1):
    k = np.arange(V, dtype=np.float64)
    p = (k + 1.0) ** (-s)
    p /= p.sum()
    seq = np.random.default_rng(seed).choice(V, size=(B, T + 1), p=p)
    seq = torch.from_numpy(seq.astype(np.int64))
    return seq[:, :-1].contiguous(), seq[:, 1:].contiguous()
