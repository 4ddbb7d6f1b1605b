"""CPU: the C-ABI library loads, exports every symbol include/fxb200.h
declares, agrees with the ctypes struct layouts, and rejects bad arguments
with FXB_EINVAL + a message (no compute call needs a GPU here). Also the
Python wrappers' input validation (the reference's ValueError / TypeError
checks) fires before any kernel would run.
"""
import ctypes
import os
import re

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "fxb200.h")


def _declared_functions():
    with open(HEADER) as f:
        src = f.read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(fxb_[a-z0-9_]+)\s*\(", src)))


@pytest.fixture(scope="module")
def lib():
    from fxb200 import _lib
    return _lib.load()


def test_library_exports_every_declared_symbol(lib):
    names = _declared_functions()
    assert len(names) >= 20
    for n in names:
        assert hasattr(lib, n), f"{n} declared in include/fxb200.h but not exported"


def test_ctypes_signatures_cover_header():
    from fxb200 import _lib
    assert set(_declared_functions()) == set(_lib.SIGNATURES)


def test_struct_layouts_match(lib):
    from fxb200 import _lib
    assert lib.fxb_abi_struct_size(0) == ctypes.sizeof(_lib.GemmArgs)
    assert lib.fxb_abi_struct_size(1) == ctypes.sizeof(_lib.AttnArgs)
    assert lib.fxb_abi_struct_size(7) == 0


def test_version_and_counters(lib):
    from fxb200 import _lib
    assert lib.fxb_version() >= 100
    assert _lib.launch_count() >= 0


def test_einval_paths_without_gpu(lib):
    from fxb200 import _lib
    # RMSNorm: D not a multiple of 8
    rc = lib.fxb_rmsnorm_fwd(2, None, None, None, None, 4, 7, 1e-6, None)
    assert rc == -1 and "D=7" in _lib.last_error()
    # CE: ld < V
    rc = lib.fxb_ce_fwd_grad(2, ctypes.c_void_p(16), 4, ctypes.c_void_p(16), None,
                             ctypes.c_void_p(16), None, 3, 8, -100, None)
    assert rc == -1 and "ce" in _lib.last_error()
    # AdamW: n not a multiple of 8
    rc = lib.fxb_adamw_update(0, 2, None, None, None, None, None, 9, None, None, 1, None, None,
                              None, None, 1e-3, None, 0.9, 0.95, 1e-8, 0.1, None)
    assert rc == -1 and "multiple of 8" in _lib.last_error()
    # GEMM: N not a multiple of 8
    a = _lib.GemmArgs()
    a.dtype, a.M, a.N, a.K = 2, 16, 12, 16
    rc = lib.fxb_gemm(ctypes.byref(a), None)
    assert rc == -1 and "N=12" in _lib.last_error()
    # GEMM: unsupported operand dtype
    a.dtype, a.N = 7, 16
    assert lib.fxb_gemm(ctypes.byref(a), None) == -2
    # GEMM: fp32 (the parity-mode kernel) still needs its operands
    a.dtype = 0
    assert lib.fxb_gemm(ctypes.byref(a), None) == -1 and "NULL" in _lib.last_error()
    # attention: head_dim 96
    at = _lib.AttnArgs()
    at.dtype, at.B, at.T, at.H, at.D = 2, 1, 8, 1, 96
    assert lib.fxb_attn_fwd(ctypes.byref(at), None) == -1
    assert "head_dim 96" in _lib.last_error()
    # attention backward at head_dim 128: checked like head_dim 64 (dout missing here)
    at.D = 128
    at.q = at.k = at.v = at.o = 256
    at.q_sb = at.q_st = at.q_sh = at.k_sb = at.k_st = at.k_sh = 8
    at.v_sb = at.v_st = at.v_sh = at.o_sb = at.o_st = at.o_sh = 8
    at.lse = 256
    assert lib.fxb_attn_bwd(ctypes.byref(at), None) == -1
    assert "dout" in _lib.last_error()
    assert lib.fxb_attn_bwd_workspace(2, 10, 3, 64) == (60 + 60 * 64) * 4
    # head_dim 128: delta, then the transposed dQ accumulator (B*H, 128, T rounded up to 64)
    assert lib.fxb_attn_bwd_workspace(2, 10, 3, 128) == (60 + 6 * 128 * 64) * 4
    # loss-only linear cross entropy: D / V must be multiples of 8
    rc = lib.fxb_linear_ce_loss(2, None, 16, None, 16, None, None, None, 4, 12, 64, -100, None)
    assert rc == -1 and "D=12" in _lib.last_error()


def test_wrapper_validation_is_host_side():
    """The reference's argument checks (attention.py:57-79, norm.py:30-42,
    cross_entropy.py:62-74,152-167) raise before any kernel launch."""
    from fxlm.attention import flash_attention
    from fxlm.norm import rms_norm
    from fxlm.cross_entropy import fused_cross_entropy, linear_cross_entropy
    q = torch.zeros(1, 4, 1, 96, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="head_dim 96"):
        flash_attention(q, q, q)
    q = torch.zeros(1, 4, 1, 64, dtype=torch.bfloat16)
    with pytest.raises(TypeError, match="cuda"):
        flash_attention(q, q, q)
    with pytest.raises(TypeError):
        flash_attention(q.float(), q.float(), q.float())
    with pytest.raises(TypeError, match="cuda"):
        rms_norm(torch.zeros(2, 8), torch.ones(8))
    with pytest.raises(TypeError):
        fused_cross_entropy(torch.zeros(2, 8, dtype=torch.bfloat16), torch.zeros(2, dtype=torch.int32))
    x = torch.zeros(4, 8, dtype=torch.bfloat16, requires_grad=True)
    with pytest.raises(TypeError, match="cuda"):
        linear_cross_entropy(x, torch.zeros(16, 8, dtype=torch.bfloat16), torch.zeros(4, dtype=torch.int64))
    with pytest.raises(TypeError, match="share"):  # x and weight of different dtypes
        linear_cross_entropy(x.float(), torch.zeros(16, 8, dtype=torch.bfloat16),
                             torch.zeros(4, dtype=torch.int64))
    with pytest.raises(TypeError, match="bf16, fp16 or fp32"):
        linear_cross_entropy(x.double(), torch.zeros(16, 8, dtype=torch.float64),
                             torch.zeros(4, dtype=torch.int64))


def test_auto_chunk_bounds_logits_buffer():
    from fxlm.cross_entropy import _auto_chunk
    assert _auto_chunk(8192, 768, 32768) == 8192           # 512 MiB of bf16 logits
    c = _auto_chunk(65536, 768, 32768)
    assert c % 128 == 0 and c * 32768 * 2 <= (1 << 30)


def test_flat_adamw_requires_cuda():
    from fxlm.optim import FlatAdamW
    with pytest.raises(TypeError, match="cuda"):
        FlatAdamW(torch.nn.Linear(8, 8))
