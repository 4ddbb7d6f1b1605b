"""ctypes binding of libfxb200.so (the C ABI in include/fxb200.h).

Replaces the reference's hiprtc/ctypes loader, ml/fxgpu/hip_kernel.py:50-145
(compile_kernel / compile_module / launch): instead of compiling kernel source
at run time and launching by hand, the ops call plain C functions of a library
built ahead of time for sm_100a. Error behaviour mirrors the reference's `_chk`
(hip_kernel.py:45-47): a failing call raises RuntimeError carrying the
library's message. There is no fallback: if the library is missing or fails to
load, every op raises.
"""
import ctypes
import os
import threading

import torch

_PKG_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.environ.get("FXB200_LIB", os.path.join(_PKG_ROOT, "lib", "libfxb200.so"))

FXB_OK = 0
DTYPE_CODE = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}

EPI_STORE, EPI_RESIDUAL, EPI_GELU, EPI_DGELU = 0, 1, 2, 3
EPI_BIAS, EPI_BIAS_GELU, EPI_BIAS_SILU, EPI_ACCUM_F32, EPI_DSILU = 4, 5, 6, 7, 8
EPI_GELU_DERIV, EPI_MUL = 9, 10

_vp = ctypes.c_void_p
_i32 = ctypes.c_int32
_i64 = ctypes.c_int64
_f32 = ctypes.c_float


class GemmArgs(ctypes.Structure):
    """Mirror of fxb_gemm_args."""
    _fields_ = [
        ("dtype", _i32), ("M", _i32), ("N", _i32), ("K", _i32),
        ("A", _vp), ("lda", _i64), ("a_trans", _i32),
        ("B", _vp), ("ldb", _i64), ("b_trans", _i32),
        ("C", _vp), ("ldc", _i64), ("c_dtype", _i32),
        ("epilogue", _i32), ("alpha", _f32),
        ("R", _vp), ("ldr", _i64),
        ("Z", _vp), ("ldz", _i64),
        ("bias", _vp),
        ("workspace", _vp), ("workspace_bytes", _i64),
    ]


class AttnArgs(ctypes.Structure):
    """Mirror of fxb_attn_args (the reference's _AttnArgs, attention.py:22-38,
    with explicit dtype, head dim and output strides)."""
    _fields_ = [
        ("dtype", _i32), ("B", _i32), ("T", _i32), ("H", _i32), ("D", _i32),
        ("scale", _f32), ("causal", _i32),
        ("q", _vp), ("q_sb", _i64), ("q_st", _i64), ("q_sh", _i64),
        ("k", _vp), ("k_sb", _i64), ("k_st", _i64), ("k_sh", _i64),
        ("v", _vp), ("v_sb", _i64), ("v_st", _i64), ("v_sh", _i64),
        ("o", _vp), ("o_sb", _i64), ("o_st", _i64), ("o_sh", _i64),
        ("lse", _vp),
        ("dout", _vp), ("do_sb", _i64), ("do_st", _i64), ("do_sh", _i64),
        ("dq", _vp), ("dq_sb", _i64), ("dq_st", _i64), ("dq_sh", _i64),
        ("dk", _vp), ("dk_sb", _i64), ("dk_st", _i64), ("dk_sh", _i64),
        ("dv", _vp), ("dv_sb", _i64), ("dv_st", _i64), ("dv_sh", _i64),
        ("workspace", _vp),
    ]


# name -> (restype, argtypes); every symbol declared in include/fxb200.h
SIGNATURES = {
    "fxb_version": (ctypes.c_int, []),
    "fxb_last_error": (ctypes.c_char_p, []),
    "fxb_device_error": (ctypes.c_int, [ctypes.POINTER(_i32), _i32]),
    "fxb_num_sms": (ctypes.c_int, [ctypes.POINTER(_i32)]),
    "fxb_abi_struct_size": (ctypes.c_size_t, [_i32]),
    "fxb_launch_count": (ctypes.c_uint64, []),
    "fxb_rmsnorm_fwd": (ctypes.c_int, [_i32, _vp, _vp, _vp, _vp, _i64, _i32, _f32, _vp]),
    "fxb_rmsnorm_bwd_workspace": (ctypes.c_size_t, [_i64, _i32]),
    "fxb_rmsnorm_bwd": (ctypes.c_int, [_i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32, _i32,
                                       _vp, _i64, _i32, _vp]),
    "fxb_rmsnorm_bwd_static_max_bytes": (ctypes.c_size_t, []),
    "fxb_rmsnorm_bwd_static": (ctypes.c_int, [_i32, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i32,
                                              _i32, _i64, _i32, _vp]),
    "fxb_ce_fwd_grad": (ctypes.c_int, [_i32, _vp, _i64, _vp, _vp, _vp, _vp, _i64, _i32,
                                       _i64, _vp]),
    "fxb_adamw_sumsq": (ctypes.c_int, [_i32, _vp, _i64, _vp, _vp, _vp]),
    "fxb_adamw_sumsq_ws_bytes": (ctypes.c_size_t, []),
    "fxb_adamw_sumsq_det": (ctypes.c_int, [_i32, _vp, _i64, _vp, _vp, _vp, _vp]),
    "fxb_adamw_final": (ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _f32, _vp]),
    "fxb_adamw_update": (ctypes.c_int, [_i32, _i32, _vp, _vp, _vp, _vp, _vp, _i64, _vp, _vp,
                                        _i32, _vp, _vp, _vp, _vp, _f32, _vp, _f32, _f32,
                                        _f32, _f32, _vp]),
    "fxb_gemm": (ctypes.c_int, [ctypes.POINTER(GemmArgs), _vp]),
    "fxb_gemm_workspace_size": (ctypes.c_size_t, []),
    "fxb_gemm_plan": (ctypes.c_int, [_i32, _i32, _i32, _i32, ctypes.POINTER(_i32),
                                     ctypes.POINTER(_i32), ctypes.POINTER(_i32)]),
    "fxb_linear_ce_loss_workspace": (ctypes.c_size_t, [_i64, _i32]),
    "fxb_linear_ce_loss": (ctypes.c_int, [_i32, _vp, _i64, _vp, _i64, _vp, _vp, _vp, _i64, _i32, _i32,
                                          _i64, _vp]),
    "fxb_attn_fwd": (ctypes.c_int, [ctypes.POINTER(AttnArgs), _vp]),
    "fxb_attn_bwd_workspace": (ctypes.c_size_t, [_i32, _i32, _i32, _i32]),
    "fxb_attn_bwd": (ctypes.c_int, [ctypes.POINTER(AttnArgs), _vp]),
    "fxb_embedding_fwd": (ctypes.c_int, [_i32, _vp, _vp, _vp, _vp, _i64, _i64, _i32, _i64, _vp]),
    "fxb_embedding_bwd": (ctypes.c_int, [_i32, _vp, _vp, _vp, _vp, _i64, _i64, _i32, _i64, _vp]),
    "fxb_axpy": (ctypes.c_int, [_i32, _vp, _i32, _vp, _vp, _i32, _i64, _vp]),
    "fxb_gather_windows": (ctypes.c_int, [_i32, _vp, _i64, _i32, _vp, _i32, _i32, _vp, _vp]),
    "fxb_colsum": (ctypes.c_int, [_i32, _vp, _i64, _i32, _vp, _i32, _vp]),
}

_LIB = None
_LOCK = threading.Lock()


def load():
    """Load (once) and return the CDLL; raises if the library is missing."""
    global _LIB
    if _LIB is not None:
        return _LIB
    with _LOCK:
        if _LIB is None:
            if not os.path.exists(LIB_PATH):
                raise RuntimeError(
                    f"libfxb200.so not found at {LIB_PATH}: build it with "
                    f"`python -m fxb200.build` (there is no CPU fallback)")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _LIB = lib
    return _LIB


def last_error():
    return load().fxb_last_error().decode(errors="replace")


def check(rc, what):
    if rc != FXB_OK:
        raise RuntimeError(f"{what} failed: fxb error {rc}: {last_error()}")


def call(name, *args):
    """Call a C-ABI function and raise RuntimeError on a non-zero status."""
    check(getattr(load(), name)(*args), name)


def stream_ptr(device=None):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else ctypes.c_void_p(0)


def dtype_code(dt):
    try:
        return DTYPE_CODE[dt]
    except KeyError:
        raise TypeError(f"unsupported dtype {dt}") from None


def gemm_plan(M, N, K, epilogue=EPI_STORE):
    """(pair, tile_n, splits) that fxb_gemm would use for this problem."""
    a, b, c = _i32(), _i32(), _i32()
    check(load().fxb_gemm_plan(M, N, K, epilogue, ctypes.byref(a), ctypes.byref(b),
                               ctypes.byref(c)), "fxb_gemm_plan")
    return bool(a.value), b.value, c.value


def launch_count():
    """Kernels launched by libfxb200 so far in this process."""
    return int(load().fxb_launch_count())


def device_error(clear=True):
    """Device error word (bounded waits that expired); synchronises."""
    v = _i32(0)
    check(load().fxb_device_error(ctypes.byref(v), 1 if clear else 0), "fxb_device_error")
    return v.value


# bits of the device error word (csrc/common.cuh)
DERR_NAMES = {1: "gemm (tensor-core pipeline or tail-split wait)", 2: "attention pipeline",
              4: "gather pipeline", 8: "cross-entropy row copy"}
DERR_GEMM_WAIT = 1

# called with the word when a check finds it non-zero, before raising
# (fxb200.ops registers the reset of its GEMM workspaces' arrival counters)
_ON_DEVICE_ERROR = []


def raise_on_device_error(where=""):
    """Read (and clear) the device error word; raise RuntimeError if a kernel's
    bounded wait expired since the last check. A training loop calls this at
    its existing host synchronisation points: results computed after an
    expired wait are not trustworthy (the kernel gave up and returned)."""
    code = device_error(clear=True)
    if code:
        for fn in _ON_DEVICE_ERROR:
            fn(code)
        what = ", ".join(n for b, n in DERR_NAMES.items() if code & b) or "unknown"
        raise RuntimeError(f"libfxb200: a kernel's bounded wait expired{' ' + where if where else ''} "
                           f"(device error word {code}: {what}); the step's results are invalid")
