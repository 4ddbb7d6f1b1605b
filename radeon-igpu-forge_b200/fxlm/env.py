"""fxlm.env: environment setup and GPU check (B200 build).

Mirrors ml/fxlm/env.py:11-48 (setup_lm_env before `import torch`,
require_gpu). The reference pins an AMD gfx1035 and disables TunableOp; here
the check is for an sm_100 (B200) device and no tuning layer is involved.
This module does not import torch at module level.
"""
import os


def require_gpu():
    """Return torch.device('cuda') after checking for an sm_100 GPU."""
    import torch

    if not torch.cuda.is_available():
        raise SystemExit("no GPU: torch.cuda.is_available() is False")
    major, minor = torch.cuda.get_device_capability(0)
    if major != 10:
        raise SystemExit(f"expected an sm_100 (B200) GPU, found sm_{major}{minor} "
                         f"({torch.cuda.get_device_name(0)})")
    return torch.device("cuda")


def setup_lm_env(tunable=False, tune_file=None):
    """Environment defaults for training (call before importing torch).

    `tunable` / `tune_file` are accepted for signature compatibility with the
    reference; the sm_100a kernels have no runtime tuning step.
    """
    os.environ.setdefault("CUDA_MODULE_LOADING", "LAZY")
    os.environ.setdefault("TORCH_NCCL_ASYNC_ERROR_HANDLING", "1")
    return None
