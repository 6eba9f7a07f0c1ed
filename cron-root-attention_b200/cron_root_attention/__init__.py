"""Cron Root Attention on B200: causal 3-phase sqrt(N) sparse attention.

Same public names as the reference package's ``cron_root_attention/__init__.py``
(lines 78-222); every op runs in libcra's hand-written sm_100a kernels.
"""
__version__ = "0.1.0"

import torch

from .core import (GPU_SM_MAP, CronRootAttentionV14Function, check_device_errors, cron_root_attention,
                   cron_root_attention_v14, cron_root_attention_varlen, get_num_sms, warmup_varlen_shapes)
from .hybrid import CronRootAttentionHybrid, cron_root_attention_hybrid
from .module import CronRootAttention, CronRootMultiheadAttention


def calibrate(H: int = 8, D: int = 64, dtype=None, S: int = 4096, verbose: bool = True) -> dict:
    """Reference __init__.py:84-180 tunes Triton (num_warps, num_stages).  The
    B200 kernels have fixed, compiled tile shapes, so there is nothing to
    tune; this runs one forward+backward at (H, D, S) to warm the library and
    returns the fixed configuration."""
    dtype = dtype or torch.float16
    dev = torch.device("cuda", torch.cuda.current_device())
    q = torch.randn(1, H, S, D, device=dev, dtype=dtype, requires_grad=True)
    k = torch.randn(1, H, S, D, device=dev, dtype=dtype, requires_grad=True)
    v = torch.randn(1, H, S, D, device=dev, dtype=dtype, requires_grad=True)
    cron_root_attention_v14(q, k, v).sum().backward()
    torch.cuda.synchronize(dev)
    cfg = {"fwd": (8, 1), "bwd": (8, 1)}  # (warps per CTA, CTAs per SM) of the compiled kernels
    if verbose:
        print(f"  H={H} D={D}: fixed sm_100a tiles {cfg}")
    return cfg


def get_gpu_info() -> dict:
    """Reference __init__.py:183-201."""
    if not torch.cuda.is_available():
        return {"gpu_name": "No GPU", "sm_count": 0, "is_known_gpu": False}
    name = torch.cuda.get_device_name()
    return {"gpu_name": name, "sm_count": get_num_sms(),
            "is_known_gpu": name in GPU_SM_MAP or any(n in name for n in GPU_SM_MAP)}


__all__ = [
    "cron_root_attention",
    "cron_root_attention_v14",
    "cron_root_attention_varlen",
    "warmup_varlen_shapes",
    "CronRootAttention",
    "CronRootMultiheadAttention",
    "cron_root_attention_hybrid",
    "CronRootAttentionHybrid",
    "calibrate",
    "get_num_sms",
    "get_gpu_info",
    "GPU_SM_MAP",
    "__version__",
]
