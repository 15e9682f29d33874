"""Device helpers of the reference API (src/rotalabs_accel/utils/device.py),
kept so code written against it imports unchanged."""

from __future__ import annotations

from typing import Any, Dict, Optional

import torch


def is_cuda_available() -> bool:
    return torch.cuda.is_available()


def is_triton_available() -> bool:
    """Whether Triton is importable.  Nothing in this package uses it."""
    try:
        import triton  # noqa: F401
        return True
    except ImportError:
        return False


def get_device(device: Optional[str] = None) -> torch.device:
    if device is not None:
        return torch.device(device)
    return torch.device("cuda" if is_cuda_available() else "cpu")


def get_device_properties(device: Optional[torch.device] = None) -> Dict[str, Any]:
    """Capability summary of a CUDA device (empty-ish dict on CPU-only hosts)."""
    if not is_cuda_available():
        return {"name": "cpu", "compute_capability": (0, 0), "total_memory": 0,
                "supports_fp16": False, "supports_bf16": False, "supports_fp8": False,
                "supports_sm100a": False, "multi_processor_count": 0}
    if device is None:
        device = torch.device("cuda", torch.cuda.current_device())
    p = torch.cuda.get_device_properties(device)
    cc = (p.major, p.minor)
    return {"name": p.name, "compute_capability": cc, "total_memory": p.total_memory,
            "supports_fp16": cc >= (5, 3), "supports_bf16": cc >= (8, 0), "supports_fp8": cc >= (8, 9),
            "supports_sm100a": cc == (10, 0), "multi_processor_count": p.multi_processor_count}
