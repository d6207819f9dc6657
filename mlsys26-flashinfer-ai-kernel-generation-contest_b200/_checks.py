"""Argument validation shared by the decode and prefill host entry points.

Errors are raised before anything is launched: ``TypeError`` for a wrong dtype
or a non-tensor, ``ValueError`` for a wrong shape, device or layout (the
flashinfer-bench harness maps either to RUNTIME_ERROR).
"""
from __future__ import annotations

import torch

HEAD_SIZE = 128


def tensor(name: str, x, dtype: torch.dtype, ndim: int, device: torch.device):
    if not isinstance(x, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor, got {type(x).__name__}")
    if x.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {x.dtype}")
    if x.dim() != ndim:
        raise ValueError(f"{name} must be {ndim}-D, got shape {tuple(x.shape)}")
    if x.device != device:
        raise ValueError(f"{name} is on {x.device}, expected {device}")
    if not x.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return x


def shape(name: str, x: torch.Tensor, expected) -> None:
    if tuple(x.shape) != tuple(expected):
        raise ValueError(f"{name} must have shape {tuple(expected)}, got {tuple(x.shape)}")


def cuda_device(q) -> torch.device:
    if not isinstance(q, torch.Tensor):
        raise TypeError(f"q must be a torch.Tensor, got {type(q).__name__}")
    if q.device.type != "cuda":
        raise ValueError(f"tensors must be on a CUDA device, got {q.device} "
                         "(there is no CPU implementation)")
    return q.device


def heads(hq: int, hk: int, hv: int, d: int) -> None:
    if d != HEAD_SIZE:
        raise ValueError(f"head_size must be {HEAD_SIZE}, got {d}")
    if hk != hq:
        raise ValueError(f"num_k_heads ({hk}) must equal num_q_heads ({hq})")
    if hq <= 0 or hv < hq or hv % hq != 0:
        raise ValueError(f"num_v_heads ({hv}) must be a positive multiple of num_q_heads ({hq})")


def scale_arg(scale) -> float:
    """None or 0.0 selects 1/sqrt(head_size) inside the kernels (passed as 0)."""
    if scale is None:
        return 0.0
    if isinstance(scale, torch.Tensor):
        if scale.numel() != 1:
            raise ValueError("scale must be a scalar")
        scale = scale.item()
    s = float(scale)
    if s < 0.0:
        raise ValueError(f"scale must be >= 0, got {s}")
    return s


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream
