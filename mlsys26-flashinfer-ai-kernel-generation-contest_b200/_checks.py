"""Argument validation shared by the decode and prefill host entry points.

Errors are raised before anything is launched: ``TypeError`` for a wrong dtype
or a non-tensor, ``ValueError`` for a wrong shape, device or layout (the
flashinfer-bench harness maps either to RUNTIME_ERROR).
"""
from __future__ import annotations

import torch

HEAD_SIZE = 128


def tensor(name: str, x, dtype: torch.dtype, ndim: int, device: torch.device,
           strided: bool = False):
    """Type, rank and device checks.  Without `strided` the tensor must be contiguous;
    with it any layout is accepted here (see `row_stride` / `rows_in` / `rows_out`)."""
    if not isinstance(x, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor, got {type(x).__name__}")
    if x.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {x.dtype}")
    if x.dim() != ndim:
        raise ValueError(f"{name} must be {ndim}-D, got shape {tuple(x.shape)}")
    if x.device != device:
        raise ValueError(f"{name} is on {x.device}, expected {device}")
    if not strided and not x.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    return x


def row_stride(x: torch.Tensor, align: int = 1):
    """Elements between consecutive rows (dim 0) of `x` when the dims after the first are
    dense (a token row of a fused projection, say), the rows do not overlap and the stride
    is a multiple of `align`; None otherwise."""
    inner = 1
    for d in range(x.dim() - 1, 0, -1):
        if x.shape[d] != 1 and x.stride(d) != inner:
            return None
        inner *= x.shape[d]
    if x.shape[0] <= 1:
        return inner
    rs = x.stride(0)
    return rs if (rs >= inner and rs % align == 0) else None


def rows_in(x: torch.Tensor, align: int = 1, ptr_align: int = 2):
    """(tensor, row stride) for a token-indexed input: strided rows whose stride is a
    multiple of `align` elements and whose first element is `ptr_align`-byte aligned are
    passed to the kernels as they are; anything else is first copied into a dense tensor
    on the device (freshly allocated, so aligned)."""
    rs = row_stride(x, align)
    if rs is None or x.data_ptr() % ptr_align != 0:
        x = x.clone(memory_format=torch.contiguous_format)
        rs = row_stride(x, align)
    return x, rs


def rows_out(x: torch.Tensor, align: int = 1, ptr_align: int = 2):
    """(target, row stride, copy_back) for a token-indexed output: strided rows (stride a
    multiple of `align`, first element `ptr_align`-byte aligned) are written in place; for
    anything else the kernels write a dense temporary that the caller copies into `x`
    afterwards (copy_back is True)."""
    rs = row_stride(x, align)
    if rs is not None and x.data_ptr() % ptr_align == 0:
        return x, rs, False
    t = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    return t, row_stride(t, align), True


def dense_or_copy(x, ptr_align: int = 4):
    """A contiguous, `ptr_align`-byte aligned tensor with x's values (x itself when it
    already is one)."""
    if x is None or (x.is_contiguous() and x.data_ptr() % ptr_align == 0):
        return x
    return x.clone(memory_format=torch.contiguous_format)


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
