"""Small helpers that turn torch tensors into C-ABI arguments."""

from __future__ import annotations

import torch


def ptr(t: torch.Tensor | None) -> int | None:
    """Device address of a tensor for a `void*` argument (None = NULL)."""
    return None if t is None else t.data_ptr()


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def stream_of(t: torch.Tensor) -> int:
    """The current CUDA stream of the tensor's device, as a `cudaStream_t` value."""
    if _raw_stream is not None:
        return _raw_stream(t.get_device())
    return torch.cuda.current_stream(t.device).cuda_stream


def require_cuda(name: str, t: torch.Tensor, dtype: torch.dtype, ndim: int | None = None,
                 align: int = 16) -> None:
    """Check device, dtype, rank, contiguity and alignment of a kernel operand."""
    # One combined test for the common case; the checks below name what is wrong.
    if (type(t) is torch.Tensor and t.is_cuda and t.dtype == dtype
            and (ndim is None or t.dim() == ndim) and t.is_contiguous()
            and t.data_ptr() % align == 0):
        return
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (the product path has no CPU fallback)")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if ndim is not None and t.dim() != ndim:
        raise ValueError(f"{name} must have {ndim} dims, got shape {tuple(t.shape)}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if t.numel() and t.data_ptr() % align:
        raise ValueError(f"{name} must be {align}-byte aligned")
