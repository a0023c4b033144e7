"""NVFP4 activation quantiser: bf16/fp16 activations -> the GEMM's A operand.

``quantize(x, global_scale)`` returns packed e2m1 codes ``[rows, cols/2]`` (uint8, element
2i in the low nibble) and E4M3 scales per 16 elements in the 128x4-blocked layout that
:func:`grouped_gemm` (and ``custom_kernel``'s reordered scale view) consumes, computed by
one CUDA kernel (``nvfp4_quantize``). Two-level scaling: per 16-element block
``sf = E4M3(amax / (6 * s_g))`` and ``q = E2M1(x / (value(sf) * s_g))``, rounded to nearest
even and saturated, so ``x ~= value(q) * value(sf) * s_g``; the GEMM result must then be
multiplied by ``s_g`` (fold it into ``alpha``). :func:`global_scale_for` gives the usual
``s_g = amax(|x|) / (6 * 448)``.

The reference has no quantiser (its inputs arrive already quantised); this is the step
that produces them from a model's activations.
"""
from __future__ import annotations

import torch

from . import _native
from .layout import blocked_sf_bytes

_DTYPES = {torch.bfloat16: _native.DTYPE_BF16, torch.float16: _native.DTYPE_FP16}


def global_scale_for(x: torch.Tensor) -> float:
    """``amax(|x|) / (6 * 448)``: the per-tensor scale that keeps every block scale finite
    in E4M3 (a device reduction and one host read)."""
    amax = float(x.detach().abs().amax().float().item())
    return amax / (6.0 * 448.0) if amax > 0 else 1.0


def quantize(x: torch.Tensor, global_scale: float, packed: torch.Tensor | None = None,
             sf: torch.Tensor | None = None,
             stream: torch.cuda.Stream | None = None) -> tuple:
    """Quantise ``x`` [rows, cols] (bf16 or fp16, CUDA, unit stride along cols, cols % 64 == 0).

    Returns ``(packed, sf_blocked)``; pass preallocated ``packed`` ([rows, cols/2] uint8, row
    stride a multiple of 16 bytes) and ``sf`` (``blocked_sf_bytes(rows, cols // 16)`` uint8 bytes)
    to write in place.
    """
    if not isinstance(x, torch.Tensor) or not x.is_cuda:
        raise ValueError("x must be a CUDA tensor")
    if x.dtype not in _DTYPES:
        raise ValueError(f"x must be bfloat16 or float16, got {x.dtype}")
    if x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("x must be 2-D with unit stride along the last dimension")
    rows, cols = int(x.shape[0]), int(x.shape[1])
    if cols % 64 != 0 or cols == 0:
        raise ValueError(f"cols={cols} must be a positive multiple of 64")
    if not (global_scale > 0.0) or global_scale == float("inf"):
        raise ValueError("global_scale must be finite and > 0")
    if packed is None:
        packed = torch.empty((rows, cols // 2), dtype=torch.uint8, device=x.device)
    if sf is None:
        sf = torch.empty(blocked_sf_bytes(rows, cols // 16), dtype=torch.uint8, device=x.device)
    if packed.dtype != torch.uint8 or tuple(packed.shape) != (rows, cols // 2) or packed.stride(1) != 1:
        raise ValueError(f"packed must be uint8 [{rows}, {cols // 2}] with unit inner stride")
    if sf.dtype != torch.uint8 or sf.numel() < blocked_sf_bytes(rows, cols // 16) or not sf.is_contiguous():
        raise ValueError("sf must be a contiguous uint8 buffer of blocked_sf_bytes(rows, cols // 16)")
    s = stream or torch.cuda.current_stream(x.device)
    with torch.cuda.device(x.device):
        _native.quantize_raw(x.data_ptr(), rows, cols, x.stride(0), _DTYPES[x.dtype],
                             float(global_scale), packed.data_ptr(), packed.stride(0),
                             sf.data_ptr(), s.cuda_stream)
    return packed, sf
