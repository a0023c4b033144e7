"""Scale-factor layouts of the NVFP4 path.

Two layouts exist for the per-16-element E4M3 scales of an [R, K] operand:

* plain: row-major ``[R, K/16]`` bytes (the harness's ``sfa``/``sfb``);
* blocked: 128-row x 4-column blocks of 512 bytes, rows padded to a multiple of
  128 and columns to a multiple of 4 with zeros. Inside a block, byte
  ``i0*16 + i1*4 + j`` holds plain row ``i1*32 + i0`` and column ``j``. Blocks are
  ordered row-block-major: ``(mm * rest_k + kk) * 512``.

The blocked bytes are what ``to_blocked`` returns (REFERENCE_IMPL.md:19-42) and are
the storage order of the harness's ``(32, 4, rest_m, 4, rest_k, l)`` "reordered"
view (REFERENCE_IMPL.md:89-137), which is an allocation of shape
``(l, rest_m, rest_k, 32, 4, 4)`` permuted by ``(3, 4, 1, 5, 2, 0)``. The kernel
reads this layout directly: one 512-byte block is one ``tcgen05.cp 32x128b``.
"""
from __future__ import annotations

import torch

SF_VEC = 16
REORDER_PERMUTE = (3, 4, 1, 5, 2, 0)


def ceil_div(a: int, b: int) -> int:
    return (a + b - 1) // b


def blocked_sf_bytes(rows: int, sf_cols: int) -> int:
    """Bytes of the blocked layout for a plain [rows, sf_cols] scale matrix."""
    if rows <= 0 or sf_cols <= 0:
        return 0
    return ceil_div(rows, 128) * ceil_div(sf_cols, 4) * 512


def reordered_shape(rows: int, k: int, l: int = 1) -> tuple:
    """Shape of the harness's reordered scale view for an [rows, k] operand."""
    return (32, 4, ceil_div(rows, 128), 4, ceil_div(ceil_div(k, SF_VEC), 4), l)


def plain_to_blocked(plain: torch.Tensor) -> torch.Tensor:
    """Blocked bytes (flat uint8) of a plain [rows, sf_cols] scale matrix, on its device.

    Pure tensor permutation (pad, split into 128x4 blocks, interleave rows by 32).
    """
    if plain.dim() != 2:
        raise ValueError(f"expected a 2-D [rows, sf_cols] tensor, got shape {tuple(plain.shape)}")
    p = plain.view(torch.uint8) if plain.element_size() == 1 else plain
    if p.dtype != torch.uint8:
        raise ValueError(f"scale factors must be 1-byte values, got {plain.dtype}")
    rows, cols = p.shape
    rm, rk = ceil_div(rows, 128), ceil_div(cols, 4)
    padded = torch.zeros((rm * 128, rk * 4), dtype=torch.uint8, device=p.device)
    padded[:rows, :cols] = p
    # [mm, i1, i0, kk, j] -> [mm, kk, i0, i1, j]
    blocks = padded.view(rm, 4, 32, rk, 4).permute(0, 3, 2, 1, 4)
    return blocks.reshape(-1).contiguous()


def blocked_to_plain(blocked: torch.Tensor, rows: int, sf_cols: int) -> torch.Tensor:
    """Inverse of plain_to_blocked (drops the padding)."""
    rm, rk = ceil_div(rows, 128), ceil_div(sf_cols, 4)
    b = blocked.reshape(-1).view(torch.uint8)[: rm * rk * 512]
    plain = b.view(rm, rk, 32, 4, 4).permute(0, 3, 2, 1, 4).reshape(rm * 128, rk * 4)
    return plain[:rows, :sf_cols].contiguous()


def blocked_as_reordered(blocked: torch.Tensor, rows: int, k: int,
                         dtype: torch.dtype | None = torch.float8_e4m3fn) -> torch.Tensor:
    """View blocked bytes as the harness's 6-D ``(32, 4, rest_m, 4, rest_k, 1)`` tensor."""
    rm = ceil_div(rows, 128)
    rk = ceil_div(ceil_div(k, SF_VEC), 4)
    t = blocked.reshape(-1)[: rm * rk * 512]
    if dtype is not None:
        t = t.view(dtype)
    return t.view(1, rm, rk, 32, 4, 4).permute(*REORDER_PERMUTE)


def reordered_storage_ok(t: torch.Tensor, rows: int, k: int) -> bool:
    """True if `t` is a (32, 4, rest_m, 4, rest_k, 1) view whose storage is blocked order."""
    shape = reordered_shape(rows, k)
    if tuple(t.shape) != shape:
        return False
    _, _, rm, _, rk, _ = shape
    expect = (16, 4, rk * 512, 1, 512, rm * rk * 512)
    return all(st == ex or sz == 1 for st, ex, sz in zip(t.stride(), expect, t.shape))


def sf_to_blocked(plain: torch.Tensor, out: torch.Tensor | None = None,
                  stream: torch.cuda.Stream | None = None) -> torch.Tensor:
    """Convert plain scales to the blocked layout on the GPU (C ABI nvfp4_sf_to_blocked)."""
    from . import _native

    if not plain.is_cuda:
        raise ValueError("sf_to_blocked needs a CUDA tensor; use plain_to_blocked on the host")
    if plain.dim() != 2 or plain.element_size() != 1 or plain.stride(1) != 1:
        raise ValueError("plain scales must be a 2-D, 1-byte, row-major tensor")
    rows, cols = plain.shape
    nbytes = blocked_sf_bytes(rows, cols)
    if out is None:
        out = torch.empty(nbytes, dtype=torch.uint8, device=plain.device)
    if out.numel() * out.element_size() < nbytes:
        raise ValueError(f"output holds {out.numel() * out.element_size()} bytes, needs {nbytes}")
    s = stream or torch.cuda.current_stream(plain.device)
    with torch.cuda.device(plain.device):
        _native.sf_to_blocked_raw(plain.data_ptr(), out.data_ptr(), rows, cols, plain.stride(0),
                                  s.cuda_stream)
    return out
