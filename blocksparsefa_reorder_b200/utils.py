"""Reference-compatible preprocessing surface (mirrors the reference ``utils.py``).

The file readers are host-side parsers with the reference's behaviour and
error messages.  Everything that touches tensors runs on the GPU through the
C ABI: the block mask build (``bsa_blockmask_from_coords``), the
permutation inverse / index remap and the row gather / scatter
(``bsa_permute_rows``).
"""

from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path
from typing import Optional

import numpy as np
import torch

from . import _lib
from .api import _check_err, _require_cuda, _stream, inverse_permutation, permute_rows


@dataclass(frozen=True)
class Args:
    """The reference's run configuration (``utils.py:14-22``)."""

    matrix_mtx: Path
    block_size: int = 128
    head_dim: int = 128
    num_heads: int = 1
    row_reorder: Optional[Path] = None
    col_reorder: Optional[Path] = None
    mode: str = "B200"


def read_mtx(path: str):
    """Headerless coordinate pattern file -> ``(rows_idx, cols_idx, seq_len)``.

    Same format and behaviour as the reference (``utils.py:25-49``): the first
    line is ``rows cols nnz``; each following line is a 1-based ``row col``
    pair, returned 0-based as int64 numpy arrays; ``seq_len = rows``.
    """
    with open(path, "r") as f:
        first_line = f.readline()
        rows, _cols, _nnz = map(int, first_line.strip().split())
    coords = np.loadtxt(path, skiprows=1, dtype=int)
    if coords.ndim == 1:
        coords = coords.reshape(1, -1)
    return coords[:, 0] - 1, coords[:, 1] - 1, rows


def read_reordering_file_to_tensor(path, *, dtype: torch.dtype = torch.int64, device="cpu",
                                   zero_based: Optional[bool] = None) -> torch.Tensor:
    """Permutation file -> ``perm`` tensor (``utils.py:139-233``).

    Format: first non-comment line ``N``, then ``N`` indices, one per line;
    ``#`` comments and blank lines are skipped.  ``zero_based=None`` detects
    the base (0-based iff the minimum is 0).  Raises ``ValueError`` with the
    reference's messages for an empty file, a bad header, a negative N, a
    count mismatch, non-integers, out-of-range values and duplicates.
    ``perm[i]`` is the old index that moves to new position ``i``.
    """
    path = Path(path)
    lines = []
    with path.open("r", encoding="utf-8") as f:
        for line in f:
            s = line.strip()
            if not s or s.startswith("#"):
                continue
            lines.append(s)
    if not lines:
        raise ValueError(f"{path}: empty reordering file")
    try:
        n = int(lines[0])
    except ValueError as e:
        raise ValueError(f"{path}: first line must be an integer N") from e
    if n < 0:
        raise ValueError(f"{path}: N must be non-negative, got {n}")
    data = lines[1:]
    if len(data) != n:
        raise ValueError(f"{path}: expected {n} indices after first line, got {len(data)}")
    try:
        vals = np.array([int(x) for x in data], dtype=np.int64)
    except ValueError as e:
        raise ValueError(f"{path}: all indices must be integers") from e
    if n == 0:
        return torch.tensor(vals, dtype=dtype, device=device)
    minv, maxv = int(vals.min()), int(vals.max())
    if zero_based is None:
        zero_based = minv == 0
    if not zero_based:
        vals = vals - 1
        minv -= 1
        maxv -= 1
    if minv < 0:
        raise ValueError(f"{path}: indices contain negatives after base adjustment (min={minv})")
    if maxv >= n:
        raise ValueError(f"{path}: index out of range after base adjustment (max={maxv}, N={n})")
    if np.unique(vals).shape[0] != n:
        raise ValueError(f"{path}: indices are not a permutation (duplicates found)")
    return torch.tensor(vals, dtype=dtype, device=device)


def _as_cuda_i64(x, device) -> torch.Tensor:
    t = x if isinstance(x, torch.Tensor) else torch.as_tensor(np.asarray(x))
    return t.to(device=device, dtype=torch.int64).contiguous()


def generate_blockmask_from_mtx_coords(rows_idx, cols_idx, seq_len: int, block_size: int, batch_size: int = 1,
                                       nheads: int = 1, device="cuda", *, row_perm=None, col_perm=None,
                                       verbose: bool = True, check_errors: bool = True):
    """Token coordinates -> bool block mask ``[B, H, nb, nb]`` on the GPU.

    Same result as the reference (``utils.py:51-84``): ``nb = ceil(seq_len /
    block)``, kept block ``(row // block, col // block)``, blocks >= nb
    dropped, one mask for every (b, h); prints ``NNZ blocks`` like the
    reference when ``verbose``.  ``row_perm`` / ``col_perm`` (optional) fuse
    ``update_idx_perm`` (``utils.py:236-258``): coordinates are mapped to
    their new positions before blocking.  Returns ``(mask, seq_len)``.
    """
    dev = torch.device(device)
    if dev.type != "cuda":
        raise ValueError("the block mask is built on the GPU; pass a CUDA device")
    rows = _as_cuda_i64(rows_idx, dev)
    cols = _as_cuda_i64(cols_idx, dev)
    if rows.shape != cols.shape or rows.dim() != 1:
        raise ValueError("rows_idx and cols_idx must be 1-D of equal length")
    nb = (seq_len + block_size - 1) // block_size
    mask = torch.empty((batch_size, nheads, nb, nb), dtype=torch.bool, device=dev)
    rinv = inverse_permutation(_as_cuda_i64(row_perm, dev)) if row_perm is not None else None
    cinv = inverse_permutation(_as_cuda_i64(col_perm, dev)) if col_perm is not None else None
    err = torch.zeros(1, dtype=torch.int32, device=dev) if check_errors else None
    _lib.check(_lib.lib().bsa_blockmask_from_coords(
        rows.data_ptr(), cols.data_ptr(), rows.shape[0], seq_len, block_size, batch_size, nheads,
        rinv.data_ptr() if rinv is not None else None, cinv.data_ptr() if cinv is not None else None,
        mask.data_ptr(), err.data_ptr() if err is not None else None, _stream(dev)),
        "bsa_blockmask_from_coords")
    _check_err(err, "generate_blockmask_from_mtx_coords")
    if verbose:
        print(f"NNZ blocks: {mask.sum().item()}")
    return mask, seq_len


def update_idx_perm(idx, perm, device="cuda"):
    """Old token indices -> new indices, ``inv_perm[idx]`` (``utils.py:236-258``),
    computed on the GPU.  Returns numpy when ``idx`` is numpy, else a tensor."""
    dev = perm.device if isinstance(perm, torch.Tensor) and perm.is_cuda else torch.device(device)
    p = _as_cuda_i64(perm, dev)
    inv = inverse_permutation(p)
    x = _as_cuda_i64(idx, dev)
    out = torch.empty_like(x)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    _lib.check(_lib.lib().bsa_remap_indices(x.data_ptr(), x.shape[0], inv.data_ptr(), p.shape[0], out.data_ptr(),
                                            err.data_ptr(), _stream(dev)), "bsa_remap_indices")
    _check_err(err, "update_idx_perm")
    return out.cpu().numpy() if isinstance(idx, np.ndarray) else out


def apply_reordering(x: torch.Tensor, perm, dim: int = 0) -> torch.Tensor:
    """``x.index_select(dim, perm)`` with the GPU row-gather kernel
    (``utils.py:260-266``)."""
    _require_cuda(x, "x")
    return permute_rows(x, perm, dim, inverse=False)


def reverse_reordering(x: torch.Tensor, perm, dim: int = 0) -> torch.Tensor:
    """Undo :func:`apply_reordering`: ``out.select(dim, perm[i]) = x.select(dim, i)``
    (``utils.py:269-288``), as a GPU row scatter."""
    _require_cuda(x, "x")
    return permute_rows(x, perm, dim, inverse=True)


__all__ = ["Args", "read_mtx", "read_reordering_file_to_tensor", "generate_blockmask_from_mtx_coords",
           "update_idx_perm", "apply_reordering", "reverse_reordering"]
