"""numpy restatement of the reference's mask / permutation preprocessing.

Test infrastructure only (see ``oracle/__init__.py``).  Every function cites
the reference lines it restates.  Permutation convention of the reference
(``utils.py:163-164``, ``main.py:27-28``): ``perm[i]`` is the OLD index that
moves to NEW position ``i``.
"""

from __future__ import annotations

import numpy as np


def blockmask_from_coords(rows_idx, cols_idx, seq_len, block_size, batch_size=1, nheads=1):
    """Token (row, col) coordinates -> bool block mask ``[B, H, nb, nb]``.

    Restates ``generate_blockmask_from_mtx_coords`` (``utils.py:51-84``):
    ``nb = ceil(seq_len / block)`` (``:66-67``), coordinates map to
    ``row // block, col // block`` (``:71-72``), block indices outside
    ``[0, nb)`` are dropped (``:75-77``; the test is on the block index, so a
    token index >= seq_len whose block is < nb is kept), and the same mask is
    written for every (b, h) (``:80-82``).
    """
    rows_idx = np.asarray(rows_idx, dtype=np.int64)
    cols_idx = np.asarray(cols_idx, dtype=np.int64)
    nb = (seq_len + block_size - 1) // block_size
    rb = rows_idx // block_size
    cb = cols_idx // block_size
    valid = (rb < nb) & (cb < nb)
    m = np.zeros((nb, nb), dtype=bool)
    m[rb[valid], cb[valid]] = True
    return np.broadcast_to(m, (batch_size, nheads, nb, nb)).copy()


def inverse_permutation(perm):
    """``inv[perm[i]] = i`` (``utils.py:253-254`` and ``:283-284``)."""
    perm = np.asarray(perm, dtype=np.int64)
    inv = np.empty_like(perm)
    inv[perm] = np.arange(perm.shape[0], dtype=np.int64)
    return inv


def is_permutation(perm, n=None):
    """The validity rules of ``read_reordering_file_to_tensor``
    (``utils.py:222-231``): values in ``[0, n)`` and no duplicates."""
    perm = np.asarray(perm, dtype=np.int64)
    n = perm.shape[0] if n is None else n
    if perm.shape[0] != n:
        return False
    if n == 0:
        return True
    if perm.min() < 0 or perm.max() >= n:
        return False
    return np.unique(perm).shape[0] == n


def update_idx_perm(idx, perm):
    """Old token index -> new token index: ``inv_perm[idx]``
    (``update_idx_perm``, ``utils.py:236-258``)."""
    return inverse_permutation(perm)[np.asarray(idx, dtype=np.int64)]


def apply_reordering(x, perm, axis):
    """``x_new[..., i, ...] = x[..., perm[i], ...]`` along ``axis``
    (``apply_reordering``, ``utils.py:260-266``; the ``torch.gather`` form at
    ``BlockSparseTriton_Naive.py:89-97``)."""
    return np.take(np.asarray(x), np.asarray(perm, dtype=np.int64), axis=axis)


def reverse_reordering(x, perm, axis):
    """``out[..., perm[i], ...] = x[..., i, ...]`` along ``axis``
    (``reverse_reordering``, ``utils.py:269-288``; the ``scatter_`` form at
    ``BlockSparseTriton_Naive.py:158-161``)."""
    return np.take(np.asarray(x), inverse_permutation(perm), axis=axis)


def tile_csr(block_mask, block):
    """Per-tile list of kept key blocks, the layout the CUDA kernels consume.

    ``block_mask``: bool ``[S, nb, nb]`` (one slice per distinct mask).  A
    tile is 128 query rows: one block row for ``block == 128``, the block rows
    ``2t`` and ``2t + 1`` for ``block == 64``.  For each tile the kept key
    blocks are listed in ascending order -- the order in which the reference
    scans them (``triton_kernels/BlockSparse_Naive.py:25-32``) -- as
    ``(flags << 24) | key_block`` where bit 0 of ``flags`` says the first
    block row of the tile keeps the key block and bit 1 the second.

    Returns ``(tile_ptr int32[S*T + 1], tile_col int32[nnz])``.
    """
    block_mask = np.asarray(block_mask, dtype=bool)
    S, nb, nb2 = block_mask.shape
    assert nb == nb2
    rows_per_tile = 128 // block
    T = (nb + rows_per_tile - 1) // rows_per_tile
    ptr = [0]
    cols = []
    for s in range(S):
        for t in range(T):
            flags = np.zeros(nb, dtype=np.int64)
            for r in range(rows_per_tile):
                br = t * rows_per_tile + r
                if br < nb:
                    flags |= block_mask[s, br].astype(np.int64) << r
            if rows_per_tile == 1:
                flags = np.where(flags != 0, 3, 0)
            kept = np.nonzero(flags)[0]
            cols.extend(((flags[kept] << 24) | kept).tolist())
            ptr.append(len(cols))
    return np.asarray(ptr, dtype=np.int32), np.asarray(cols, dtype=np.int32)
