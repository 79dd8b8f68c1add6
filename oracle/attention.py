"""numpy restatement of the reference's block-sparse attention forward.

Test infrastructure only (see ``oracle/__init__.py``).

* :func:`dense_masked_attention` is the mathematical definition in float64:
  ``O = softmax(mask_tok * (Q K^T * sm_scale), -inf elsewhere) V`` with rows
  that keep no key giving ``O = 0`` and ``lse = -inf`` (the reference's empty
  rows: ``l_i`` starts at 1 and ``acc`` at 0, ``BlockSparse_Naive.py:91-93,
  119-125``).  The LSE is returned in the reference's log2 units
  (``M = m_i + log2(l_i)``, ``BlockSparse_Naive.py:119``).
* :func:`block_sparse_online` ports the reference's per-query-block loop
  (``triton_kernels/BlockSparse_Naive.py:5-125``) to float32 numpy: it visits
  only kept key blocks in ascending order and applies the same online
  softmax in base 2, rounding P to the input's 16-bit type before the PV
  product as the Triton kernel does (``p.to(dtype)``, ``:54``).
  :func:`block_sparse_online_batched` applies the same per-row update
  sequence batched over query blocks (large GEMMs); it is the timed CPU
  baseline.
* :func:`reordered_attention` is the "with reordering" pipeline of the
  reference runners (``BlockSparseTriton_Naive.py:129-161``): gather Q by the
  row permutation and K/V by the column permutation, attend with the mask in
  the new order, scatter O back by the row permutation.
"""

from __future__ import annotations

import math
from concurrent.futures import ThreadPoolExecutor

import numpy as np

from .preprocess import apply_reordering, reverse_reordering

LOG2E = 1.4426950408889634  # the constant of BlockSparse_Naive.py:96


def _mask_slice(block_mask, b, h):
    Bm, Hm = block_mask.shape[:2]
    return block_mask[0 if Bm == 1 else b, 0 if Hm == 1 else h]


def token_mask(block_mask_2d, block, n):
    """Expand a ``[nb, nb]`` block mask to ``[n, n]`` tokens."""
    m = np.repeat(np.repeat(np.asarray(block_mask_2d, bool), block, 0), block, 1)
    return m[:n, :n]


def dense_masked_attention(q, k, v, block_mask, block, sm_scale=None, row_chunk=1024):
    """float64 dense masked softmax attention.  q, k, v: ``[B, H, N, D]``;
    block_mask: bool ``[1|B, 1|H, nb, nb]``.  Returns ``(o float64, lse_log2
    float64 [B, H, N])``."""
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    block_mask = np.asarray(block_mask, dtype=bool)
    B, H, N, D = q.shape
    scale = 1.0 / math.sqrt(D) if sm_scale is None else float(sm_scale)
    o = np.zeros((B, H, N, D), dtype=np.float64)
    lse = np.full((B, H, N), -np.inf, dtype=np.float64)
    for b in range(B):
        for h in range(H):
            tm = token_mask(_mask_slice(block_mask, b, h), block, N)
            for r0 in range(0, N, row_chunk):
                r1 = min(N, r0 + row_chunk)
                s = (q[b, h, r0:r1] @ k[b, h].T) * scale
                mk = tm[r0:r1]
                s = np.where(mk, s, -np.inf)
                mx = s.max(axis=1, keepdims=True)
                alive = np.isfinite(mx[:, 0])
                mx = np.where(np.isfinite(mx), mx, 0.0)
                p = np.where(mk, np.exp(s - mx), 0.0)
                l = p.sum(axis=1, keepdims=True)
                safe_l = np.where(l > 0, l, 1.0)
                o[b, h, r0:r1] = np.where(alive[:, None], (p @ v[b, h]) / safe_l, 0.0)
                lse[b, h, r0:r1] = np.where(alive, (mx[:, 0] + np.log(safe_l[:, 0])) * LOG2E, -np.inf)
    return o, lse


def _round_to(x, dtype_name):
    """Round float32 values to a 16-bit float type and back (the Triton
    kernel's ``p.to(dtype)`` before the PV dot)."""
    if dtype_name == "float16":
        return x.astype(np.float16).astype(np.float32)
    if dtype_name == "bfloat16":
        u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
        rounded = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)
        return rounded.view(np.float32)
    return x


def _query_block(qb, kh, vh, kept, block, qk_scale, p_dtype):
    """One query block of ``_attn_fwd_block_sparse`` (BlockSparse_Naive.py:68-125)."""
    bm, d = qb.shape
    acc = np.zeros((bm, d), dtype=np.float32)
    m_i = np.full((bm,), -np.inf, dtype=np.float32)
    l_i = np.ones((bm,), dtype=np.float32)
    for j in kept:  # ascending key blocks, masked blocks skipped (:25-32)
        kb = kh[j * block:(j + 1) * block]
        vb = vh[j * block:(j + 1) * block]
        qk = qb @ kb.T                                        # :39
        m_ij = np.maximum(m_i, qk.max(axis=1) * qk_scale)     # :40
        p = np.exp2(qk * qk_scale - m_ij[:, None])            # :41-42
        alpha = np.exp2(m_i - m_ij)                           # :44
        l_ij = p.sum(axis=1)                                  # :45
        acc = acc * alpha[:, None]                            # :47
        acc = acc + _round_to(p, p_dtype) @ vb                # :54-56
        l_i = l_i * alpha + l_ij                              # :59
        m_i = m_ij                                            # :60
    with np.errstate(divide="ignore"):
        m_out = m_i + np.log2(l_i)                            # :119
    return acc / l_i[:, None], m_out                          # :120


def _head_by_key_blocks(qh, kh, vh, mask2d, block, qk_scale, p_dtype, query_blocks=None):
    """The same per-row update sequence as :func:`_query_block`, batched: for
    each key block j (ascending), every query block that keeps j is updated
    at once, so each step is one large GEMM.  Each row still sees its kept
    key blocks in ascending order with the reference's update rule."""
    n, d = qh.shape
    nb = mask2d.shape[0]
    sel = np.zeros(nb, dtype=bool)
    sel[np.arange(nb) if query_blocks is None else np.asarray(list(query_blocks), dtype=np.int64)] = True
    acc = np.zeros((n, d), dtype=np.float32)
    m_i = np.full((n,), -np.inf, dtype=np.float32)
    l_i = np.ones((n,), dtype=np.float32)
    offs = np.arange(block)
    for j in range(nb):
        rb = np.nonzero(mask2d[:, j] & sel)[0]
        if rb.size == 0:
            continue
        idx = (rb[:, None] * block + offs[None, :]).ravel()
        idx = idx[idx < n]
        kb = kh[j * block:(j + 1) * block]
        vb = vh[j * block:(j + 1) * block]
        qk = qh[idx] @ kb.T
        mi = m_i[idx]
        m_ij = np.maximum(mi, qk.max(axis=1) * qk_scale)
        p = np.exp2(qk * qk_scale - m_ij[:, None])
        alpha = np.exp2(mi - m_ij)
        acc[idx] = acc[idx] * alpha[:, None] + _round_to(p, p_dtype) @ vb
        l_i[idx] = l_i[idx] * alpha + p.sum(axis=1)
        m_i[idx] = m_ij
    with np.errstate(divide="ignore"):
        return acc / l_i[:, None], m_i + np.log2(l_i)


def block_sparse_online_batched(q, k, v, block_mask, block, sm_scale=None, p_dtype=None, heads=None,
                                query_blocks=None):
    """:func:`block_sparse_online` with the key-block batching of
    :func:`_head_by_key_blocks` (large GEMMs that a threaded BLAS spreads over
    the host cores).  Same outputs up to float32 rounding order."""
    qf = np.asarray(q, dtype=np.float32)
    kf = np.asarray(k, dtype=np.float32)
    vf = np.asarray(v, dtype=np.float32)
    block_mask = np.asarray(block_mask, dtype=bool)
    B, H, N, D = qf.shape
    scale = 1.0 / math.sqrt(D) if sm_scale is None else float(sm_scale)
    qk_scale = np.float32(scale * LOG2E)
    o = np.zeros((B, H, N, D), dtype=np.float32)
    M = np.full((B, H, N), -np.inf, dtype=np.float32)
    for u in (range(B * H) if heads is None else heads):
        b, h = divmod(u, H)
        ob, mb = _head_by_key_blocks(qf[b, h], kf[b, h], vf[b, h], _mask_slice(block_mask, b, h), block,
                                     qk_scale, p_dtype, query_blocks)
        o[b, h], M[b, h] = ob, mb
    return o, M


def block_sparse_online(q, k, v, block_mask, block, sm_scale=None, p_dtype=None,
                        heads=None, query_blocks=None, threads=1):
    """float32 port of the reference's block loop.

    q, k, v: ``[B, H, N, D]`` (any float dtype; computed in float32).
    ``p_dtype``: ``"float16"`` / ``"bfloat16"`` to round P like the GPU
    kernels, ``None`` for no rounding.  ``heads``: optional list of flattened
    ``b * H + h`` units to compute (others are left zero); ``query_blocks``:
    optional list of query-block indices.  ``threads``: worker threads.
    Returns ``(o float32, M float32)``.
    """
    qf = np.asarray(q, dtype=np.float32)
    kf = np.asarray(k, dtype=np.float32)
    vf = np.asarray(v, dtype=np.float32)
    block_mask = np.asarray(block_mask, dtype=bool)
    B, H, N, D = qf.shape
    nb = (N + block - 1) // block
    scale = 1.0 / math.sqrt(D) if sm_scale is None else float(sm_scale)
    qk_scale = np.float32(scale * LOG2E)
    o = np.zeros((B, H, N, D), dtype=np.float32)
    M = np.full((B, H, N), -np.inf, dtype=np.float32)
    units = list(range(B * H)) if heads is None else list(heads)
    qblocks = list(range(nb)) if query_blocks is None else list(query_blocks)
    jobs = []
    for u in units:
        b, h = divmod(u, H)
        ms = _mask_slice(block_mask, b, h)
        for mb in qblocks:
            jobs.append((b, h, mb, np.nonzero(ms[mb])[0]))

    def run(job):
        b, h, mb, kept = job
        r0, r1 = mb * block, min(N, (mb + 1) * block)
        ob, mo = _query_block(qf[b, h, r0:r1], kf[b, h], vf[b, h], kept, block, qk_scale, p_dtype)
        o[b, h, r0:r1] = ob
        M[b, h, r0:r1] = mo

    if threads <= 1:
        for job in jobs:
            run(job)
    else:
        with ThreadPoolExecutor(max_workers=threads) as ex:
            list(ex.map(run, jobs))
    return o, M


def reordered_attention(q, k, v, block_mask, block, q_perm=None, kv_perm=None, sm_scale=None):
    """The runners' "with reordering" semantics (``BlockSparseTriton_Naive.py:
    129-161``) on the float64 dense definition.  ``block_mask`` is in the NEW
    (permuted) order.  Returns ``(o, lse)`` in the ORIGINAL row order."""
    qn = apply_reordering(q, q_perm, 2) if q_perm is not None else np.asarray(q)
    kn = apply_reordering(k, kv_perm, 2) if kv_perm is not None else np.asarray(k)
    vn = apply_reordering(v, kv_perm, 2) if kv_perm is not None else np.asarray(v)
    o, lse = dense_masked_attention(qn, kn, vn, block_mask, block, sm_scale)
    if q_perm is not None:
        o = reverse_reordering(o, q_perm, 2)
        lse = reverse_reordering(lse, q_perm, 2)
    return o, lse


def effective_flops(block_mask, block, B, H, D):
    """Algorithmic flops on kept blocks: ``4 * block^2 * D * nnz`` summed over
    (b, h) (two GEMMs, 2 flops per MAC)."""
    block_mask = np.asarray(block_mask, dtype=bool)
    Bm, Hm = block_mask.shape[:2]
    per_slice = block_mask.reshape(Bm, Hm, -1).sum(axis=2)
    nnz = int(np.broadcast_to(per_slice, (B, H)).sum())
    return 4.0 * block * block * D * nnz, nnz
