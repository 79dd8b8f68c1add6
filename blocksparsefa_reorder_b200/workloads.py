"""Seeded synthetic workloads: block masks, token permutations and q, k, v.

The reference's experiment inputs (reordered ``.mtx`` attention patterns) are
not shipped with it, so these generators stand in for them with the shapes,
densities and value distributions of the benchmark configurations:

===========  =======================================================================
name         description
===========  =======================================================================
plumbing     B1 H4 N1024 D64 fp32 BLOCK64; q,k,v ~ N(0,1)/sqrt(D); 16x16 mask,
             diagonal + Bernoulli(0.25); no permutation
random       B2 H16 N8192 D64 bf16 BLOCK128; N(0,1); diagonal + Bernoulli(0.10),
             shared across heads; identity permutation
sbm          B1 H16 N16384 D128 bf16 BLOCK128; stochastic block model token graph
             (32 communities x 512 tokens, p_in 0.05, p_out 5e-4, self loops) in a
             shuffled token order, reordered by the community-sorting permutation;
             a block is kept if any token pair in it is an edge
headline     B1 H16 N16384 D128 bf16 BLOCK128; diagonal + Bernoulli(0.10)
             (the "N=16K, D=128, 10% density" operating point)
longctx      B1 H32 N65536 D128 bf16 BLOCK128; band of +-4 blocks + 64 seeded
             random key blocks per query block
sweep_pXX    B4 H32 N32768 D128 fp16 BLOCK64; lower-triangular, diagonal kept,
             below-diagonal Bernoulli(p), p in {0.01, 0.05, 0.2, 0.5}
===========  =======================================================================

Masks are shared across (b, h) (shape ``[1, 1, nb, nb]``).  Everything is
generated from fixed seeds; q, k, v are drawn on the target device.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Optional

import numpy as np
import torch


@dataclass
class Workload:
    name: str
    B: int
    H: int
    N: int
    D: int
    block: int
    dtype: torch.dtype
    mask: np.ndarray                      # bool [nb, nb] in the (new) kernel token order
    q_perm: Optional[np.ndarray] = None   # perm[i] = old index at new position i
    kv_perm: Optional[np.ndarray] = None
    coords: Optional[tuple] = None        # token-level (rows, cols) in the ORIGINAL order, if any
    qkv_scale: float = 1.0
    seed: int = 0
    extra: dict = field(default_factory=dict)

    @property
    def nb(self) -> int:
        return self.mask.shape[0]

    @property
    def nnz_blocks(self) -> int:
        """Kept (query block, key block) pairs summed over (b, h)."""
        return int(self.mask.sum()) * self.B * self.H

    @property
    def density(self) -> float:
        return float(self.mask.mean())

    @property
    def flops(self) -> float:
        """Algorithmic flops on kept blocks: 4 * BLOCK^2 * D per kept block."""
        return 4.0 * self.block * self.block * self.D * self.nnz_blocks

    def make_qkv(self, device, seed: Optional[int] = None):
        g = torch.Generator(device=device).manual_seed(self.seed if seed is None else seed)
        shape = (self.B, self.H, self.N, self.D)
        out = []
        for _ in range(3):
            t = torch.randn(shape, generator=g, device=device, dtype=torch.float32)
            if self.qkv_scale != 1.0:
                t.mul_(self.qkv_scale)
            out.append(t.to(self.dtype))
        return tuple(out)

    def mask_tensor(self, device) -> torch.Tensor:
        return torch.from_numpy(self.mask).to(device)[None, None]


def diag_bernoulli(nb: int, p: float, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    m = rng.random((nb, nb)) < p
    m[np.arange(nb), np.arange(nb)] = True
    return m


def causal_bernoulli(nb: int, p: float, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    m = np.tril(rng.random((nb, nb)) < p, k=-1)
    m[np.arange(nb), np.arange(nb)] = True
    return m


def band_random(nb: int, half_band: int, n_random: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    m = np.zeros((nb, nb), dtype=bool)
    for i in range(nb):
        m[i, max(0, i - half_band):min(nb, i + half_band + 1)] = True
        m[i, rng.choice(nb, size=min(n_random, nb), replace=False)] = True
    return m


def sbm_coords(n_comm: int, comm_size: int, p_in: float, p_out: float, seed: int):
    """Token-level edges of a stochastic block model in a shuffled token order.

    Returns ``(rows, cols, labels)``: int64 edge coordinates (with one self
    loop per token) and each token's community, all in the shuffled
    (original) order."""
    rng = np.random.default_rng(seed)
    n = n_comm * comm_size
    labels = rng.permutation(np.repeat(np.arange(n_comm), comm_size))
    members = [np.nonzero(labels == c)[0] for c in range(n_comm)]
    rows, cols = [np.arange(n)], [np.arange(n)]
    for ci in range(n_comm):
        for cj in range(n_comm):
            p = p_in if ci == cj else p_out
            cnt = rng.binomial(comm_size * comm_size, p)
            rows.append(members[ci][rng.integers(0, comm_size, cnt)])
            cols.append(members[cj][rng.integers(0, comm_size, cnt)])
    return np.concatenate(rows).astype(np.int64), np.concatenate(cols).astype(np.int64), labels


def blockmask_np(rows, cols, n: int, block: int) -> np.ndarray:
    nb = (n + block - 1) // block
    m = np.zeros((nb, nb), dtype=bool)
    rb, cb = rows // block, cols // block
    ok = (rb < nb) & (cb < nb)
    m[rb[ok], cb[ok]] = True
    return m


def make(name: str, scale: float = 1.0) -> Workload:
    """Build a named workload.  ``scale`` < 1 shrinks N (and H, B) for tests
    while keeping the mask recipe; the mask seed is fixed per workload."""
    if name == "plumbing":
        return Workload(name, 1, 4, 1024, 64, 64, torch.float32, diag_bernoulli(16, 0.25, 11),
                        qkv_scale=1.0 / math.sqrt(64), seed=1)
    if name == "random":
        n = max(256, int(8192 * scale))
        return Workload(name, 2, 16 if scale >= 1 else 2, n, 64, 128, torch.bfloat16,
                        diag_bernoulli(n // 128, 0.10, 12), seed=2)
    if name == "headline":
        n = max(256, int(16384 * scale))
        return Workload(name, 1, 16 if scale >= 1 else 2, n, 128, 128, torch.bfloat16,
                        diag_bernoulli(n // 128, 0.10, 13), seed=3)
    if name == "sbm":
        comm = 32 if scale >= 1 else 8
        size = 512 if scale >= 1 else max(16, int(512 * scale))
        n = comm * size
        rows, cols, labels = sbm_coords(comm, size, 0.05, 5e-4, 14)
        perm = np.argsort(labels, kind="stable").astype(np.int64)   # community sort
        inv = np.empty_like(perm)
        inv[perm] = np.arange(n)
        mask = blockmask_np(inv[rows], inv[cols], n, 128)
        return Workload(name, 1, 16 if scale >= 1 else 2, n, 128, 128, torch.bfloat16, mask, q_perm=perm,
                        kv_perm=perm, coords=(rows, cols), seed=4)
    if name == "longctx":
        n = max(1024, int(65536 * scale))
        nb = n // 128
        return Workload(name, 1, 32 if scale >= 1 else 2, n, 128, 128, torch.bfloat16,
                        band_random(nb, 4, min(64, nb), 15), seed=5)
    if name.startswith("sweep_p"):
        p = {"sweep_p01": 0.01, "sweep_p05": 0.05, "sweep_p20": 0.2, "sweep_p50": 0.5}[name]
        n = max(512, int(32768 * scale))
        big = scale >= 1
        return Workload(name, 4 if big else 1, 32 if big else 2, n, 128, 64, torch.float16,
                        causal_bernoulli(n // 64, p, 16), seed=6)
    raise KeyError(f"unknown workload {name!r}")


NAMES = ["plumbing", "random", "sbm", "headline", "longctx", "sweep_p01", "sweep_p05", "sweep_p20", "sweep_p50"]
