"""Every benchmark configuration at its full shape on the B200, and the
BLOCK 64 kernel form that takes a tile's kept blocks in pairs.

The full-shape tests run the whole forward through the public API and check
sampled (b, h) units and query blocks (first, middle and last block rows)
against the oracle's port of the reference block loop
(``triton_kernels/BlockSparse_Naive.py:5-125``); the permuted configuration
follows the runners' "with reordering" semantics
(``BlockSparseTriton_Naive.py:129-161``: inputs and output in the original
token order, mask in the new order).  Outputs are NaN-prefilled and a second
run must be bitwise identical.

Tolerances (fixed by the parity spec): max |err| <= 2e-2 for bf16 / fp16;
log2 LSE within 2e-2 where finite, -inf exactly where the oracle's is.
"""

import numpy as np
import pytest
import torch

from blocksparsefa_reorder_b200 import BlockSparsePlan, block_sparse_attention
from blocksparsefa_reorder_b200 import workloads as W
from oracle import attention as OA

pytestmark = pytest.mark.gpu

TOL_16 = 2e-2
TOL_LSE = 2e-2
PAIR_MIN_ENTRIES = 4  # the plan average (entries per tile) from which BLOCK 64 runs the paired form


def _units_numpy(t, units):
    """[B, H, N, D] CUDA tensor -> float32 numpy [1, len(units), N, D] of the chosen (b, h)."""
    return np.stack([t[b, h].float().cpu().numpy() for b, h in units])[None]


def _check_sampled(wl, o, lse, q, k, v, units, qblocks):
    qs, ks, vs = (_units_numpy(t, units) for t in (q, k, v))
    if wl.q_perm is not None:
        qs = qs[:, :, wl.q_perm]
    if wl.kv_perm is not None:
        ks, vs = ks[:, :, wl.kv_perm], vs[:, :, wl.kv_perm]
    ref, ref_lse = OA.block_sparse_online(qs, ks, vs, wl.mask[None, None], wl.block, query_blocks=qblocks)
    for i, (b, h) in enumerate(units):
        got = o[b, h].float().cpu().numpy()
        gl = lse[b, h].cpu().numpy()
        for mb in qblocks:
            r0, r1 = mb * wl.block, min(wl.N, (mb + 1) * wl.block)
            rows = np.arange(r0, r1) if wl.q_perm is None else wl.q_perm[r0:r1]
            err = np.abs(got[rows] - ref[0, i, r0:r1]).max()
            assert err <= TOL_16, (wl.name, b, h, mb, err)
            rl = ref_lse[0, i, r0:r1]
            fin = np.isfinite(rl)
            assert np.array_equal(np.isfinite(gl[rows]), fin), (wl.name, b, h, mb)
            assert np.abs(gl[rows][fin] - rl[fin]).max() <= TOL_LSE, (wl.name, b, h, mb)


def _run_full(wl, dev):
    q, k, v = wl.make_qkv(dev)
    plan = BlockSparsePlan(wl.mask_tensor(dev), wl.block)
    qp = torch.from_numpy(wl.q_perm).to(dev) if wl.q_perm is not None else None
    kp = torch.from_numpy(wl.kv_perm).to(dev) if wl.kv_perm is not None else None
    o = torch.full_like(q, float("nan"))
    lse = torch.full(q.shape[:3], float("nan"), device=dev)
    block_sparse_attention(q, k, v, plan=plan, q_perm=qp, kv_perm=kp, return_lse=True, out=o, lse_out=lse,
                           check_errors=True)
    o2 = block_sparse_attention(q, k, v, plan=plan, q_perm=qp, kv_perm=kp)
    assert torch.equal(o, o2), "second run differs"
    assert torch.isfinite(o.float()).all()
    return q, k, v, o, lse, plan


def test_random_config_full_size(dev):
    """Random block-sparse: B2 H16 N8192 D64 bf16 BLOCK128, ~11% kept."""
    wl = W.make("random")
    assert (wl.B, wl.H, wl.N, wl.D, wl.block) == (2, 16, 8192, 64, 128)
    q, k, v, o, lse, _ = _run_full(wl, dev)
    _check_sampled(wl, o, lse, q, k, v, [(0, 0), (1, 15)], [0, 31, 63])


def test_sbm_reordered_config_full_size(dev):
    """Reordered graph mask: B1 H16 N16384 D128 bf16 BLOCK128 with the
    community-sort permutation as q_perm = kv_perm (the fused Q gather and
    O / lse scatter at full size, K and V permuted beforehand)."""
    wl = W.make("sbm")
    assert (wl.B, wl.H, wl.N, wl.D, wl.block) == (1, 16, 16384, 128, 128) and wl.q_perm is not None
    q, k, v, o, lse, _ = _run_full(wl, dev)
    _check_sampled(wl, o, lse, q, k, v, [(0, 0), (0, 15)], [0, 64, 127])


@pytest.mark.parametrize("name", ["sweep_p01", "sweep_p05", "sweep_p20", "sweep_p50"])
def test_density_sweep_config_full_size(dev, name):
    """Density sweep: B4 H32 N32768 D128 fp16 BLOCK64, causal with the
    diagonal kept.  Every density runs the paired form (tiles average 7 kept
    blocks at p = 0.01; asserted from the plan's entry total, the value the
    kernels select on)."""
    wl = W.make(name)
    assert (wl.B, wl.H, wl.N, wl.D, wl.block, wl.dtype) == (4, 32, 32768, 128, 64, torch.float16)
    q, k, v, o, lse, plan = _run_full(wl, dev)
    tiles = plan.mask_b * plan.mask_h * plan.tiles_per_row
    paired = plan.nnz_entries() >= PAIR_MIN_ENTRIES * tiles
    assert paired
    _check_sampled(wl, o, lse, q, k, v, [(0, 0), (3, 31)], [0, 1, 300, 510, 511])


def _pairing_mask(nb, H, p, seed):
    """A dense BLOCK 64 mask (tiles average well over PAIR_MIN_ENTRIES
    entries) with the edge cases of the paired form planted in it."""
    rng = np.random.default_rng(seed)
    mask = rng.random((1, H, nb, nb)) < p
    mask[..., np.arange(nb), np.arange(nb)] = True
    # head 0, tile 2 (block rows 4 and 5): rows keep disjoint blocks, odd total
    mask[:, 0, 4:6, :] = False
    mask[:, 0, 4, [0, 5, 9, 40]] = True
    mask[:, 0, 5, [1, 4, 13]] = True
    # head 0, tile 3: one row keeps only the partial last key block
    mask[:, 0, 6, :] = False
    mask[:, 0, 6, nb - 1] = True
    # head 1: key block 11 kept by nobody (its keys and values become NaN)
    mask[:, 1, :, 11] = False
    return mask


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("D", [64, 128])
def test_block64_paired_form(dev, dtype, D):
    """BLOCK 64 with tiles averaging many kept key blocks, so the kernel form
    that takes a tile's entries two at a time (128-key steps) runs: odd entry
    counts (the repeated, masked second entry), blocks kept by only one of a
    tile's two block rows, rows with disjoint kept sets, a row keeping only the
    partial last key block (N % 64 = 23) and a partial last 128-row tile (odd
    number of block rows), NaN keys and values in a block nobody keeps,
    NaN-prefilled outputs, three runs bitwise identical.  O and lse against the
    float64 masked-softmax oracle."""
    B, H, block = 1, 2, 64
    N = 64 * 98 + 23
    nb = (N + block - 1) // block
    assert nb % 2 == 1
    mask = _pairing_mask(nb, H, 0.6, seed=D + (1 if dtype == torch.float16 else 2))
    g = torch.Generator(device="cpu").manual_seed(D)
    q, k, v = ((torch.randn(B, H, N, D, generator=g)).to(dtype).to(dev) for _ in range(3))
    k[:, 1, 11 * block:12 * block] = float("nan")
    v[:, 1, 11 * block:12 * block] = float("nan")
    plan = BlockSparsePlan(torch.from_numpy(mask).to(dev), block)
    tiles = plan.mask_b * plan.mask_h * plan.tiles_per_row
    assert plan.nnz_entries() >= PAIR_MIN_ENTRIES * tiles, "mask too sparse for the paired form"
    runs = []
    for _ in range(3):
        o = torch.full_like(q, float("nan"))
        lse = torch.full((B, H, N), float("nan"), device=dev)
        block_sparse_attention(q, k, v, plan=plan, kernel="tcgen05", return_lse=True, out=o, lse_out=lse,
                               check_errors=True)
        runs.append((o, lse))
    for o, lse in runs[1:]:
        assert torch.equal(o, runs[0][0]) and torch.equal(lse, runs[0][1])
    o, lse = runs[0]
    assert torch.isfinite(o.float()).all()
    kc, vc = k.clone(), v.clone()
    kc[:, 1, 11 * block:12 * block] = 0
    vc[:, 1, 11 * block:12 * block] = 0
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    ref, ref_lse = OA.dense_masked_attention(f(q), f(kc), f(vc), mask, block)
    assert np.abs(f(o) - ref).max() <= TOL_16
    lv = lse.cpu().numpy()
    fin = np.isfinite(ref_lse)
    assert np.array_equal(np.isfinite(lv), fin)
    assert np.abs(lv[fin] - ref_lse[fin]).max() <= TOL_LSE


def test_block64_paired_form_fused_permutation(dev):
    """The paired form with the query permutation gathered and scattered
    inside the kernel and a key permutation: int32 permutations, against the
    oracle's reordered attention."""
    B, H, block, D = 2, 2, 64, 128
    N = 64 * 71
    nb = N // block
    rng = np.random.default_rng(5)
    mask = rng.random((1, H, nb, nb)) < 0.7
    mask[..., np.arange(nb), np.arange(nb)] = True
    g = torch.Generator(device="cpu").manual_seed(9)
    q, k, v = (torch.randn(B, H, N, D, generator=g).to(torch.float16).to(dev) for _ in range(3))
    qp = torch.randperm(N, generator=g).to(torch.int32).to(dev)
    kp = torch.randperm(N, generator=g).to(torch.int32).to(dev)
    plan = BlockSparsePlan(torch.from_numpy(mask).to(dev), block)
    assert plan.nnz_entries() >= PAIR_MIN_ENTRIES * plan.mask_b * plan.mask_h * plan.tiles_per_row
    o = torch.full_like(q, float("nan"))
    o, lse = block_sparse_attention(q, k, v, plan=plan, q_perm=qp, kv_perm=kp, return_lse=True, out=o,
                                    kernel="tcgen05", check_errors=True)
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    ref, ref_lse = OA.reordered_attention(f(q), f(k), f(v), mask, block, qp.cpu().numpy(), kp.cpu().numpy())
    assert np.abs(f(o) - ref).max() <= TOL_16
    assert np.abs(lse.cpu().numpy() - ref_lse).max() <= TOL_LSE


@pytest.mark.parametrize("which", ["q", "kv"])
def test_repeated_permutation_value_flagged(dev, which):
    """With check_errors the reordered forward checks both permutations on
    the device first: a repeated value (two new rows from one old row) is
    reported, on the fused path too, where the kernel's own gather and
    scatter could not see it."""
    B, H, N, D, block = 1, 2, 1024, 128, 128
    rng = np.random.default_rng(3)
    mask = rng.random((1, 1, N // block, N // block)) < 0.5
    mask[..., np.arange(N // block), np.arange(N // block)] = True
    q, k, v = (torch.randn(B, H, N, D).to(torch.bfloat16).to(dev) for _ in range(3))
    perm = torch.randperm(N)
    perm[17] = perm[500]
    perm = perm.to(dev)
    kw = {"q_perm": perm} if which == "q" else {"kv_perm": perm}
    with pytest.raises(RuntimeError, match="permutation value repeated"):
        block_sparse_attention(q, k, v, torch.from_numpy(mask).to(dev), kernel="tcgen05", check_errors=True, **kw)
    # a true permutation passes the same check
    good = torch.randperm(N).to(dev)
    kw = {"q_perm": good} if which == "q" else {"kv_perm": good}
    block_sparse_attention(q, k, v, torch.from_numpy(mask).to(dev), kernel="tcgen05", check_errors=True, **kw)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_block64_dense_reference_point_guard(dev, dtype):
    """The paired BLOCK 64 form (dense plans) takes each row's reference point
    from the exact max of its first kept step and redoes a step with the exact
    max (O and the row sum rescaled) when a score leaves the slack: one key
    block scaled by 30 (~40 log2 units above the reference, past fp16's range
    for P without the redo), an early block scaled down.  O (finite) and lse
    against the float64 oracle."""
    B, H, block, D = 1, 2, 64, 128
    N = 64 * 60
    nb = N // block
    rng = np.random.default_rng(17)
    mask = rng.random((1, H, nb, nb)) < 0.8
    mask[..., np.arange(nb), np.arange(nb)] = True
    mask[..., :, nb - 3] = True
    g = torch.Generator(device="cpu").manual_seed(18)
    q, k, v = (torch.randn(B, H, N, D, generator=g).to(dtype).to(dev) for _ in range(3))
    k[:, :, (nb - 3) * block:(nb - 2) * block] *= 30
    k[:, :, :block] *= 0.1
    plan = BlockSparsePlan(torch.from_numpy(mask).to(dev), block)
    assert plan.nnz_entries() >= PAIR_MIN_ENTRIES * plan.mask_b * plan.mask_h * plan.tiles_per_row
    o, lse = block_sparse_attention(q, k, v, plan=plan, return_lse=True, kernel="tcgen05", check_errors=True)
    assert torch.isfinite(o.float()).all()
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    ref, ref_lse = OA.dense_masked_attention(f(q), f(k), f(v), mask, block)
    assert np.abs(f(o) - ref).max() <= TOL_16
    lv = lse.cpu().numpy()
    fin = np.isfinite(ref_lse)
    assert np.array_equal(np.isfinite(lv), fin)
    assert np.abs(lv[fin] - ref_lse[fin]).max() <= TOL_LSE * max(1.0, float(np.abs(ref_lse[fin]).max()) / 8)


def test_block64_dense_wait_timeout(dev):
    """The bounded-wait timeout on the paired BLOCK 64 form: one softmax warp
    of CTA 0 withholds its first arrival (test hook, 1 ms limit); the host sees
    the timeout and the next forwards, including the one that reuses the
    work-counter slot, equal the result before."""
    from blocksparsefa_reorder_b200 import _lib

    B, H, block, D = 1, 4, 64, 128
    N = 64 * 64
    nb = N // block
    rng = np.random.default_rng(19)
    mask = rng.random((1, 1, nb, nb)) < 0.7
    mask[..., np.arange(nb), np.arange(nb)] = True
    g = torch.Generator(device="cpu").manual_seed(20)
    q, k, v = (torch.randn(B, H, N, D, generator=g).to(torch.bfloat16).to(dev) for _ in range(3))
    plan = BlockSparsePlan(torch.from_numpy(mask).to(dev), block)
    assert plan.nnz_entries() >= PAIR_MIN_ENTRIES * plan.tiles_per_row
    good = block_sparse_attention(q, k, v, plan=plan, kernel="tcgen05", check_errors=True)
    assert _lib.lib().bsa_test_arm_wait_timeout(1000) == 0
    with pytest.raises(RuntimeError, match="device wait timed out"):
        block_sparse_attention(q, k, v, plan=plan, kernel="tcgen05", check_errors=True)
    for _ in range(65):
        o = block_sparse_attention(q, k, v, plan=plan, kernel="tcgen05", check_errors=True)
        assert torch.equal(o, good)
