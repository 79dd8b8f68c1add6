"""GPU preprocessing kernels against the oracle and the reference's own
outputs (golden): bit-exact, since all of this is integer / index / copy
work."""

import math

import numpy as np
import pytest
import torch

from blocksparsefa_reorder_b200 import BlockSparsePlan, inverse_permutation, permute_rows, runners, sharding, utils
from blocksparsefa_reorder_b200 import block_sparse_attention
from oracle import preprocess as OP

pytestmark = pytest.mark.gpu


# the last two cases exceed the one-kernel plan build (T > 1024 tiles per
# slice; > 4096 tiles in all) and take the multi-kernel path
@pytest.mark.parametrize("block,nb,shape,p", [(128, 64, (1, 1), 0.1), (64, 33, (2, 3), 0.3), (64, 8, (1, 2), 0.0),
                                             (128, 5, (2, 1), 1.0), (64, 512, (1, 1), 0.05),
                                             (128, 1100, (1, 1), 0.01), (64, 40, (16, 16), 0.2)])
def test_plan_build_bitexact(dev, block, nb, shape, p):
    rng = np.random.default_rng(nb)
    m = rng.random(shape + (nb, nb)) < p
    plan = BlockSparsePlan(torch.from_numpy(m).to(dev), block)
    ptr, col = OP.tile_csr(m.reshape(-1, nb, nb), block)
    assert np.array_equal(plan.tile_ptr.cpu().numpy(), ptr)
    n = int(ptr[-1])
    assert np.array_equal(plan.tile_col[:n].cpu().numpy(), col)


@pytest.mark.parametrize("block,nb,shape,p", [(128, 64, (1, 1), 0.1), (64, 33, (2, 3), 0.3), (64, 8, (1, 2), 0.0),
                                             (128, 700, (1, 2), 0.02), (64, 600, (1, 1), 0.5),
                                             (128, 1100, (1, 1), 0.01), (64, 40, (16, 16), 0.2)])
def test_tile_order(dev, block, nb, shape, p):
    """The plan's work order: per slice, the tile rows by decreasing number of
    kept blocks, ties by increasing row (a stable descending sort), including
    slices with more than one 256-row chunk."""
    rng = np.random.default_rng(nb + 1)
    m = rng.random(shape + (nb, nb)) < p
    m[..., : nb // 3, :] = False  # some empty rows
    plan = BlockSparsePlan(torch.from_numpy(m).to(dev), block)
    T = plan.tiles_per_row
    n = np.diff(plan.tile_ptr.cpu().numpy()).reshape(-1, T)
    want = np.argsort(-n, axis=1, kind="stable")
    got = plan.tile_order.cpu().numpy().reshape(-1, T)
    assert np.array_equal(got, want)


def test_plan_from_strided_mask(dev):
    rng = np.random.default_rng(5)
    big = torch.from_numpy(rng.random((2, 3, 16, 20)) < 0.4).to(dev)
    view = big[:, :, :, 2:18]  # non-contiguous rows
    plan = BlockSparsePlan(view, 128)
    ptr, col = OP.tile_csr(view.cpu().numpy().reshape(-1, 16, 16), 128)
    assert np.array_equal(plan.tile_ptr.cpu().numpy(), ptr)
    assert np.array_equal(plan.tile_col[:int(ptr[-1])].cpu().numpy(), col)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("idx_dtype", [torch.int32, torch.int64])
def test_permute_rows_gather_scatter(dev, dtype, idx_dtype):
    g = torch.Generator().manual_seed(1)
    x = torch.randn(2, 3, 300, 72, generator=g).to(dtype).to(dev)
    perm = torch.randperm(300, generator=g).to(idx_dtype).to(dev)
    y = permute_rows(x, perm, 2, inverse=False)
    assert torch.equal(y, x.index_select(2, perm.long()))
    z = permute_rows(y, perm, 2, inverse=True)
    assert torch.equal(z, x)
    # a 3-D [(B*S), H, D] tensor permuted along dim 0 (the BSFA layout)
    w = torch.randn(300, 4, 16, generator=g).to(dtype).to(dev)
    assert torch.equal(permute_rows(w, perm, 0, inverse=False), w.index_select(0, perm.long()))


def test_inverse_permutation_and_checks(dev):
    g = torch.Generator().manual_seed(2)
    p = torch.randperm(1000, generator=g).to(dev)
    inv = inverse_permutation(p)
    assert np.array_equal(inv.cpu().numpy(), OP.inverse_permutation(p.cpu().numpy()))
    dup = p.clone()
    dup[5] = dup[6]
    with pytest.raises(RuntimeError, match="repeated"):
        inverse_permutation(dup)
    bad = p.clone()
    bad[0] = 1000
    with pytest.raises(RuntimeError, match="out of range"):
        inverse_permutation(bad)
    with pytest.raises(RuntimeError, match="out of range"):
        permute_rows(torch.zeros(1, 1, 1000, 8, device=dev), bad, 2, inverse=False, check_errors=True)


def test_reference_preprocessing_golden(dev, golden_dir):
    gd = np.load(golden_dir / "preprocess_golden.npz")
    for ci in range(int(gd["n_cases"])):
        n, blk, bsz, nh = (int(x) for x in gd[f"c{ci}_meta"])
        m, sl = utils.generate_blockmask_from_mtx_coords(gd[f"c{ci}_rows"], gd[f"c{ci}_cols"], n, blk, bsz, nh,
                                                        device=dev, verbose=False)
        assert sl == n and m.dtype == torch.bool
        assert np.array_equal(m.cpu().numpy(), gd[f"c{ci}_mask_plain"])
        rn = utils.update_idx_perm(gd[f"c{ci}_r_in"], torch.from_numpy(gd[f"c{ci}_perm_r"]).to(dev))
        assert isinstance(rn, np.ndarray) and np.array_equal(rn, gd[f"c{ci}_r_new"])
        # fused remap + mask build gives the reference's permuted mask
        m2, _ = utils.generate_blockmask_from_mtx_coords(gd[f"c{ci}_r_in"], gd[f"c{ci}_c_in"], n, blk, bsz, nh,
                                                         device=dev, row_perm=gd[f"c{ci}_perm_r"],
                                                         col_perm=gd[f"c{ci}_perm_c"], verbose=False)
        assert np.array_equal(m2.cpu().numpy(), gd[f"c{ci}_mask_perm"])
        x = torch.from_numpy(gd[f"c{ci}_x"]).to(dev)
        pr = torch.from_numpy(gd[f"c{ci}_perm_r"]).to(dev)
        assert np.array_equal(utils.apply_reordering(x, pr, dim=2).cpu().numpy(), gd[f"c{ci}_applied"])
        assert np.array_equal(utils.reverse_reordering(x, pr, dim=2).cpu().numpy(), gd[f"c{ci}_reversed"])


def test_negative_coordinates_flagged(dev):
    with pytest.raises(RuntimeError, match="coordinate"):
        utils.generate_blockmask_from_mtx_coords(np.array([0, -1]), np.array([0, 3]), 128, 64, device=dev,
                                                 verbose=False)


def test_runner_prints_reference_lines(dev, capsys):
    args = utils.Args(matrix_mtx="unused.mtx", block_size=64, head_dim=64, num_heads=2)
    nb = 8
    mask = torch.eye(nb, dtype=torch.bool, device=dev)[None, None]
    perm = torch.randperm(nb * 64, generator=torch.Generator().manual_seed(0))
    r = runners.run_experiments_B200(args, mask, nb * 64, row_perm=perm, col_perm=perm, warmup=2, reps=3)
    out = capsys.readouterr().out
    assert "Average time with reordering:" in out and "Average time without reordering:" in out
    assert r["ms_with_reordering"] > 0 and r["ms_without_reordering"] > 0


def test_head_sharding_reassembles_full_output(dev):
    """The multi-GPU partition run on one GPU: each 'rank' computes its head
    range alone; concatenating the shards equals the unsharded output."""
    B, H, N, D, block = 1, 8, 1024, 128, 128
    rng = np.random.default_rng(3)
    mask = torch.from_numpy(rng.random((1, 1, N // block, N // block)) < 0.3).to(dev)
    g = torch.Generator().manual_seed(4)
    q, k, v = (torch.randn(B, H, N, D, generator=g).to(torch.bfloat16).to(dev) for _ in range(3))
    full = block_sparse_attention(q, k, v, mask)
    parts = []
    for rank in range(4):
        h0, h1 = sharding.local_heads(H, rank, 4)
        parts.append(block_sparse_attention(q[:, h0:h1].contiguous(), k[:, h0:h1].contiguous(),
                                            v[:, h0:h1].contiguous(), mask))
    assert torch.equal(torch.cat(parts, dim=1), full)
    assert math.isfinite(full.float().abs().max().item())


def test_cli_end_to_end(dev, tmp_path, capsys):
    """The main.py-compatible command line on a small pattern file with row
    and column permutation files (1-based, as the reference's files are):
    prints the mask's NNZ line and the runner's two timing lines."""
    from blocksparsefa_reorder_b200 import __main__ as cli

    n = 512
    rng = np.random.default_rng(3)
    pairs = {(i, i) for i in range(n)} | {tuple(x) for x in rng.integers(0, n, size=(2000, 2))}
    rows = np.array(sorted(pairs))
    mtx = tmp_path / "pattern.mtx"
    mtx.write_text(f"{n} {n} {len(rows)}\n" + "".join(f"{r + 1} {c + 1}\n" for r, c in rows))
    for name, seed in (("rows.txt", 1), ("cols.txt", 2)):
        perm = np.random.default_rng(seed).permutation(n) + 1
        (tmp_path / name).write_text(f"{n}\n" + "".join(f"{v}\n" for v in perm))
    assert cli.main([str(mtx), "--block-size", "64", "--head-dim", "64", "--row-reorder", str(tmp_path / "rows.txt"),
                     "--col-reorder", str(tmp_path / "cols.txt")]) == 0
    out = capsys.readouterr().out
    assert "NNZ blocks:" in out
    assert "Average time with reordering:" in out and "Average time without reordering:" in out
