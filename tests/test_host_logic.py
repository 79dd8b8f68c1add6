"""Host-side logic that runs without a GPU: the reference-compatible file
readers against what the reference itself returned (golden), partitioning,
block inference, workload generators and the API's argument checks."""

import json
from pathlib import Path

import numpy as np
import pytest
import torch

from blocksparsefa_reorder_b200 import api, kernels, sharding, utils
from blocksparsefa_reorder_b200 import workloads as W
from oracle import preprocess as OP


@pytest.fixture(scope="module")
def files(golden_dir):
    return json.loads((golden_dir / "reorder_files.json").read_text())


def test_read_reordering_file_matches_reference(tmp_path, files):
    for name, ent in files["perm_files"].items():
        p = tmp_path / name
        p.write_text(ent["text"])
        if ent["ok"]:
            got = utils.read_reordering_file_to_tensor(p, zero_based=ent["zero_based"])
            assert got.dtype == torch.int64 and got.tolist() == ent["perm"], name
        else:
            with pytest.raises(ValueError) as e:
                utils.read_reordering_file_to_tensor(p, zero_based=ent["zero_based"])
            assert str(e.value).replace(str(p), "<path>") == ent["error"], name


def test_read_mtx_matches_reference(tmp_path, files):
    for name, ent in files["mtx"].items():
        p = tmp_path / name
        p.write_text(ent["text"])
        r, c, n = utils.read_mtx(str(p))
        assert r.tolist() == ent["rows"] and c.tolist() == ent["cols"] and n == ent["seq_len"], name


def test_partition_units_even_and_weighted():
    assert sharding.partition_units(16, 8) == [(2 * i, 2 * i + 2) for i in range(8)]
    assert sharding.partition_units(5, 2) == [(0, 3), (3, 5)]
    assert sharding.partition_units(2, 4) == [(0, 1), (1, 2), (2, 2), (2, 2)]
    w = [10, 1, 1, 1, 1, 1, 1, 4]
    parts = sharding.partition_units(8, 2, w)
    assert parts[0][0] == 0 and parts[-1][1] == 8
    assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))
    loads = [sum(w[lo:hi]) for lo, hi in parts]
    assert max(loads) <= 11
    with pytest.raises(ValueError):
        sharding.partition_units(4, 0)
    with pytest.raises(ValueError):
        sharding.partition_units(3, 2, [1, 2])


def test_infer_block():
    assert api.infer_block(16384, 128) == 128
    assert api.infer_block(16384, 256) == 64
    assert api.infer_block(200, 4) == 64
    with pytest.raises(ValueError):
        api.infer_block(1000, 3)


def test_workloads_match_their_recipes():
    hl = W.make("headline")
    assert (hl.B, hl.H, hl.N, hl.D, hl.block) == (1, 16, 16384, 128, 128)
    assert 0.09 < hl.density < 0.12 and hl.mask.diagonal().all()
    assert hl.flops == 4.0 * 128 * 128 * 128 * int(hl.mask.sum()) * 16
    sw = W.make("sweep_p05")
    assert not np.triu(sw.mask, 1).any() and sw.mask.diagonal().all()
    lc = W.make("longctx", scale=0.0625)
    assert lc.mask.shape == (32, 32) and all(lc.mask[i, max(0, i - 4):i + 5].all() for i in range(32))
    sb = W.make("sbm", scale=0.125)
    assert OP.is_permutation(sb.q_perm)
    # the mask is the reordered coordinates' block mask
    rows, cols = sb.coords
    m = OP.blockmask_from_coords(OP.update_idx_perm(rows, sb.q_perm), OP.update_idx_perm(cols, sb.kv_perm), sb.N,
                                 sb.block)
    assert np.array_equal(m[0, 0], sb.mask)


def test_api_rejects_cpu_tensors_and_bad_shapes():
    q = torch.zeros(1, 1, 128, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        api.block_sparse_attention(q, q, q, torch.ones(1, 1, dtype=torch.bool))
    with pytest.raises(ValueError, match="CUDA"):
        api.BlockSparsePlan(torch.ones(2, 2, dtype=torch.bool), 64)
    with pytest.raises(ValueError):
        kernels._check_blocks(64, 128, 256, torch.ones(4, 4))
    with pytest.raises(ValueError):
        kernels._check_blocks(64, 64, 256, torch.ones(3, 3))
    assert api._perm_vector(torch.arange(8).view(1, 1, 8, 1).expand(2, 3, 8, 4), 8, "cpu", "p").tolist() == \
        list(range(8))
    with pytest.raises(ValueError):
        api._perm_vector(torch.arange(7), 8, "cpu", "p")


def test_utils_requires_gpu_device():
    with pytest.raises(ValueError):
        utils.generate_blockmask_from_mtx_coords(np.array([0]), np.array([0]), 64, 64, device="cpu")


def test_build_script_lists_every_source():
    from blocksparsefa_reorder_b200 import build

    on_disk = sorted(p.name for p in build.CSRC.glob("*.cu"))
    assert sorted(build.SOURCES) == on_disk
    assert Path(build.LIB_PATH).name == "libbsattn_b200.so"


def test_cli_arguments_follow_main_py(tmp_path):
    """``python -m blocksparsefa_reorder_b200`` parses main.py's arguments
    (main.py:102-160): defaults, the .mtx extension check, and the
    reference's comparator modes reported as not included."""
    from blocksparsefa_reorder_b200 import __main__ as cli

    a = cli.parse_args([str(tmp_path / "p.mtx")])
    assert (a.block_size, a.head_dim, a.num_heads, a.mode) == (128, 128, 1, "B200")
    assert a.row_reorder is None and a.col_reorder is None
    a = cli.parse_args([str(tmp_path / "p.MTX"), "--block-size", "64", "--head-dim", "64", "--num-heads", "4",
                        "--row-reorder", "r.txt", "--col-reorder", "c.txt"])
    assert (a.block_size, a.head_dim, a.num_heads) == (64, 64, 4)
    assert str(a.row_reorder) == "r.txt" and str(a.col_reorder) == "c.txt"
    for bad in (["p.txt"], ["p.mtx", "--mode", "BSFA"], ["p.mtx", "--block-size", "96"],
                ["p.mtx", "--head-dim", "0"], ["p.mtx", "--mode", "XYZ"]):
        with pytest.raises(SystemExit):
            cli.parse_args(bad)
