"""Pin the CPU oracle to the reference: golden vectors recorded from the
reference's own utils.py and Triton kernels (tests/golden/make_golden.py).

Preprocessing is integer / index work: bit-exact.  Attention: the oracle's
float64 definition against the reference's fp16 outputs within fp16 output
rounding; the float32 port of the reference block loop reproduces the
reference's log2 LSE (M)."""

import numpy as np
import pytest

from oracle import attention as OA
from oracle import preprocess as OP


@pytest.fixture(scope="module")
def pre(golden_dir):
    return np.load(golden_dir / "preprocess_golden.npz")


@pytest.fixture(scope="module")
def att(golden_dir):
    return np.load(golden_dir / "attention_golden.npz")


def _cases(pre):
    return range(int(pre["n_cases"]))


def test_blockmask_from_coords_bitexact(pre):
    for ci in _cases(pre):
        n, blk, bsz, nh = (int(x) for x in pre[f"c{ci}_meta"])
        m = OP.blockmask_from_coords(pre[f"c{ci}_rows"], pre[f"c{ci}_cols"], n, blk, bsz, nh)
        assert m.dtype == bool and m.shape == pre[f"c{ci}_mask_plain"].shape
        assert np.array_equal(m, pre[f"c{ci}_mask_plain"])


def test_update_idx_perm_and_permuted_mask_bitexact(pre):
    for ci in _cases(pre):
        n, blk, bsz, nh = (int(x) for x in pre[f"c{ci}_meta"])
        rn = OP.update_idx_perm(pre[f"c{ci}_r_in"], pre[f"c{ci}_perm_r"])
        cn = OP.update_idx_perm(pre[f"c{ci}_c_in"], pre[f"c{ci}_perm_c"])
        assert np.array_equal(rn, pre[f"c{ci}_r_new"])
        assert np.array_equal(cn, pre[f"c{ci}_c_new"])
        m = OP.blockmask_from_coords(rn, cn, n, blk, bsz, nh)
        assert np.array_equal(m, pre[f"c{ci}_mask_perm"])


def test_apply_and_reverse_reordering_bitexact(pre):
    for ci in _cases(pre):
        x, p = pre[f"c{ci}_x"], pre[f"c{ci}_perm_r"]
        assert np.array_equal(OP.apply_reordering(x, p, 2), pre[f"c{ci}_applied"])
        assert np.array_equal(OP.reverse_reordering(x, p, 2), pre[f"c{ci}_reversed"])
        # round trip
        assert np.array_equal(OP.reverse_reordering(OP.apply_reordering(x, p, 2), p, 2), x)


def test_is_permutation():
    assert OP.is_permutation([2, 0, 1])
    assert not OP.is_permutation([0, 0, 1])
    assert not OP.is_permutation([0, 3, 1])
    assert OP.is_permutation([])


def test_attention_oracles_against_reference_kernels(att):
    for name in att["names"]:
        B, H, N, D, BL = (int(x) for x in att[f"{name}_meta"])
        q, k, v, m = (att[f"{name}_{t}"] for t in ("q", "k", "v", "mask"))
        qp = att[f"{name}_q_perm"] if f"{name}_q_perm" in att else None
        kp = att[f"{name}_kv_perm"] if f"{name}_kv_perm" in att else None
        ref_o = att[f"{name}_o"].astype(np.float64)
        ref_M = att[f"{name}_M"]
        o, lse = OA.reordered_attention(q, k, v, m, BL, qp, kp)
        fin = np.isfinite(ref_M)
        assert np.array_equal(np.isfinite(lse), fin), name
        # the reference stores O in fp16: half an ulp at |o| < 1 is < 5e-4
        assert np.abs(o - ref_o).max() < 1e-3, name
        assert np.abs(lse[fin] - ref_M[fin]).max() < 1e-4, name
        # rows with no kept block: O = 0 exactly in both
        assert np.all(ref_o[~fin] == 0) and np.all(o[~fin] == 0)
        if qp is None:
            o2, M2 = OA.block_sparse_online(q, k, v, m, BL, p_dtype="float16")
            assert np.abs(o2 - ref_o).max() < 1e-3, name
            assert np.abs(M2[fin] - ref_M[fin]).max() < 1e-5, name
            o3, M3 = OA.block_sparse_online_batched(q, k, v, m, BL, p_dtype="float16")
            assert np.abs(o3 - o2).max() < 1e-5, name
            assert np.abs(M3[fin] - M2[fin]).max() < 1e-5, name


def test_tile_csr_matches_mask():
    rng = np.random.default_rng(0)
    for block, nb in ((128, 8), (64, 9), (64, 8)):
        m = rng.random((3, nb, nb)) < 0.3
        ptr, col = OP.tile_csr(m, block)
        rpt = 128 // block
        T = (nb + rpt - 1) // rpt
        assert ptr.shape == (3 * T + 1,)
        for s in range(3):
            for t in range(T):
                ents = col[ptr[s * T + t]:ptr[s * T + t + 1]]
                kb = ents & 0xFFFFFF
                fl = ents >> 24
                assert np.all(np.diff(kb) > 0)
                for r in range(rpt):
                    br = t * rpt + r
                    want = np.nonzero(m[s, br])[0] if br < nb else np.array([], dtype=np.int64)
                    bit = 1 if block == 128 else (1 << r)
                    assert np.array_equal(kb[(fl & bit) != 0], want)
