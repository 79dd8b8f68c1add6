"""Generate the golden vectors that pin the CPU oracle to the reference.

Run on a machine that has the reference checkout (read-only is enough):

    python tests/golden/make_golden.py --reference <path of the reference checkout>

It imports the reference's own code from that checkout and records its
outputs on small seeded inputs:

* ``utils.py`` (run on CPU; the unconditional ``import block_sparse_attn`` at
  ``utils.py:4`` is satisfied with an empty stub module):
  ``generate_blockmask_from_mtx_coords``, ``update_idx_perm``,
  ``apply_reordering``, ``reverse_reordering``, ``read_mtx`` and
  ``read_reordering_file_to_tensor`` (valid files and every error branch).
* ``triton_kernels/BlockSparse_Naive.py`` and ``BlockSparse_Fused.py`` run on
  CPU tensors under ``TRITON_INTERPRET=1``, launched the way the runners
  launch them (``BlockSparseTriton_Naive.py:99-113``,
  ``BlockSparseTriton_Fused.py:95-111``), fp16 only (the only dtype they
  compile for).

Outputs (committed): ``preprocess_golden.npz``, ``reorder_files.json``,
``attention_golden.npz``.  Nothing at test time reads the reference.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import sys
import tempfile
import types
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

HERE = Path(__file__).resolve().parent


def _import_reference(ref: Path):
    sys.path.insert(0, str(ref))
    stub = types.ModuleType("block_sparse_attn")
    stub.block_sparse_attn_func = None
    sys.modules["block_sparse_attn"] = stub
    import utils  # noqa: E402  (reference module)
    from triton_kernels.BlockSparse_Naive import _attn_fwd_block_sparse  # noqa: E402
    from triton_kernels.BlockSparse_Fused import _attn_fwd_block_sparse_perm  # noqa: E402
    return utils, _attn_fwd_block_sparse, _attn_fwd_block_sparse_perm


def make_preprocess(utils, out: dict):
    import numpy as np
    import torch

    rng = np.random.default_rng(1234)
    cases = [
        # (seq_len, block, batch, heads, n_coords, coord_hi)
        (256, 64, 1, 1, 300, 256),
        (200, 64, 2, 3, 400, 270),    # nb = 4; tokens 200..255 keep (block 3), 256..269 drop
        (1000, 128, 1, 2, 2000, 1000),
    ]
    for ci, (n, blk, bsz, nh, nnz, hi) in enumerate(cases):
        rows = rng.integers(0, hi, size=nnz)
        cols = rng.integers(0, hi, size=nnz)
        perm_r = rng.permutation(n)
        perm_c = rng.permutation(n)
        # coordinates outside [0, n) cannot be remapped through a permutation
        # of length n; remap only the in-range ones, as main.py would.
        inr = (rows < n) & (cols < n)
        r_in, c_in = rows[inr], cols[inr]
        r_new = utils.update_idx_perm(r_in, torch.from_numpy(perm_r))
        c_new = utils.update_idx_perm(c_in, torch.from_numpy(perm_c))
        mask_plain, _ = utils.generate_blockmask_from_mtx_coords(rows, cols, n, blk, bsz, nh, device="cpu")
        mask_perm, _ = utils.generate_blockmask_from_mtx_coords(r_new, c_new, n, blk, bsz, nh, device="cpu")
        x = rng.standard_normal((bsz, nh, n, 8)).astype(np.float32)
        xt = torch.from_numpy(x)
        pr = torch.from_numpy(perm_r)
        applied = utils.apply_reordering(xt, pr, dim=2).numpy()
        reversed_ = utils.reverse_reordering(xt, pr, dim=2).numpy()
        out.update({
            f"c{ci}_meta": np.array([n, blk, bsz, nh], dtype=np.int64),
            f"c{ci}_rows": rows, f"c{ci}_cols": cols,
            f"c{ci}_perm_r": perm_r, f"c{ci}_perm_c": perm_c,
            f"c{ci}_r_in": r_in, f"c{ci}_c_in": c_in,
            f"c{ci}_r_new": np.asarray(r_new), f"c{ci}_c_new": np.asarray(c_new),
            f"c{ci}_mask_plain": mask_plain.numpy(), f"c{ci}_mask_perm": mask_perm.numpy(),
            f"c{ci}_x": x, f"c{ci}_applied": applied, f"c{ci}_reversed": reversed_,
        })
    out["n_cases"] = np.array(len(cases))


def make_reorder_files(utils) -> dict:
    """Text files for ``read_reordering_file_to_tensor`` / ``read_mtx`` and
    what the reference returns (or raises) for each."""
    files = {
        "zero_based.txt": "5\n3\n0\n4\n1\n2\n",
        "one_based.txt": "5\n3\n1\n5\n2\n4\n",
        "comments_blank.txt": "# a permutation\n\n4\n  2\n# mid comment\n0\n3\n\n1\n",
        "forced_zero.txt": "3\n1\n2\n3\n",
        "empty.txt": "\n# nothing\n",
        "bad_header.txt": "four\n1\n2\n",
        "negative_n.txt": "-1\n",
        "count_mismatch.txt": "4\n0\n1\n2\n",
        "non_int.txt": "3\n0\n1.5\n2\n",
        "duplicates.txt": "4\n0\n1\n1\n3\n",
        "out_of_range.txt": "3\n0\n1\n7\n",
        "negative_after_base.txt": "3\n-2\n0\n1\n",
        "n_zero.txt": "0\n",
    }
    zero_based_arg = {"forced_zero.txt": True}
    result = {"perm_files": {}, "mtx": {}}
    with tempfile.TemporaryDirectory() as td:
        for name, text in files.items():
            p = Path(td) / name
            p.write_text(text)
            entry = {"text": text, "zero_based": zero_based_arg.get(name)}
            try:
                perm = utils.read_reordering_file_to_tensor(p, zero_based=zero_based_arg.get(name))
                entry["ok"] = True
                entry["perm"] = perm.tolist()
            except ValueError as e:
                entry["ok"] = False
                entry["error"] = str(e).replace(str(p), "<path>")
            result["perm_files"][name] = entry
        mtx_files = {
            "small.mtx": "6 6 5\n1 1\n2 3\n6 6\n4 2\n5 5\n",
            "single.mtx": "3 3 1\n2 3\n",
        }
        for name, text in mtx_files.items():
            p = Path(td) / name
            p.write_text(text)
            r, c, n = utils.read_mtx(str(p))
            result["mtx"][name] = {"text": text, "rows": [int(x) for x in r], "cols": [int(x) for x in c],
                                   "seq_len": int(n)}
    return result


def make_attention(naive, fused, out: dict):
    import numpy as np
    import torch

    def mask(bsz, nh, nb, p, seed, empty_row=None):
        g = torch.Generator().manual_seed(seed)
        m = torch.rand(bsz, nh, nb, nb, generator=g) < p
        m |= torch.eye(nb, dtype=torch.bool)
        if empty_row is not None:
            m[:, :, empty_row, :] = False
        return m

    # (name, B, H, N, D, BLOCK, kind, mask-p, empty block row)
    cases = [
        ("naive_a", 1, 1, 256, 64, 64, "naive", 0.4, 2),
        ("naive_b", 2, 2, 256, 64, 64, "naive", 0.5, None),
        ("naive_c", 1, 1, 256, 128, 64, "naive", 0.3, 1),
        ("naive_d", 1, 2, 256, 128, 128, "naive", 0.5, None),
        ("fused_a", 1, 1, 256, 64, 64, "fused", 0.4, 3),
        ("fused_b", 1, 1, 256, 128, 128, "fused", 0.5, None),
    ]
    names = []
    for ci, (name, B, H, N, D, BL, kind, p, er) in enumerate(cases):
        torch.manual_seed(100 + ci)
        q, k, v = [torch.randn(B, H, N, D, dtype=torch.float16) for _ in range(3)]
        nb = N // BL
        bm = mask(B, H, nb, p, 7 + ci, er)
        M = torch.empty(B, H, N, dtype=torch.float32)
        o = torch.empty_like(q)
        grid = (N // BL, B * H, 1)
        sc = 1.0 / math.sqrt(D)
        rec = {}
        if kind == "naive":
            naive[grid](sc, M, B, H, q, k, v, o, bm, N_CTX=N, HEAD_DIM=D, BLOCK_M=BL, BLOCK_N=BL,
                        STAGE=1, warp_specialize=False, IS_HOPPER=False, num_warps=4, num_stages=3)
        else:
            g = torch.Generator().manual_seed(55 + ci)
            q_perm = torch.randperm(N, generator=g)
            kv_perm = torch.randperm(N, generator=g)
            rp = q_perm.view(1, 1, N, 1).expand(B, H, N, D)
            cp = kv_perm.view(1, 1, N, 1).expand(B, H, N, D)
            fused[grid](sc, M, B, H, q, k, v, o, bm, N_CTX=N, q_perm=rp, kv_perm=cp, HEAD_DIM=D,
                        BLOCK_M=BL, BLOCK_N=BL, STAGE=1, warp_specialize=False, IS_HOPPER=False,
                        num_warps=4, num_stages=3)
            rec["q_perm"] = q_perm.numpy()
            rec["kv_perm"] = kv_perm.numpy()
        rec.update({"meta": np.array([B, H, N, D, BL], dtype=np.int64), "q": q.numpy(), "k": k.numpy(),
                    "v": v.numpy(), "mask": bm.numpy(), "o": o.numpy(), "M": M.numpy()})
        for key, val in rec.items():
            out[f"{name}_{key}"] = val
        names.append(name)
    out["names"] = np.array(names)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", type=Path, required=True, help="path of the reference checkout")
    args = ap.parse_args()
    import numpy as np

    utils, naive, fused = _import_reference(args.reference)
    pre = {}
    make_preprocess(utils, pre)
    np.savez_compressed(HERE / "preprocess_golden.npz", **pre)
    files = make_reorder_files(utils)
    (HERE / "reorder_files.json").write_text(json.dumps(files, indent=1, sort_keys=True))
    att = {}
    make_attention(naive, fused, att)
    np.savez_compressed(HERE / "attention_golden.npz", **att)
    print("wrote", sorted(p.name for p in HERE.glob("*.npz")), "and reorder_files.json")


if __name__ == "__main__":
    main()
