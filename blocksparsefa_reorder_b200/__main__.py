"""Command line with the reference's ``main.py`` interface (``main.py:102-167``).

    python -m blocksparsefa_reorder_b200 pattern.mtx [--block-size 128] [--head-dim 128]
        [--num-heads 1] [--row-reorder rows.txt] [--col-reorder cols.txt] [--mode B200]

Same positional pattern file, options, defaults and argument checks as the
reference; ``--mode B200`` (the default here) runs this library: read the
pattern (``read_mtx``), read the permutations, build the block mask on the GPU
with the coordinates moved to their new positions (``update_idx_perm`` fused
into the mask build, ``main.py:27-49, 54-63``), then time the forward with
and without reordering and print the reference runner's lines
(``run_experiments_B200``).  The reference's other modes run its comparator
backends (BSFA, FlexAttention, its Triton kernels), which this library does not
include.  Deliberate difference: ``--num-heads`` may exceed 1 (the kernels
take any number of heads; the reference refuses values other than 1).
"""

from __future__ import annotations

import argparse
from pathlib import Path
from typing import Optional

REFERENCE_MODES = ("BSFA", "BSFlexAttention", "BSTF", "BSTN")


def _positive_int(x: str) -> int:
    v = int(x)
    if v <= 0:
        raise argparse.ArgumentTypeError("must be a positive integer")
    return v


def parse_args(argv: Optional[list] = None):
    from .utils import Args

    p = argparse.ArgumentParser(prog="python -m blocksparsefa_reorder_b200",
                                description="Sparse attention matrix reordering test (MTX input).")
    p.add_argument("matrix_mtx", type=Path, help="Input sparse attention matrix in Matrix Market (.mtx) format.")
    p.add_argument("--block-size", type=_positive_int, default=128, help="Block size: 64 or 128 (default: 128).")
    p.add_argument("--head-dim", type=_positive_int, default=128, help="Head dimension (default: 128).")
    p.add_argument("--num-heads", type=_positive_int, default=1, help="Number of heads (default: 1).")
    p.add_argument("--row-reorder", type=Path, default=None,
                   help="Optional input file for row reorderings (default: None).")
    p.add_argument("--col-reorder", type=Path, default=None,
                   help="Optional input file for column reorderings (default: None).")
    p.add_argument("--mode", type=str, choices=["B200", *REFERENCE_MODES], default="B200",
                   help="Attention backend (default: B200, this library).")
    ns = p.parse_args(argv)
    if ns.matrix_mtx.suffix.lower() != ".mtx":
        p.error("Input matrix file must have .mtx extension.")
    if ns.mode in REFERENCE_MODES:
        p.error(f"--mode {ns.mode} runs one of the reference's comparator backends, which this library does not "
                "include; use --mode B200")
    if ns.block_size not in (64, 128):
        p.error("--block-size must be 64 or 128 for the B200 kernels.")
    return Args(matrix_mtx=ns.matrix_mtx, block_size=ns.block_size, head_dim=ns.head_dim, num_heads=ns.num_heads,
                row_reorder=ns.row_reorder, col_reorder=ns.col_reorder, mode=ns.mode)


def run_sparse_attention_reordering_test(args, device: str = "cuda:0") -> None:
    """The reference's driver (``main.py:19-96``) for the B200 backend."""
    from .runners import run_experiments_B200
    from .utils import generate_blockmask_from_mtx_coords, read_mtx, read_reordering_file_to_tensor

    rows_idx, cols_idx, seq_len = read_mtx(str(args.matrix_mtx))
    row_perm = (read_reordering_file_to_tensor(str(args.row_reorder), device=device, zero_based=None)
                if args.row_reorder is not None else None)
    col_perm = (read_reordering_file_to_tensor(str(args.col_reorder), device=device, zero_based=None)
                if args.col_reorder is not None else None)
    block_mask, seq_len = generate_blockmask_from_mtx_coords(
        rows_idx, cols_idx, seq_len, args.block_size, batch_size=1, nheads=args.num_heads, device=device,
        row_perm=row_perm, col_perm=col_perm)
    run_experiments_B200(args, block_mask, seq_len, row_perm=row_perm, col_perm=col_perm, device=device)


def main(argv: Optional[list] = None) -> int:
    run_sparse_attention_reordering_test(parse_args(argv))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
