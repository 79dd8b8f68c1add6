"""One backward pass (dq, dk, dv) of a benchmark workload, for profiler captures.

    python -m blocksparsefa_reorder_b200.profile_bwd [--workload headline] [--reps 3]

Builds the forward's plan and the transposed plan, runs the forward once for
o / lse, then ``--reps`` backward calls (Delta, dQ and dK/dV kernels) on the
current stream and prints their mean device time.
"""

from __future__ import annotations

import argparse


def main(argv=None):
    import torch

    from . import BlockSparsePlan, block_sparse_attention, block_sparse_attention_backward, transposed_plan
    from . import workloads as W

    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--workload", default="headline")
    ap.add_argument("--reps", type=int, default=3)
    args = ap.parse_args(argv)
    dev = torch.device("cuda", 0)
    wl = W.make(args.workload)
    q, k, v = wl.make_qkv(dev)
    g = torch.Generator(device="cpu").manual_seed(wl.seed + 7)
    dout = torch.randn(q.shape, generator=g).to(q.dtype).to(dev)
    m = wl.mask_tensor(dev)
    plan = BlockSparsePlan(m, wl.block)
    plan_t = transposed_plan(plan, m)
    o, lse = block_sparse_attention(q, k, v, plan=plan, return_lse=True, kernel="tcgen05")
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.reps):
        block_sparse_attention_backward(q, k, v, o, lse, dout, plan=plan, plan_t=plan_t)
    e1.record()
    torch.cuda.synchronize()
    print(f"{wl.name}: backward {e0.elapsed_time(e1) / args.reps:.3f} ms per call ({args.reps} calls)")


if __name__ == "__main__":
    main()
