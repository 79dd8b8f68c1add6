"""Parity of the CUDA attention forward (tcgen05 and SIMT kernels) against the
CPU oracle and against the reference kernels' own outputs (golden vectors).

Tolerances (fixed by the parity spec): max |err| <= 2e-2 for bf16 / fp16
against the float64 masked-softmax definition, <= 1e-5 for fp32; exactly
zero contribution from key blocks outside the mask.
"""

import math

import numpy as np
import pytest
import torch

from blocksparsefa_reorder_b200 import BlockSparsePlan, block_sparse_attention
from blocksparsefa_reorder_b200 import kernels as K
from blocksparsefa_reorder_b200 import workloads as W
from oracle import attention as OA

pytestmark = pytest.mark.gpu

TOL_16 = 2e-2
TOL_32 = 1e-5
TOL_LSE = 2e-2


def _rand_mask(nb, p, seed, shape=(1, 1), empty_rows=()):
    rng = np.random.default_rng(seed)
    m = rng.random(shape + (nb, nb)) < p
    idx = np.arange(nb)
    m[..., idx, idx] = True
    for r in empty_rows:
        m[..., r, :] = False
    return m


def _qkv(B, H, N, D, dtype, seed, dev, scale=1.0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    ts = [(torch.randn(B, H, N, D, generator=g) * scale).to(dtype) for _ in range(3)]
    return [t.to(dev) for t in ts]


def _oracle(q, k, v, mask, block, q_perm=None, kv_perm=None, sm_scale=None):
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    qp = None if q_perm is None else q_perm.cpu().numpy()
    kp = None if kv_perm is None else kv_perm.cpu().numpy()
    return OA.reordered_attention(f(q), f(k), f(v), mask, block, qp, kp, sm_scale)


def _maxerr(o, ref):
    return float(np.abs(o.float().cpu().numpy().astype(np.float64) - ref).max())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("block", [128, 64])
def test_tcgen05_matches_oracle(dev, dtype, D, block):
    B, H, N = 1, 2, 1024
    nb = N // block
    mask = _rand_mask(nb, 0.3, seed=D + block, shape=(1, H), empty_rows=(3,))
    q, k, v = _qkv(B, H, N, D, dtype, seed=7, dev=dev)
    o, lse = block_sparse_attention(q, k, v, torch.from_numpy(mask).to(dev), return_lse=True, kernel="tcgen05",
                                    check_errors=True)
    ref, ref_lse = _oracle(q, k, v, mask, block)
    assert _maxerr(o, ref) <= TOL_16
    lv = lse.cpu().numpy()
    fin = np.isfinite(ref_lse)
    assert np.array_equal(np.isfinite(lv), fin)
    assert np.abs(lv[fin] - ref_lse[fin]).max() <= TOL_LSE
    # the empty block row gives exactly zero and lse = -inf
    assert torch.count_nonzero(o[:, :, 3 * block:4 * block]) == 0
    assert np.all(np.isneginf(lv[:, :, 3 * block:4 * block]))


@pytest.mark.parametrize("D,block", [(64, 64), (128, 64), (64, 128), (128, 128)])
def test_tcgen05_repeatable(dev, D, block):
    """Pipeline races show up as run-to-run differences: 25 runs of the same
    call into NaN-prefilled outputs must be bitwise identical and in tolerance.
    The masks include tiles whose trailing key blocks are kept by only one of
    the two block rows of a 128-row tile (BLOCK 64), the pattern that exposed
    an epilogue ordering bug."""
    B, H, N = 1, 2, 1024
    mask = _rand_mask(N // block, 0.3, seed=D + block, shape=(1, H), empty_rows=(3,))
    q, k, v = _qkv(B, H, N, D, torch.bfloat16, seed=7, dev=dev)
    plan = BlockSparsePlan(torch.from_numpy(mask).to(dev), block)
    ref, _ = _oracle(q, k, v, mask, block)
    first = None
    for _ in range(25):
        o = torch.full_like(q, float("nan"))
        block_sparse_attention(q, k, v, plan=plan, kernel="tcgen05", out=o)
        if first is None:
            first = o.clone()
            assert _maxerr(first, ref) <= TOL_16
        assert torch.equal(o, first)


def test_fp32_simt_plumbing_config(dev):
    wl = W.make("plumbing")
    q, k, v = wl.make_qkv(dev)
    o = block_sparse_attention(q, k, v, wl.mask_tensor(dev), block=wl.block, check_errors=True)
    ref, _ = _oracle(q, k, v, wl.mask[None, None], wl.block)
    assert _maxerr(o, ref) <= TOL_32


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_permuted_path_matches_oracle(dev, dtype):
    B, H, N, D, block = 2, 2, 1024, 128, 128
    nb = N // block
    mask = _rand_mask(nb, 0.4, seed=5)
    q, k, v = _qkv(B, H, N, D, dtype, seed=9, dev=dev)
    g = torch.Generator().manual_seed(3)
    qp = torch.randperm(N, generator=g).to(dev)
    kp = torch.randperm(N, generator=g).to(dev)
    o, lse = block_sparse_attention(q, k, v, torch.from_numpy(mask).to(dev), q_perm=qp, kv_perm=kp,
                                    return_lse=True, check_errors=True)
    ref, ref_lse = _oracle(q, k, v, mask, block, qp, kp)
    assert _maxerr(o, ref) <= TOL_16
    assert np.abs(lse.cpu().numpy() - ref_lse).max() <= TOL_LSE


@pytest.mark.parametrize("which", ["q", "kv", "both"])
@pytest.mark.parametrize("D,block,N,idx", [(128, 128, 1024, torch.int64), (64, 64, 64 * 13, torch.int32),
                                           (128, 64, 64 * 9, torch.int64), (128, 128, 1000, torch.int32),
                                           (64, 64, 64 * 7 + 40, torch.int64)])
def test_fused_permutation(dev, which, D, block, N, idx):
    """The reordered forward on the tcgen05 path gathers Q rows and scatters
    O / lse rows through q_perm inside the attention kernel (K and V are
    permuted beforehand): every combination of permutations, BLOCK 64 with a
    partial last 128-row tile, N not a multiple of BLOCK (a partial last key
    block), int32 and int64 permutations, NaN-prefilled outputs, against the oracle's reordered attention (BlockSparse_Fused.py
    semantics: mask in the new order, output in the original order)."""
    B, H = 2, 2
    nb = (N + block - 1) // block
    mask = _rand_mask(nb, 0.35, seed=D + N, shape=(1, H), empty_rows=(1,))
    q, k, v = _qkv(B, H, N, D, torch.bfloat16, seed=N, dev=dev)
    g = torch.Generator().manual_seed(N + D)
    qp = torch.randperm(N, generator=g).to(idx).to(dev) if which in ("q", "both") else None
    kp = torch.randperm(N, generator=g).to(idx).to(dev) if which in ("kv", "both") else None
    o = torch.full_like(q, float("nan"))
    lse = torch.full((B, H, N), float("nan"), device=dev)
    o, lse = block_sparse_attention(q, k, v, torch.from_numpy(mask).to(dev), q_perm=qp, kv_perm=kp, return_lse=True,
                                    out=o, lse_out=lse, kernel="tcgen05", check_errors=True)
    ref, ref_lse = _oracle(q, k, v, mask, block, qp, kp)
    assert _maxerr(o, ref) <= TOL_16
    lv = lse.cpu().numpy()
    fin = np.isfinite(ref_lse)
    assert np.array_equal(np.isfinite(lv), fin)
    assert np.abs(lv[fin] - ref_lse[fin]).max() <= TOL_LSE


def test_fused_permutation_out_of_range_flagged(dev):
    """A query permutation value outside [0, N) is reported through the error
    word (the row is not read or written), not read out of bounds."""
    B, H, N, D, block = 1, 1, 512, 128, 128
    mask = _rand_mask(N // block, 0.5, seed=1)
    q, k, v = _qkv(B, H, N, D, torch.bfloat16, seed=2, dev=dev)
    qp = torch.arange(N, device=dev)
    qp[7] = N + 5
    with pytest.raises(RuntimeError, match="permutation value out of range"):
        block_sparse_attention(q, k, v, torch.from_numpy(mask).to(dev), q_perm=qp, kernel="tcgen05",
                               check_errors=True)


def test_golden_reference_kernels(dev, golden_dir):
    """Our kernels against the reference Triton kernels' outputs, through the
    kernel-level drop-ins called like the reference runners call Triton."""
    g = np.load(golden_dir / "attention_golden.npz")
    for name in g["names"]:
        B, H, N, D, BL = (int(x) for x in g[f"{name}_meta"])
        q, k, v = (torch.from_numpy(g[f"{name}_{t}"]).to(dev) for t in "qkv")
        bm = torch.from_numpy(g[f"{name}_mask"]).to(dev)
        M = torch.empty(B, H, N, dtype=torch.float32, device=dev)
        o = torch.empty_like(q)
        sc = 1.0 / math.sqrt(D)
        if f"{name}_q_perm" in g:
            qp = torch.from_numpy(g[f"{name}_q_perm"]).to(dev)
            kp = torch.from_numpy(g[f"{name}_kv_perm"]).to(dev)
            rp = qp.view(1, 1, N, 1).expand(B, H, N, D)
            cp = kp.view(1, 1, N, 1).expand(B, H, N, D)
            K.attn_fwd_block_sparse_perm(sc, M, B, H, q, k, v, o, bm, N_CTX=N, q_perm=rp, kv_perm=cp, HEAD_DIM=D,
                                         BLOCK_M=BL, BLOCK_N=BL, STAGE=1, warp_specialize=False, IS_HOPPER=False,
                                         num_warps=4, num_stages=3)
        else:
            K.attn_fwd_block_sparse(sc, M, B, H, q, k, v, o, bm, N_CTX=N, HEAD_DIM=D, BLOCK_M=BL, BLOCK_N=BL,
                                    STAGE=1, warp_specialize=False, IS_HOPPER=False, num_warps=4, num_stages=3)
        ref_o = g[f"{name}_o"].astype(np.float64)
        ref_M = g[f"{name}_M"]
        assert np.abs(o.float().cpu().numpy() - ref_o).max() <= TOL_16, name
        m = M.cpu().numpy()
        fin = np.isfinite(ref_M)
        assert np.array_equal(np.isfinite(m), fin), name
        assert np.abs(m[fin] - ref_M[fin]).max() <= TOL_LSE, name


@pytest.mark.parametrize("block,N,p", [(128, 1024, 0.2), (64, 1024, 0.2), (64, 3072, 0.85)])
def test_masked_blocks_contribute_nothing(dev, block, N, p):
    """NaN/Inf-poison every K/V row in key blocks that no query block keeps,
    and perturb them: O must stay finite and bitwise equal.  Then perturb (by
    finite amounts) every key block the first block row does not keep: that
    block row's output must stay bitwise equal, also at BLOCK 64 where the
    perturbed blocks include ones its sibling row in the 128-row tile keeps
    (loaded for the tile, scored and given P = 0 for these rows).  The last
    case is dense enough for the paired BLOCK 64 form."""
    B, H, D = 1, 2, 128
    nb = N // block
    mask = _rand_mask(nb, p, seed=21)
    mask[..., :, nb - 2:] = False
    unused = np.nonzero(~mask[0, 0].any(axis=0))[0]
    assert unused.size > 0
    q, k, v = _qkv(B, H, N, D, torch.bfloat16, seed=4, dev=dev)
    mt = torch.from_numpy(mask).to(dev)
    o1 = block_sparse_attention(q, k, v, mt)
    k2, v2 = k.clone(), v.clone()
    for j in unused:
        k2[:, :, j * block:(j + 1) * block] = float("nan")
        v2[:, :, j * block:(j + 1) * block] = float("inf")
    o2 = block_sparse_attention(q, k2, v2, mt)
    assert torch.isfinite(o2.float()).all()
    assert torch.equal(o1, o2)
    # finite perturbation of every K/V row outside the kept blocks of the
    # first tile row block leaves that block row bitwise unchanged
    k3, v3 = k.clone(), v.clone()
    for j in np.nonzero(~mask[0, 0, 0])[0]:
        k3[:, :, j * block:(j + 1) * block] += 3.0
        v3[:, :, j * block:(j + 1) * block] -= 5.0
    o3 = block_sparse_attention(q, k3, v3, mt)
    assert torch.equal(o1[:, :, :block], o3[:, :, :block])


def test_tcgen05_vs_simt_crosscheck(dev):
    B, H, N, D, block = 1, 2, 2048, 128, 128
    mask = _rand_mask(N // block, 0.25, seed=8)
    q, k, v = _qkv(B, H, N, D, torch.bfloat16, seed=12, dev=dev)
    mt = torch.from_numpy(mask).to(dev)
    a = block_sparse_attention(q, k, v, mt, kernel="tcgen05")
    b = block_sparse_attention(q, k, v, mt, kernel="simt")
    assert (a.float() - b.float()).abs().max().item() <= TOL_16


def test_strided_bnhd_layout(dev):
    """q, k, v as [B, N, H, D] memory viewed as [B, H, N, D] (the layout the
    reference's BSFA runner uses, BlockSparseFA.py:28-34): TMA takes the
    strides directly, no copy."""
    B, H, N, D, block = 2, 3, 512, 64, 128
    mask = _rand_mask(N // block, 0.5, seed=30)
    base = [torch.randn(B, N, H, D, generator=torch.Generator().manual_seed(i)).to(torch.bfloat16).to(dev)
            for i in range(3)]
    q, k, v = (t.permute(0, 2, 1, 3) for t in base)
    o = block_sparse_attention(q, k, v, torch.from_numpy(mask).to(dev), kernel="tcgen05")
    ref, _ = _oracle(q, k, v, mask, block)
    assert _maxerr(o, ref) <= TOL_16


@pytest.mark.parametrize("block", [128, 64])
def test_permutations_on_strided_layout(dev, block):
    """q, k, v as [B, N, H, D] memory viewed as [B, H, N, D] with both
    permutations: K / V are permuted into the workspace (contiguous), Q is
    gathered inside the kernel through its own strides and O / lse scattered
    through q_perm."""
    B, H, N, D = 2, 3, 1024, 128
    mask = _rand_mask(N // block, 0.4, seed=33, shape=(1, H))
    base = [torch.randn(B, N, H, D, generator=torch.Generator().manual_seed(50 + i)).to(torch.bfloat16).to(dev)
            for i in range(3)]
    q, k, v = (t.permute(0, 2, 1, 3) for t in base)
    g = torch.Generator().manual_seed(51)
    qp = torch.randperm(N, generator=g).to(dev)
    kp = torch.randperm(N, generator=g).to(dev)
    o, lse = block_sparse_attention(q, k, v, torch.from_numpy(mask).to(dev), q_perm=qp, kv_perm=kp, return_lse=True,
                                    kernel="tcgen05", check_errors=True)
    ref, ref_lse = _oracle(q, k, v, mask, block, qp, kp)
    assert _maxerr(o, ref) <= TOL_16
    assert np.abs(lse.cpu().numpy() - ref_lse).max() <= TOL_LSE


def test_partial_last_tile(dev):
    """N = 64 * odd with BLOCK 64: the last 128-row tile has one block row;
    TMA zero-fills the missing rows and clips the store."""
    B, H, N, D, block = 1, 2, 64 * 9, 128, 64
    mask = _rand_mask(N // block, 0.4, seed=31, shape=(1, H))
    q, k, v = _qkv(B, H, N, D, torch.float16, seed=3, dev=dev)
    o = block_sparse_attention(q, k, v, torch.from_numpy(mask).to(dev), kernel="tcgen05", check_errors=True)
    ref, _ = _oracle(q, k, v, mask, block)
    assert _maxerr(o, ref) <= TOL_16


def test_per_batch_head_masks(dev):
    B, H, N, D, block = 2, 3, 1024, 128, 128
    mask = _rand_mask(N // block, 0.3, seed=40, shape=(B, H))
    q, k, v = _qkv(B, H, N, D, torch.bfloat16, seed=41, dev=dev)
    o = block_sparse_attention(q, k, v, torch.from_numpy(mask).to(dev), check_errors=True)
    ref, _ = _oracle(q, k, v, mask, block)
    assert _maxerr(o, ref) <= TOL_16


def test_headline_full_size_sampled(dev):
    """Full-size headline workload (B1 H16 N16384 D128 bf16, 10% blocks):
    sampled query blocks against the oracle's block loop; a second run is
    bitwise identical (deterministic)."""
    wl = W.make("headline")
    q, k, v = wl.make_qkv(dev)
    plan = BlockSparsePlan(wl.mask_tensor(dev), wl.block)
    o = block_sparse_attention(q, k, v, plan=plan, check_errors=True)
    o2 = block_sparse_attention(q, k, v, plan=plan)
    assert torch.equal(o, o2)
    heads = [0, 15]
    qblocks = [0, 37, 127]
    sub = lambda t: t[:, heads].float().cpu().numpy()  # noqa: E731
    ref, _ = OA.block_sparse_online(sub(q), sub(k), sub(v), wl.mask[None, None], wl.block, query_blocks=qblocks)
    got = o[:, heads].float().cpu().numpy()
    for mb in qblocks:
        r0, r1 = mb * wl.block, (mb + 1) * wl.block
        assert np.abs(got[:, :, r0:r1] - ref[:, :, r0:r1]).max() <= TOL_16


def _torch_masked_reference(q, k, v, mask, block, sm_scale):
    """fp32 masked softmax attention on the GPU, one (b, h) slice at a time:
    rows with no kept key give O = 0 and lse = -inf."""
    B, H, N, _ = q.shape
    o = torch.zeros(B, H, N, q.shape[-1], dtype=torch.float32, device=q.device)
    lse = torch.full((B, H, N), float("-inf"), dtype=torch.float32, device=q.device)
    mt = torch.from_numpy(mask).to(q.device)
    for b in range(B):
        for h in range(H):
            m = mt[b % mt.shape[0], h % mt.shape[1]]
            full = m.repeat_interleave(block, 0).repeat_interleave(block, 1)[:N, :N]
            s = (q[b, h].float() @ k[b, h].float().T) * sm_scale
            s = s.masked_fill(~full, float("-inf"))
            ls = torch.logsumexp(s, dim=-1)
            p = torch.exp(s - ls[:, None].clamp_min(-1e30))
            p = torch.where(full, p, torch.zeros_like(p))
            o[b, h] = p @ v[b, h].float()
            lse[b, h] = ls / math.log(2.0)  # the API's lse is in log2 units
    return o, lse


@pytest.mark.parametrize("block", [64, 128])
def test_runs_of_empty_tiles(dev, block):
    """Each head keeps key blocks only in its first 128-row tile (many key
    blocks, so that tile has many steps) and every other tile of the head is
    empty, so a CTA claims one long tile and then runs of empty tiles, which
    fill the producer's tile ring without any load: the tile's last V and
    last PV must still be issued while the ring is full (the roles that free
    the ring wait for that tile's output).  No timeout, and O / lse against
    the fp32 reference on sampled heads (the empty rows: O = 0, lse = -inf)."""
    B, H, D = 1, 160, 64
    N = 40 * 128 - 32  # 40 tiles per head, a partial last key block
    nb = (N + block - 1) // block
    mask = np.zeros((1, H, nb, nb), dtype=bool)
    rows = 128 // block
    rng = np.random.default_rng(23)
    mask[0, :, :rows, :] = rng.random((H, rows, nb)) < 0.5
    mask[0, :, :rows, 0] = True
    q, k, v = _qkv(B, H, N, D, torch.bfloat16, seed=24, dev=dev)
    plan = BlockSparsePlan(torch.from_numpy(mask).to(dev), block)
    for _ in range(3):
        o, lse = block_sparse_attention(q, k, v, plan=plan, kernel="tcgen05", return_lse=True, check_errors=True)
    heads = [0, 77, H - 1]
    ref_o, ref_lse = _torch_masked_reference(q[:, heads], k[:, heads], v[:, heads], mask[:, heads], block,
                                             1.0 / math.sqrt(D))
    assert (o[:, heads].float() - ref_o).abs().max().item() <= TOL_16
    fin = torch.isfinite(ref_lse)
    assert torch.equal(torch.isfinite(lse[:, heads]), fin)
    assert (lse[:, heads][fin] - ref_lse[fin]).abs().max().item() <= TOL_LSE
    assert torch.count_nonzero(o[:, :, 128:]) == 0


@pytest.mark.parametrize("D,block", [(64, 64), (128, 64), (64, 128), (128, 128)])
def test_many_tiles_per_cta(dev, D, block):
    """Several times more 128-row tiles than SMs, so each CTA of the
    persistent kernel runs many tiles back to back: per-(b, h) masks with
    empty block rows scattered through them and one head with no kept block
    at all, a partial last tile, NaN-prefilled outputs, lse checked, and three
    runs bitwise identical."""
    B, H, N = 2, 8, 4096 - 64
    nb = (N + block - 1) // block
    mask = _rand_mask(nb, 0.2, seed=D * 7 + block, shape=(B, H))
    rng = np.random.default_rng(D + block)
    for r in rng.choice(nb, size=nb // 4, replace=False):
        mask[rng.integers(B), rng.integers(H), r, :] = False
    mask[1, 5] = False
    q, k, v = _qkv(B, H, N, D, torch.bfloat16, seed=D + block, dev=dev)
    plan = BlockSparsePlan(torch.from_numpy(mask).to(dev), block)
    scale = 1.0 / math.sqrt(D)
    ref_o, ref_lse = _torch_masked_reference(q, k, v, mask, block, scale)
    first = None
    for _ in range(3):
        o = torch.full_like(q, float("nan"))
        o, lse = block_sparse_attention(q, k, v, plan=plan, kernel="tcgen05", return_lse=True, out=o,
                                        check_errors=True)
        if first is None:
            first = (o.clone(), lse.clone())
            assert (o.float() - ref_o).abs().max().item() <= TOL_16
            fin = torch.isfinite(ref_lse)
            assert torch.equal(torch.isfinite(lse), fin)
            assert (lse[fin] - ref_lse[fin]).abs().max().item() <= TOL_LSE
            assert torch.count_nonzero(o[1, 5]) == 0
        assert torch.equal(o, first[0]) and torch.equal(lse, first[1])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("D,block", [(64, 64), (128, 64), (64, 128), (128, 128)])
def test_reference_point_guard(dev, D, block, dtype):
    """The kernels take a row's softmax reference point from its first kept
    block and redo a block with the exact max only when its sum leaves the
    slack: keys of one later block scaled by 30 force that path (scores ~40
    log2 units above the reference: past fp16's range for P without the redo),
    and an earlier block scaled down makes the first reference point low.
    Checked against the float64 oracle, O and lse, with finite outputs."""
    B, H, N = 1, 2, 1024
    nb = N // block
    mask = _rand_mask(nb, 0.6, seed=D + block + 3, shape=(1, H))
    mask[..., :, nb - 2] = True
    q, k, v = _qkv(B, H, N, D, dtype, seed=D + block, dev=dev)
    k[:, :, (nb - 2) * block:(nb - 1) * block] *= 30
    k[:, :, :block] *= 0.1
    o, lse = block_sparse_attention(q, k, v, torch.from_numpy(mask).to(dev), return_lse=True, kernel="tcgen05",
                                    check_errors=True)
    assert torch.isfinite(o.float()).all()
    ref, ref_lse = _oracle(q, k, v, mask, block)
    assert _maxerr(o, ref) <= TOL_16
    lv = lse.cpu().numpy()
    fin = np.isfinite(ref_lse)
    assert np.array_equal(np.isfinite(lv), fin)
    assert np.abs(lv[fin] - ref_lse[fin]).max() <= TOL_LSE * max(1.0, float(np.abs(ref_lse[fin]).max()) / 8)


def test_concurrent_streams(dev):
    """Forwards running at the same time on different streams: each launch
    claims tiles from its own work-counter slot, so every result equals the
    one computed alone (bitwise), also when the launches are repeated many
    times (slots are reused after 64 launches)."""
    B, H, N, D, block = 1, 4, 2048, 128, 128
    nb = N // block
    masks = [_rand_mask(nb, 0.2 + 0.1 * i, seed=60 + i, shape=(1, H)) for i in range(4)]
    qkv = [_qkv(B, H, N, D, torch.bfloat16, seed=70 + i, dev=dev) for i in range(4)]
    plans = [BlockSparsePlan(torch.from_numpy(m).to(dev), block) for m in masks]
    alone = []
    for (q, k, v), plan in zip(qkv, plans):
        alone.append(block_sparse_attention(q, k, v, plan=plan, kernel="tcgen05"))
    torch.cuda.synchronize()
    streams = [torch.cuda.Stream(dev) for _ in range(4)]
    outs = [torch.full_like(qkv[i][0], float("nan")) for i in range(4)]
    for _ in range(40):
        for i, st in enumerate(streams):
            st.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(st):
                q, k, v = qkv[i]
                block_sparse_attention(q, k, v, plan=plans[i], kernel="tcgen05", out=outs[i])
        torch.cuda.synchronize()
        for i in range(4):
            assert torch.equal(outs[i], alone[i])


def test_long_context_sampled(dev):
    """The long-context shape at full length (N = 65536, 512 block rows: the
    mask is 256 KiB, so the plan takes the multi-kernel path, and each head has
    512 tiles of ~72 kept blocks), two heads: sampled query blocks against the
    oracle's block loop, lse included."""
    wl = W.make("longctx")
    q, k, v = (t[:, :2].contiguous() for t in wl.make_qkv(dev))
    plan = BlockSparsePlan(wl.mask_tensor(dev), wl.block)
    o, lse = block_sparse_attention(q, k, v, plan=plan, return_lse=True, check_errors=True)
    qblocks = [0, 257, 511]
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    ref, ref_lse = OA.block_sparse_online(f(q), f(k), f(v), wl.mask[None, None], wl.block, query_blocks=qblocks)
    got, gl = o.float().cpu().numpy(), lse.cpu().numpy()
    for mb in qblocks:
        r0, r1 = mb * wl.block, (mb + 1) * wl.block
        assert np.abs(got[:, :, r0:r1] - ref[:, :, r0:r1]).max() <= TOL_16
        assert np.abs(gl[:, :, r0:r1] - ref_lse[:, :, r0:r1]).max() <= TOL_LSE


@pytest.mark.parametrize("density,paired", [(0.05, False), (0.3, True)])
@pytest.mark.parametrize("D", [64, 128])
def test_block64_forms_edges(dev, D, density, paired):
    """BLOCK 64 with a sparse plan (tiles average fewer than 4 kept blocks:
    the form that runs one kept block per step is selected) and a denser one
    (the paired form): tiles with an odd number of kept blocks, blocks kept by
    only one of the tile's two query block rows, a tile whose rows keep
    disjoint blocks, a partial last key block (N % 64 != 0), and key blocks no
    query keeps filled with NaN."""
    B, H, block = 1, 3, 64
    N = 64 * 13 + 23
    nb = (N + block - 1) // block
    rng = np.random.default_rng(D)
    mask = rng.random((1, H, nb, nb)) < density
    mask[..., np.arange(nb), np.arange(nb)] = True
    mask[:, 0, 2, :] = False                       # rows 2 and 3 (one tile) keep disjoint blocks
    mask[:, 0, 3, :] = False
    mask[:, 0, 2, [0, 5, 9]] = True
    mask[:, 0, 3, [1, 4, 13]] = True
    mask[:, 1, 4, :] = False                       # row 4 keeps only the partial last block,
    mask[:, 1, 4, nb - 1] = True                   # row 5 keeps three blocks: odd count in the tile
    mask[:, 1, 5, :] = False
    mask[:, 1, 5, [0, 7, nb - 1]] = True
    mask[:, 2, :, 11] = False                      # head 2: block 11 kept by nobody -> NaN keys and values
    q, k, v = _qkv(B, H, N, D, torch.bfloat16, seed=D + 5, dev=dev)
    k[:, 2, 11 * block:12 * block] = float("nan")
    v[:, 2, 11 * block:12 * block] = float("nan")
    plan = BlockSparsePlan(torch.from_numpy(mask).to(dev), block)
    # the form the kernels select from the plan's entry total (4 per tile)
    assert (plan.nnz_entries() >= 4 * plan.mask_b * plan.mask_h * plan.tiles_per_row) == paired
    o, lse = block_sparse_attention(q, k, v, plan=plan, kernel="tcgen05", return_lse=True, check_errors=True)
    kc, vc = k.clone(), v.clone()
    kc[:, 2, 11 * block:12 * block] = 0
    vc[:, 2, 11 * block:12 * block] = 0
    ref_o, ref_lse = _torch_masked_reference(q, kc, vc, mask, block, 1.0 / math.sqrt(D))
    assert torch.isfinite(o).all()
    assert (o.float() - ref_o).abs().max().item() <= TOL_16
    fin = torch.isfinite(ref_lse)
    assert torch.equal(torch.isfinite(lse), fin)
    assert (lse[fin] - ref_lse[fin]).abs().max().item() <= TOL_LSE
