"""PyTorch-facing API of the B200 block-sparse attention forward.

PyTorch provides device memory and the current stream; every computation
runs in the CUDA kernels of ``_lib/libbsattn_b200.so`` through the C ABI
(``include/bsattn_b200.h``).  There is no CPU path: CPU tensors are rejected.

The call surface keeps what the reference's runners consume
(``BlockSparseTriton_Naive.py:10-18``): q, k, v ``[B, H, N, D]``, a
BLOCK x BLOCK bool block mask in the permuted (new) token order, optional row
(query) and column (key/value) permutations with ``perm[i]`` = old index that
moves to new position ``i``; the output comes back in the original order.
"""

from __future__ import annotations

import ctypes
import math
from typing import Optional

import torch

from . import _lib

_DTYPES = {torch.float32: _lib.DTYPE_F32, torch.float16: _lib.DTYPE_F16, torch.bfloat16: _lib.DTYPE_BF16}
_KERNELS = {"auto": _lib.KERNEL_AUTO, "simt": _lib.KERNEL_SIMT, "tcgen05": _lib.KERNEL_TCGEN05}


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(t, name: str) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (this library has no CPU path)")


def _t4(t: torch.Tensor) -> _lib.Tensor4d:
    """A [B, H, N, D] view as the C descriptor (innermost stride 1)."""
    if t.stride(3) != 1:
        raise ValueError("the last (head) dimension must be contiguous")
    return _lib.Tensor4d(t.data_ptr(), t.stride(0), t.stride(1), t.stride(2))


def _index_dtype(p: torch.Tensor) -> int:
    if p.dtype == torch.int64:
        return _lib.INDEX_I64
    if p.dtype == torch.int32:
        return _lib.INDEX_I32
    raise TypeError(f"permutation dtype must be int32 or int64, got {p.dtype}")


def _perm_vector(p, n: int, device, name: str) -> Optional[torch.Tensor]:
    """Accept ``[N]`` or the runners' expanded ``[B, H, N, D]`` views."""
    if p is None:
        return None
    if not isinstance(p, torch.Tensor):
        p = torch.as_tensor(p)
    if p.dim() == 4:
        p = p[0, 0, :, 0]
    if p.dim() != 1 or p.shape[0] != n:
        raise ValueError(f"{name} must have shape [N] (N={n}), got {tuple(p.shape)}")
    if p.dtype not in (torch.int32, torch.int64):
        p = p.to(torch.int64)
    return p.to(device).contiguous()


def infer_block(n: int, nb: int) -> int:
    """The BLOCK (64 or 128) for which ``ceil(n / BLOCK) == nb``."""
    for b in (128, 64):
        if (n + b - 1) // b == nb:
            return b
    raise ValueError(f"cannot infer BLOCK from N={n} and {nb} mask blocks (supported BLOCK: 64, 128)")


class BlockSparsePlan:
    """Per-tile list of kept key blocks, built on the GPU from a block mask.

    ``block_mask``: bool (or uint8) CUDA tensor ``[nb, nb]`` or
    ``[1|B, 1|H, nb, nb]``.  The plan replaces the reference kernel's scan of
    every mask byte (``BlockSparse_Naive.py:25-32``) and can be reused across
    calls with the same mask.  It also holds the work order the tcgen05
    kernel hands tiles out in (each slice's tiles by decreasing kept-block
    count).  Building it enqueues one kernel for small masks (four for large
    ones) and does not synchronise.
    """

    def __init__(self, block_mask: torch.Tensor, block: int):
        m = self._as_mask(block_mask)
        self.mask_b, self.mask_h, self.nb = int(m.shape[0]), int(m.shape[1]), int(m.shape[2])
        self.block = int(block)
        self.device = m.device
        L = _lib.lib()
        ptr_len, cap, ws = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_size_t()
        _lib.check(L.bsa_plan_sizes(self.mask_b, self.mask_h, self.nb, self.block, ctypes.byref(ptr_len),
                                    ctypes.byref(cap), ctypes.byref(ws)), "bsa_plan_sizes")
        self.tile_ptr = torch.empty(ptr_len.value, dtype=torch.int32, device=self.device)
        self.tile_col = torch.empty(max(1, cap.value), dtype=torch.int32, device=self.device)
        self._ws_bytes = ws.value
        self._work = torch.empty(max(1, (ws.value + 3) // 4), dtype=torch.int32, device=self.device)
        self.tile_order = torch.empty(max(1, ptr_len.value - 1), dtype=torch.int32, device=self.device)
        self._build(m)

    @staticmethod
    def _as_mask(block_mask: torch.Tensor) -> torch.Tensor:
        _require_cuda(block_mask, "block_mask")
        m = block_mask
        if m.dim() == 2:
            m = m[None, None]
        if m.dim() != 4 or m.shape[-1] != m.shape[-2]:
            raise ValueError(f"block_mask must be [nb, nb] or [B, H, nb, nb], got {tuple(block_mask.shape)}")
        if m.dtype == torch.bool:
            m = m.view(torch.uint8)
        elif m.dtype != torch.uint8:
            m = (m != 0).view(torch.uint8)
        if m.stride(3) != 1:
            m = m.contiguous()
        return m

    def _build(self, m: torch.Tensor) -> None:
        _lib.check(_lib.lib().bsa_build_plan(m.data_ptr(), m.stride(0), m.stride(1), m.stride(2), self.mask_b,
                                             self.mask_h, self.nb, self.block, self.tile_ptr.data_ptr(),
                                             self.tile_col.data_ptr(), self.tile_order.data_ptr(),
                                             self._work.data_ptr(), self._ws_bytes, _stream(self.device)),
                   "bsa_build_plan")
        self._mask_ref = m  # keep the mask alive until the kernels ran

    def update(self, block_mask: torch.Tensor) -> "BlockSparsePlan":
        """Rebuild the plan from a new mask of the same shape into the same
        device buffers (no allocation; enqueued on the current stream, so a
        forward already enqueued with this plan still reads the old one)."""
        m = self._as_mask(block_mask)
        if (int(m.shape[0]), int(m.shape[1]), int(m.shape[2])) != (self.mask_b, self.mask_h, self.nb):
            raise ValueError(f"mask shape {tuple(m.shape)} differs from the plan's "
                             f"({self.mask_b}, {self.mask_h}, {self.nb}, {self.nb})")
        if m.device != self.device:
            raise ValueError("mask is on another device")
        self._build(m)
        return self

    @property
    def tiles_per_row(self) -> int:
        return (self.nb * self.block + 127) // 128

    def nnz_entries(self) -> int:
        """Number of (tile, key block) entries (synchronises)."""
        return int(self.tile_ptr[-1].item())

    def c_plan(self) -> _lib.Plan:
        return _lib.Plan(self.tile_ptr.data_ptr(), self.tile_col.data_ptr(), self.mask_b, self.mask_h, self.nb,
                         self.block, self.tile_order.data_ptr())


def _check_err(err: Optional[torch.Tensor], what: str) -> None:
    if err is None:
        return
    v = int(err.item())
    if v:
        names = [(_lib.DEVERR_TIMEOUT, "device wait timed out"),
                 (_lib.DEVERR_PERM_RANGE, "permutation value out of range"),
                 (_lib.DEVERR_PERM_DUP, "permutation value repeated"),
                 (_lib.DEVERR_COORD, "coordinate out of range"),
                 (_lib.DEVERR_PLAN, "plan entry out of range"),
                 (_lib.DEVERR_ALIGN, "dynamic shared memory misaligned")]
        bits = [n for b, n in names if v & b]
        status = _lib.STATUS_NAMES[7] if v & _lib.DEVERR_TIMEOUT else _lib.STATUS_NAMES[6]
        raise RuntimeError(f"{what}: device check failed ({status}): {', '.join(bits)}")


def block_sparse_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                           block_mask: Optional[torch.Tensor] = None, *, plan: Optional[BlockSparsePlan] = None,
                           block: Optional[int] = None, q_perm=None, kv_perm=None, sm_scale: Optional[float] = None,
                           return_lse: bool = False, kernel: str = "auto", check_errors: bool = False,
                           out: Optional[torch.Tensor] = None, lse_out: Optional[torch.Tensor] = None):
    """Block-sparse attention forward.

    ``o = softmax(QK^T * sm_scale restricted to kept blocks) V`` per (b, h).

    q, k, v: CUDA ``[B, H, N, D]`` of one dtype (bf16 / fp16 run on the
    tcgen05 tensor cores, fp32 on the CUDA cores), last dim contiguous.
    block_mask: bool ``[nb, nb]`` or ``[1|B, 1|H, nb, nb]`` in the permuted
    (new) token order, as the reference builds it (``utils.py:51-84`` after
    ``update_idx_perm``); or pass a prebuilt ``plan``.
    q_perm / kv_perm: optional ``[N]`` int permutations (``perm[i]`` = old
    index at new position ``i``), or the runners' expanded ``[B,H,N,D]``
    views.  Inputs are taken in the ORIGINAL order and the output is returned
    in the ORIGINAL order (``BlockSparseTriton_Naive.py:129-161``).  On the
    tensor-core path the query permutation is applied inside the attention
    kernel (Q rows gathered, O / lse rows scattered) and K, V are permuted by
    one pass each into a workspace; the fp32 path permutes every tensor.
    return_lse: also return the per-row log-sum-exp in log2 units (the
    reference kernel's ``M``), ``-inf`` for rows that keep no block.
    check_errors: synchronise and raise if a device-side check fired.
    """
    for name, t in (("q", q), ("k", k), ("v", v)):
        _require_cuda(t, name)
    if q.dim() != 4 or k.shape != q.shape or v.shape != q.shape:
        raise ValueError(f"q, k, v must share one [B, H, N, D] shape, got {tuple(q.shape)}, {tuple(k.shape)}, "
                         f"{tuple(v.shape)}")
    if not (q.dtype == k.dtype == v.dtype) or q.dtype not in _DTYPES:
        raise TypeError(f"q, k, v must share a dtype in (float32, float16, bfloat16), got {q.dtype}, {k.dtype}, "
                        f"{v.dtype}")
    if not (q.device == k.device == v.device):
        raise ValueError("q, k, v must be on one device")
    if kernel not in _KERNELS:
        raise ValueError(f"kernel must be one of {sorted(_KERNELS)}")
    B, H, N, D = (int(x) for x in q.shape)
    if plan is None:
        if block_mask is None:
            raise ValueError("pass block_mask or plan")
        nb = int(block_mask.shape[-1])
        plan = BlockSparsePlan(block_mask, block if block is not None else infer_block(N, nb))
    elif block is not None and block != plan.block:
        raise ValueError("block does not match the plan")
    if plan.device != q.device:
        raise ValueError("plan is on another device")
    if plan.mask_b not in (1, B) or plan.mask_h not in (1, H):
        raise ValueError(f"mask batch/head dims ({plan.mask_b}, {plan.mask_h}) do not broadcast to ({B}, {H})")
    if plan.nb != (N + plan.block - 1) // plan.block:
        raise ValueError(f"mask has {plan.nb} blocks per row; N={N} with BLOCK={plan.block} needs "
                         f"{(N + plan.block - 1) // plan.block}")
    scale = 1.0 / math.sqrt(D) if sm_scale is None else float(sm_scale)
    if not scale > 0:
        raise ValueError("sm_scale must be positive")
    qp = _perm_vector(q_perm, N, q.device, "q_perm")
    kp = _perm_vector(kv_perm, N, q.device, "kv_perm")
    if qp is not None and kp is not None and qp.dtype != kp.dtype:
        kp = kp.to(qp.dtype)

    o = out if out is not None else torch.empty((B, H, N, D), dtype=q.dtype, device=q.device)
    if tuple(o.shape) != (B, H, N, D) or o.dtype != q.dtype or o.device != q.device:
        raise ValueError("out has the wrong shape, dtype or device")
    lse = None
    if return_lse:
        lse = lse_out if lse_out is not None else torch.empty((B, H, N), dtype=torch.float32, device=q.device)
        if not lse.is_contiguous() or tuple(lse.shape) != (B, H, N) or lse.dtype != torch.float32:
            raise ValueError("lse_out must be a contiguous float32 [B, H, N] tensor")
    err = torch.zeros(1, dtype=torch.int32, device=q.device) if check_errors else None

    args = _lib.FwdArgs()
    args.B, args.H, args.N, args.D = B, H, N, D
    args.dtype = _DTYPES[q.dtype]
    args.q, args.k, args.v, args.o = _t4(q), _t4(k), _t4(v), _t4(o)
    args.sm_scale = scale
    args.lse = lse.data_ptr() if lse is not None else None
    args.plan = plan.c_plan()
    args.err_flag = err.data_ptr() if err is not None else None
    args.kernel = _KERNELS[kernel]
    L = _lib.lib()
    stream = _stream(q.device)
    if qp is None and kp is None:
        _lib.check(L.bsa_fwd(ctypes.byref(args), stream), "bsa_fwd")
    else:
        nbytes = ctypes.c_size_t()
        _lib.check(L.bsa_fwd_reordered_workspace_bytes(ctypes.byref(args), ctypes.byref(nbytes)),
                   "bsa_fwd_reordered_workspace_bytes")
        ws = torch.empty(max(1, nbytes.value), dtype=torch.uint8, device=q.device)
        pdt = _index_dtype(qp if qp is not None else kp)
        _lib.check(L.bsa_fwd_reordered(ctypes.byref(args), qp.data_ptr() if qp is not None else None,
                                       kp.data_ptr() if kp is not None else None, pdt, ws.data_ptr(),
                                       nbytes.value, stream), "bsa_fwd_reordered")
    _check_err(err, "block_sparse_attention")
    return (o, lse) if return_lse else o


def transposed_plan(plan: BlockSparsePlan, block_mask: torch.Tensor) -> BlockSparsePlan:
    """The plan of ``block_mask`` with its last two dims swapped: per key
    block, the query blocks that keep it (what the backward's dK / dV kernel
    walks)."""
    m = BlockSparsePlan._as_mask(block_mask)
    if (int(m.shape[0]), int(m.shape[1]), int(m.shape[2])) != (plan.mask_b, plan.mask_h, plan.nb):
        raise ValueError("block_mask does not match the plan")
    return BlockSparsePlan(m.transpose(-1, -2).contiguous(), plan.block)


def block_sparse_attention_backward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, o: torch.Tensor,
                                    lse: torch.Tensor, dout: torch.Tensor, *, plan: BlockSparsePlan,
                                    plan_t: BlockSparsePlan, sm_scale: Optional[float] = None,
                                    check_errors: bool = False):
    """Gradients of :func:`block_sparse_attention` (no token permutation):
    returns ``dq, dk, dv`` for the output gradient ``dout``.

    ``o`` and ``lse`` are the forward's output and log2 LSE
    (``return_lse=True``); ``plan`` is the forward's plan and ``plan_t`` the
    plan of the transposed block mask (:func:`transposed_plan`).  bf16 /
    fp16, D 64 or 128, BLOCK 64 or 128, on the tcgen05 kernels; P is recomputed
    from ``lse`` and every gradient row is written by one CTA (no atomics,
    deterministic).  The reference has no backward pass.
    """
    for name, t in (("q", q), ("k", k), ("v", v), ("o", o), ("dout", dout), ("lse", lse)):
        _require_cuda(t, name)
    if q.dim() != 4 or any(t.shape != q.shape for t in (k, v, o, dout)):
        raise ValueError("q, k, v, o, dout must share one [B, H, N, D] shape")
    if q.dtype not in (torch.float16, torch.bfloat16) or any(t.dtype != q.dtype for t in (k, v, o, dout)):
        raise TypeError("the backward takes float16 or bfloat16 q, k, v, o, dout of one dtype")
    B, H, N, D = (int(x) for x in q.shape)
    if tuple(lse.shape) != (B, H, N) or lse.dtype != torch.float32 or not lse.is_contiguous():
        raise ValueError("lse must be the forward's contiguous float32 [B, H, N] LSE")
    for pl in (plan, plan_t):
        if pl.device != q.device:
            raise ValueError("plan is on another device")
    scale = 1.0 / math.sqrt(D) if sm_scale is None else float(sm_scale)
    dq, dk, dv = (torch.empty_like(q) for _ in range(3))
    delta = torch.empty((B, H, N), dtype=torch.float32, device=q.device)
    err = torch.zeros(1, dtype=torch.int32, device=q.device) if check_errors else None
    args = _lib.BwdArgs()
    args.B, args.H, args.N, args.D = B, H, N, D
    args.dtype = _DTYPES[q.dtype]
    args.q, args.k, args.v, args.o, args.dout = _t4(q), _t4(k), _t4(v), _t4(o), _t4(dout)
    args.dq, args.dk, args.dv = _t4(dq), _t4(dk), _t4(dv)
    args.sm_scale = scale
    args.lse = lse.data_ptr()
    args.delta = delta.data_ptr()
    args.plan = plan.c_plan()
    args.plan_t = plan_t.c_plan()
    args.err_flag = err.data_ptr() if err is not None else None
    _lib.check(_lib.lib().bsa_bwd(ctypes.byref(args), _stream(q.device)), "bsa_bwd")
    _check_err(err, "block_sparse_attention_backward")
    return dq, dk, dv


class _BlockSparseAttentionFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, q, k, v, plan, plan_t, sm_scale):
        o, lse = block_sparse_attention(q, k, v, plan=plan, sm_scale=sm_scale, return_lse=True, kernel="tcgen05")
        ctx.save_for_backward(q, k, v, o, lse)
        ctx.plan, ctx.plan_t, ctx.sm_scale = plan, plan_t, sm_scale
        return o

    @staticmethod
    def backward(ctx, dout):
        q, k, v, o, lse = ctx.saved_tensors
        dq, dk, dv = block_sparse_attention_backward(q, k, v, o, lse, dout.contiguous(), plan=ctx.plan,
                                                     plan_t=ctx.plan_t, sm_scale=ctx.sm_scale)
        return dq, dk, dv, None, None, None


def block_sparse_attention_autograd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                                    block_mask: torch.Tensor, *, block: int = 128,
                                    sm_scale: Optional[float] = None) -> torch.Tensor:
    """The forward as a differentiable op: ``o.backward(g)`` runs
    :func:`block_sparse_attention_backward` (same restrictions)."""
    plan = BlockSparsePlan(block_mask, block)
    plan_t = transposed_plan(plan, block_mask)
    scale = 1.0 / math.sqrt(int(q.shape[-1])) if sm_scale is None else float(sm_scale)
    return _BlockSparseAttentionFn.apply(q, k, v, plan, plan_t, scale)


def permute_rows(x: torch.Tensor, perm, dim: int, inverse: bool, out: Optional[torch.Tensor] = None,
                 check_errors: bool = False) -> torch.Tensor:
    """Gather (``inverse=False``: ``out.select(dim, i) = x.select(dim, perm[i])``)
    or scatter (``inverse=True``: ``out.select(dim, perm[i]) = x.select(dim, i)``)
    of a CUDA tensor along ``dim`` with the row-copy kernel."""
    _require_cuda(x, "x")
    if x.dtype not in _DTYPES:
        raise TypeError(f"unsupported dtype {x.dtype}")
    dim = dim % x.dim()
    x = x.contiguous()
    n = int(x.shape[dim])
    p = _perm_vector(perm, n, x.device, "perm")
    outer = int(math.prod(x.shape[:dim]))
    inner = int(math.prod(x.shape[dim + 1:]))
    y = out if out is not None else torch.empty_like(x)
    if y.shape != x.shape or not y.is_contiguous():
        raise ValueError("out must be contiguous with the input's shape")
    if x.numel() == 0:
        return y
    err = torch.zeros(1, dtype=torch.int32, device=x.device) if check_errors else None
    src = _lib.Tensor4d(x.data_ptr(), n * inner, 0, inner)
    dst = _lib.Tensor4d(y.data_ptr(), n * inner, 0, inner)
    _lib.check(_lib.lib().bsa_permute_rows(dst, src, outer, 1, n, inner, _DTYPES[x.dtype], p.data_ptr(),
                                           _index_dtype(p), 1 if inverse else 0,
                                           err.data_ptr() if err is not None else None, _stream(x.device)),
               "bsa_permute_rows")
    _check_err(err, "permute_rows")
    return y


def inverse_permutation(perm: torch.Tensor, check_errors: bool = True) -> torch.Tensor:
    """``inv[perm[i]] = i`` on the GPU, validating that ``perm`` is a permutation."""
    _require_cuda(perm, "perm")
    p = perm.contiguous()
    inv = torch.empty(p.shape[0], dtype=torch.int64, device=p.device)
    err = torch.zeros(1, dtype=torch.int32, device=p.device) if check_errors else None
    _lib.check(_lib.lib().bsa_inverse_permutation(p.data_ptr(), _index_dtype(p), p.shape[0], inv.data_ptr(),
                                                  err.data_ptr() if err is not None else None, _stream(p.device)),
               "bsa_inverse_permutation")
    _check_err(err, "inverse_permutation")
    return inv
