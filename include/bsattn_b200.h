/*
 * bsattn_b200.h -- C ABI of the B200 (sm_100a) block-sparse attention forward.
 *
 * Drop-in boundary for the hot path of KutayTasci/BlockSparseFA_Reorder:
 * q, k, v [B,H,N,D] + a BLOCK x BLOCK block mask (+ optional token
 * permutations) in, attention output in original token order out.
 *
 * Conventions
 *  - Every pointer is a device pointer unless stated otherwise.  The library
 *    never allocates device memory: scratch space is passed in as a
 *    workspace whose size a *_sizes / *_workspace_bytes query returns.
 *  - Every entry point is enqueued on `stream` (a cudaStream_t passed as
 *    void*; NULL = legacy default stream) and does not synchronise.
 *  - Return value: a bsa_status code (0 = success).  Nothing aborts.
 *  - Permutation convention (reference utils.py:163-164, main.py:27-28):
 *    perm[i] is the OLD index that moves to NEW position i.
 *  - Tensors are 4-D [B, H, N, D] views given by a base pointer and element
 *    strides for b, h and n; the innermost (D) stride must be 1.
 */
#ifndef BSATTN_B200_H
#define BSATTN_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define BSA_API __attribute__((visibility("default")))
#else
#define BSA_API
#endif

#define BSA_ABI_VERSION 2

typedef enum bsa_status {
  BSA_OK = 0,
  BSA_ERR_INVALID_ARG = 1,     /* null pointer / non-positive size / bad enum      */
  BSA_ERR_SHAPE = 2,           /* inconsistent shapes (mask vs N, strides, ...)    */
  BSA_ERR_DTYPE = 3,           /* unsupported element type                         */
  BSA_ERR_ALIGNMENT = 4,       /* pointer or stride not 16-byte aligned (TMA)      */
  BSA_ERR_UNSUPPORTED = 5,     /* head dim / block size / scale not supported      */
  BSA_ERR_NOT_PERMUTATION = 6, /* device check found a value out of range / dup    */
  BSA_ERR_TIMEOUT = 7,         /* a bounded device wait ran out (err flag)         */
  BSA_ERR_CUDA = 8,            /* CUDA runtime error (launch / attribute)          */
  BSA_ERR_WORKSPACE = 9,       /* workspace missing or too small                   */
  BSA_ERR_DEVICE = 10          /* current device is not sm_100                     */
} bsa_status;

typedef enum bsa_dtype { BSA_DTYPE_F32 = 0, BSA_DTYPE_F16 = 1, BSA_DTYPE_BF16 = 2 } bsa_dtype;
typedef enum bsa_index_dtype { BSA_INDEX_I32 = 0, BSA_INDEX_I64 = 1 } bsa_index_dtype;

/* Kernel choice for bsa_fwd (AUTO picks tcgen05 for f16/bf16 with D in
 * {64,128} and BLOCK in {64,128}, the SIMT kernel otherwise). */
typedef enum bsa_kernel { BSA_KERNEL_AUTO = 0, BSA_KERNEL_SIMT = 1, BSA_KERNEL_TCGEN05 = 2 } bsa_kernel;

/* Bits that kernels OR into the optional device error word (int32). */
#define BSA_DEVERR_TIMEOUT 1     /* bounded mbarrier wait ran out                 */
#define BSA_DEVERR_PERM_RANGE 2  /* permutation value outside [0, n)              */
#define BSA_DEVERR_PERM_DUP 4    /* permutation value repeated                    */
#define BSA_DEVERR_COORD 8       /* coordinate negative or outside the perm      */
#define BSA_DEVERR_PLAN 16       /* plan entry outside [0, nb)                    */
#define BSA_DEVERR_ALIGN 32      /* dynamic shared memory not 1024-byte aligned   */

typedef struct bsa_tensor4d {
  void* data;
  int64_t stride_b, stride_h, stride_n; /* in elements; stride_d == 1 */
} bsa_tensor4d;

/* Per-tile list of kept key blocks (output of bsa_build_plan).  A tile is
 * 128 query rows: one block row for BLOCK 128, block rows 2t and 2t+1 for
 * BLOCK 64.  Tiles of mask slice s = (mask_b==1 ? 0 : b) * mask_h +
 * (mask_h==1 ? 0 : h) are tile_ptr[s*T + t] .. tile_ptr[s*T + t + 1] in
 * tile_col, T = ceil(nb * BLOCK / 128).  Each entry is (flags << 24) |
 * key_block, ascending in key_block; flags bit 0 / bit 1 = the first /
 * second block row of the tile keeps that key block.
 * tile_order (optional, output of bsa_build_tile_order, NULL = natural
 * order): for each slice, its T tile rows by decreasing number of kept
 * blocks; the tcgen05 kernel hands tiles to CTAs in that order. */
typedef struct bsa_plan {
  const int32_t* tile_ptr;
  const int32_t* tile_col;
  int32_t mask_b, mask_h;
  int32_t nb;    /* ceil(N / block) */
  int32_t block; /* 64 or 128 */
  const int32_t* tile_order;
} bsa_plan;

typedef struct bsa_fwd_args {
  int32_t B, H, N, D;
  int32_t dtype;            /* bsa_dtype of q, k, v and o                         */
  bsa_tensor4d q, k, v, o;
  float sm_scale;           /* softmax scale, > 0 (reference: 1/sqrt(D))          */
  float* lse;               /* optional contiguous [B,H,N] fp32 LSE in log2 units
                               (the reference's M); NULL = not written            */
  bsa_plan plan;
  int32_t* err_flag;        /* optional device int32 for BSA_DEVERR_* bits        */
  int32_t kernel;           /* bsa_kernel                                         */
} bsa_fwd_args;

/* Library identity. */
BSA_API int bsa_abi_version(void);
BSA_API const char* bsa_status_string(int status);
/* 1 in *supported when `device` is an sm_100 part the kernels were built for. */
BSA_API int bsa_device_supported(int device, int* supported);

/* Sizes for a plan over a [mask_b, mask_h, nb, nb] mask: tile_ptr length,
 * tile_col capacity (worst case: every block kept) and workspace bytes. */
BSA_API int bsa_plan_sizes(int32_t mask_b, int32_t mask_h, int32_t nb, int32_t block, int64_t* tile_ptr_len,
                           int64_t* tile_col_capacity, size_t* workspace_bytes);

/* Block mask (bytes, nonzero = kept, [mask_b, mask_h, nb, nb] with the given
 * element strides) -> per-tile CSR.  Replaces the per-query-block scan of
 * every mask byte inside the reference kernel
 * (triton_kernels/BlockSparse_Naive.py:25-32, BlockSparse_Fused.py:29-35).
 * tile_order (optional, tile_ptr_len - 1 entries) also receives the plan's
 * work order (see bsa_build_tile_order).  Small plans (<= 4096 tiles, <= 1024
 * per slice) are built by a single one-CTA kernel. */
BSA_API int bsa_build_plan(const uint8_t* mask, int64_t stride_b, int64_t stride_h, int64_t stride_row,
                           int32_t mask_b, int32_t mask_h, int32_t nb, int32_t block, int32_t* tile_ptr,
                           int32_t* tile_col, int32_t* tile_order, void* workspace, size_t workspace_bytes,
                           void* stream);

/* Work order for a built plan: tile_order[s*T + r] = the tile row with the
 * r-th largest kept-block count in slice s (ties by increasing row), for the
 * mask_b*mask_h slices (tile_order holds tile_ptr_len - 1 entries).  With it
 * the tcgen05 kernel's CTAs claim tiles dynamically, longest first, which
 * balances their load.  No counterpart in the reference, whose grid is one
 * static program per query block (BlockSparseTriton_Naive.py:56-57,
 * triton_kernels/BlockSparse_Naive.py:80-81).  Needs no workspace; enqueued on
 * `stream`. */
BSA_API int bsa_build_tile_order(const int32_t* tile_ptr, int32_t mask_b, int32_t mask_h, int32_t nb, int32_t block,
                                 int32_t* tile_order, void* stream);

/* bsa_build_plan for callers that may not allocate device memory (a host
 * framework that owns every device buffer through its own pool, a serving
 * loop that cannot afford an allocation's implicit synchronisation).  No
 * counterpart in the reference.  Same inputs and outputs as bsa_build_plan
 * minus the workspace: the per-tile scratch lives in a fixed device array
 * inside the library (BSA_PLAN_NOALLOC_MAX_TILES int32 = 4 MiB, held by every
 * GPU that loads the library until exit).  Returns BSA_ERR_WORKSPACE when the
 * mask has more than BSA_PLAN_NOALLOC_MAX_TILES tiles (mask_b * mask_h *
 * ceil(nb * block / 128)).  The first call on a device looks the array's
 * address up (cudaGetSymbolAddress), so make it before any stream capture.
 * Calls share the array: calls that overlap on the GPU race and must be
 * serialised by the caller.  Allocates nothing. */
#define BSA_PLAN_NOALLOC_MAX_TILES (1 << 20)
BSA_API int bsa_build_plan_noalloc(const uint8_t* mask, int64_t stride_b, int64_t stride_h, int64_t stride_row,
                                   int32_t mask_b, int32_t mask_h, int32_t nb, int32_t block, int32_t* tile_ptr,
                                   int32_t* tile_col, void* stream);

/* Attention forward on tensors already in the mask's token order.
 * Replaces _attn_fwd_block_sparse (triton_kernels/BlockSparse_Naive.py:68-125)
 * as launched at BlockSparseTriton_Naive.py:142-156: o = softmax over kept
 * blocks of (q k^T * sm_scale) v; rows that keep no block give o = 0 and
 * lse = -inf.  At BLOCK 64 a 128-row tile reads every key block that either
 * of its two 64-row query blocks keeps, and the rows whose block does not
 * keep it add 0 x V: the masked blocks contribute exactly nothing when V is
 * finite in the blocks a tile's other query block keeps (NaN / Inf there
 * would reach those rows).  BLOCK 128 has no such condition. */
BSA_API int bsa_fwd(const bsa_fwd_args* args, void* stream);

/* Row gather / scatter along N for every (b, h); D = elements per row:
 *   inverse == 0: dst[b,h,i,:] = src[b,h,perm[i],:]
 *     (apply_reordering, utils.py:260-266; torch.gather at
 *      BlockSparseTriton_Naive.py:89-97)
 *   inverse != 0: dst[b,h,perm[i],:] = src[b,h,i,:]
 *     (reverse_reordering, utils.py:269-288; scatter_ at
 *      BlockSparseTriton_Naive.py:158-161)
 * Out-of-range perm values set BSA_DEVERR_PERM_RANGE and skip the row. */
BSA_API int bsa_permute_rows(bsa_tensor4d dst, bsa_tensor4d src, int32_t B, int32_t H, int32_t N, int32_t D,
                             int32_t dtype, const void* perm, int32_t perm_dtype, int32_t inverse,
                             int32_t* err_flag, void* stream);

/* inv[perm[i]] = i with validation (utils.py:253-254, 283-284; the checks of
 * read_reordering_file_to_tensor, utils.py:222-231): out-of-range values set
 * BSA_DEVERR_PERM_RANGE, repeated values BSA_DEVERR_PERM_DUP. */
BSA_API int bsa_inverse_permutation(const void* perm, int32_t perm_dtype, int64_t n, int64_t* inv_out,
                                    int32_t* err_flag, void* stream);

/* out[i] = inv_perm[idx[i]]  (update_idx_perm, utils.py:236-258, given the
 * inverse permutation).  Indices outside [0, n) set BSA_DEVERR_COORD and
 * copy the index unchanged. */
BSA_API int bsa_remap_indices(const int64_t* idx, int64_t count, const int64_t* inv_perm, int64_t n,
                              int64_t* out, int32_t* err_flag, void* stream);

/* Token coordinates -> bool block mask [B, H, nb, nb] (uint8 0/1, contiguous),
 * nb = ceil(seq_len / block); coordinates whose block index is >= nb are
 * dropped, negative ones set BSA_DEVERR_COORD.  The same mask is written to
 * every (b, h).  `row_inv` / `col_inv` (optional, length seq_len) remap the
 * coordinates through inverse permutations first, fusing update_idx_perm.
 * Replaces generate_blockmask_from_mtx_coords (utils.py:51-84). */
BSA_API int bsa_blockmask_from_coords(const int64_t* rows, const int64_t* cols, int64_t count, int64_t seq_len,
                                      int32_t block, int32_t B, int32_t H, const int64_t* row_inv,
                                      const int64_t* col_inv, uint8_t* mask_out, int32_t* err_flag,
                                      void* stream);

/* "With reordering" forward: q rows taken through q_perm, k / v rows
 * through kv_perm, attention with the mask in the new order, o (and lse)
 * rows returned through q_perm to the ORIGINAL order.  Either permutation may
 * be NULL (identity).  Mirrors the timed loop of
 * BlockSparseTriton_Naive.py:129-161 and the fused kernel
 * triton_kernels/BlockSparse_Fused.py:115-223.  On the tcgen05 path the
 * query gather and the o / lse scatter run inside the attention kernel and
 * k, v are permuted into the workspace; the SIMT path permutes every tensor.
 * With `args->err_flag` set, both permutations are first checked on the
 * device (values outside [0, N) set BSA_DEVERR_PERM_RANGE, repeated values
 * BSA_DEVERR_PERM_DUP); the workspace then also holds the check's bits, so
 * query the size with the same args. */
BSA_API int bsa_fwd_reordered_workspace_bytes(const bsa_fwd_args* args, size_t* bytes);
BSA_API int bsa_fwd_reordered(const bsa_fwd_args* args, const void* q_perm, const void* kv_perm,
                              int32_t perm_dtype, void* workspace, size_t workspace_bytes, void* stream);

/* Backward pass (gradients of bsa_fwd), beyond the reference, whose kernels
 * write the row LSE M (triton_kernels/BlockSparse_Naive.py:119-122) but have
 * no backward.  tcgen05 path only: bf16 / fp16, D 64 or 128, BLOCK 64 or
 * 128 (both plans of one BLOCK), no token permutation, 16-byte aligned rows.  From dout and the forward's o
 * and lse it writes dq = sm_scale dS K, dk = sm_scale dS^T Q, dv = P^T dout
 * (P recomputed from lse, dS = P o (dout V^T - rowsum(dout o o))), each
 * output row by one CTA (deterministic, no atomics).
 *  - lse: the forward's [B,H,N] fp32 LSE (log2 units), contiguous;
 *  - delta: workspace, contiguous [B,H,N] fp32 (rowsum(dout o o) is written
 *    there first);
 *  - plan: the forward's plan (query tiles); plan_t: the plan of the
 *    transposed block mask, mask[..., j, i] (key tiles), same BLOCK.
 * Enqueues three kernels on `stream`. */
typedef struct bsa_bwd_args {
  int32_t B, H, N, D;
  int32_t dtype;            /* bsa_dtype of every tensor below (f16 or bf16)      */
  bsa_tensor4d q, k, v, o, dout;
  bsa_tensor4d dq, dk, dv;  /* outputs                                            */
  float sm_scale;           /* the forward's softmax scale                        */
  const float* lse;
  float* delta;
  bsa_plan plan;
  bsa_plan plan_t;
  int32_t* err_flag;        /* optional device int32 for BSA_DEVERR_* bits        */
} bsa_bwd_args;
BSA_API int bsa_bwd(const bsa_bwd_args* args, void* stream);

/* Test hook for the bounded device waits, not for production use.  Arms the
 * NEXT tcgen05 forward (bsa_fwd / bsa_fwd_reordered) of the process: every
 * mbarrier wait of its launch gives up after `wait_us` microseconds (100 ..
 * 2,000,000) instead of 2 s, and one softmax warp of CTA 0 withholds its
 * arrival for that CTA's first step, so the MMA issuer's wait for it runs
 * out.  The kernel then ORs BSA_DEVERR_TIMEOUT into the error word, every
 * role of the CTA drains its loads and MMAs, frees its tensor memory and
 * returns; the other CTAs finish normally.  No TMA load or MMA is ever counted
 * on the withheld barrier.  No counterpart in the reference. */
BSA_API int bsa_test_arm_wait_timeout(uint32_t wait_us);

#ifdef __cplusplus
}
#endif

#endif /* BSATTN_B200_H */
