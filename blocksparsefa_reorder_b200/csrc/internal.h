// Launchers shared between the translation units of the library.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/bsattn_b200.h"

namespace bsa {

// Element size in bytes of a bsa_dtype (0 when invalid).
inline int dtype_bytes(int dt) {
  return dt == BSA_DTYPE_F32 ? 4 : (dt == BSA_DTYPE_F16 || dt == BSA_DTYPE_BF16) ? 2 : 0;
}

inline int tiles_per_row(int nb, int block) { return (nb * block + 127) / 128; }

// preprocess.cu
int launch_plan_count(const uint8_t* mask, int64_t sb, int64_t sh, int64_t srow, int mask_b, int mask_h, int nb,
                      int block, int32_t* counts, cudaStream_t st);
int launch_plan_scan(const int32_t* counts, int64_t n, int32_t* tile_ptr, cudaStream_t st);
int launch_plan_fill(const uint8_t* mask, int64_t sb, int64_t sh, int64_t srow, int mask_b, int mask_h, int nb,
                     int block, const int32_t* tile_ptr, int32_t* tile_col, cudaStream_t st);
// Bits of a permutation check (ceil(n / 32) words) and the check itself:
// zeroes `scratch`, then sets BSA_DEVERR_PERM_RANGE / _DUP in `err`.
size_t perm_check_bytes(int64_t n);
int launch_perm_check(const void* perm, int perm_dtype, int64_t n, void* scratch, int32_t* err, cudaStream_t st);
int launch_permute_rows(bsa_tensor4d dst, bsa_tensor4d src, int B, int H, int N, int row_elems, int elt_bytes,
                        const void* perm, int perm_dtype, int inverse, int32_t* err, cudaStream_t st);

// attn_simt.cu
int launch_attn_simt(const bsa_fwd_args* a, cudaStream_t st);
// The backward kernels (attn_bwd.cu): Delta, dQ, dK / dV; arguments validated.
int launch_attn_bwd(const bsa_bwd_args* a, cudaStream_t st);

// tma_maps.cu: whether the tcgen05 path takes these arguments (bf16 / fp16,
// D 64 or 128, BLOCK 64 or 128, 16-byte-aligned rows), and the 4-D TMA map
// over a [B, H, N, D] 16-bit tensor, box 64 x rows, 128-byte swizzle.
bool attn_tc_supported(const bsa_fwd_args* a);
int make_tensor_map_4d(CUtensorMap* m, const bsa_tensor4d& t, int B, int H, int N, int D, bool bf16, int rows);

// attn_tcp.cu: the persistent tcgen05 attention forward
// q_perm (optional, bsa_index_dtype perm_dtype): gather Q rows from and
// scatter O / lse rows to q_perm[row] inside the kernel.
int launch_attn_tcp(const bsa_fwd_args* a, cudaStream_t st, const void* q_perm = nullptr,
                    int perm_dtype = BSA_INDEX_I64);
// Arms the timeout test for the next launch_attn_tcp call (see
// bsa_test_arm_wait_timeout).
int arm_test_wait_timeout(uint32_t wait_us);


}  // namespace bsa

#define BSA_CUDA_CHECK(expr)                    \
  do {                                          \
    cudaError_t e_ = (expr);                    \
    if (e_ != cudaSuccess) return BSA_ERR_CUDA; \
  } while (0)
