// Host helpers of the tcgen05 attention path: TMA tensor maps over the
// caller's [B, H, N, D] tensors and the support predicate for the path.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "internal.h"

namespace bsa {

namespace {

bool aligned16(const bsa_tensor4d& t) {
  return (reinterpret_cast<uintptr_t>(t.data) % 16) == 0 && (t.stride_n * 2) % 16 == 0 &&
         (t.stride_h * 2) % 16 == 0 && (t.stride_b * 2) % 16 == 0;
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

}  // namespace

// 4-D map over [B, H, N, D] (TMA order: D, N, H, B), box = 64 x rows, 128B
// swizzle; strides are the caller's, so [B,H,N,D] and [B,N,H,D] memory both
// work without a copy.
int make_tensor_map_4d(CUtensorMap* m, const bsa_tensor4d& tdesc, int B, int H, int N, int D, bool bf16, int rows) {
  auto enc = get_encode_fn();
  if (!enc) return BSA_ERR_CUDA;
  const cuuint64_t dims[4] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(H),
                              static_cast<cuuint64_t>(B)};
  const cuuint64_t strides[3] = {static_cast<cuuint64_t>(tdesc.stride_n) * 2,
                                 static_cast<cuuint64_t>(tdesc.stride_h) * 2,
                                 static_cast<cuuint64_t>(tdesc.stride_b) * 2};
  const cuuint32_t box[4] = {64, static_cast<cuuint32_t>(rows), 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, tdesc.data, dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? BSA_OK : BSA_ERR_ALIGNMENT;
}

// 2-D map over the rows of a [B, H, N, D] tensor whose b and h strides are
// whole multiples of its row stride: rows of D elements, row (b, h, n) =
// b * stride_b / stride_n + h * stride_h / stride_n + n; box 64 x 1 (the row
// gathers load four such boxes), 128B swizzle.
int make_tensor_map_rows(CUtensorMap* m, const bsa_tensor4d& tdesc, int64_t rows, int D, bool bf16) {
  auto enc = get_encode_fn();
  if (!enc) return BSA_ERR_CUDA;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(tdesc.stride_n) * 2};
  const cuuint32_t box[2] = {64, 1};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, tdesc.data, dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? BSA_OK : BSA_ERR_ALIGNMENT;
}

bool rows_gatherable(const bsa_tensor4d& t, int B, int H, int N, int64_t* rb, int64_t* rh, int64_t* rows) {
  if (t.stride_n <= 0 || t.stride_h % t.stride_n || t.stride_b % t.stride_n) return false;
  *rb = t.stride_b / t.stride_n;
  *rh = t.stride_h / t.stride_n;
  *rows = (B - 1) * *rb + (H - 1) * *rh + N;
  return *rows < (int64_t(1) << 31) - 1;
}

bool attn_tc_supported(const bsa_fwd_args* a) {
  if (a->dtype != BSA_DTYPE_F16 && a->dtype != BSA_DTYPE_BF16) return false;
  if (a->D != 64 && a->D != 128) return false;
  if (a->plan.block != 64 && a->plan.block != 128) return false;
  return aligned16(a->q) && aligned16(a->k) && aligned16(a->v) && aligned16(a->o);
}

}  // namespace bsa
