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

bool attn_tc_supported(const bsa_fwd_args* a) {
  if (a->dtype != BSA_DTYPE_F16 && a->dtype != BSA_DTYPE_BF16) return false;
  if (a->D != 64 && a->D != 128) return false;
  if (a->plan.block != 64 && a->plan.block != 128) return false;
  return aligned16(a->q) && aligned16(a->k) && aligned16(a->v) && aligned16(a->o);
}

}  // namespace bsa
