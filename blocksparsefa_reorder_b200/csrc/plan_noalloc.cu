// bsa_build_plan_noalloc: the plan build for callers that cannot allocate.
//
// Some host programs that embed this library never let a component call
// cudaMalloc: an application that hands all device memory out of its own
// pre-reserved pool, a serving loop that must not take the implicit device
// synchronisation of an allocation, or a memory-budgeted process that has
// already claimed the GPU.  bsa_build_plan needs a small scratch array (one
// int32 per tile: the per-tile counts before the scan) and asks its caller
// for it; this variant instead keeps that scratch in a fixed array inside the
// library, so the caller only passes the mask and the two output arrays.
//
// The array is a file-scope __device__ variable: every GPU that loads the
// library holds its BSA_PLAN_NOALLOC_MAX_TILES * 4 bytes until the process
// exits.  Host code cannot use the variable's name as a device pointer, so
// the first call on each device looks its address up with
// cudaGetSymbolAddress (with that device current) and caches it; that first
// call should therefore come before any stream capture.  All calls share the
// one array, so calls whose kernels overlap on the GPU (different streams, or
// different host threads) race on it and must be serialised by the caller.
// The count kernel writes every element it later reads, so nothing has to be
// cleared between calls.
#include <mutex>

#include "common.cuh"
#include "internal.h"

namespace {

static __device__ __align__(256) int32_t g_plan_counts[BSA_PLAN_NOALLOC_MAX_TILES];

std::mutex g_mu;
int32_t* g_counts_addr[64] = {};  // per device, filled on first use

int counts_address(int32_t** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return BSA_ERR_CUDA;
  if (dev < 0 || dev >= 64) return BSA_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_counts_addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_plan_counts) != cudaSuccess || !p) {
      cudaGetLastError();
      return BSA_ERR_CUDA;
    }
    g_counts_addr[dev] = static_cast<int32_t*>(p);
  }
  *out = g_counts_addr[dev];
  return BSA_OK;
}

}  // namespace

extern "C" int bsa_build_plan_noalloc(const uint8_t* mask, int64_t stride_b, int64_t stride_h, int64_t stride_row,
                                      int32_t mask_b, int32_t mask_h, int32_t nb, int32_t block, int32_t* tile_ptr,
                                      int32_t* tile_col, void* stream) {
  size_t need = 0;
  int64_t ptr_len = 0, cap = 0;
  int rc = bsa_plan_sizes(mask_b, mask_h, nb, block, &ptr_len, &cap, &need);
  if (rc != BSA_OK) return rc;
  if (!mask || !tile_ptr || !tile_col) return BSA_ERR_INVALID_ARG;
  if (ptr_len - 1 > BSA_PLAN_NOALLOC_MAX_TILES) return BSA_ERR_WORKSPACE;  // more tiles than the fixed scratch
  if (cap > INT32_MAX) return BSA_ERR_UNSUPPORTED;
  int32_t* counts = nullptr;
  if ((rc = counts_address(&counts))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  rc = bsa::launch_plan_count(mask, stride_b, stride_h, stride_row, mask_b, mask_h, nb, block, counts, st);
  if (rc) return rc;
  rc = bsa::launch_plan_scan(counts, ptr_len - 1, tile_ptr, st);
  if (rc) return rc;
  return bsa::launch_plan_fill(mask, stride_b, stride_h, stride_row, mask_b, mask_h, nb, block, tile_ptr, tile_col,
                               st);
}
