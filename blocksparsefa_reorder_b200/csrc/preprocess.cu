// Mask / permutation preprocessing kernels.
//
// * Plan build: block mask -> per-tile CSR of kept key blocks (count, scan,
//   fill).  One warp per tile reads the tile's mask rows with coalesced byte
//   loads and compacts kept columns with ballot + popc, so the list comes out
//   in ascending key-block order (the order the reference kernel scans,
//   triton_kernels/BlockSparse_Naive.py:25-32).
// * Row gather / scatter along N (apply_reordering / reverse_reordering,
//   utils.py:260-288) with 16-byte vector copies.
// * Inverse permutation with range / duplicate checks (utils.py:253-254,
//   222-231), index remap (update_idx_perm, utils.py:236-258) and token
//   coordinates -> block mask (generate_blockmask_from_mtx_coords,
//   utils.py:51-84).
#include <type_traits>

#include "common.cuh"
#include "internal.h"

namespace bsa {

namespace {

constexpr int kWarpsPerBlock = 8;

__device__ __forceinline__ uint32_t tile_flags(const uint8_t* base, int64_t srow, int nb, int rows_per_tile, int t,
                                               int j) {
  uint32_t f = 0;
  if (j < nb) {
    for (int r = 0; r < rows_per_tile; ++r) {
      const int br = t * rows_per_tile + r;
      if (br < nb && base[br * srow + j]) f |= 1u << r;
    }
    if (rows_per_tile == 1 && f) f = 3u;
  }
  return f;
}

__global__ void plan_count_kernel(const uint8_t* __restrict__ mask, int64_t sb, int64_t sh, int64_t srow, int mask_b,
                                  int mask_h, int nb, int rows_per_tile, int T, int32_t* __restrict__ counts) {
  const int64_t total = static_cast<int64_t>(mask_b) * mask_h * T;
  const int lane = threadIdx.x & 31;
  for (int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; w < total;
       w += (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5) {
    const int64_t s = w / T;
    const int t = static_cast<int>(w % T);
    const uint8_t* base = mask + (s / mask_h) * sb + (s % mask_h) * sh;
    int count = 0;
    for (int j0 = 0; j0 < nb; j0 += 32) {
      const uint32_t f = tile_flags(base, srow, nb, rows_per_tile, t, j0 + lane);
      count += __popc(__ballot_sync(0xffffffffu, f != 0));
    }
    if (lane == 0) counts[w] = count;
  }
}

__global__ void plan_fill_kernel(const uint8_t* __restrict__ mask, int64_t sb, int64_t sh, int64_t srow, int mask_b,
                                 int mask_h, int nb, int rows_per_tile, int T, const int32_t* __restrict__ tile_ptr,
                                 int32_t* __restrict__ tile_col) {
  const int64_t total = static_cast<int64_t>(mask_b) * mask_h * T;
  const int lane = threadIdx.x & 31;
  const uint32_t lt_mask = (1u << lane) - 1u;
  for (int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; w < total;
       w += (static_cast<int64_t>(gridDim.x) * blockDim.x) >> 5) {
    const int64_t s = w / T;
    const int t = static_cast<int>(w % T);
    const uint8_t* base = mask + (s / mask_h) * sb + (s % mask_h) * sh;
    int pos = tile_ptr[w];
    for (int j0 = 0; j0 < nb; j0 += 32) {
      const int j = j0 + lane;
      const uint32_t f = tile_flags(base, srow, nb, rows_per_tile, t, j);
      const uint32_t bal = __ballot_sync(0xffffffffu, f != 0);
      if (f) tile_col[pos + __popc(bal & lt_mask)] = static_cast<int32_t>((f << 24) | static_cast<uint32_t>(j));
      pos += __popc(bal);
    }
  }
}

// Exclusive scan of counts[0, n) into tile_ptr[0, n]; one block of 1024
// threads, each owning a contiguous chunk.
__global__ void __launch_bounds__(1024) plan_scan_kernel(const int32_t* __restrict__ counts, int64_t n,
                                                         int32_t* __restrict__ tile_ptr) {
  __shared__ int32_t warp_sums[32];
  const int tid = threadIdx.x;
  const int64_t chunk = (n + blockDim.x - 1) / blockDim.x;
  const int64_t lo = tid * chunk;
  const int64_t hi = lo + chunk < n ? lo + chunk : n;
  int32_t local = 0;
  for (int64_t i = lo; i < hi; ++i) local += counts[i];
  int32_t x = local;  // inclusive warp scan
  const int lane = tid & 31, wid = tid >> 5;
  for (int o = 1; o < 32; o <<= 1) {
    const int32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[wid] = x;
  __syncthreads();
  if (wid == 0) {
    int32_t ws = warp_sums[lane];
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t y = __shfl_up_sync(0xffffffffu, ws, o);
      if (lane >= o) ws += y;
    }
    warp_sums[lane] = ws;
  }
  __syncthreads();
  int32_t run = x - local + (wid > 0 ? warp_sums[wid - 1] : 0);
  for (int64_t i = lo; i < hi; ++i) {
    tile_ptr[i] = run;
    run += counts[i];
  }
  if (tid == blockDim.x - 1) tile_ptr[n] = run;
}

// Whole plan (and optionally its work order) in one CTA for small masks,
// where the multi-kernel path is all launch latency: the mask is staged in
// shared memory by all threads at once (independent loads); one thread per
// (tile, 16-column chunk) turns its chunk into kept-column bit masks and
// counts them; a block-wide exclusive scan of the tile counts gives
// tile_ptr; each chunk thread then writes its entries at the tile's offset
// plus the counts of the tile's earlier chunks; the tile ranks of the work
// order are computed by groups of threads.  Limits: n = slices * T tiles <=
// kSmallPlanTiles, n * chunks <= kSmallPlanChunks, mask <= kSmallPlanMaskBytes.
constexpr int kSmallPlanTiles = 4096;
constexpr int kSmallPlanSliceTiles = 1024;
constexpr int kSmallPlanMaskBytes = 96 * 1024;
constexpr int kSmallPlanChunks = 8192;

// bit k = byte k of p[0, jmax) is nonzero; `aligned`: p is 16-byte aligned and jmax == 16
__device__ __forceinline__ uint32_t nonzero_bits16(const uint8_t* p, int jmax, bool aligned) {
  uint32_t m = 0;
  if (aligned) {
    const uint4 v = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int b = 0; b < 4; ++b) m |= (((w[k] >> (8 * b)) & 0xFFu) != 0u ? 1u : 0u) << (4 * k + b);
  } else {
    for (int k = 0; k < jmax; ++k) m |= (p[k] != 0 ? 1u : 0u) << k;
  }
  return m;
}

__global__ void __launch_bounds__(1024) plan_small_kernel(const uint8_t* __restrict__ mask, int64_t sb, int64_t sh,
                                                          int64_t srow, int mask_h, int nb, int rows_per_tile, int T,
                                                          int n, bool vec16, int32_t* __restrict__ tile_ptr,
                                                          int32_t* __restrict__ tile_col,
                                                          int32_t* __restrict__ tile_order) {
  // dynamic shared memory: [mask slices x nb x nb][cnt n][off n + 1][chunk bits n * cpr]
  extern __shared__ __align__(16) uint8_t sm[];
  __shared__ int32_t warp_sums[32];
  // the attention kernel that follows may start its set-up on the other SMs;
  // it waits for this kernel's completion before reading the plan
  allow_dependents();
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int slices = n / T;
  const int nn = nb * nb;  // <= kSmallPlanMaskBytes
  const int rows = slices * nb;
  const int cpr = (nb + 15) / 16;
  const int tasks = n * cpr;
  uint8_t* smask = sm;
  int32_t* cnt = reinterpret_cast<int32_t*>(sm + ((slices * nn + 15) & ~15));
  int32_t* off = cnt + n;
  uint32_t* kbits = reinterpret_cast<uint32_t*>(off + n + 1);
  if (vec16) {
    // 16-byte vectors: every load of the CTA is independent and coalesced
    const int vpr = nb / 16;
    for (int i = tid; i < rows * vpr; i += 1024) {
      const int rr = i / vpr, v = i - rr * vpr;
      const int s = rr / nb, r = rr - s * nb;
      const uint8_t* src = mask + static_cast<int64_t>(s / mask_h) * sb + static_cast<int64_t>(s % mask_h) * sh +
                           r * srow + v * 16;
      *reinterpret_cast<uint4*>(smask + rr * nb + v * 16) = *reinterpret_cast<const uint4*>(src);
    }
  } else {
    for (int i = tid; i < rows * nb; i += 1024) {
      const int rr = i / nb, c = i - rr * nb;
      const int s = rr / nb, r = rr - s * nb;
      smask[i] = mask[static_cast<int64_t>(s / mask_h) * sb + static_cast<int64_t>(s % mask_h) * sh + r * srow + c];
    }
  }
  for (int i = tid; i < n; i += 1024) cnt[i] = 0;
  __syncthreads();
  // kept columns of each (tile, chunk): bits 0-15 first block row, 16-31 second
  const bool aligned = nb % 16 == 0;
  for (int task = tid; task < tasks; task += 1024) {
    const int w = task / cpr, c = task - w * cpr;
    const int s = w / T, t = w - s * T;
    const int r0 = t * rows_per_tile;
    const int jmax = nb - c * 16 < 16 ? nb - c * 16 : 16;
    const uint8_t* base = smask + s * nn + c * 16;
    const uint32_t m0 = nonzero_bits16(base + r0 * nb, jmax, aligned);
    const uint32_t m1 = rows_per_tile == 2 && r0 + 1 < nb ? nonzero_bits16(base + (r0 + 1) * nb, jmax, aligned) : 0u;
    kbits[task] = m0 | (m1 << 16);
    atomicAdd(&cnt[w], __popc(m0 | m1));
  }
  __syncthreads();
  // exclusive scan: each thread a contiguous chunk, then warp and block totals
  const int chunk = (n + 1023) / 1024;
  const int lo = tid * chunk < n ? tid * chunk : n;
  const int hi = lo + chunk < n ? lo + chunk : n;
  int32_t local = 0;
  for (int i = lo; i < hi; ++i) local += cnt[i];
  int32_t x = local;
  for (int o = 1; o < 32; o <<= 1) {
    const int32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[wid] = x;
  __syncthreads();
  if (wid == 0) {
    int32_t ws = warp_sums[lane];
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t y = __shfl_up_sync(0xffffffffu, ws, o);
      if (lane >= o) ws += y;
    }
    warp_sums[lane] = ws;
  }
  __syncthreads();
  int32_t run = x - local + (wid > 0 ? warp_sums[wid - 1] : 0);
  for (int i = lo; i < hi; ++i) {
    off[i] = run;
    run += cnt[i];
  }
  if (tid == 1023) off[n] = run;
  __syncthreads();
  for (int i = tid; i <= n; i += 1024) tile_ptr[i] = off[i];
  // fill: each chunk's entries in ascending column order
  for (int task = tid; task < tasks; task += 1024) {
    const int w = task / cpr, c = task - w * cpr;
    const uint32_t kb = kbits[task];
    int pos = off[w];
    for (int c2 = 0; c2 < c; ++c2) {
      const uint32_t k2 = kbits[w * cpr + c2];
      pos += __popc((k2 | (k2 >> 16)) & 0xFFFFu);
    }
    uint32_t kept = (kb | (kb >> 16)) & 0xFFFFu;
    while (kept) {
      const int k = __ffs(kept) - 1;
      kept &= kept - 1;
      const uint32_t f = rows_per_tile == 1 ? 3u : (((kb >> k) & 1u) | (((kb >> (16 + k)) & 1u) << 1));
      tile_col[pos++] = static_cast<int32_t>((f << 24) | static_cast<uint32_t>(c * 16 + k));
    }
  }
  // work order: rank by (decreasing count, increasing row) within the slice,
  // g threads of one warp per tile
  if (tile_order) {
    int g = 1;
    while (g < 32 && 2 * g * n <= 1024) g *= 2;
    const int gi = tid & (g - 1);
    const int per_round = 1024 / g;
    const int rounds = (n + per_round - 1) / per_round;
    for (int rd = 0; rd < rounds; ++rd) {
      const int w = rd * per_round + tid / g;
      const bool valid = w < n;
      const int s0 = valid ? (w / T) * T : 0, t = valid ? w - s0 : 0;
      const int mine = valid ? cnt[w] : 0;
      int rank = 0;
      if (valid)
        for (int u = gi; u < T; u += g) {
          const int c = cnt[s0 + u];
          rank += (c > mine) || (c == mine && u < t);
        }
      for (int o = g / 2; o > 0; o >>= 1) rank += __shfl_xor_sync(0xffffffffu, rank, o);
      if (valid && gi == 0) tile_order[s0 + rank] = t;
    }
  }
}

__device__ __forceinline__ int64_t load_index(const void* p, int dtype, int64_t i) {
  return dtype == BSA_INDEX_I64 ? static_cast<const int64_t*>(p)[i]
                                : static_cast<int64_t>(static_cast<const int32_t*>(p)[i]);
}

// Copy rows of `VB`-byte vectors, one vector per thread.  Rows are (b, h, i)
// with i in [0, N); the permutation is the same for every (b, h).
// Work order of a plan: the rank of tile row t among its slice's rows by
// (decreasing kept-block count, increasing row), stored as
// order[s*T + rank] = t.  One thread per row; the slice's counts are streamed
// through shared memory 256 at a time.  Ranks are distinct, so the result is
// a permutation of 0..T-1 per slice and deterministic.
__global__ void __launch_bounds__(256) tile_order_kernel(const int32_t* __restrict__ tile_ptr, int T,
                                                         int32_t* __restrict__ order) {
  __shared__ int cnt[256];
  const int64_t base_s = static_cast<int64_t>(blockIdx.y) * T;
  const int t = blockIdx.x * 256 + threadIdx.x;
  const int32_t* ptr = tile_ptr + base_s;
  const int mine = t < T ? ptr[t + 1] - ptr[t] : 0;
  int rank = 0;
  for (int base = 0; base < T; base += 256) {
    const int u = base + threadIdx.x;
    cnt[threadIdx.x] = u < T ? ptr[u + 1] - ptr[u] : 0;
    __syncthreads();
    const int lim = T - base < 256 ? T - base : 256;
    for (int i = 0; i < lim; ++i) {
      const int c = cnt[i];
      rank += (c > mine) || (c == mine && base + i < t);
    }
    __syncthreads();
  }
  if (t < T) order[base_s + rank] = t;
}

template <int VB>
__global__ void permute_rows_kernel(uint8_t* __restrict__ dst, const uint8_t* __restrict__ src, int64_t dsb,
                                    int64_t dsh, int64_t dsn, int64_t ssb, int64_t ssh, int64_t ssn, int H, int N,
                                    int vecs_per_row, int64_t total_vecs, const void* __restrict__ perm,
                                    int perm_dtype, int inverse, int32_t* err) {
  using V = typename std::conditional<
      VB == 16, uint4,
      typename std::conditional<VB == 8, uint2,
                                typename std::conditional<VB == 4, uint32_t, uint16_t>::type>::type>::type;
  for (int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < total_vecs;
       g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = g / vecs_per_row;
    const int vi = static_cast<int>(g - r * vecs_per_row);
    const int64_t bh = r / N;
    const int i = static_cast<int>(r - bh * N);
    const int64_t b = bh / H, h = bh - (bh / H) * H;
    const int64_t p = load_index(perm, perm_dtype, i);
    if (p < 0 || p >= N) {
      if (vi == 0) set_err(err, BSA_DEVERR_PERM_RANGE);
      continue;
    }
    const int64_t si = inverse ? i : p;
    const int64_t di = inverse ? p : i;
    const V* s = reinterpret_cast<const V*>(src + b * ssb + h * ssh + si * ssn) + vi;
    V* d = reinterpret_cast<V*>(dst + b * dsb + h * dsh + di * dsn) + vi;
    *d = __ldg(s);
  }
}

__global__ void inverse_perm_kernel(const void* __restrict__ perm, int perm_dtype, int64_t n,
                                    unsigned long long* __restrict__ inv, int32_t* err) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t p = load_index(perm, perm_dtype, i);
    if (p < 0 || p >= n) {
      set_err(err, BSA_DEVERR_PERM_RANGE);
      continue;
    }
    const unsigned long long old = atomicCAS(inv + p, ~0ull, static_cast<unsigned long long>(i));
    if (old != ~0ull) set_err(err, BSA_DEVERR_PERM_DUP);
  }
}

// Permutation check with a bit per value: values outside [0, n) set
// BSA_DEVERR_PERM_RANGE, a value seen twice sets BSA_DEVERR_PERM_DUP.
// `seen` holds ceil(n / 32) words, zeroed beforehand.
__global__ void perm_check_kernel(const void* __restrict__ perm, int perm_dtype, int64_t n,
                                  uint32_t* __restrict__ seen, int32_t* err) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t p = load_index(perm, perm_dtype, i);
    if (p < 0 || p >= n) {
      set_err(err, BSA_DEVERR_PERM_RANGE);
      continue;
    }
    const uint32_t bit = 1u << (p & 31);
    if (atomicOr(seen + (p >> 5), bit) & bit) set_err(err, BSA_DEVERR_PERM_DUP);
  }
}

__global__ void remap_kernel(const int64_t* __restrict__ idx, int64_t count, const int64_t* __restrict__ inv,
                             int64_t n, int64_t* __restrict__ out, int32_t* err) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t x = idx[i];
    if (x < 0 || x >= n) {
      set_err(err, BSA_DEVERR_COORD);
      out[i] = x;
    } else {
      out[i] = inv[x];
    }
  }
}

__global__ void coords_to_mask_kernel(const int64_t* __restrict__ rows, const int64_t* __restrict__ cols,
                                      int64_t count, int64_t seq_len, int block, int64_t nb,
                                      const int64_t* __restrict__ row_inv, const int64_t* __restrict__ col_inv,
                                      uint8_t* __restrict__ mask, int32_t* err) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int64_t r = rows[i], c = cols[i];
    if (r < 0 || c < 0) {
      set_err(err, BSA_DEVERR_COORD);
      continue;
    }
    if (row_inv) {
      if (r >= seq_len) {
        set_err(err, BSA_DEVERR_COORD);
        continue;
      }
      r = row_inv[r];
    }
    if (col_inv) {
      if (c >= seq_len) {
        set_err(err, BSA_DEVERR_COORD);
        continue;
      }
      c = col_inv[c];
    }
    const int64_t rb = r / block, cb = c / block;
    if (rb < nb && cb < nb) mask[rb * nb + cb] = 1;  // identical values: the race is benign
  }
}

// Copy slice 0 of a contiguous [S, nb*nb] byte mask to slices 1..S-1.
__global__ void broadcast_slices_kernel(uint8_t* __restrict__ mask, int64_t slice_bytes, int64_t S) {
  const int64_t total = slice_bytes * (S - 1);
  for (int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < total;
       g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    mask[slice_bytes + g] = mask[g % slice_bytes];
  }
}

inline int grid_for(int64_t work, int threads, int cap = 148 * 16) {
  int64_t g = (work + threads - 1) / threads;
  if (g < 1) g = 1;
  if (g > cap) g = cap;
  return static_cast<int>(g);
}

}  // namespace

int launch_plan_count(const uint8_t* mask, int64_t sb, int64_t sh, int64_t srow, int mask_b, int mask_h, int nb,
                      int block, int32_t* counts, cudaStream_t st) {
  const int T = tiles_per_row(nb, block);
  const int64_t warps = static_cast<int64_t>(mask_b) * mask_h * T;
  plan_count_kernel<<<grid_for(warps * 32, 32 * kWarpsPerBlock), 32 * kWarpsPerBlock, 0, st>>>(
      mask, sb, sh, srow, mask_b, mask_h, nb, 128 / block, T, counts);
  return cudaGetLastError() == cudaSuccess ? BSA_OK : BSA_ERR_CUDA;
}

int launch_plan_scan(const int32_t* counts, int64_t n, int32_t* tile_ptr, cudaStream_t st) {
  plan_scan_kernel<<<1, 1024, 0, st>>>(counts, n, tile_ptr);
  return cudaGetLastError() == cudaSuccess ? BSA_OK : BSA_ERR_CUDA;
}

int launch_plan_fill(const uint8_t* mask, int64_t sb, int64_t sh, int64_t srow, int mask_b, int mask_h, int nb,
                     int block, const int32_t* tile_ptr, int32_t* tile_col, cudaStream_t st) {
  const int T = tiles_per_row(nb, block);
  const int64_t warps = static_cast<int64_t>(mask_b) * mask_h * T;
  plan_fill_kernel<<<grid_for(warps * 32, 32 * kWarpsPerBlock), 32 * kWarpsPerBlock, 0, st>>>(
      mask, sb, sh, srow, mask_b, mask_h, nb, 128 / block, T, tile_ptr, tile_col);
  return cudaGetLastError() == cudaSuccess ? BSA_OK : BSA_ERR_CUDA;
}

int launch_permute_rows(bsa_tensor4d dst, bsa_tensor4d src, int B, int H, int N, int row_elems, int elt_bytes,
                        const void* perm, int perm_dtype, int inverse, int32_t* err, cudaStream_t st) {
  const int64_t row_bytes = static_cast<int64_t>(row_elems) * elt_bytes;
  const int64_t dsb = dst.stride_b * elt_bytes, dsh = dst.stride_h * elt_bytes, dsn = dst.stride_n * elt_bytes;
  const int64_t ssb = src.stride_b * elt_bytes, ssh = src.stride_h * elt_bytes, ssn = src.stride_n * elt_bytes;
  auto aligned = [&](int vb) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(dst.data) | reinterpret_cast<uintptr_t>(src.data);
    return (a % vb) == 0 && row_bytes % vb == 0 && dsb % vb == 0 && dsh % vb == 0 && dsn % vb == 0 &&
           ssb % vb == 0 && ssh % vb == 0 && ssn % vb == 0;
  };
  const int vb = aligned(16) ? 16 : aligned(8) ? 8 : aligned(4) ? 4 : 2;
  const int vecs = static_cast<int>(row_bytes / vb);
  const int64_t total = static_cast<int64_t>(B) * H * N * vecs;
  const int threads = 256;
  const int grid = grid_for(total, threads, 148 * 32);
  uint8_t* d = static_cast<uint8_t*>(dst.data);
  const uint8_t* s = static_cast<const uint8_t*>(src.data);
#define BSA_PERM_LAUNCH(VB)                                                                                         \
  permute_rows_kernel<VB><<<grid, threads, 0, st>>>(d, s, dsb, dsh, dsn, ssb, ssh, ssn, H, N, vecs, total, perm, \
                                                    perm_dtype, inverse, err)
  switch (vb) {
    case 16: BSA_PERM_LAUNCH(16); break;
    case 8: BSA_PERM_LAUNCH(8); break;
    case 4: BSA_PERM_LAUNCH(4); break;
    default: BSA_PERM_LAUNCH(2); break;
  }
#undef BSA_PERM_LAUNCH
  return cudaGetLastError() == cudaSuccess ? BSA_OK : BSA_ERR_CUDA;
}

size_t perm_check_bytes(int64_t n) { return static_cast<size_t>((n + 31) / 32) * 4; }

int launch_perm_check(const void* perm, int perm_dtype, int64_t n, void* scratch, int32_t* err, cudaStream_t st) {
  BSA_CUDA_CHECK(cudaMemsetAsync(scratch, 0, perm_check_bytes(n), st));
  perm_check_kernel<<<grid_for(n, 256), 256, 0, st>>>(perm, perm_dtype, n, static_cast<uint32_t*>(scratch), err);
  return cudaGetLastError() == cudaSuccess ? BSA_OK : BSA_ERR_CUDA;
}

}  // namespace bsa

using namespace bsa;

extern "C" int bsa_plan_sizes(int32_t mask_b, int32_t mask_h, int32_t nb, int32_t block, int64_t* tile_ptr_len,
                              int64_t* tile_col_capacity, size_t* workspace_bytes) {
  if (mask_b <= 0 || mask_h <= 0 || nb <= 0) return BSA_ERR_INVALID_ARG;
  if (block != 64 && block != 128) return BSA_ERR_UNSUPPORTED;
  if (nb >= (1 << 24)) return BSA_ERR_UNSUPPORTED;
  const int64_t T = tiles_per_row(nb, block);
  const int64_t tiles = static_cast<int64_t>(mask_b) * mask_h * T;
  if (tile_ptr_len) *tile_ptr_len = tiles + 1;
  if (tile_col_capacity) *tile_col_capacity = tiles * nb;
  if (workspace_bytes) *workspace_bytes = static_cast<size_t>(tiles) * sizeof(int32_t);
  return BSA_OK;
}

extern "C" int bsa_build_plan(const uint8_t* mask, int64_t stride_b, int64_t stride_h, int64_t stride_row,
                              int32_t mask_b, int32_t mask_h, int32_t nb, int32_t block, int32_t* tile_ptr,
                              int32_t* tile_col, int32_t* tile_order, void* workspace, size_t workspace_bytes,
                              void* stream) {
  size_t need = 0;
  int64_t ptr_len = 0, cap = 0;
  const int rc = bsa_plan_sizes(mask_b, mask_h, nb, block, &ptr_len, &cap, &need);
  if (rc != BSA_OK) return rc;
  if (!mask || !tile_ptr || !tile_col) return BSA_ERR_INVALID_ARG;
  if (!workspace || workspace_bytes < need) return BSA_ERR_WORKSPACE;
  if (cap > INT32_MAX) return BSA_ERR_UNSUPPORTED;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int T = tiles_per_row(nb, block);
  const int64_t n = ptr_len - 1;
  const int64_t mask_bytes = static_cast<int64_t>(mask_b) * mask_h * nb * nb;
  const int64_t chunks = n * ((nb + 15) / 16);
  if (n <= kSmallPlanTiles && T <= kSmallPlanSliceTiles && mask_bytes <= kSmallPlanMaskBytes &&
      chunks <= kSmallPlanChunks) {
    constexpr int kMaxDyn = kSmallPlanMaskBytes + 4 * (2 * kSmallPlanTiles + 1) + 4 * kSmallPlanChunks + 16;
    static bool attr_set[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return BSA_ERR_CUDA;
    if (!attr_set[dev]) {
      BSA_CUDA_CHECK(cudaFuncSetAttribute(plan_small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDyn));
      attr_set[dev] = true;
    }
    const size_t dyn = static_cast<size_t>((mask_bytes + 15) & ~int64_t(15)) + 4 * (2 * n + 1) + 4 * chunks;
    const bool vec16 = reinterpret_cast<uintptr_t>(mask) % 16 == 0 && nb % 16 == 0 && stride_row % 16 == 0 &&
                       (mask_b == 1 || stride_b % 16 == 0) && (mask_h == 1 || stride_h % 16 == 0);
    plan_small_kernel<<<1, 1024, dyn, st>>>(
        mask, stride_b, stride_h, stride_row, mask_h, nb, 128 / block, T, static_cast<int>(n), vec16, tile_ptr,
        tile_col, tile_order);
    return cudaGetLastError() == cudaSuccess ? BSA_OK : BSA_ERR_CUDA;
  }
  int32_t* counts = static_cast<int32_t*>(workspace);
  int r = launch_plan_count(mask, stride_b, stride_h, stride_row, mask_b, mask_h, nb, block, counts, st);
  if (r) return r;
  r = launch_plan_scan(counts, n, tile_ptr, st);
  if (r) return r;
  r = launch_plan_fill(mask, stride_b, stride_h, stride_row, mask_b, mask_h, nb, block, tile_ptr, tile_col, st);
  if (r || !tile_order) return r;
  return bsa_build_tile_order(tile_ptr, mask_b, mask_h, nb, block, tile_order, stream);
}

extern "C" int bsa_build_tile_order(const int32_t* tile_ptr, int32_t mask_b, int32_t mask_h, int32_t nb,
                                    int32_t block, int32_t* tile_order, void* stream) {
  const int rc = bsa_plan_sizes(mask_b, mask_h, nb, block, nullptr, nullptr, nullptr);
  if (rc != BSA_OK) return rc;
  if (!tile_ptr || !tile_order) return BSA_ERR_INVALID_ARG;
  const int64_t T = tiles_per_row(nb, block);
  const int64_t slices = static_cast<int64_t>(mask_b) * mask_h;
  if (slices > 65535) return BSA_ERR_UNSUPPORTED;  // grid.y
  const dim3 grid(static_cast<unsigned>((T + 255) / 256), static_cast<unsigned>(slices));
  tile_order_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(tile_ptr, static_cast<int>(T), tile_order);
  return cudaGetLastError() == cudaSuccess ? BSA_OK : BSA_ERR_CUDA;
}

extern "C" int bsa_permute_rows(bsa_tensor4d dst, bsa_tensor4d src, int32_t B, int32_t H, int32_t N, int32_t D,
                                int32_t dtype, const void* perm, int32_t perm_dtype, int32_t inverse,
                                int32_t* err_flag, void* stream) {
  if (B <= 0 || H <= 0 || N <= 0 || D <= 0) return BSA_ERR_INVALID_ARG;
  if (!dst.data || !src.data || !perm) return BSA_ERR_INVALID_ARG;
  const int eb = dtype_bytes(dtype);
  if (!eb) return BSA_ERR_DTYPE;
  if (perm_dtype != BSA_INDEX_I32 && perm_dtype != BSA_INDEX_I64) return BSA_ERR_DTYPE;
  if (dst.data == src.data) return BSA_ERR_INVALID_ARG;
  return launch_permute_rows(dst, src, B, H, N, D, eb, perm, perm_dtype, inverse, err_flag,
                             static_cast<cudaStream_t>(stream));
}

extern "C" int bsa_inverse_permutation(const void* perm, int32_t perm_dtype, int64_t n, int64_t* inv_out,
                                       int32_t* err_flag, void* stream) {
  if (n < 0) return BSA_ERR_INVALID_ARG;
  if (n == 0) return BSA_OK;
  if (!perm || !inv_out) return BSA_ERR_INVALID_ARG;
  if (perm_dtype != BSA_INDEX_I32 && perm_dtype != BSA_INDEX_I64) return BSA_ERR_DTYPE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  BSA_CUDA_CHECK(cudaMemsetAsync(inv_out, 0xFF, static_cast<size_t>(n) * sizeof(int64_t), st));
  inverse_perm_kernel<<<grid_for(n, 256), 256, 0, st>>>(perm, perm_dtype, n,
                                                        reinterpret_cast<unsigned long long*>(inv_out), err_flag);
  return cudaGetLastError() == cudaSuccess ? BSA_OK : BSA_ERR_CUDA;
}

extern "C" int bsa_remap_indices(const int64_t* idx, int64_t count, const int64_t* inv_perm, int64_t n, int64_t* out,
                                 int32_t* err_flag, void* stream) {
  if (count < 0 || n < 0) return BSA_ERR_INVALID_ARG;
  if (count == 0) return BSA_OK;
  if (!idx || !inv_perm || !out) return BSA_ERR_INVALID_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  remap_kernel<<<grid_for(count, 256), 256, 0, st>>>(idx, count, inv_perm, n, out, err_flag);
  return cudaGetLastError() == cudaSuccess ? BSA_OK : BSA_ERR_CUDA;
}

extern "C" int bsa_blockmask_from_coords(const int64_t* rows, const int64_t* cols, int64_t count, int64_t seq_len,
                                         int32_t block, int32_t B, int32_t H, const int64_t* row_inv,
                                         const int64_t* col_inv, uint8_t* mask_out, int32_t* err_flag,
                                         void* stream) {
  if (count < 0 || seq_len <= 0 || block <= 0 || B <= 0 || H <= 0) return BSA_ERR_INVALID_ARG;
  if (!mask_out || (count > 0 && (!rows || !cols))) return BSA_ERR_INVALID_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t nb = (seq_len + block - 1) / block;
  const int64_t slice = nb * nb;
  const int64_t S = static_cast<int64_t>(B) * H;
  BSA_CUDA_CHECK(cudaMemsetAsync(mask_out, 0, static_cast<size_t>(slice), st));
  if (count > 0) {
    coords_to_mask_kernel<<<grid_for(count, 256), 256, 0, st>>>(rows, cols, count, seq_len, block, nb, row_inv,
                                                               col_inv, mask_out, err_flag);
    BSA_CUDA_CHECK(cudaGetLastError());
  }
  if (S > 1) {
    broadcast_slices_kernel<<<grid_for(slice * (S - 1), 256), 256, 0, st>>>(mask_out, slice, S);
    BSA_CUDA_CHECK(cudaGetLastError());
  }
  return BSA_OK;
}
