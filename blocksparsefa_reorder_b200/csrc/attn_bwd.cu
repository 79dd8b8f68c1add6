// Block-sparse attention backward for sm_100a: BLOCK 64 or 128, head dim 64
// or 128, bf16 / fp16, no token permutation.
//
// The reference has no backward pass: its kernels write the row log-sum-exp
// M (triton_kernels/BlockSparse_Naive.py:119-122) and nothing consumes it.
// This is the gradient of the forward in attn_tcp.cu, recomputing P from
// that LSE (log2 units) instead of storing it:
//   P = 2^(s * scale_log2 - lse)      s = q . k, per kept block
//   dP = dO V^T,  Delta = rowsum(dO o O),  dS = P o (dP - Delta)
//   dQ = sm_scale dS K,  dK = sm_scale dS^T Q,  dV = P^T dO
// Three kernels, no atomics (every output row is written by one CTA, so the
// result is deterministic):
//  * bwd_delta_kernel: Delta per query row (16-byte loads);
//  * bwd_dq_kernel: one CTA per 128-row query tile over the tile's plan
//    entries (kept key blocks of BN keys, one per step): S = Q K^T and
//    dP = dO V^T on tcgen05 into TMEM, dS by the elementwise warpgroup
//    (written back as 16-bit pairs over S's first BN/2 columns), dQ += dS K
//    (A from TMEM, K as the MN-major B).  At BLOCK 64 a tile holds two query
//    blocks and an entry's flags say which of them keeps it: the other
//    block's rows get P = 0;
//  * bwd_dkdv_kernel: one CTA per 128-key tile over the entries of the
//    transposed mask's plan (query blocks of BN rows that keep a key block
//    of the tile): S^T = K Q^T and dP^T = V dO^T into TMEM, P^T and dS^T by
//    the elementwise warpgroup (the query rows' LSE and Delta staged in
//    shared memory per step; at BLOCK 64 the key rows of a key block the
//    query block does not keep get P = 0), dV += P^T dO and dK += dS^T Q (dO
//    and Q as MN-major B operands).
// Roles per CTA (192 threads): warp 0 one thread, TMA producer; warp 1
// allocates TMEM and one thread issues the MMAs; warps 2-5, one row per
// thread (TMEM lane quarter = warp % 4), the elementwise work and the
// epilogue.  K/V (or Q/dO) stages are double-buffered; every wait is bounded.
#include <cudaTypedefs.h>

#include <atomic>

#include "common.cuh"
#include "internal.h"

namespace bsa {

namespace {

constexpr int kBwdThreads = 192;

struct BwdParams {
  const int32_t* tile_ptr;
  const int32_t* tile_col;
  int mask_b, mask_h, T, nb;
  int H, N;
  float scale_log2, sm_scale;
  const float* lse;    // [B, H, N] log2 units
  const float* delta;  // [B, H, N]
  uint8_t* out;        // dQ (dq kernel) or dK (dkdv kernel), 16-bit elements
  int64_t os_b, os_h, os_n;
  uint8_t* out2;       // dV (dkdv kernel)
  int64_t os2_b, os2_h, os2_n;
  int32_t* err;
  uint64_t wait_ns;
};

// BN: the block size; the streamed operand of each kernel (K / V in the dQ
// kernel, Q / dO in the dK/dV kernel) comes in tiles of BN rows, the
// resident one (Q / dO, resp. K / V) in 128-row tiles.
template <int D, int BN>
struct BwdCfg {
  static constexpr int NCHUNK = D / 64;
  static constexpr int CHUNK = 128 * 128;    // one 64-column chunk of a 128-row tile (128-byte swizzle)
  static constexpr int TILE = 128 * D * 2;   // a 128-row tile of D 16-bit columns
  static constexpr int SCHUNK = BN * 128;    // one 64-column chunk of a BN-row tile
  static constexpr int STILE = BN * D * 2;   // a BN-row tile
  static constexpr int BAR_BYTES = 256;
};

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void ew_bar_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// The 128x(D) accumulator in TMEM columns [col, col + D) of this thread's
// lane, times `scale`, as one 16-bit row in global memory.
template <int D, bool BF16>
__device__ __forceinline__ void store_acc_row(uint32_t lane_base, int col, float scale, uint8_t* row, bool store) {
#pragma unroll
  for (int c = 0; c < D / 32; ++c) {
    uint32_t a[32];
    tmem_ld32(lane_base + col + c * 32, a);
    tmem_wait_ld();
    if (store) {
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        uint4 v;
        v.x = pack2<BF16>(__uint_as_float(a[8 * g + 0]) * scale, __uint_as_float(a[8 * g + 1]) * scale);
        v.y = pack2<BF16>(__uint_as_float(a[8 * g + 2]) * scale, __uint_as_float(a[8 * g + 3]) * scale);
        v.z = pack2<BF16>(__uint_as_float(a[8 * g + 4]) * scale, __uint_as_float(a[8 * g + 5]) * scale);
        v.w = pack2<BF16>(__uint_as_float(a[8 * g + 6]) * scale, __uint_as_float(a[8 * g + 7]) * scale);
        reinterpret_cast<uint4*>(row)[c * 4 + g] = v;
      }
    }
  }
}

template <int D>
__device__ __forceinline__ void zero_row(uint8_t* row) {
#pragma unroll
  for (int i = 0; i < D / 8; ++i) reinterpret_cast<uint4*>(row)[i] = make_uint4(0, 0, 0, 0);
}

// Delta[b, h, n] = sum_d dO[n, d] * O[n, d] in fp32: each row read by D / 8
// lanes with 16-byte loads (two rows per warp at D = 128, four at D = 64).
template <bool BF16, int D>
__global__ void __launch_bounds__(256) bwd_delta_kernel(const uint8_t* o, int64_t o_b, int64_t o_h, int64_t o_n,
                                                        const uint8_t* dout, int64_t d_b, int64_t d_h, int64_t d_n,
                                                        float* delta, int B, int H, int N) {
  constexpr int LPR = D / 8;  // lanes per row
  const int lane = threadIdx.x & 31;
  const int64_t r = (static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5)) * (32 / LPR) + lane / LPR;
  const bool live = r < static_cast<int64_t>(B) * H * N;
  float acc = 0.f;
  if (live) {
    const int64_t bh = r / N, n = r - bh * N, b = bh / H, h = bh - b * H;
    const int d = (lane % LPR) * 8;
    const uint4 ov = *reinterpret_cast<const uint4*>(o + 2 * (b * o_b + h * o_h + n * o_n + d));
    const uint4 dv = *reinterpret_cast<const uint4*>(dout + 2 * (b * d_b + h * d_h + n * d_n + d));
    const uint32_t ow[4] = {ov.x, ov.y, ov.z, ov.w}, dw[4] = {dv.x, dv.y, dv.z, dv.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float o0, o1, d0, d1;
      if constexpr (BF16) {
        o0 = __uint_as_float(ow[k] << 16), o1 = __uint_as_float(ow[k] & 0xFFFF0000u);
        d0 = __uint_as_float(dw[k] << 16), d1 = __uint_as_float(dw[k] & 0xFFFF0000u);
      } else {
        const __half2 oh = *reinterpret_cast<const __half2*>(&ow[k]);
        const __half2 dh = *reinterpret_cast<const __half2*>(&dw[k]);
        o0 = __low2float(oh), o1 = __high2float(oh), d0 = __low2float(dh), d1 = __high2float(dh);
      }
      acc = fmaf(o0, d0, fmaf(o1, d1, acc));
    }
  }
#pragma unroll
  for (int off = LPR / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (live && lane % LPR == 0) delta[r] = acc;
}

// ---------------------------------------------------------------------------
// dQ: one CTA per 128-row query tile.
// TMEM columns: S_j / dS_j in [128 (j & 1), +128), dP [256, 384), dQ
// [384, 384 + D).  S is double-buffered: S_j+1 is computed while the
// elementwise warpgroup turns S_j and dP_j into dS_j; then dP_j+1 is issued
// before dQ_j, so the next elementwise step waits for one MMA group, not
// three.
// ---------------------------------------------------------------------------
template <int D, int BN, bool BF16>
__global__ void __launch_bounds__(kBwdThreads, 1)
    bwd_dq_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                  const BwdParams p) {
  using C = BwdCfg<D, BN>;
  extern __shared__ __align__(1024) uint8_t smem[];
  if (smem_u32(smem) & 1023u) {
    if (threadIdx.x == 0) set_err(p.err, BSA_DEVERR_ALIGN);
    return;
  }
  uint8_t* sQ = smem;
  uint8_t* sDO = sQ + C::TILE;
  uint8_t* sK = sDO + C::TILE;      // [2][STILE]
  uint8_t* sV = sK + 2 * C::STILE;  // [2][STILE]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + 2 * C::STILE);
  uint64_t* q_full = bars;        // Q and dO of the tile landed
  uint64_t* kv_full = bars + 1;   // [2] K_j, V_j landed
  uint64_t* kv_empty = bars + 3;  // [2] dQ_j (the last reader of K_j) completed
  uint64_t* s_full = bars + 5;    // [2] S_j complete, by S buffer j & 1
  uint64_t* dp_full = bars + 7;   // dP_j complete
  uint64_t* ds_ready = bars + 8;  // 4 elementwise warps wrote dS_j (and are done with dP_j)
  uint64_t* done = bars + 9;      // every MMA complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 10);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x / p.T, t = blockIdx.x - bh * p.T;
  const int b = bh / p.H, h = bh - b * p.H;
  const int sl = (p.mask_b == 1 ? 0 : b) * p.mask_h + (p.mask_h == 1 ? 0 : h);
  const int e0 = p.tile_ptr[sl * p.T + t];
  const int n = p.tile_ptr[sl * p.T + t + 1] - e0;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) mbar_init(&s_full[i], 1);
    mbar_init(dp_full, 1);
    mbar_init(ds_ready, 4);
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  constexpr uint32_t kDP = 256, kDQ = 384;  // TMEM columns of dP and dQ
  // plan entry j: (flags << 24) | key block
  auto entry = [&](int j) -> uint32_t {
    uint32_t en = static_cast<uint32_t>(p.tile_col[e0 + j]);
    if (static_cast<int>(en & 0xFFFFFFu) >= p.nb) {
      set_err(p.err, BSA_DEVERR_PLAN);
      en &= 0xFF000000u;
    }
    return en;
  };

  if (warp == 0 && lane == 0 && n > 0) {
    // ------------------------------------------------------------- producer
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmDO);
    mbar_arrive_expect_tx(q_full, 2 * C::TILE);
    for (int c = 0; c < C::NCHUNK; ++c) {
      tma_load_4d(sQ + c * C::CHUNK, &tmQ, q_full, c * 64, t * 128, h, b);
      tma_load_4d(sDO + c * C::CHUNK, &tmDO, q_full, c * 64, t * 128, h, b);
    }
    int j = 0;
    for (; j < n; ++j) {
      const int st = j & 1;
      if (j >= 2 && !mbar_wait(&kv_empty[st], ((j >> 1) - 1) & 1, abort_flag, p.err, p.wait_ns)) break;
      const int kb = static_cast<int>(entry(j) & 0xFFFFFFu);
      mbar_arrive_expect_tx(&kv_full[st], 2 * C::STILE);
      for (int c = 0; c < C::NCHUNK; ++c) {
        tma_load_4d(sK + st * C::STILE + c * C::SCHUNK, &tmK, &kv_full[st], c * 64, kb * BN, h, b);
        tma_load_4d(sV + st * C::STILE + c * C::SCHUNK, &tmV, &kv_full[st], c * 64, kb * BN, h, b);
      }
    }
    // every load issued lands before the CTA exits
    mbar_wait(q_full, 0, nullptr, nullptr, p.wait_ns);
    for (int i = j > 2 ? j - 2 : 0; i < j; ++i) mbar_wait(&kv_full[i & 1], (i >> 1) & 1, nullptr, nullptr, p.wait_ns);
  } else if (warp == 1 && lane == 0 && n > 0) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc_s = make_idesc_f16(BF16, 128, BN, false, false);
    constexpr uint32_t idesc_dq = make_idesc_f16(BF16, 128, D, false, true);
    const uint32_t q_addr = smem_u32(sQ), do_addr = smem_u32(sDO), k_addr = smem_u32(sK), v_addr = smem_u32(sV);
    // S_j = Q K_j^T into S buffer j & 1; dP_j = dO V_j^T
    auto issue_s = [&](int j) {
      const int st = j & 1;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint32_t off = (kk & 3) * 32;
        tc_mma_ss(tmem + st * 128, make_sw128_desc(q_addr + (kk >> 2) * C::CHUNK + off, 16, 1024),
                  make_sw128_desc(k_addr + st * C::STILE + (kk >> 2) * C::SCHUNK + off, 16, 1024), idesc_s,
                  kk > 0 ? 1u : 0u);
      }
      tc_commit(&s_full[st]);
    };
    auto issue_dp = [&](int j) {
      const int st = j & 1;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint32_t off = (kk & 3) * 32;
        tc_mma_ss(tmem + kDP, make_sw128_desc(do_addr + (kk >> 2) * C::CHUNK + off, 16, 1024),
                  make_sw128_desc(v_addr + st * C::STILE + (kk >> 2) * C::SCHUNK + off, 16, 1024), idesc_s,
                  kk > 0 ? 1u : 0u);
      }
      tc_commit(dp_full);
    };
    bool ok = mbar_wait(q_full, 0, abort_flag, p.err, p.wait_ns) && mbar_wait(&kv_full[0], 0, abort_flag, p.err, p.wait_ns);
    if (ok) {
      tc_fence_after();
      issue_s(0);
      issue_dp(0);
    }
    for (int j = 0; ok && j < n; ++j) {
      const int st = j & 1;
      // S_j+1 into the other buffer while the elementwise warps work on step j
      // (that buffer's dS_j-1 was read by dQ_j-1, issued before)
      if (j + 1 < n) {
        if (!(ok = mbar_wait(&kv_full[st ^ 1], ((j + 1) >> 1) & 1, abort_flag, p.err, p.wait_ns))) break;
        tc_fence_after();
        issue_s(j + 1);
      }
      if (!(ok = mbar_wait(ds_ready, j & 1, abort_flag, p.err, p.wait_ns))) break;
      tc_fence_after();
      // dP's buffer is free again: dP_j+1 first, so that step j+1 can start
      if (j + 1 < n) issue_dp(j + 1);
      // dQ += dS_j K_j: dS in the first BN/2 columns of S buffer j & 1, K_j MN-major (N = D)
#pragma unroll
      for (int kk = 0; kk < BN / 16; ++kk)
        tc_mma_ts(tmem + kDQ, tmem + st * 128 + kk * 8,
                  make_sw128_desc(k_addr + st * C::STILE + kk * 16 * 128, C::SCHUNK, 1024), idesc_dq,
                  (j > 0 || kk > 0) ? 1u : 0u);
      tc_commit(&kv_empty[st]);
    }
    tc_commit(done);
    mbar_wait(done, 0, nullptr, nullptr, p.wait_ns);
  } else if (warp >= 2) {
    // ------------------------------------------------- elementwise, epilogue
    const int q4 = warp & 3;
    const int row = q4 * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q4 * 32) << 16);
    const int grow = t * 128 + row;
    const bool live = grow < p.N;
    uint8_t* orow = p.out + 2 * (b * p.os_b + h * p.os_h + static_cast<int64_t>(grow) * p.os_n);
    if (n == 0) {
      if (live) zero_row<D>(orow);
    } else {
      const int64_t ri = (static_cast<int64_t>(b) * p.H + h) * p.N + grow;
      // rows past N: P = 0 (lse = +inf)
      const float neg_lse = live ? -__ldg(&p.lse[ri]) : -INFINITY;
      const float dlt = live ? __ldg(&p.delta[ri]) : 0.f;
      bool ok = true;
      for (int j = 0; j < n; ++j) {
        if (!(ok = ok && __all_sync(0xffffffffu, mbar_wait(&s_full[j & 1], (j >> 1) & 1, abort_flag, p.err,
                                                              p.wait_ns) &&
                                                       mbar_wait(dp_full, j & 1, abort_flag, p.err, p.wait_ns))))
          break;
        tc_fence_after();
        const uint32_t s_col = (j & 1) * 128;
        const uint32_t en = entry(j);
        // keys at or past N, and at BLOCK 64 every key of an entry this row's
        // query block does not keep: P = 0
        const int kvalid = ((en >> 24 >> (BN == 64 ? row >> 6 : 0)) & 1u)
                               ? p.N - static_cast<int>(en & 0xFFFFFFu) * BN : 0;
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t sv[32], dp[32], ds[16];
          tmem_ld32(lane_base + s_col + c * 32, sv);
          tmem_ld32(lane_base + kDP + c * 32, dp);
          tmem_wait_ld();
#pragma unroll
          for (int k = 0; k < 32; k += 2) {
            const float p0 = c * 32 + k < kvalid ? ex2_approx(fmaf(__uint_as_float(sv[k]), p.scale_log2, neg_lse)) : 0.f;
            const float p1 =
                c * 32 + k + 1 < kvalid ? ex2_approx(fmaf(__uint_as_float(sv[k + 1]), p.scale_log2, neg_lse)) : 0.f;
            ds[k / 2] = pack2<BF16>(p0 * (__uint_as_float(dp[k]) - dlt), p1 * (__uint_as_float(dp[k + 1]) - dlt));
          }
          // dS columns [16c, 16c + 16) hold S columns already read (chunks <= c)
          tmem_st16(lane_base + s_col + c * 16, ds);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(ds_ready);
      }
      ok = ok && __all_sync(0xffffffffu, mbar_wait(done, 0, abort_flag, p.err, p.wait_ns));
      if (ok) {
        tc_fence_after();
        store_acc_row<D, BF16>(lane_base, kDQ, p.sm_scale, orow, live);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------
// dK, dV: one CTA per 128-key block, over the query blocks that keep it.
// TMEM columns: S^T / P^T [0, 128), dP^T / dS^T [128, 256), dV [256, 256 + D),
// dK [256 + D, 256 + 2D).
// ---------------------------------------------------------------------------
template <int D, int BN, bool BF16>
__global__ void __launch_bounds__(kBwdThreads, 1)
    bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                    const BwdParams p) {
  using C = BwdCfg<D, BN>;
  extern __shared__ __align__(1024) uint8_t smem[];
  if (smem_u32(smem) & 1023u) {
    if (threadIdx.x == 0) set_err(p.err, BSA_DEVERR_ALIGN);
    return;
  }
  uint8_t* sK = smem;
  uint8_t* sV = sK + C::TILE;
  uint8_t* sQ = sV + C::TILE;        // [2][STILE]
  uint8_t* sDO = sQ + 2 * C::STILE;  // [2][STILE]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sDO + 2 * C::STILE);
  float* col_lse = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + C::BAR_BYTES);  // [2][128]
  float* col_dlt = col_lse + 256;                                                                  // [2][128]
  uint64_t* kv_full = bars;       // K and V of the key block landed
  uint64_t* qd_full = bars + 1;   // [2] Q_i, dO_i landed
  uint64_t* qd_empty = bars + 3;  // [2] dV_i and dK_i (the last readers) completed
  uint64_t* s_full = bars + 5;    // S^T_i and dP^T_i complete
  uint64_t* pt_ready = bars + 6;  // 4 elementwise warps wrote P^T_i, dS^T_i
  uint64_t* done = bars + 7;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 8);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.x / p.T, jt = blockIdx.x - bh * p.T;
  const int b = bh / p.H, h = bh - b * p.H;
  const int sl = (p.mask_b == 1 ? 0 : b) * p.mask_h + (p.mask_h == 1 ? 0 : h);
  const int e0 = p.tile_ptr[sl * p.T + jt];
  const int n = p.tile_ptr[sl * p.T + jt + 1] - e0;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&qd_full[i], 1);
      mbar_init(&qd_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(pt_ready, 4);
    mbar_init(done, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // entry i of the transposed plan: (flags << 24) | query block; flag bit
  // 0 / 1 = the tile's first / second key block is kept by that query block
  auto entry = [&](int i) -> uint32_t {
    uint32_t en = static_cast<uint32_t>(p.tile_col[e0 + i]);
    if (static_cast<int>(en & 0xFFFFFFu) >= p.nb) {
      set_err(p.err, BSA_DEVERR_PLAN);
      en &= 0xFF000000u;
    }
    return en;
  };

  if (warp == 0 && lane == 0 && n > 0) {
    // ------------------------------------------------------------- producer
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmDO);
    mbar_arrive_expect_tx(kv_full, 2 * C::TILE);
    for (int c = 0; c < C::NCHUNK; ++c) {
      tma_load_4d(sK + c * C::CHUNK, &tmK, kv_full, c * 64, jt * 128, h, b);
      tma_load_4d(sV + c * C::CHUNK, &tmV, kv_full, c * 64, jt * 128, h, b);
    }
    int i = 0;
    for (; i < n; ++i) {
      const int st = i & 1;
      if (i >= 2 && !mbar_wait(&qd_empty[st], ((i >> 1) - 1) & 1, abort_flag, p.err, p.wait_ns)) break;
      const int qb = static_cast<int>(entry(i) & 0xFFFFFFu);
      mbar_arrive_expect_tx(&qd_full[st], 2 * C::STILE);
      for (int c = 0; c < C::NCHUNK; ++c) {
        tma_load_4d(sQ + st * C::STILE + c * C::SCHUNK, &tmQ, &qd_full[st], c * 64, qb * BN, h, b);
        tma_load_4d(sDO + st * C::STILE + c * C::SCHUNK, &tmDO, &qd_full[st], c * 64, qb * BN, h, b);
      }
    }
    mbar_wait(kv_full, 0, nullptr, nullptr, p.wait_ns);
    for (int k = i > 2 ? i - 2 : 0; k < i; ++k) mbar_wait(&qd_full[k & 1], (k >> 1) & 1, nullptr, nullptr, p.wait_ns);
  } else if (warp == 1 && lane == 0 && n > 0) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc_s = make_idesc_f16(BF16, 128, BN, false, false);
    constexpr uint32_t idesc_acc = make_idesc_f16(BF16, 128, D, false, true);
    const uint32_t k_addr = smem_u32(sK), v_addr = smem_u32(sV), q_addr = smem_u32(sQ), do_addr = smem_u32(sDO);
    bool ok = mbar_wait(kv_full, 0, abort_flag, p.err, p.wait_ns);
    for (int i = 0; ok && i < n; ++i) {
      const int st = i & 1;
      if (!(ok = mbar_wait(&qd_full[st], (i >> 1) & 1, abort_flag, p.err, p.wait_ns))) break;
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint32_t off = (kk & 3) * 32;
        tc_mma_ss(tmem, make_sw128_desc(k_addr + (kk >> 2) * C::CHUNK + off, 16, 1024),
                  make_sw128_desc(q_addr + st * C::STILE + (kk >> 2) * C::SCHUNK + off, 16, 1024), idesc_s,
                  kk > 0 ? 1u : 0u);
      }
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint32_t off = (kk & 3) * 32;
        tc_mma_ss(tmem + 128, make_sw128_desc(v_addr + (kk >> 2) * C::CHUNK + off, 16, 1024),
                  make_sw128_desc(do_addr + st * C::STILE + (kk >> 2) * C::SCHUNK + off, 16, 1024), idesc_s,
                  kk > 0 ? 1u : 0u);
      }
      tc_commit(s_full);
      if (!(ok = mbar_wait(pt_ready, i & 1, abort_flag, p.err, p.wait_ns))) break;
      tc_fence_after();
      // dV += P^T dO_i, dK += dS^T Q_i (P^T, dS^T as 16-bit pairs in TMEM; dO_i, Q_i MN-major, N = D)
#pragma unroll
      for (int kk = 0; kk < BN / 16; ++kk)
        tc_mma_ts(tmem + 256, tmem + kk * 8,
                  make_sw128_desc(do_addr + st * C::STILE + kk * 16 * 128, C::SCHUNK, 1024), idesc_acc,
                  (i > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
      for (int kk = 0; kk < BN / 16; ++kk)
        tc_mma_ts(tmem + 256 + D, tmem + 128 + kk * 8,
                  make_sw128_desc(q_addr + st * C::STILE + kk * 16 * 128, C::SCHUNK, 1024), idesc_acc,
                  (i > 0 || kk > 0) ? 1u : 0u);
      tc_commit(&qd_empty[st]);
    }
    tc_commit(done);
    mbar_wait(done, 0, nullptr, nullptr, p.wait_ns);
  } else if (warp >= 2) {
    // ------------------------------------------------- elementwise, epilogue
    const int q4 = warp & 3;
    const int row = q4 * 32 + lane;  // key row of the block; also the query column it stages
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q4 * 32) << 16);
    const int krow = jt * 128 + row;
    const bool live = krow < p.N;
    uint8_t* krow_out = p.out + 2 * (b * p.os_b + h * p.os_h + static_cast<int64_t>(krow) * p.os_n);
    uint8_t* vrow_out = p.out2 + 2 * (b * p.os2_b + h * p.os2_h + static_cast<int64_t>(krow) * p.os2_n);
    if (n == 0) {
      if (live) {
        zero_row<D>(krow_out);
        zero_row<D>(vrow_out);
      }
    } else {
      const int64_t base = (static_cast<int64_t>(b) * p.H + h) * p.N;
      bool ok = true;
      for (int i = 0; i < n; ++i) {
        // the query rows' LSE and Delta for this step (rows past N: P = 0)
        const uint32_t en = entry(i);
        const int qrow = static_cast<int>(en & 0xFFFFFFu) * BN + row;
        float* lb = col_lse + (i & 1) * 128;
        float* db = col_dlt + (i & 1) * 128;
        if (row < BN) {
          lb[row] = qrow < p.N ? -__ldg(&p.lse[base + qrow]) : -INFINITY;
          db[row] = qrow < p.N ? __ldg(&p.delta[base + qrow]) : 0.f;
        }
        // at BLOCK 64: a key row of the tile's block that this query block does not keep gets P = 0
        const bool act = BN == 128 || ((en >> 24 >> (row >> 6)) & 1u) != 0;
        // (a warp whose wait failed keeps taking part in this barrier, which
        // has no time limit, and skips the rest of each step)
        ew_bar_sync();
        if (!(ok = ok && __all_sync(0xffffffffu, mbar_wait(s_full, i & 1, abort_flag, p.err, p.wait_ns)))) continue;
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t sv[32], dp[32], pt[16], ds[16];
          tmem_ld32(lane_base + c * 32, sv);
          tmem_ld32(lane_base + 128 + c * 32, dp);
          tmem_wait_ld();
#pragma unroll
          for (int k = 0; k < 32; k += 2) {
            const int q = c * 32 + k;
            const float p0 = act ? ex2_approx(fmaf(__uint_as_float(sv[k]), p.scale_log2, lb[q])) : 0.f;
            const float p1 = act ? ex2_approx(fmaf(__uint_as_float(sv[k + 1]), p.scale_log2, lb[q + 1])) : 0.f;
            pt[k / 2] = pack2<BF16>(p0, p1);
            ds[k / 2] = pack2<BF16>(p0 * (__uint_as_float(dp[k]) - db[q]), p1 * (__uint_as_float(dp[k + 1]) - db[q + 1]));
          }
          // columns [16c, 16c + 16) of both buffers were read already (chunks <= c)
          tmem_st16(lane_base + c * 16, pt);
          tmem_st16(lane_base + 128 + c * 16, ds);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(pt_ready);
      }
      ok = ok && __all_sync(0xffffffffu, mbar_wait(done, 0, abort_flag, p.err, p.wait_ns));
      if (ok) {
        tc_fence_after();
        store_acc_row<D, BF16>(lane_base, 256, 1.f, vrow_out, live);
        store_acc_row<D, BF16>(lane_base, 256 + D, p.sm_scale, krow_out, live);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int D, int BN, bool BF16>
int launch_bwd_t(const bsa_bwd_args* a, cudaStream_t st) {
  using C = BwdCfg<D, BN>;
  constexpr int kSmemDq = 2 * C::TILE + 4 * C::STILE + C::BAR_BYTES;
  constexpr int kSmemDkdv = 2 * C::TILE + 4 * C::STILE + C::BAR_BYTES + 2048;
  static_assert(kSmemDkdv <= 232448, "shared memory budget");
  static std::atomic<bool> attr_set[64] = {};
  int dev = 0;
  BSA_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return BSA_ERR_DEVICE;
  if (!attr_set[dev].load(std::memory_order_acquire)) {
    BSA_CUDA_CHECK(
        cudaFuncSetAttribute(bwd_dq_kernel<D, BN, BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemDq));
    BSA_CUDA_CHECK(
        cudaFuncSetAttribute(bwd_dkdv_kernel<D, BN, BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemDkdv));
    attr_set[dev].store(true, std::memory_order_release);
  }
  // 128-row tiles of the resident operands, BN-row tiles of the streamed ones
  CUtensorMap mq, mk, mv, mdo, mq_s, mk_s, mv_s, mdo_s;
  int r;
  if ((r = make_tensor_map_4d(&mq, a->q, a->B, a->H, a->N, D, BF16, 128))) return r;
  if ((r = make_tensor_map_4d(&mk, a->k, a->B, a->H, a->N, D, BF16, 128))) return r;
  if ((r = make_tensor_map_4d(&mv, a->v, a->B, a->H, a->N, D, BF16, 128))) return r;
  if ((r = make_tensor_map_4d(&mdo, a->dout, a->B, a->H, a->N, D, BF16, 128))) return r;
  if ((r = make_tensor_map_4d(&mq_s, a->q, a->B, a->H, a->N, D, BF16, BN))) return r;
  if ((r = make_tensor_map_4d(&mk_s, a->k, a->B, a->H, a->N, D, BF16, BN))) return r;
  if ((r = make_tensor_map_4d(&mv_s, a->v, a->B, a->H, a->N, D, BF16, BN))) return r;
  if ((r = make_tensor_map_4d(&mdo_s, a->dout, a->B, a->H, a->N, D, BF16, BN))) return r;

  const int64_t rows = static_cast<int64_t>(a->B) * a->H * a->N;
  const int64_t rows_per_block = 8 * (32 / (D / 8));
  bwd_delta_kernel<BF16, D><<<static_cast<unsigned>((rows + rows_per_block - 1) / rows_per_block), 256, 0, st>>>(
      static_cast<const uint8_t*>(a->o.data), a->o.stride_b, a->o.stride_h, a->o.stride_n,
      static_cast<const uint8_t*>(a->dout.data), a->dout.stride_b, a->dout.stride_h, a->dout.stride_n, a->delta,
      a->B, a->H, a->N);
  BSA_CUDA_CHECK(cudaGetLastError());

  BwdParams p{};
  p.H = a->H;
  p.N = a->N;
  p.scale_log2 = a->sm_scale * 1.4426950408889634f;
  p.sm_scale = a->sm_scale;
  p.lse = a->lse;
  p.delta = a->delta;
  p.err = a->err_flag;
  p.wait_ns = kWaitNs;

  p.tile_ptr = a->plan.tile_ptr;
  p.tile_col = a->plan.tile_col;
  p.mask_b = a->plan.mask_b;
  p.mask_h = a->plan.mask_h;
  p.nb = a->plan.nb;
  p.T = tiles_per_row(a->plan.nb, BN);
  p.out = static_cast<uint8_t*>(a->dq.data);
  p.os_b = a->dq.stride_b;
  p.os_h = a->dq.stride_h;
  p.os_n = a->dq.stride_n;
  bwd_dq_kernel<D, BN, BF16>
      <<<static_cast<unsigned>(a->B * a->H * p.T), kBwdThreads, kSmemDq, st>>>(mq, mk_s, mv_s, mdo, p);
  BSA_CUDA_CHECK(cudaGetLastError());

  p.tile_ptr = a->plan_t.tile_ptr;
  p.tile_col = a->plan_t.tile_col;
  p.mask_b = a->plan_t.mask_b;
  p.mask_h = a->plan_t.mask_h;
  p.nb = a->plan_t.nb;
  p.T = tiles_per_row(a->plan_t.nb, BN);
  p.out = static_cast<uint8_t*>(a->dk.data);
  p.os_b = a->dk.stride_b;
  p.os_h = a->dk.stride_h;
  p.os_n = a->dk.stride_n;
  p.out2 = static_cast<uint8_t*>(a->dv.data);
  p.os2_b = a->dv.stride_b;
  p.os2_h = a->dv.stride_h;
  p.os2_n = a->dv.stride_n;
  bwd_dkdv_kernel<D, BN, BF16>
      <<<static_cast<unsigned>(a->B * a->H * p.T), kBwdThreads, kSmemDkdv, st>>>(mq_s, mk, mv, mdo_s, p);
  BSA_CUDA_CHECK(cudaGetLastError());
  return BSA_OK;
}

}  // namespace

int launch_attn_bwd(const bsa_bwd_args* a, cudaStream_t st) {
  const bool bf16 = a->dtype == BSA_DTYPE_BF16;
#define BSA_BWD_CASE(D_, BN_)                                                                  \
  if (a->D == D_ && a->plan.block == BN_)                                                     \
    return bf16 ? launch_bwd_t<D_, BN_, true>(a, st) : launch_bwd_t<D_, BN_, false>(a, st);
  BSA_BWD_CASE(128, 128)
  BSA_BWD_CASE(64, 128)
  BSA_BWD_CASE(128, 64)
  BSA_BWD_CASE(64, 64)
#undef BSA_BWD_CASE
  return BSA_ERR_UNSUPPORTED;
}

}  // namespace bsa
