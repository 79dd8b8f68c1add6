// Persistent tcgen05 block-sparse attention forward for sm_100a.
//
// The pipeline of attn_tc.cu (one 128-row query tile at a time: TMA
// producer warp, one MMA-issuing thread, one softmax warpgroup, S
// double-buffered in TMEM) run by one CTA per SM over many tiles, so that
// one tile's epilogue and the next tile's start overlap instead of leaving
// the tensor cores idle between CTAs.  Replaces _attn_fwd_block_sparse
// (triton_kernels/BlockSparse_Naive.py:68-125); results are those of the
// reference's online softmax (:39-60, 119-125): rows with no kept block give
// O = 0 and lse = -inf.
//
// Work: CTA c takes tiles w = c, c + G, c + 2G, ... of the (b, h)-major tile
// order (w = bh * T + t), so the CTAs in flight share a head's K / V in L2.
//
// Across tiles:
//  * block counter j runs on from tile to tile: S_j goes to TMEM buffer j&1
//    and P_j is written back into the first columns of that buffer (the
//    next S into the buffer is issued after the PV that reads P, and one
//    thread's tcgen05.mma operations execute in issue order);
//  * non-empty tiles alternate between two Q buffers in shared memory and
//    two O accumulators in TMEM (counter e);
//  * the MMA thread issues the last PV of a tile after the first S of the
//    next, and waits for the epilogue to have read an O buffer (o_empty)
//    before the first PV that overwrites it;
//  * the epilogue stages O in the tile's Q buffer for the TMA store and
//    releases that buffer to the producer (q_empty) once the store has read
//    it, which is checked during the next tile's first block.
// TMEM columns: S0 [0,BN), S1 [BN,2BN), O0 [2BN, 2BN+D), O1 [2BN+D, 2BN+2D).
//
// Every wait is bounded by %globaltimer; a timeout sets BSA_DEVERR_TIMEOUT
// and all roles drain and exit.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "internal.h"
#include "softmax.cuh"

namespace bsa {

namespace {

struct TcpParams {
  const int32_t* tile_ptr;
  const int32_t* tile_col;
  float* lse;
  void* o_raw;  // for the zero rows of empty tiles (plain stores)
  int64_t os_b, os_h, os_n;
  int32_t* err;
  int H, N, nb, T, mask_b, mask_h, total_tiles;
  float scale_log2;
};

constexpr int kSmemLimitP = 232448;

template <int D, int BN>
struct TcpCfg {
  static constexpr int BM = 128;
  static constexpr int NCHUNK = D / 64;
  static constexpr int Q_CHUNK = BM * 128;
  static constexpr int KV_CHUNK = BN * 128;
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_BYTES = BN * D * 2;
  static constexpr int BAR_BYTES = 512;
  // K and V have their own rings: K_j is released when S_j completes, V_j only
  // when PV_j does, one block later, so K gets the deeper ring.
  static constexpr bool fits(int ks, int vs) { return 2 * Q_BYTES + (ks + vs) * KV_BYTES + BAR_BYTES <= kSmemLimitP; }
  static constexpr int KS = fits(4, 4) || fits(4, 3) ? 4 : 3;
  static constexpr int VS = fits(4, 4) ? 4 : fits(4, 3) ? 3 : 2;
  static constexpr int SMEM = 2 * Q_BYTES + (KS + VS) * KV_BYTES + BAR_BYTES;
  static constexpr int O_COL0 = 2 * BN;
  static constexpr int TMEM_COLS = 2 * BN + 2 * D <= 256 ? 256 : 512;
  static_assert(SMEM <= kSmemLimitP, "shared memory budget");
  static_assert(2 * BN + 2 * D <= 512, "TMEM budget");
  static_assert((2 * KS + 2 * VS + 14) * 8 + 16 <= BAR_BYTES, "barrier area");
};

template <int D, int BN, bool BF16>
__global__ void __launch_bounds__(192, 1)
    attn_tcp_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                    const TcpParams p) {
  using C = TcpCfg<D, BN>;
  constexpr int KS = C::KS, VS = C::VS;
  extern __shared__ __align__(1024) uint8_t smem[];
  if (smem_u32(smem) & 1023u) {
    if (threadIdx.x == 0) set_err(p.err, BSA_DEVERR_ALIGN);
    return;
  }
  uint8_t* sQ = smem;  // [2][Q_BYTES]
  uint8_t* sK = sQ + 2 * C::Q_BYTES;  // [KS][KV_BYTES]
  uint8_t* sV = sK + KS * C::KV_BYTES;  // [VS][KV_BYTES]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + VS * C::KV_BYTES);
  uint64_t* q_full = bars;          // [2]
  uint64_t* q_empty = q_full + 2;   // [2] epilogue's TMA store has read the buffer
  uint64_t* k_full = q_empty + 2;   // [KS]
  uint64_t* k_empty = k_full + KS;  // [KS] S MMA has read K
  uint64_t* v_full = k_empty + KS;  // [VS]
  uint64_t* v_empty = v_full + VS;  // [VS] PV MMA has read V
  uint64_t* s_full = v_empty + VS;  // [2]
  uint64_t* p_ready = s_full + 2;        // [2]
  uint64_t* o_empty = p_ready + 2;       // [2] epilogue has read O buffer
  uint64_t* pv_done = o_empty + 2;       // one phase per PV (rescale waits for PV_{j-1})
  uint64_t* o_final = pv_done + 1;       // one phase per non-empty tile: its last PV completed
  uint64_t* drain = o_final + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int G = gridDim.x;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_ready[i], 4);
      mbar_init(&o_empty[i], 4);
    }
    for (int i = 0; i < KS; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < VS; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    mbar_init(pv_done, 1);
    mbar_init(o_final, 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // tile w -> (slice s, entries e0 .. e0+n, b, h, t)
  auto tile_info = [&](int w, int& e0, int& n, int& b, int& h, int& t) {
    const int bh = w / p.T;
    t = w - bh * p.T;
    b = bh / p.H;
    h = bh - b * p.H;
    const int s = (p.mask_b == 1 ? 0 : b) * p.mask_h + (p.mask_h == 1 ? 0 : h);
    e0 = p.tile_ptr[s * p.T + t];
    n = p.tile_ptr[s * p.T + t + 1] - e0;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      // Loads in the order Q(tile), K_g, V_{g-1}: V runs one block behind K
      // because PV_{g-1} is issued after S_g.
      int e = 0, g = 0, gv = 0;  // non-empty tiles, K loads, V loads so far
      int pv_b = 0, pv_h = 0, pv_kb = 0;  // the block whose V is still to load (gv < g)
      bool ok = true;
      auto load_v = [&]() -> bool {
        const int st = gv % VS;
        if (gv >= VS && !mbar_wait(&v_empty[st], ((gv / VS) - 1) & 1, abort_flag, p.err)) return false;
        mbar_arrive_expect_tx(&v_full[st], C::KV_BYTES);
        for (int c = 0; c < C::NCHUNK; ++c)
          tma_load_4d(sV + st * C::KV_BYTES + c * C::KV_CHUNK, &tmV, &v_full[st], c * 64, pv_kb * BN, pv_h, pv_b);
        ++gv;
        return true;
      };
      for (int w = blockIdx.x; ok && w < p.total_tiles; w += G) {
        int e0, n, b, h, t;
        tile_info(w, e0, n, b, h, t);
        if (n == 0) continue;
        const int qb = e & 1;
        if (e >= 2 && !(ok = mbar_wait(&q_empty[qb], ((e >> 1) - 1) & 1, abort_flag, p.err))) break;
        mbar_arrive_expect_tx(&q_full[qb], C::Q_BYTES);
        for (int c = 0; c < C::NCHUNK; ++c)
          tma_load_4d(sQ + qb * C::Q_BYTES + c * C::Q_CHUNK, &tmQ, &q_full[qb], c * 64, t * 128, h, b);
        ++e;
        for (int j = 0; j < n; ++j, ++g) {
          const int st = g % KS;
          if (g >= KS && !(ok = mbar_wait(&k_empty[st], ((g / KS) - 1) & 1, abort_flag, p.err))) break;
          int kb = static_cast<int>(static_cast<uint32_t>(p.tile_col[e0 + j]) & 0xFFFFFFu);
          if (kb >= p.nb) {
            set_err(p.err, BSA_DEVERR_PLAN);
            kb = 0;
          }
          mbar_arrive_expect_tx(&k_full[st], C::KV_BYTES);
          for (int c = 0; c < C::NCHUNK; ++c)
            tma_load_4d(sK + st * C::KV_BYTES + c * C::KV_CHUNK, &tmK, &k_full[st], c * 64, kb * BN, h, b);
          if (gv < g && !(ok = load_v())) break;
          pv_b = b;
          pv_h = h;
          pv_kb = kb;
        }
      }
      if (ok && gv < g) ok = load_v();
      if (*abort_flag) {
        for (int j = g > KS ? g - KS : 0; j < g; ++j) mbar_wait(&k_full[j % KS], (j / KS) & 1, nullptr, nullptr);
        for (int j = gv > VS ? gv - VS : 0; j < gv; ++j) mbar_wait(&v_full[j % VS], (j / VS) & 1, nullptr, nullptr);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = make_idesc_f16(BF16, 128, BN, false, false);
      constexpr uint32_t idesc_pv = make_idesc_f16(BF16, 128, D, false, true);
      const uint32_t q_addr = smem_u32(sQ);
      const uint32_t k_addr = smem_u32(sK);
      const uint32_t v_addr = smem_u32(sV);
      int e = 0;   // non-empty tiles so far
      int jg = 0;  // blocks (S MMAs) so far
      // the PV still to issue: block index, its stage, O buffer, first / last block of its tile
      int pend_j = -1, pend_ob = 0;
      bool pend_first = false, pend_last = false;
      bool ok = true;
      int pv_issued_tiles = 0;  // non-empty tiles whose first PV was issued (o_empty accounting)
      auto do_pv = [&]() -> bool {
        const int i = pend_j, st = i % VS;
        if (pend_first && pv_issued_tiles >= 2 &&
            !mbar_wait(&o_empty[pend_ob], ((pv_issued_tiles >> 1) - 1) & 1, abort_flag, p.err))
          return false;
        if (!mbar_wait(&p_ready[i & 1], (i >> 1) & 1, abort_flag, p.err)) return false;
        if (!mbar_wait(&v_full[st], (i / VS) & 1, abort_flag, p.err)) return false;
        tc_fence_after();
        const uint32_t p_tmem = tmem + (i & 1) * BN;  // P_i lives in the first columns of S buffer i&1
        const uint32_t o_tmem = tmem + C::O_COL0 + pend_ob * D;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t bd = make_sw128_desc(v_addr + st * C::KV_BYTES + kk * 16 * 128, C::KV_CHUNK, 1024);
          tc_mma_ts(o_tmem, p_tmem + kk * 8, bd, idesc_pv, (!pend_first || kk > 0) ? 1u : 0u);
        }
        tc_commit(&v_empty[st]);
        tc_commit(pv_done);
        if (pend_last) tc_commit(o_final);
        if (pend_first) ++pv_issued_tiles;
        pend_j = -1;
        return true;
      };
      for (int w = blockIdx.x; ok && w < p.total_tiles; w += G) {
        int e0, n, b, h, t;
        tile_info(w, e0, n, b, h, t);
        if (n == 0) continue;
        const int qb = e & 1;
        if (!(ok = mbar_wait(&q_full[qb], (e >> 1) & 1, abort_flag, p.err))) break;
        tc_fence_after();
        for (int j = 0; j < n; ++j, ++jg) {
          const int st = jg % KS;
          if (!(ok = mbar_wait(&k_full[st], (jg / KS) & 1, abort_flag, p.err))) break;
          tc_fence_after();
          const uint32_t d_tmem = tmem + (jg & 1) * BN;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk & 3) * 32;  // 16 elements = 32 bytes inside the 128-byte swizzle row
            const uint64_t a = make_sw128_desc(q_addr + qb * C::Q_BYTES + (kk >> 2) * C::Q_CHUNK + off, 16, 1024);
            const uint64_t bd = make_sw128_desc(k_addr + st * C::KV_BYTES + (kk >> 2) * C::KV_CHUNK + off, 16, 1024);
            tc_mma_ss(d_tmem, a, bd, idesc_qk, kk > 0 ? 1u : 0u);
          }
          tc_commit(&s_full[jg & 1]);
          tc_commit(&k_empty[st]);
          if (pend_j >= 0 && !(ok = do_pv())) break;
          pend_j = jg;
          pend_ob = e & 1;
          pend_first = j == 0;
          pend_last = j == n - 1;
        }
        ++e;
      }
      if (ok && pend_j >= 0) ok = do_pv();
      tc_commit(drain);
      mbar_wait(drain, 0, nullptr, nullptr);
    }
  } else {
    // ------------------------------------------------------------ softmax warpgroup + epilogue
    const int q4 = warp & 3;
    const int row = q4 * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q4 * 32) << 16);
    const int half = row >> 6;
    const bool store_thread = warp == 2 && lane == 0;
    int e = 0, jg = 0;
    int pending_store_qb = -1;  // Q buffer whose TMA store still has to be waited for
    bool ok = true;
    for (int w = blockIdx.x; w < p.total_tiles; w += G) {
      int e0, n, b, h, t;
      tile_info(w, e0, n, b, h, t);
      const int grow0 = t * 128;
      if (n == 0) {
        // no kept block: O = 0 and lse = -inf for the tile's rows (plain stores)
        const int grow = grow0 + row;
        if (grow < p.N) {
          const int64_t bh = static_cast<int64_t>(b) * p.H + h;
          uint4* dst = reinterpret_cast<uint4*>(static_cast<uint8_t*>(p.o_raw) +
                                                2 * (b * p.os_b + h * p.os_h + grow * p.os_n));
#pragma unroll
          for (int i = 0; i < D / 8; ++i) dst[i] = make_uint4(0, 0, 0, 0);
          if (p.lse) p.lse[bh * p.N + grow] = -INFINITY;
        }
        continue;
      }
      const int ob = e & 1;
      float m_run = -INFINITY, l_run = 0.f;
      for (int j = 0; j < n; ++j, ++jg) {
        const int sb = jg & 1;
        // after a failed wait (ok false) every later wait returns at once (abort flag); the
        // loops still run to keep all warps on the same named-barrier sequence
        if (!(ok = ok && __all_sync(0xffffffffu, mbar_wait(&s_full[sb], (jg >> 1) & 1, abort_flag, p.err))))
          continue;
        tc_fence_after();
        uint32_t sr[BN];
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) tmem_ld32(lane_base + sb * BN + c * 32, &sr[c * 32]);
        tmem_wait_ld();
        const uint32_t entry = static_cast<uint32_t>(__ldg(&p.tile_col[e0 + j]));
        const uint32_t flags = entry >> 24;
        const bool active = BN == 128 ? true : (((flags >> half) & 1u) != 0);
        // keys at or past N (a partial last key block; TMA zero-filled them) are
        // masked out: only the one block that crosses N takes this branch
        {
          const int kvalid = p.N - static_cast<int>(entry & 0xFFFFFFu) * BN;
          if (kvalid < BN) {
#pragma unroll
            for (int i = 0; i < BN; ++i)
              if (i >= kvalid) sr[i] = __float_as_uint(-INFINITY);
          }
        }
        uint32_t pr[BN / 2];
        if (active) {
          const float alpha = softmax_block<BN, BF16>(sr, pr, p.scale_log2, m_run, l_run);
          if (__any_sync(0xffffffffu, alpha != 1.f)) {
            // O holds the sum up to block j-1 of this tile: wait for that PV, rescale in TMEM.
            if (!(ok = __all_sync(0xffffffffu, mbar_wait(pv_done, (jg - 1) & 1, abort_flag, p.err)))) continue;
            tc_fence_after();
#pragma unroll
            for (int c = 0; c < D / 32; ++c) {
              uint32_t o[32];
              tmem_ld32(lane_base + C::O_COL0 + ob * D + c * 32, o);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
              tmem_st32(lane_base + C::O_COL0 + ob * D + c * 32, o);
            }
          }
        } else {
#pragma unroll
          for (int i = 0; i < BN / 2; ++i) pr[i] = 0u;
        }
        // P_j into the first BN/2 columns of its S buffer (all of S is in registers)
#pragma unroll
        for (int c = 0; c < BN / 64; ++c) tmem_st32(lane_base + sb * BN + c * 32, &pr[c * 32]);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_ready[sb]);
        if (j == 0 && store_thread && pending_store_qb >= 0) {
          // the previous tile's output store must have read its Q buffer
          tma_store_wait_read0();
          mbar_arrive(&q_empty[pending_store_qb]);
          pending_store_qb = -1;
        }
      }
      // ---------------------------------------------------------- epilogue of this tile
      ok = ok && __all_sync(0xffffffffu, mbar_wait(o_final, e & 1, abort_flag, p.err));
      if (ok) {
      tc_fence_after();
      uint32_t o_all[D];
#pragma unroll
      for (int c = 0; c < D / 32; ++c) tmem_ld32(lane_base + C::O_COL0 + ob * D + c * 32, &o_all[c * 32]);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&o_empty[ob]);  // the MMA may start the tile after next in this buffer
      const float inv_l = l_run > 0.f ? 1.f / l_run : 0.f;
      uint8_t* orow = sQ + (e & 1) * C::Q_BYTES + row * 128;  // this tile's Q buffer: no MMA reads it any more
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint8_t* chunk_row = orow + (c >> 1) * C::Q_CHUNK;
#pragma unroll
        for (int g2 = 0; g2 < 4; ++g2) {
          const uint32_t* o = &o_all[c * 32 + 8 * g2];
          uint4 v;
          v.x = pack2<BF16>(__uint_as_float(o[0]) * inv_l, __uint_as_float(o[1]) * inv_l);
          v.y = pack2<BF16>(__uint_as_float(o[2]) * inv_l, __uint_as_float(o[3]) * inv_l);
          v.z = pack2<BF16>(__uint_as_float(o[4]) * inv_l, __uint_as_float(o[5]) * inv_l);
          v.w = pack2<BF16>(__uint_as_float(o[6]) * inv_l, __uint_as_float(o[7]) * inv_l);
          const int gran = ((c & 1) * 4 + g2) ^ (row & 7);  // 128-byte swizzle
          *reinterpret_cast<uint4*>(chunk_row + gran * 16) = v;
        }
      }
      fence_proxy_async_smem();
      const int grow = grow0 + row;
      if (p.lse && grow < p.N)
        p.lse[(static_cast<int64_t>(b) * p.H + h) * p.N + grow] = l_run > 0.f ? m_run + log2f(l_run) : -INFINITY;
      }
      named_bar_sync(1, 128);  // every softmax warp, once per non-empty tile, also after a failure
      if (store_thread && !*abort_flag) {
        // (the previous tile's buffer was released at this tile's block 0)
        for (int c = 0; c < C::NCHUNK; ++c)
          tma_store_4d(&tmO, sQ + (e & 1) * C::Q_BYTES + c * C::Q_CHUNK, c * 64, grow0, h, b);
        tma_store_commit();
        pending_store_qb = e & 1;
      }
      ++e;
    }
    if (store_thread) tma_store_wait0();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

int sm_count() {
  static int count[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!count[dev]) {
    int c = 0;
    count[dev] = cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && c > 0 ? c : 148;
  }
  return count[dev];
}

template <int D, int BN, bool BF16>
int launch_p(const bsa_fwd_args* a, cudaStream_t st) {
  using C = TcpCfg<D, BN>;
  CUtensorMap mq, mk, mv, mo;
  int r;
  if ((r = make_tensor_map_4d(&mq, a->q, a->B, a->H, a->N, D, BF16, 128))) return r;
  if ((r = make_tensor_map_4d(&mk, a->k, a->B, a->H, a->N, D, BF16, BN))) return r;
  if ((r = make_tensor_map_4d(&mv, a->v, a->B, a->H, a->N, D, BF16, BN))) return r;
  if ((r = make_tensor_map_4d(&mo, a->o, a->B, a->H, a->N, D, BF16, 128))) return r;
  TcpParams p;
  p.tile_ptr = a->plan.tile_ptr;
  p.tile_col = a->plan.tile_col;
  p.lse = a->lse;
  p.o_raw = a->o.data;
  p.os_b = a->o.stride_b;
  p.os_h = a->o.stride_h;
  p.os_n = a->o.stride_n;
  p.err = a->err_flag;
  p.H = a->H;
  p.N = a->N;
  p.nb = a->plan.nb;
  p.T = tiles_per_row(a->plan.nb, a->plan.block);
  p.mask_b = a->plan.mask_b;
  p.mask_h = a->plan.mask_h;
  p.total_tiles = a->B * a->H * p.T;
  p.scale_log2 = a->sm_scale * 1.4426950408889634f;
  auto kern = attn_tcp_kernel<D, BN, BF16>;
  BSA_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
  int per_sm = 1;
  BSA_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 192, C::SMEM));
  if (per_sm < 1) per_sm = 1;
  if (C::TMEM_COLS * per_sm > 512) per_sm = 512 / C::TMEM_COLS;
  int grid = sm_count() * per_sm;
  if (grid > p.total_tiles) grid = p.total_tiles;
  kern<<<grid, 192, C::SMEM, st>>>(mq, mk, mv, mo, p);
  return cudaGetLastError() == cudaSuccess ? BSA_OK : BSA_ERR_CUDA;
}

}  // namespace

int launch_attn_tcp(const bsa_fwd_args* a, cudaStream_t st) {
  const bool bf16 = a->dtype == BSA_DTYPE_BF16;
  const int bn = a->plan.block;
#define BSA_TCP_CASE(D_, BN_) \
  if (a->D == D_ && bn == BN_) return bf16 ? launch_p<D_, BN_, true>(a, st) : launch_p<D_, BN_, false>(a, st);
  BSA_TCP_CASE(64, 64)
  BSA_TCP_CASE(64, 128)
  BSA_TCP_CASE(128, 64)
  BSA_TCP_CASE(128, 128)
#undef BSA_TCP_CASE
  return BSA_ERR_UNSUPPORTED;
}

}  // namespace bsa
