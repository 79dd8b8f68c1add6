// tcgen05 block-sparse attention forward for BLOCK 64, D 128 and dense plans,
// computed per 64-row query block in the transposed orientation (sm_100a).
//
// Same contract as _attn_fwd_block_sparse (triton_kernels/BlockSparse_Naive.py:
// 68-125) with its online softmax (:39-60) and epilogue (:119-125): rows with
// no kept block give O = 0 and lse = -inf; keys at or past N are masked; with
// a query permutation (BlockSparse_Fused.py:173-223) Q rows are read from
// q_perm[row] and O / lse rows written to q_perm[row].
//
// Why transposed: the reference visits, for each 64-row query block, only the
// 64-key blocks that block keeps.  An M = 128 MMA over a 128-row tile of two
// query blocks wastes half its rows on every key block only one of them
// keeps (most of them, on random masks).  Here the 128 MMA rows are keys:
// two key blocks the query block keeps (one "pair" per step), the 64 query
// rows are the MMA's N:
//   S^T (128 keys x 64 queries) = K_pair Q^T      (A = K, B = Q, both K-major)
//   O^T (D x 64 queries)       += V_pair^T P^T    (A = V MN-major, B = P^T in
//                                                   shared memory, MN-major)
// so every multiply is useful, and so is every exponential.  A 128-row plan
// tile is processed as its two 64-row query blocks ("sub-tiles") in turn, each
// walking the tile's plan entries that its block row keeps.
//
// One softmax thread per key (TMEM lane): it holds its key's 64 scores, so
// the per-query reference point (the exact max of the sub-tile's first pair,
// see softmax.cuh) and the row sums are reductions across the warpgroup:
// shuffle reduce-scatters (64 columns over 32 lanes) and shared memory.  Each
// step the warpgroup votes (barrier.red.or) whether any score left the slack
// of its reference point; then that step is redone with the exact column max
// and O^T, l rescaled.  P^T (bf16 / fp16) is written to shared memory,
// 128-byte swizzled, one key row per thread.
//
// Roles as in attn_tcp.cu: warp 0 = producer (claims tiles, counts each block
// row's entries, loads Q, K and V pairs), warp 1 = TMEM and MMA issuer,
// warps 2-3 = Q gather with a query permutation, warpgroup 1 = softmax,
// warpgroup 2 = epilogue (O^T / l from TMEM to global memory).
// Ordering facts (one thread issues every MMA, in order; a commit tracks all
// earlier MMAs of the thread): S_g+2 reuses S_g's TMEM after PV_g was issued;
// S_g complete implies PV_g-2 complete, so the softmax may overwrite P^T buffer
// g&1 once it has S_g; step_done[g % 4] after PV_g frees K_g+1's and V_g's
// stages; q_empty after a tile's last S frees the (single) Q buffer; o_empty /
// o_final per O^T buffer (two, by sub-tile).  Every wait is bounded.
#include <cudaTypedefs.h>

#include <atomic>

#include "common.cuh"
#include "internal.h"
#include "softmax.cuh"

namespace bsa {

namespace {

constexpr int kSlotsT = 64;
__device__ uint32_t g_tt_next[kSlotsT];
__device__ uint32_t g_tt_done[kSlotsT];
std::atomic<unsigned> g_tt_launches{0};

constexpr int kRingT = 8;
constexpr int kUsersT = 9;        // MMA thread + 4 softmax + 4 epilogue warps
constexpr int kUsersGatherT = 11;  // + the 2 Q-gather warps
constexpr int kPairMinEntriesT = 32;

// One claimed tile: number (-1 = no more), plan entries e0 .. e0+n, (b, h),
// tile row, and per block row r the number of entries it keeps (bits 0-29)
// with bit 30 set when it keeps the partial last key block (N % 64 != 0).
struct TTTile {
  int w, e0, n, b, h, t, c0, c1;
};

struct TtParams {
  const int32_t* tile_ptr;
  const int32_t* tile_col;
  const int32_t* tile_order;
  float* lse;
  uint8_t* o;
  int64_t os_b, os_h, os_n;
  int32_t* err;
  const uint8_t* q;
  int64_t qs_b, qs_h, qs_n;
  const void* q_perm;
  int perm_dtype;
  int H, N, nb, T, mask_b, mask_h, total_tiles;
  int slot;
  float scale_log2;
  uint64_t wait_ns;
  int withhold_arrive;
};

constexpr int kThreadsT = 384;
constexpr int kRegsIssueT = 80;
constexpr int kRegsSoftmaxT = 240;
constexpr int kRegsEpilogueT = 128;
static_assert(128 * (kRegsIssueT + kRegsSoftmaxT + kRegsEpilogueT) <= kThreadsT * 168, "register split");

struct TtCfg {
  static constexpr int D = 128;
  static constexpr int Q_BYTES = 128 * D * 2;   // one 128-row tile, 2 chunks of 64 columns
  static constexpr int CHUNK = 128 * 128;       // 128 rows of one 64-column chunk
  static constexpr int BOX_BYTES = 64 * 128;    // one 64-row key block of a chunk
  static constexpr int KV_BYTES = 128 * D * 2;  // a pair of key blocks
  static constexpr int P_BYTES = 128 * 64 * 2;  // P^T: 128 key rows x 64 queries
  static constexpr int KS = 3, VS = 2;
  static constexpr int BAR_BYTES = 1024;
  static constexpr int STATS_BYTES = 2 * 2 * 64 * 4;  // [buffer][m, l][query]
  static constexpr int RED_BYTES = 4 * 64 * 4;        // [warp][column]
  static constexpr int SMEM = Q_BYTES + (KS + VS) * KV_BYTES + 2 * P_BYTES + BAR_BYTES + STATS_BYTES + RED_BYTES;
  static constexpr int RING_OFF = 512;
  static_assert(SMEM <= 232448, "shared memory budget");
  static_assert(RING_OFF + kRingT * 32 <= BAR_BYTES, "ring area");
};

__device__ __forceinline__ int64_t load_perm_t(const void* perm, int dtype, int64_t i) {
  return dtype == BSA_INDEX_I64 ? __ldg(static_cast<const int64_t*>(perm) + i)
                                : static_cast<int64_t>(__ldg(static_cast<const int32_t*>(perm) + i));
}

// Named barrier 1 over the 128 softmax threads; the second form ORs a
// predicate over them.
__device__ __forceinline__ void sm_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
__device__ __forceinline__ bool sm_bar_or(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "barrier.cta.red.or.pred p, 1, 128, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(v ? 1u : 0u)
      : "memory");
  return r != 0;
}

// One level of a reduce-scatter across the lanes at distance `o`: each lane
// keeps the lower or upper half of its S values (by lane bit o) combined with
// the partner's copy of that half.
template <int S, bool MAX>
__device__ __forceinline__ void rs_level(const float (&in)[S], float (&out)[S / 2], int lane, int o) {
  const bool hi = (lane & o) != 0;
#pragma unroll
  for (int i = 0; i < S / 2; ++i) {
    const float keep = hi ? in[S / 2 + i] : in[i];
    const float send = hi ? in[i] : in[S / 2 + i];
    const float got = __shfl_xor_sync(0xffffffffu, send, o);
    out[i] = MAX ? fmaxf(keep, got) : keep + got;
  }
}

// Column max of v[64] over the 128 softmax threads: one redux per column
// within the warp, then the four warps' maxima through shared memory.
// Afterwards red_w[q] (q = 0..63) holds the result.
__device__ __forceinline__ void column_max(const float (&v)[64], float* red_w, int q4, int lane) {
#pragma unroll
  for (int q = 0; q < 64; ++q) {
    const float r = warp_max_f32(v[q]);
    if (lane == (q & 31)) red_w[q4 * 64 + q] = r;
  }
  sm_bar();
  if (q4 == 0) {
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int c = 2 * lane + k;
      red_w[c] = fmaxf(fmaxf(red_w[c], red_w[64 + c]), fmaxf(red_w[128 + c], red_w[192 + c]));
    }
  }
  sm_bar();
}

// Column reduction of v[64] over the 128 softmax threads (4 warps x 32 lanes):
// max or sum per column q, returned through red[q] ... with the per-warp
// partials in red_w[warp][q]; every softmax thread calls it.  After return,
// red_w[0][q] holds the result for q = 0..63 (written by warp 0).
template <bool MAX>
__device__ __forceinline__ void column_reduce(const float (&v)[64], float* red_w, int q4, int lane) {
  float a32[32], a16[16], a8[8], a4[4], a2[2];
  rs_level<64, MAX>(v, a32, lane, 16);
  rs_level<32, MAX>(a32, a16, lane, 8);
  rs_level<16, MAX>(a16, a8, lane, 4);
  rs_level<8, MAX>(a8, a4, lane, 2);
  rs_level<4, MAX>(a4, a2, lane, 1);
  // lane l now holds columns 2l and 2l + 1 of its warp
  red_w[q4 * 64 + 2 * lane] = a2[0];
  red_w[q4 * 64 + 2 * lane + 1] = a2[1];
  sm_bar();
  if (q4 == 0) {
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int c = 2 * lane + k;
      float x = red_w[c];
#pragma unroll
      for (int w = 1; w < 4; ++w) x = MAX ? fmaxf(x, red_w[w * 64 + c]) : x + red_w[w * 64 + c];
      red_w[c] = x;
    }
  }
  sm_bar();
}

template <bool BF16>
__global__ void __launch_bounds__(kThreadsT, 1)
    attn_tt_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const TtParams p) {
  using C = TtCfg;
  constexpr int KS = C::KS, VS = C::VS, D = C::D;
  extern __shared__ __align__(1024) uint8_t smem[];
  if (smem_u32(smem) & 1023u) {
    if (threadIdx.x == 0) set_err(p.err, BSA_DEVERR_ALIGN);
    return;
  }
  uint8_t* sQ = smem;                      // [Q_BYTES]
  uint8_t* sK = sQ + C::Q_BYTES;           // [KS][KV_BYTES]
  uint8_t* sV = sK + KS * C::KV_BYTES;     // [VS][KV_BYTES]
  uint8_t* sP = sV + VS * C::KV_BYTES;     // [2][P_BYTES]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * C::P_BYTES);
  float* stats = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + C::BAR_BYTES);  // [2][m, l][64]
  float* red_w = stats + 2 * 2 * 64;                                                           // [4][64]
  uint64_t* q_full = bars;                // [1]
  uint64_t* q_empty = q_full + 1;         // [1]
  uint64_t* kv_full = q_empty + 1;        // [KS]
  uint64_t* s_full = kv_full + KS;        // [2]
  uint64_t* p_ready = s_full + 2;         // [2] 4 softmax warps wrote P^T
  uint64_t* o_final = p_ready + 2;        // [2] by O^T buffer: the sub-tile's last PV completed
  uint64_t* o_empty = o_final + 2;        // [2] 4 epilogue warps read O^T
  uint64_t* stats_ready = o_empty + 2;    // [2]
  uint64_t* stats_empty = stats_ready + 2;  // [2]
  uint64_t* step_done = stats_empty + 2;  // [4]
  uint64_t* drain = step_done + 4;        // [1]
  uint64_t* tile_ready = drain + 1;       // [kRingT]
  uint64_t* tile_free = tile_ready + kRingT;  // [kRingT]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tile_free + kRingT);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile TTTile* ring = reinterpret_cast<volatile TTTile*>(reinterpret_cast<uint8_t*>(bars) + C::RING_OFF);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(q_full, p.q_perm ? 2 : 1);
    mbar_init(q_empty, 1);
    for (int i = 0; i < KS; ++i) mbar_init(&kv_full[i], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_ready[i], 4);
      mbar_init(&o_final[i], 1);
      mbar_init(&o_empty[i], 4);
      mbar_init(&stats_ready[i], 4);
      mbar_init(&stats_empty[i], 4);
    }
    for (int i = 0; i < 4; ++i) mbar_init(&step_done[i], 1);
    mbar_init(drain, 1);
    for (int i = 0; i < kRingT; ++i) {
      mbar_init(&tile_ready[i], 1);
      mbar_init(&tile_free[i], p.q_perm ? kUsersGatherT : kUsersT);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  grid_dependency_wait();
  {
    // run only when the plan averages at least kPairMinEntriesT kept blocks
    // per tile (the one-block-per-step form of attn_tcp.cu takes the others);
    // every CTA reads the same total and the form not chosen exits here
    const int tiles = p.mask_b * p.mask_h * p.T;
    if (__ldg(&p.tile_ptr[tiles]) < kPairMinEntriesT * tiles) {
      if (warp == 1) tmem_dealloc(tmem, 256);
      return;
    }
  }

  auto tile_info = [&](int w, int& e0, int& n, int& b, int& h, int& t) {
    const int bh = w / p.T;
    const int r = w - bh * p.T;
    b = bh / p.H;
    h = bh - b * p.H;
    const int sl = (p.mask_b == 1 ? 0 : b) * p.mask_h + (p.mask_h == 1 ? 0 : h);
    t = p.tile_order ? p.tile_order[sl * p.T + r] : r;
    e0 = p.tile_ptr[sl * p.T + t];
    n = p.tile_ptr[sl * p.T + t + 1] - e0;
  };
  auto next_tile = [&](int i, TTTile& tl) -> bool {
    const int ri = i % kRingT;
    if (!mbar_wait(&tile_ready[ri], (i / kRingT) & 1, abort_flag, p.err, p.wait_ns)) return false;
    tl.w = ring[ri].w;
    tl.e0 = ring[ri].e0;
    tl.n = ring[ri].n;
    tl.b = ring[ri].b;
    tl.h = ring[ri].h;
    tl.t = ring[ri].t;
    tl.c0 = ring[ri].c0;
    tl.c1 = ring[ri].c1;
    return tl.w >= 0;
  };
  constexpr int kCountMask = (1 << 30) - 1;

  if (warp < 4) {
    regs_dec<kRegsIssueT>();
    if (warp == 0) {
      // ------------------------------------------------------------ producer (whole warp)
      if (lane == 0) {
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
      }
      int e = 0, g = 0, gv = 0, armed = 0, qarmed = 0;
      int pv_b = 0, pv_h = 0, pv_kb0 = 0, pv_kb1 = 0;
      bool ok = true;
      auto wait0 = [&](uint64_t* bar, uint32_t parity) -> bool {
        int r = 1;
        if (lane == 0) r = mbar_wait(bar, parity, abort_flag, p.err, p.wait_ns) ? 1 : 0;
        return __shfl_sync(0xffffffffu, r, 0) != 0;
      };
      auto wait_k_stage = [&](int gs) -> bool {
        const int sd = gs - KS - 1 > 0 ? gs - KS - 1 : 0;
        return gs < KS || wait0(&step_done[sd & 3], (sd >> 2) & 1);
      };
      auto wait_v_stage = [&]() -> bool {
        return gv < VS || wait0(&step_done[(gv - VS) & 3], ((gv - VS) >> 2) & 1);
      };
      // two key blocks into a stage: block kb0 in rows 0-63, kb1 in rows 64-127
      auto load_pair = [&](uint8_t* stage, const CUtensorMap* tm, uint64_t* bar, int kb0, int kb1, int h, int b) {
        if (lane == 0)
          for (int c = 0; c < D / 64; ++c) {
            tma_load_4d(stage + c * C::CHUNK, tm, bar, c * 64, kb0 * 64, h, b);
            tma_load_4d(stage + c * C::CHUNK + C::BOX_BYTES, tm, bar, c * 64, kb1 * 64, h, b);
          }
      };
      auto load_v = [&](uint64_t* bar) {
        load_pair(sV + (gv % VS) * C::KV_BYTES, &tmV, bar, pv_kb0, pv_kb1, pv_h, pv_b);
        ++gv;
      };
      for (int i = 0; ok; ++i) {
        int w = -1, e0 = 0, n = 0, b = 0, h = 0, t = 0;
        if (lane == 0) {
          const uint32_t claim = atomicAdd(&g_tt_next[p.slot], 1u);
          w = claim < static_cast<uint32_t>(p.total_tiles) ? static_cast<int>(claim) : -1;
          if (w >= 0) tile_info(w, e0, n, b, h, t);
        }
        w = __shfl_sync(0xffffffffu, w, 0);
        e0 = __shfl_sync(0xffffffffu, e0, 0);
        n = __shfl_sync(0xffffffffu, n, 0);
        b = __shfl_sync(0xffffffffu, b, 0);
        h = __shfl_sync(0xffffffffu, h, 0);
        t = __shfl_sync(0xffffffffu, t, 0);
        // entries kept by each block row (flag bits 24 / 25), eight windows of
        // 32 entries per round of loads; the partial last key block can only be
        // the tile's last entry
        int cnt[2] = {0, 0};
        for (int base = 0; base < n; base += 256) {
          uint32_t ev[8];
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const int idx = base + k * 32 + lane;
            ev[k] = idx < n ? static_cast<uint32_t>(__ldg(&p.tile_col[e0 + idx])) : 0u;
          }
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            cnt[0] += __popc(__ballot_sync(0xffffffffu, (ev[k] >> 24) & 1u));
            cnt[1] += __popc(__ballot_sync(0xffffffffu, (ev[k] >> 25) & 1u));
          }
        }
        if (n > 0 && p.N % 64 != 0) {
          const uint32_t last = static_cast<uint32_t>(__ldg(&p.tile_col[e0 + n - 1]));
          if (static_cast<int>(last & 0xFFFFFFu) == p.nb - 1) {
            if ((last >> 24) & 1u) cnt[0] |= 1 << 30;
            if ((last >> 25) & 1u) cnt[1] |= 1 << 30;
          }
        }
        const int ri = i % kRingT;
        if (i >= kRingT && !(ok = wait0(&tile_free[ri], ((i / kRingT) - 1) & 1))) break;
        if (lane == 0) {
          ring[ri].w = w;
          ring[ri].e0 = e0;
          ring[ri].n = n;
          ring[ri].b = b;
          ring[ri].h = h;
          ring[ri].t = t;
          ring[ri].c0 = cnt[0];
          ring[ri].c1 = cnt[1];
          mbar_arrive(&tile_ready[ri]);
        }
        if (w < 0) break;
        if (n == 0) continue;
        if (!p.q_perm) {
          if (e >= 1 && !(ok = wait0(q_empty, (e - 1) & 1))) break;
          if (lane == 0) {
            mbar_arrive_expect_tx(q_full, C::Q_BYTES);
            for (int c = 0; c < D / 64; ++c) tma_load_4d(sQ + c * C::CHUNK, &tmQ, q_full, c * 64, t * 128, h, b);
          }
          ++qarmed;
        }
        ++e;
        for (int r = 0; r < 2 && ok; ++r) {
          const int c = (r ? cnt[1] : cnt[0]) & kCountMask;
          const int ns = (c + 1) >> 1;
          // the block row's entries in order: a window of 32 plan entries, a
          // ballot of the row's flag, lowest set bit first
          int win_base = -32;
          uint32_t win_mask = 0, win_val = 0;
          auto next_entry = [&]() -> int {
            while (win_mask == 0 && win_base + 32 < n) {
              win_base += 32;
              const int idx = win_base + lane;
              win_val = idx < n ? static_cast<uint32_t>(__ldg(&p.tile_col[e0 + idx])) : 0u;
              win_mask = __ballot_sync(0xffffffffu, (win_val >> (24 + r)) & 1u);
            }
            if (win_mask == 0) {  // fewer flagged entries than counted: a corrupt plan
              if (lane == 0) set_err(p.err, BSA_DEVERR_PLAN);
              return 0;
            }
            const int pos = __ffs(win_mask) - 1;
            win_mask &= win_mask - 1;
            return static_cast<int>(__shfl_sync(0xffffffffu, win_val, pos) & 0xFFFFFFu);
          };
          for (int j = 0; j < ns; ++j, ++g) {
            int kb0 = next_entry();
            int kb1 = 2 * j + 1 < c ? next_entry() : kb0;  // a missing second entry repeats the first (masked)
            if (kb0 >= p.nb || kb1 >= p.nb) {
              if (lane == 0) set_err(p.err, BSA_DEVERR_PLAN);
              kb0 = kb0 < p.nb ? kb0 : 0;
              kb1 = kb1 < p.nb ? kb1 : 0;
            }
            const int st = g % KS;
            if (!(ok = wait_k_stage(g))) break;
            ++armed;
            if (lane == 0) mbar_expect_tx(&kv_full[st], C::KV_BYTES);
            load_pair(sK + st * C::KV_BYTES, &tmK, &kv_full[st], kb0, kb1, h, b);
            if (gv < g && (ok = wait_v_stage())) {
              if (lane == 0) mbar_expect_tx(&kv_full[st], C::KV_BYTES);
              load_v(&kv_full[st]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&kv_full[st]);
            if (!ok) break;
            pv_b = b;
            pv_h = h;
            pv_kb0 = kb0;
            pv_kb1 = kb1;
          }
        }
      }
      if (ok && gv < g) {
        // the last V pair alone, on the barrier of step g (no K)
        if ((ok = wait_k_stage(g) && wait_v_stage())) {
          ++armed;
          if (lane == 0) mbar_expect_tx(&kv_full[g % KS], C::KV_BYTES);
          load_v(&kv_full[g % KS]);
          __syncwarp();
          if (lane == 0) mbar_arrive(&kv_full[g % KS]);
        }
      }
      // every load lands before the CTA exits (the last phase armed on each barrier)
      if (lane == 0) {
        for (int j = armed > KS ? armed - KS : 0; j < armed; ++j)
          mbar_wait(&kv_full[j % KS], (j / KS) & 1, nullptr, nullptr, p.wait_ns);
        if (qarmed > 0) mbar_wait(q_full, (qarmed - 1) & 1, nullptr, nullptr, p.wait_ns);
      }
    } else if (warp == 1 && lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      // S^T: M = 128 keys, N = 64 queries, A = K pair and B = Q rows, K-major.
      // O^T: M = 128 (D), N = 64 queries, A = V pair (MN-major), B = P^T (MN-major).
      constexpr uint32_t idesc_s = make_idesc_f16(BF16, 128, 64, false, false);
      constexpr uint32_t idesc_o = make_idesc_f16(BF16, 128, 64, true, true);
      const uint32_t q_addr = smem_u32(sQ);
      const uint32_t k_addr = smem_u32(sK);
      const uint32_t v_addr = smem_u32(sV);
      const uint32_t p_addr = smem_u32(sP);
      int e = 0, jg = 0, u = 0, pv_subs = 0;
      int pend_j = -1, pend_u = 0;
      bool pend_first = false, pend_last = false, ok = true;
      auto do_pv = [&](bool last_pv) -> bool {
        const int i = pend_j;
        if (pend_first && pv_subs >= 2 &&
            !mbar_wait(&o_empty[pend_u & 1], ((pv_subs >> 1) - 1) & 1, abort_flag, p.err, p.wait_ns))
          return false;
        if (!mbar_wait(&p_ready[i & 1], (i >> 1) & 1, abort_flag, p.err, p.wait_ns)) return false;
        // V_i landed with K_i+1 (waited before S_i+1), or alone after the last step
        if (last_pv && !mbar_wait(&kv_full[(i + 1) % KS], ((i + 1) / KS) & 1, abort_flag, p.err, p.wait_ns))
          return false;
        tc_fence_after();
        const uint32_t o_tmem = tmem + 128 + (pend_u & 1) * 64;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t a = make_sw128_desc(v_addr + (i % VS) * C::KV_BYTES + kk * 16 * 128, C::CHUNK, 1024);
          const uint64_t bd = make_sw128_desc(p_addr + (i & 1) * C::P_BYTES + kk * 16 * 128, C::P_BYTES, 1024);
          tc_mma_ss(o_tmem, a, bd, idesc_o, (!pend_first || kk > 0) ? 1u : 0u);
        }
        tc_commit(&step_done[i & 3]);
        if (pend_last) tc_commit(&o_final[pend_u & 1]);
        if (pend_first) ++pv_subs;
        pend_j = -1;
        return true;
      };
      for (int i = 0; ok; ++i) {
        TTTile tl;
        const bool have = next_tile(i, tl);
        mbar_arrive(&tile_free[i % kRingT]);
        if (!have) break;
        if (tl.n == 0) continue;
        if (!(ok = mbar_wait(q_full, e & 1, abort_flag, p.err, p.wait_ns))) break;
        tc_fence_after();
        const int c0 = tl.c0 & kCountMask, c1 = tl.c1 & kCountMask;
        const int last_r = c1 > 0 ? 1 : 0;
        for (int r = 0; r < 2 && ok; ++r) {
          const int ns = ((r ? c1 : c0) + 1) >> 1;
          for (int j = 0; j < ns; ++j, ++jg) {
            const int st = jg % KS;
            if (!(ok = mbar_wait(&kv_full[st], (jg / KS) & 1, abort_flag, p.err, p.wait_ns))) break;
            tc_fence_after();
            const uint32_t d_tmem = tmem + (jg & 1) * 64;
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const uint32_t off = (kk & 3) * 32;  // 16 elements = 32 bytes inside the 128-byte swizzle row
              const uint64_t a = make_sw128_desc(k_addr + st * C::KV_BYTES + (kk >> 2) * C::CHUNK + off, 16, 1024);
              const uint64_t bd =
                  make_sw128_desc(q_addr + (kk >> 2) * C::CHUNK + r * C::BOX_BYTES + off, 16, 1024);
              tc_mma_ss(d_tmem, a, bd, idesc_s, kk > 0 ? 1u : 0u);
            }
            tc_commit(&s_full[jg & 1]);
            if (r == last_r && j == ns - 1) tc_commit(q_empty);
            if (pend_j >= 0 && !(ok = do_pv(false))) break;
            pend_j = jg;
            pend_u = u;
            pend_first = j == 0;
            pend_last = j == ns - 1;
          }
          if (ns > 0) ++u;
        }
        ++e;
      }
      if (ok && pend_j >= 0) ok = do_pv(true);
      tc_commit(drain);
      mbar_wait(drain, 0, nullptr, nullptr, p.wait_ns);
    } else if (warp >= 2 && p.q_perm) {
      // ------------------------------------------------- Q gather (permuted queries)
      // Warp 2 fills rows 0-63 of the tile, warp 3 rows 64-127, as 16-byte
      // granules into the 128-byte-swizzled chunks the MMA reads.
      const int gw = warp - 2;
      int e = 0;
      bool ok = true;
      for (int i = 0;; ++i) {
        TTTile tl;
        const bool have = next_tile(i, tl);
        __syncwarp();
        if (lane == 0) mbar_arrive(&tile_free[i % kRingT]);
        if (!have) break;
        if (tl.n == 0) continue;
        if (e >= 1) ok = ok && __all_sync(0xffffffffu, mbar_wait(q_empty, (e - 1) & 1, abort_flag, p.err, p.wait_ns));
        ++e;
        if (!ok) continue;
        for (int k = 0; k < 2; ++k) {
          const int r = gw * 64 + k * 32 + lane;
          const int grow = tl.t * 128 + r;
          const uint4* src = nullptr;
          if (grow < p.N) {
            const int64_t old = load_perm_t(p.q_perm, p.perm_dtype, grow);
            if (old >= 0 && old < p.N)
              src = reinterpret_cast<const uint4*>(p.q + 2 * (tl.b * p.qs_b + tl.h * p.qs_h + old * p.qs_n));
            else
              set_err(p.err, BSA_DEVERR_PERM_RANGE);
          }
#pragma unroll
          for (int c = 0; c < D / 64; ++c) {
            uint8_t* dst = sQ + c * C::CHUNK + r * 128;
            uint4 v[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) v[u] = src ? __ldg(src + c * 8 + u) : make_uint4(0, 0, 0, 0);
#pragma unroll
            for (int u = 0; u < 8; ++u) *reinterpret_cast<uint4*>(dst + ((u ^ (r & 7)) * 16)) = v[u];
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(q_full);
      }
    }
  } else if (warp < 8) {
    regs_inc<kRegsSoftmaxT>();
    // -------------------------------------------------------------- softmax
    // thread = one key of the step's pair (TMEM lane k; keys 0-63 the first
    // block, 64-127 the second), its 64 scores = the sub-tile's queries
    const int q4 = warp & 3;
    const int k = q4 * 32 + lane;
    const int half = k >> 6;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q4 * 32) << 16);
    const float thresh = BF16 ? 30.f : 14.f;  // largest x = s*scale - m kept without a redo (fp16: P < 2^15)
    int jg = 0, u = 0;
    bool ok = true;
    for (int i = 0;; ++i) {
      TTTile tl;
      const bool have = next_tile(i, tl);
      __syncwarp();
      if (lane == 0) mbar_arrive(&tile_free[i % kRingT]);
      if (!have) break;
      if (tl.n == 0) continue;
      for (int r = 0; r < 2; ++r) {
        const int cw = r ? tl.c1 : tl.c0;
        const int c = cw & kCountMask;
        const bool keeps_partial = (cw >> 30) & 1;
        const int ns = (c + 1) >> 1;
        if (ns == 0) continue;
        const int ub = u & 1;
        float* m_s = stats + ub * 128;
        float* l_s = m_s + 64;
        // the epilogue has read this buffer's statistics of sub-tile u-2
        if (u >= 2)
          ok = ok && __all_sync(0xffffffffu, mbar_wait(&stats_empty[ub], ((u >> 1) - 1) & 1, abort_flag, p.err,
                                                       p.wait_ns));
        float lp[64];
#pragma unroll
        for (int q = 0; q < 64; ++q) lp[q] = 0.f;
        for (int j = 0; j < ns; ++j, ++jg) {
          const int sb = jg & 1;
          if (!(ok = ok && __all_sync(0xffffffffu, mbar_wait(&s_full[sb], (jg >> 1) & 1, abort_flag, p.err,
                                                             p.wait_ns))))
            continue;
          tc_fence_after();
          // this thread's key: the pair's missing second block (odd count) and
          // keys at or past N in the partial last block are masked
          bool valid = true;
          if (j == ns - 1) {
            if ((c & 1) && half == 1) valid = false;
            if (keeps_partial && half == ((c - 1) & 1) && (p.nb - 1) * 64 + (k & 63) >= p.N) valid = false;
          }
          // x = scaled scores (log2 units), -inf for a masked key
          float x[64];
          auto load_scaled = [&]() {
            uint32_t sr[64];
            tmem_ld32(lane_base + sb * 64, &sr[0]);
            tmem_ld32(lane_base + sb * 64 + 32, &sr[32]);
            tmem_wait_ld();
#pragma unroll
            for (int q = 0; q < 64; ++q) x[q] = valid ? __uint_as_float(sr[q]) * p.scale_log2 : -INFINITY;
          };
          load_scaled();
          if (j == 0) {
            // the sub-tile's reference point: the exact column max of this pair
            column_max(x, red_w, q4, lane);
            if (q4 == 0) {
              m_s[2 * lane] = red_w[2 * lane];
              m_s[2 * lane + 1] = red_w[2 * lane + 1];
            }
            sm_bar();
          }
          float xmax = -INFINITY;
#pragma unroll
          for (int q = 0; q < 64; q += 4) {
            const float4 m4 = *reinterpret_cast<const float4*>(m_s + q);
            x[q] -= m4.x;
            x[q + 1] -= m4.y;
            x[q + 2] -= m4.z;
            x[q + 3] -= m4.w;
            xmax = fmaxf(fmaxf(xmax, fmaxf(x[q], x[q + 1])), fmaxf(x[q + 2], x[q + 3]));
          }
          // a score past the slack (or not finite) anywhere in the warpgroup:
          // redo the step with the exact column max, rescale O^T and l (S^T is
          // still in TMEM: S_g+2 is issued only after this step's P is used)
          if (sm_bar_or(!(xmax <= thresh))) {
            load_scaled();
            column_max(x, red_w, q4, lane);
            if (q4 == 0) {
#pragma unroll
              for (int kk = 0; kk < 2; ++kk) {
                const int col = 2 * lane + kk;
                const float m_old = m_s[col];
                const float m_new = fmaxf(m_old, red_w[col]);
                red_w[col] = ex2_approx(m_old - m_new);  // alpha of the column
                m_s[col] = m_new;
              }
            }
            sm_bar();
            // O^T holds the sum through the previous pair: wait for its PV
            if (j > 0) {
              ok = ok && __all_sync(0xffffffffu, mbar_wait(&step_done[(jg - 1) & 3], ((jg - 1) >> 2) & 1, abort_flag,
                                                           p.err, p.wait_ns));
              tc_fence_after();
#pragma unroll
              for (int cc = 0; cc < 2; ++cc) {
                uint32_t o[32];
                tmem_ld32(lane_base + 128 + ub * 64 + cc * 32, o);
                tmem_wait_ld();
#pragma unroll
                for (int q = 0; q < 32; ++q) o[q] = __float_as_uint(__uint_as_float(o[q]) * red_w[cc * 32 + q]);
                tmem_st32(lane_base + 128 + ub * 64 + cc * 32, o);
              }
              tmem_wait_st();
            }
#pragma unroll
            for (int q = 0; q < 64; ++q) {
              lp[q] *= red_w[q];
              x[q] -= m_s[q];
            }
            sm_bar();  // every thread read alpha before red_w is reused
          }
          // P^T row k: 64 queries as 16-bit pairs, 16-byte granules swizzled
          uint8_t* prow = sP + sb * C::P_BYTES + k * 128;
#pragma unroll
          for (int g8 = 0; g8 < 8; ++g8) {
            uint32_t w4[4];
#pragma unroll
            for (int z = 0; z < 4; ++z) {
              const int q = g8 * 8 + 2 * z;
              const float p0 = ex2_approx(x[q]), p1 = ex2_approx(x[q + 1]);
              lp[q] += p0;
              lp[q + 1] += p1;
              w4[z] = pack2<BF16>(p0, p1);
            }
            *reinterpret_cast<uint4*>(prow + ((g8 ^ (k & 7)) * 16)) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
          }
          fence_proxy_async_smem();  // generic-proxy writes, read by the tensor cores
          tc_fence_before();
          __syncwarp();
          if (lane == 0 && !(p.withhold_arrive && jg == 0 && q4 == 0 && blockIdx.x == 0)) mbar_arrive(&p_ready[sb]);
        }
        // the sub-tile's row sums: a column sum over the 128 keys' partials;
        // the epilogue gets 1/l (0 for an empty row) and lse = m + log2(l) in
        // place of m and l
        column_reduce<false>(lp, red_w, q4, lane);
        if (q4 == 0) {
#pragma unroll
          for (int kk = 0; kk < 2; ++kk) {
            const int col = 2 * lane + kk;
            const float l = red_w[col];
            const float m = m_s[col];
            l_s[col] = l > 0.f ? m + log2f(l) : -INFINITY;
            m_s[col] = l > 0.f ? 1.f / l : 0.f;
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&stats_ready[ub]);
        ++u;
      }
    }
  } else {
    regs_dec<kRegsEpilogueT>();
    // ------------------------------------------------------------- epilogue
    // thread = one output column d (TMEM lane of O^T); per sub-tile it writes
    // element d of the block row's 64 query rows
    const int q4 = warp & 3;
    const int d = q4 * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q4 * 32) << 16);
    int u = 0;
    bool ok = true;
    auto dst_row = [&](int grow) -> int64_t {
      if (grow >= p.N) return -1;
      if (!p.q_perm) return grow;
      const int64_t drow = load_perm_t(p.q_perm, p.perm_dtype, grow);
      return drow >= 0 && drow < p.N ? drow : -1;
    };
    for (int i = 0;; ++i) {
      TTTile tl;
      const bool have = next_tile(i, tl);
      __syncwarp();
      if (lane == 0) mbar_arrive(&tile_free[i % kRingT]);
      if (!have) break;
      uint8_t* obase = p.o + 2 * (tl.b * p.os_b + tl.h * p.os_h);
      float* lbase = p.lse ? p.lse + (static_cast<int64_t>(tl.b) * p.H + tl.h) * p.N : nullptr;
      for (int r = 0; r < 2; ++r) {
        const int c = (r ? tl.c1 : tl.c0) & kCountMask;
        const int row0 = tl.t * 128 + r * 64;
        if (tl.n == 0 || c == 0) {
          // the block row keeps no block: O = 0, lse = -inf
          for (int q = 0; q < 64; ++q) {
            const int64_t drow = dst_row(row0 + q);
            if (drow >= 0) {
              reinterpret_cast<uint16_t*>(obase + 2 * drow * p.os_n)[d] = 0;
              if (lbase && d == 0) lbase[drow] = -INFINITY;
            }
          }
          continue;
        }
        const int ub = u & 1;
        const float* inv_s = stats + ub * 128;  // 1/l per query
        const float* lse_s = inv_s + 64;        // lse per query
        ok = ok && __all_sync(0xffffffffu, mbar_wait(&stats_ready[ub], (u >> 1) & 1, abort_flag, p.err, p.wait_ns));
        ok = ok && __all_sync(0xffffffffu, mbar_wait(&o_final[ub], (u >> 1) & 1, abort_flag, p.err, p.wait_ns));
        if (ok) {
          tc_fence_after();
          // eight columns (queries) of this thread's O^T row at a time
#pragma unroll 1
          for (int c8 = 0; c8 < 8; ++c8) {
            uint32_t o[8];
            tmem_ld8(lane_base + 128 + ub * 64 + c8 * 8, o);
            tmem_wait_ld();
#pragma unroll
            for (int z = 0; z < 8; ++z) {
              const int q = c8 * 8 + z;
              const int64_t drow = dst_row(row0 + q);
              if (drow >= 0) {
                const uint32_t bits = pack2<BF16>(__uint_as_float(o[z]) * inv_s[q], 0.f);
                reinterpret_cast<uint16_t*>(obase + 2 * drow * p.os_n)[d] = static_cast<uint16_t>(bits & 0xFFFFu);
              }
            }
          }
          // every read of O^T is done: the MMA may start sub-tile u+2 in this buffer
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&o_empty[ub]);
          if (lbase && d < 64) {
            const int64_t drow = dst_row(row0 + d);
            if (drow >= 0) lbase[drow] = lse_s[d];
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&stats_empty[ub]);
        ++u;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(&g_tt_done[p.slot], 1u) == gridDim.x - 1) {
      g_tt_next[p.slot] = 0;
      g_tt_done[p.slot] = 0;
      __threadfence();
    }
  }
}

template <bool BF16>
int launch_tt(const bsa_fwd_args* a, cudaStream_t st, const void* q_perm, int perm_dtype, uint32_t test_wait_us) {
  using C = TtCfg;
  auto kern = attn_tt_kernel<BF16>;
  static std::atomic<int> checked{0};
  if (!checked.load(std::memory_order_relaxed)) {
    cudaFuncAttributes fa;
    BSA_CUDA_CHECK(cudaFuncGetAttributes(&fa, kern));
    checked.store(fa.numRegs * kThreadsT >= 128 * (kRegsIssueT + kRegsSoftmaxT + kRegsEpilogueT) ? 1 : 2);
  }
  if (checked.load(std::memory_order_relaxed) != 1) return BSA_ERR_UNSUPPORTED;
  static std::atomic<bool> smem_set[64] = {};
  int dev = 0;
  BSA_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return BSA_ERR_DEVICE;
  if (!smem_set[dev].load(std::memory_order_acquire)) {
    BSA_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    smem_set[dev].store(true, std::memory_order_release);
  }
  CUtensorMap mq, mk, mv;
  int r;
  if ((r = tensor_maps(a, C::D, BF16, 64, &mq, &mk, &mv))) return r;
  TtParams p;
  p.tile_ptr = a->plan.tile_ptr;
  p.tile_col = a->plan.tile_col;
  p.tile_order = a->plan.tile_order;
  p.q = static_cast<const uint8_t*>(a->q.data);
  p.qs_b = a->q.stride_b;
  p.qs_h = a->q.stride_h;
  p.qs_n = a->q.stride_n;
  p.q_perm = q_perm;
  p.perm_dtype = perm_dtype;
  p.lse = a->lse;
  p.o = static_cast<uint8_t*>(a->o.data);
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
  p.wait_ns = test_wait_us ? static_cast<uint64_t>(test_wait_us) * 1000ull : kWaitNs;
  p.withhold_arrive = test_wait_us ? 1 : 0;
  p.slot = static_cast<int>(g_tt_launches.fetch_add(1, std::memory_order_relaxed) % kSlotsT);
  int grid = sm_count();
  if (grid > p.total_tiles) grid = p.total_tiles;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreadsT);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  BSA_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, mq, mk, mv, p));
  return BSA_OK;
}

}  // namespace

int launch_attn_tt(const bsa_fwd_args* a, cudaStream_t st, const void* q_perm, int perm_dtype,
                   uint32_t test_wait_us) {
  if (a->plan.block != 64 || a->D != 128) return BSA_ERR_UNSUPPORTED;
  return a->dtype == BSA_DTYPE_BF16 ? launch_tt<true>(a, st, q_perm, perm_dtype, test_wait_us)
                                    : launch_tt<false>(a, st, q_perm, perm_dtype, test_wait_us);
}

}  // namespace bsa
