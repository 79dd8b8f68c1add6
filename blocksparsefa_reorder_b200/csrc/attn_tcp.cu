// Persistent tcgen05 block-sparse attention forward for sm_100a.
//
// Replaces _attn_fwd_block_sparse (triton_kernels/BlockSparse_Naive.py:68-125)
// with its online softmax (:39-60) and epilogue (:119-125): rows with no kept
// block give O = 0 and lse = -inf.  Keys at or past N (a partial last key
// block) are masked.
//
// One CTA per SM loops over 128-row query tiles.  The tiles are numbered
// w = bh * T + r in (b, h)-major order, r ranking the rows of the head's mask
// slice by decreasing kept-block count (the plan's tile_order; natural order
// without one), and CTAs claim them from a global counter: longest tiles
// first within a head, dynamically, so the CTAs finish together, while the
// CTAs in flight still share a head's K / V in L2.  The producer claims a
// tile and passes its number, plan range, (b, h) and row to the other roles
// through a small ring in shared memory.  The counter is one of kWorkSlots per device, taken in turn
// by successive launches; the last CTA to finish resets it.  Roles:
//  * warp 0, one thread: TMA producer (Q per tile, then K_g and V_g-1 per
//    step, V one step behind K because PV_g-1 is issued after S_g; each on
//    its own barrier).  Before it blocks on a full tile ring it loads the V
//    still pending, and the MMA issuer issues a pending PV before it blocks
//    on a ring entry not yet written: the tile those end may be the one the
//    ring waits for (runs of empty tiles fill the ring without any load);
//  * warp 1, one thread: tcgen05.mma issuer (S_g = Q K_g^T, then PV_g-1);
//  * warpgroups 1 and 2: softmax, two threads per query row (lanes i and
//    i ^ 16 of a warp, half of the step's scores each; warpgroup 1 takes
//    lanes 0-15 of every 32-lane TMEM quarter, warpgroup 2 lanes 16-31), P
//    written back into the first BS/2 columns of S's TMEM.  Two softmax warps
//    share each SM sub-partition, so one's waits and TMEM round trips overlap
//    the other's exponentials;
//  * warpgroup 3: epilogue, one query row per thread: O / l from TMEM
//    straight to global memory, lse, and the zero rows of empty tiles;
//  * warps 2-3, with a query permutation only: gather the tile's Q rows
//    q[q_perm[row]] into the Q buffer (the layout the TMA load would give).
// With a query permutation (the fused variant, BlockSparse_Fused.py:173-223)
// Q rows are read from q_perm[row] and O / lse rows written to q_perm[row];
// the mask is in the permuted order.
// The epilogue has its own warps so that the softmax goes straight on to the
// next tile while the previous tile's output is written.
//
// Buffers: S double-buffered in TMEM by global block counter g (S_g in
// buffer g&1); O double-buffered by non-empty-tile counter e (O_e in buffer
// e&1); Q double-buffered in shared memory by e; K and V in rings of KS and
// VS stages; a step is BS keys: one kept block at BLOCK 128, two in the
// paired BLOCK-64 form (BS = 128), one in the single BLOCK-64 form (BS = 64).
// TMEM columns: S0 [0,BS), S1 [BS,2BS), O0 [2BS,2BS+D), O1 [2BS+D,2BS+2D).
// Ordering facts (one thread's tcgen05.mma operations execute in issue order
// and tcgen05.commit tracks every earlier one):
//  * S_g+2 reuses S_g's TMEM and is issued after PV_g, which reads P_g there;
//  * S_g complete implies PV_g-2 complete, and PV_g-1 completes before any
//    later MMA: the softmax's rescale of O waits step_done of PV_g-1;
//  * S_g complete (s_full, seen by the first softmax warp, warp 4, which
//    then arrives on k_empty) frees K_g's stage; the commit after PV_g (step_done[g % 4])
//    frees V_g's stage and lets a rescale of O go ahead;
//  * Q_e's buffer is released (q_empty) by a commit after the tile's last S;
//  * the first PV of tile e+2 waits o_empty[e&1]: the epilogue has read O_e.
// Every wait is bounded by %globaltimer; a timeout sets BSA_DEVERR_TIMEOUT
// and all roles drain and exit.
#include <cudaTypedefs.h>

#include <atomic>

#include "common.cuh"
#include "internal.h"
#include "softmax.cuh"

namespace bsa {

namespace {

// Tile counters for dynamic claiming: launch k uses slot k % kWorkSlots, so
// up to kWorkSlots launches may run at the same time on different streams.
constexpr int kWorkSlots = 64;
__device__ uint32_t g_work_next[kWorkSlots];
__device__ uint32_t g_work_done[kWorkSlots];
// Launch counter shared by every instantiation of the kernel (they share the slots).
std::atomic<unsigned> g_launches{0};
// Armed by bsa_test_arm_wait_timeout: the wait limit (us) of the next forward.
std::atomic<uint32_t> g_test_wait_us{0};

constexpr int kTileRing = 8;   // tile numbers in flight between the producer and the other roles
// readers of each tile-ring entry: MMA thread + 8 softmax + 4 epilogue warps,
// and the 2 Q-gather warps when there is a query permutation (without one they
// leave at once rather than poll the ring next to the softmax warps)
constexpr int kTileUsers = 13;
constexpr int kTileUsersGather = 15;
constexpr int kSoftmaxWarps = 8;


// One claimed tile as the producer hands it to the other roles: the tile
// number (-1 = no more), its plan entries e0 .. e0+n, its (b, h) and tile row.
struct TileSlot {
  int w, e0, n, b, h, t, pad0, pad1;
};

struct TcpParams {
  const int32_t* tile_ptr;
  const int32_t* tile_col;
  const int32_t* tile_order;  // optional: per slice, rows by decreasing kept-block count
  float* lse;
  uint8_t* o;                // output base (16-bit elements)
  int64_t os_b, os_h, os_n;  // output strides in elements
  int32_t* err;
  const uint8_t* q;           // query base, for the gather of permuted rows
  int64_t qs_b, qs_h, qs_n;   // query strides in elements
  const void* q_perm;         // optional query permutation (new row -> old row)
  int perm_dtype;             // bsa_index_dtype of q_perm
  int H, N, nb, T, mask_b, mask_h, total_tiles;
  int slot;  // work counter slot
  float scale_log2;
  // 0: run.  1 / 2: run only if the plan averages at least / fewer than
  // kPairMinEntries kept blocks per tile (the two forms launched for BLOCK 64).
  int select;
  // limit of every bounded wait (kWaitNs unless a test shortened it)
  uint64_t wait_ns;
  // test of the timeout path: softmax warp 0 of CTA 0 withholds its arrival on
  // p_ready for the CTA's first step, so the MMA issuer's wait for that step
  // runs out (no TMA load or MMA is ever counted on that barrier)
  int withhold_arrive;
};

// BLOCK 64: tiles averaging at least this many kept key blocks run the form
// that takes them in pairs (128-key steps); sparser plans run one block per
// step.  Measured on the causal sweep masks, the paired form is faster from
// 7 kept blocks per tile up (359 vs 320 TF/s at 7, 446-458 vs 366-370 at
// 26.6); below 4 a tile has so few steps that pairing saves little.
constexpr int kPairMinEntries = 4;

constexpr int kSmemLimitP = 232448;
constexpr int kThreadsP = 512;
// setmaxnreg split over the four warpgroups (producer / MMA / Q gather, two
// softmax, epilogue); the launch holds 128 per thread (65536 / 512).
constexpr int kRegsLaunchP = 128;
constexpr int kRegsIssueP = 64;
constexpr int kRegsSoftmaxP = 176;
constexpr int kRegsEpilogueP = 96;
constexpr int kRegsSplitP = kRegsIssueP + 2 * kRegsSoftmaxP + kRegsEpilogueP;
static_assert(128 * kRegsSplitP <= kThreadsP * kRegsLaunchP, "register split");

__device__ __forceinline__ int64_t load_perm(const void* perm, int dtype, int64_t i) {
  return dtype == BSA_INDEX_I64 ? __ldg(static_cast<const int64_t*>(perm) + i)
                                : static_cast<int64_t>(__ldg(static_cast<const int32_t*>(perm) + i));
}

// BN is the mask's block size (64 or 128).  A pipeline step covers BS keys:
// one kept key block, or with PAIR (BN 64) two -- the tile's plan entries
// taken in pairs, each 64-row box landing in one half of the stage -- so that
// the S MMAs are 128 wide, the PV MMAs 128 deep, and the per-step hand-offs
// between the roles are paid once per 128 keys.
template <int D, int BN, bool PAIR>
struct TcpCfg {
  static constexpr int BM = 128;
  static constexpr int BS = PAIR ? 128 : BN;  // keys per step
  static constexpr int SUB = BS / BN;   // plan entries per step
  static constexpr int NCHUNK = D / 64;
  static constexpr int Q_CHUNK = BM * 128;
  static constexpr int KV_CHUNK = BS * 128;
  static constexpr int BOX_BYTES = BN * 128;  // one entry's rows of one 64-column chunk
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_BYTES = BS * D * 2;
  // barriers (2 KS + VS + 21 + 2 kTileRing), TMEM slot and abort flag, then the tile ring
  static constexpr int ring_off(int ks, int vs) { return ((2 * ks + vs + 21 + 2 * kTileRing) * 8 + 8 + 15) / 16 * 16; }
  static constexpr int bar_bytes(int ks, int vs) {
    return (ring_off(ks, vs) + kTileRing * static_cast<int>(sizeof(TileSlot)) + 127) / 128 * 128;
  }
  static constexpr int STATS_BYTES = 2 * 2 * BM * 4;  // [buffer][m, l][row] fp32
  static constexpr bool fits(int ks, int vs) {
    return 2 * Q_BYTES + (ks + vs) * KV_BYTES + bar_bytes(ks, vs) + STATS_BYTES <= kSmemLimitP;
  }
  // K_j is released when S_j completes, V_j only when PV_j does: K gets the deeper ring.
  static constexpr int KS = fits(4, 4) || fits(4, 3) ? 4 : 3;
  static constexpr int VS = fits(4, 4) ? 4 : fits(4, 3) ? 3 : 2;
  static constexpr int BAR_BYTES = bar_bytes(KS, VS);
  static constexpr int SMEM = 2 * Q_BYTES + (KS + VS) * KV_BYTES + BAR_BYTES + STATS_BYTES;
  static constexpr int O_COL0 = 2 * BS;
  static constexpr int TMEM_COLS = 2 * BS + 2 * D <= 256 ? 256 : 512;
  static_assert(SMEM <= kSmemLimitP, "shared memory budget");
  static_assert(2 * BS + 2 * D <= 512, "TMEM budget");
  static_assert(SUB * BN == BS && (SUB == 1 || SUB == 2) && (!PAIR || BN == 64), "block size");
  static constexpr int RING_OFF = ring_off(KS, VS);
  static_assert(RING_OFF + kTileRing * static_cast<int>(sizeof(TileSlot)) <= BAR_BYTES, "barrier area");
};

template <int D, int BN, bool BF16, bool PAIR>
__global__ void __launch_bounds__(kThreadsP, 1)
    attn_tcp_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, const TcpParams p) {
  using C = TcpCfg<D, BN, PAIR>;
  constexpr int KS = C::KS, VS = C::VS;
  extern __shared__ __align__(1024) uint8_t smem[];
  if (smem_u32(smem) & 1023u) {
    if (threadIdx.x == 0) set_err(p.err, BSA_DEVERR_ALIGN);
    return;
  }
  uint8_t* sQ = smem;                   // [2][Q_BYTES]
  uint8_t* sK = sQ + 2 * C::Q_BYTES;    // [KS][KV_BYTES]
  uint8_t* sV = sK + KS * C::KV_BYTES;  // [VS][KV_BYTES]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + VS * C::KV_BYTES);
  float* stats = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + C::BAR_BYTES);
  uint64_t* q_full = bars;               // [2]
  uint64_t* q_empty = q_full + 2;        // [2] the tile's last S has read Q
  uint64_t* k_full = q_empty + 2;        // [KS] by step g % KS: K_g landed
  uint64_t* k_empty = k_full + KS;       // [KS] by step g % KS: S_g completed (K_g's stage free)
  uint64_t* v_full = k_empty + KS;       // [VS] by step g % VS: V_g landed
  uint64_t* s_full = v_full + VS;        // [2] by S buffer
  uint64_t* p_ready = s_full + 2;        // [2] by S buffer, 8 softmax warps
  uint64_t* o_final = p_ready + 2;       // [2] by O buffer: the tile's last PV completed
  uint64_t* o_empty = o_final + 2;       // [2] by O buffer: 4 epilogue warps read O
  uint64_t* stats_ready = o_empty + 2;   // [2] 8 softmax warps wrote (m, l)
  uint64_t* stats_empty = stats_ready + 2;  // [2] 4 epilogue warps read (m, l)
  // [4] by step g % 4: the commit after PV_g (V_g's stage free, O up to PV_g complete)
  uint64_t* step_done = stats_empty + 2;
  uint64_t* drain = step_done + 4;
  uint64_t* tile_ready = drain + 1;              // [kTileRing] producer wrote the entry
  uint64_t* tile_free = tile_ready + kTileRing;  // [kTileRing] all kTileUsers read it
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tile_free + kTileRing);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // [kTileRing] claimed tiles with their plan range, (b, h) and row
  volatile TileSlot* tile_ring = reinterpret_cast<volatile TileSlot*>(reinterpret_cast<uint8_t*>(bars) + C::RING_OFF);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], p.q_perm ? 2 : 1);  // gather warps, or the TMA transaction
      mbar_init(&q_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_ready[i], kSoftmaxWarps);
      mbar_init(&o_final[i], 1);
      mbar_init(&o_empty[i], 4);
      mbar_init(&stats_ready[i], kSoftmaxWarps);
      mbar_init(&stats_empty[i], 4);
    }
    for (int i = 0; i < KS; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < VS; ++i) mbar_init(&v_full[i], 1);
    for (int i = 0; i < 4; ++i) mbar_init(&step_done[i], 1);
    mbar_init(drain, 1);
    for (int i = 0; i < kTileRing; ++i) {
      mbar_init(&tile_ready[i], 1);
      mbar_init(&tile_free[i], p.q_perm ? kTileUsersGather : kTileUsers);
    }
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
  // Launched as a programmatic dependent of the plan build (or whatever ran
  // before on the stream): everything above touched only this CTA's shared
  // memory and TMEM; from here on global memory is read and written.
  grid_dependency_wait();
  if constexpr (BN == 64) {
    if (p.select) {
      // one of the two BLOCK 64 forms: every CTA reads the same plan total, so
      // all take the same decision; the form not chosen frees TMEM and exits
      // before it claims a tile
      const int tiles = p.mask_b * p.mask_h * p.T;
      const bool dense = __ldg(&p.tile_ptr[tiles]) >= kPairMinEntries * tiles;
      if (dense != (p.select == 1)) {
        if (warp == 1) tmem_dealloc(tmem, C::TMEM_COLS);
        return;
      }
    }
  }

  // tile w -> (entries e0 .. e0+n of the plan, b, h, tile row t); the producer
  // reads it when it claims the tile and passes it on through the ring
  auto tile_info = [&](int w, int& e0, int& n, int& b, int& h, int& t) {
    const int bh = w / p.T;
    const int r = w - bh * p.T;
    b = bh / p.H;
    h = bh - b * p.H;
    const int s = (p.mask_b == 1 ? 0 : b) * p.mask_h + (p.mask_h == 1 ? 0 : h);
    t = p.tile_order ? p.tile_order[s * p.T + r] : r;
    e0 = p.tile_ptr[s * p.T + t];
    n = p.tile_ptr[s * p.T + t + 1] - e0;
  };
  // i-th tile of this CTA from the ring (every calling thread waits and reads
  // it; w = -1 when there are no more or a wait failed)
  auto next_tile = [&](int i, int& w, int& e0, int& n, int& b, int& h, int& t) {
    const int ri = i % kTileRing;
    if (!mbar_wait(&tile_ready[ri], (i / kTileRing) & 1, abort_flag, p.err, p.wait_ns)) {
      w = -1;
      return;
    }
    w = tile_ring[ri].w;
    e0 = tile_ring[ri].e0;
    n = tile_ring[ri].n;
    b = tile_ring[ri].b;
    h = tile_ring[ri].h;
    t = tile_ring[ri].t;
  };

  if (warp < 4) {
    regs_dec<kRegsIssueP>();
    if (warp == 0 && lane == 0) {
      // ------------------------------------------------------------ producer
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      int e = 0, g = 0, gv = 0;  // non-empty tiles, K steps, V steps loaded so far
      int pv_b = 0, pv_h = 0;    // the step whose V is still to load (gv < g)
      int pv_kb[C::SUB] = {};
      bool ok = true;
      int qarmed = 0;  // Q tiles loaded by TMA so far
      // step gs's K stage is free once S_gs-KS completed
      auto wait_k_stage = [&](int gs) -> bool {
        return gs < KS || mbar_wait(&k_empty[gs % KS], ((gs / KS) - 1) & 1, abort_flag, p.err, p.wait_ns);
      };
      // V of step gv (one step behind K: PV_gv is issued after S_gv+1) into
      // its stage, free once PV_gv-VS completed
      auto load_v = [&]() -> bool {
        if (gv >= VS && !mbar_wait(&step_done[(gv - VS) & 3], ((gv - VS) >> 2) & 1, abort_flag, p.err, p.wait_ns))
          return false;
        const int st = gv % VS;
        mbar_arrive_expect_tx(&v_full[st], C::KV_BYTES);
#pragma unroll
        for (int u = 0; u < C::SUB; ++u)
          for (int c = 0; c < C::NCHUNK; ++c)
            tma_load_4d(sV + st * C::KV_BYTES + c * C::KV_CHUNK + u * C::BOX_BYTES, &tmV, &v_full[st], c * 64,
                        pv_kb[u] * BN, pv_h, pv_b);
        ++gv;
        return true;
      };
      for (int i = 0; ok; ++i) {
        // claim the next tile and pass its number on
        const uint32_t claim = atomicAdd(&g_work_next[p.slot], 1u);
        const int w = claim < static_cast<uint32_t>(p.total_tiles) ? static_cast<int>(claim) : -1;
        const int ri = i % kTileRing;
        int e0 = 0, n = 0, b = 0, h = 0, t = 0;
        if (w >= 0) tile_info(w, e0, n, b, h, t);
        if (i >= kTileRing) {
          const uint32_t par = ((i / kTileRing) - 1) & 1;
          // a full ring: a role is still on an earlier tile, whose last PV may
          // need the V not loaded yet
          if (!mbar_try_wait(&tile_free[ri], par) && gv < g && !(ok = load_v())) break;
          if (!(ok = mbar_wait(&tile_free[ri], par, abort_flag, p.err, p.wait_ns))) break;
        }
        tile_ring[ri].w = w;
        tile_ring[ri].e0 = e0;
        tile_ring[ri].n = n;
        tile_ring[ri].b = b;
        tile_ring[ri].h = h;
        tile_ring[ri].t = t;
        mbar_arrive(&tile_ready[ri]);  // release: the entry is visible to every waiter
        if (w < 0) {
          // No more tiles for this CTA: the next kernel on the stream (launched
          // as a programmatic dependent) may start its set-up on SMs as they
          // free up; it reads global memory only after this grid completed.
          allow_dependents();
          break;
        }
        if (n == 0) continue;
        const int qb = e & 1;
        if (!p.q_perm) {  // (permuted queries: warps 2-3 gather Q)
          if (e >= 2 && !(ok = mbar_wait(&q_empty[qb], ((e >> 1) - 1) & 1, abort_flag, p.err, p.wait_ns))) break;
          mbar_arrive_expect_tx(&q_full[qb], C::Q_BYTES);
          ++qarmed;
          for (int c = 0; c < C::NCHUNK; ++c)
            tma_load_4d(sQ + qb * C::Q_BYTES + c * C::Q_CHUNK, &tmQ, &q_full[qb], c * 64, t * 128, h, b);
        }
        ++e;
        const int nsteps = (n + C::SUB - 1) / C::SUB;
        for (int j = 0; j < nsteps; ++j, ++g) {
          const int st = g % KS;
          if (!(ok = wait_k_stage(g))) break;
          int kb[C::SUB];
#pragma unroll
          for (int u = 0; u < C::SUB; ++u) {
            // a missing second entry (odd count) repeats the first: the softmax masks it out
            const int ei = j * C::SUB + u < n ? j * C::SUB + u : j * C::SUB;
            kb[u] = static_cast<int>(static_cast<uint32_t>(p.tile_col[e0 + ei]) & 0xFFFFFFu);
            if (kb[u] >= p.nb) {
              set_err(p.err, BSA_DEVERR_PLAN);
              kb[u] = 0;
            }
          }
          mbar_arrive_expect_tx(&k_full[st], C::KV_BYTES);
#pragma unroll
          for (int u = 0; u < C::SUB; ++u)
            for (int c = 0; c < C::NCHUNK; ++c)
              tma_load_4d(sK + st * C::KV_BYTES + c * C::KV_CHUNK + u * C::BOX_BYTES, &tmK, &k_full[st], c * 64,
                          kb[u] * BN, h, b);
          if (gv < g && !(ok = load_v())) break;
          pv_b = b;
          pv_h = h;
#pragma unroll
          for (int u = 0; u < C::SUB; ++u) pv_kb[u] = kb[u];
        }
      }
      if (ok && gv < g) ok = load_v();  // the last step's V
      // Every load this thread issued lands before the CTA exits, also when a
      // role gave up and the loads were never consumed: the last phase armed on
      // each K, V and Q barrier (all earlier phases completed before their
      // stage was loaded again).
      for (int j = g > KS ? g - KS : 0; j < g; ++j) mbar_wait(&k_full[j % KS], (j / KS) & 1, nullptr, nullptr, p.wait_ns);
      for (int j = gv > VS ? gv - VS : 0; j < gv; ++j)
        mbar_wait(&v_full[j % VS], (j / VS) & 1, nullptr, nullptr, p.wait_ns);
      for (int j = qarmed > 2 ? qarmed - 2 : 0; j < qarmed; ++j)
        mbar_wait(&q_full[j & 1], (j >> 1) & 1, nullptr, nullptr, p.wait_ns);
    } else if (warp == 1 && lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      constexpr uint32_t idesc_qk = make_idesc_f16(BF16, 128, C::BS, false, false);
      constexpr uint32_t idesc_pv = make_idesc_f16(BF16, 128, D, false, true);
      const uint32_t q_addr = smem_u32(sQ);
      const uint32_t k_addr = smem_u32(sK);
      const uint32_t v_addr = smem_u32(sV);
      int e = 0;   // non-empty tiles so far
      int jg = 0;  // blocks (S MMAs) so far
      // the PV still to issue: block index, O buffer, first / last block of its tile
      int pend_j = -1, pend_ob = 0;
      bool pend_first = false, pend_last = false;
      bool ok = true;
      int pv_issued_tiles = 0;  // non-empty tiles whose first PV was issued (o_empty accounting)
      auto do_pv = [&]() -> bool {
        const int i = pend_j, st = i % VS;
        if (pend_first && pv_issued_tiles >= 2 &&
            !mbar_wait(&o_empty[pend_ob], ((pv_issued_tiles >> 1) - 1) & 1, abort_flag, p.err, p.wait_ns))
          return false;
        if (!mbar_wait(&p_ready[i & 1], (i >> 1) & 1, abort_flag, p.err, p.wait_ns)) return false;
        if (!mbar_wait(&v_full[st], (i / VS) & 1, abort_flag, p.err, p.wait_ns)) return false;
        tc_fence_after();
        const uint32_t p_tmem = tmem + (i & 1) * C::BS;  // P_i lives in the first columns of S buffer i&1
        const uint32_t o_tmem = tmem + C::O_COL0 + pend_ob * D;
#pragma unroll
        for (int kk = 0; kk < C::BS / 16; ++kk) {
          const uint64_t bd = make_sw128_desc(v_addr + st * C::KV_BYTES + kk * 16 * 128, C::KV_CHUNK, 1024);
          tc_mma_ts(o_tmem, p_tmem + kk * 8, bd, idesc_pv, (!pend_first || kk > 0) ? 1u : 0u);
        }
        tc_commit(&step_done[i & 3]);
        if (pend_last) tc_commit(&o_final[pend_ob]);
        if (pend_first) ++pv_issued_tiles;
        pend_j = -1;
        return true;
      };
      for (int i = 0; ok; ++i) {
        // the next tile not announced yet: issue the pending PV now (the tile
        // it ends may be what the ring waits for)
        if (pend_j >= 0 && !mbar_try_wait(&tile_ready[i % kTileRing], (i / kTileRing) & 1) && !(ok = do_pv())) break;
        int w, e0, n, b, h, t;
        next_tile(i, w, e0, n, b, h, t);
        mbar_arrive(&tile_free[i % kTileRing]);
        if (w < 0) break;
        if (n == 0) continue;
        const int qb = e & 1;
        if (!(ok = mbar_wait(&q_full[qb], (e >> 1) & 1, abort_flag, p.err, p.wait_ns))) break;
        tc_fence_after();
        const int nsteps = (n + C::SUB - 1) / C::SUB;
        for (int j = 0; j < nsteps; ++j, ++jg) {
          const int st = jg % KS;
          if (!(ok = mbar_wait(&k_full[st], (jg / KS) & 1, abort_flag, p.err, p.wait_ns))) break;
          tc_fence_after();
          const uint32_t d_tmem = tmem + (jg & 1) * C::BS;
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk & 3) * 32;  // 16 elements = 32 bytes inside the 128-byte swizzle row
            const uint64_t a = make_sw128_desc(q_addr + qb * C::Q_BYTES + (kk >> 2) * C::Q_CHUNK + off, 16, 1024);
            const uint64_t bd = make_sw128_desc(k_addr + st * C::KV_BYTES + (kk >> 2) * C::KV_CHUNK + off, 16, 1024);
            tc_mma_ss(d_tmem, a, bd, idesc_qk, kk > 0 ? 1u : 0u);
          }
          tc_commit(&s_full[jg & 1]);
          if (j == nsteps - 1) tc_commit(&q_empty[qb]);
          if (pend_j >= 0 && !(ok = do_pv())) break;
          pend_j = jg;
          pend_ob = e & 1;
          pend_first = j == 0;
          pend_last = j == nsteps - 1;
        }
        ++e;
      }
      if (ok && pend_j >= 0) ok = do_pv();
      tc_commit(drain);
      mbar_wait(drain, 0, nullptr, nullptr, p.wait_ns);
    } else if (warp >= 2 && p.q_perm) {
      // ------------------------------------------------- Q gather (permuted queries)
      // Warp 2 fills rows 0-63 of the tile, warp 3 rows 64-127, each row
      // as 16-byte granules into the 128-byte-swizzled chunks the MMA reads.
      const int gw = warp - 2;
      int e = 0;
      bool ok = true;
      for (int i = 0;; ++i) {
        int w, e0, n, b, h, t;
        next_tile(i, w, e0, n, b, h, t);
        __syncwarp();
        if (lane == 0) mbar_arrive(&tile_free[i % kTileRing]);
        if (w < 0) break;
        if (!p.q_perm || n == 0) continue;
        const int qb = e & 1;
        if (e >= 2)
          ok = ok && __all_sync(0xffffffffu, mbar_wait(&q_empty[qb], ((e >> 1) - 1) & 1, abort_flag, p.err, p.wait_ns));
        ++e;
        if (!ok) continue;
        for (int k = 0; k < 2; ++k) {
          const int r = gw * 64 + k * 32 + lane;
          const int grow = t * 128 + r;
          const uint4* src = nullptr;
          if (grow < p.N) {
            const int64_t old = load_perm(p.q_perm, p.perm_dtype, grow);
            if (old >= 0 && old < p.N)
              src = reinterpret_cast<const uint4*>(p.q + 2 * (b * p.qs_b + h * p.qs_h + old * p.qs_n));
            else
              set_err(p.err, BSA_DEVERR_PERM_RANGE);
          }
#pragma unroll
          for (int c = 0; c < C::NCHUNK; ++c) {
            uint8_t* dst = sQ + qb * C::Q_BYTES + c * C::Q_CHUNK + r * 128;
            uint4 v[8];
#pragma unroll
            for (int g = 0; g < 8; ++g) v[g] = src ? __ldg(src + c * 8 + g) : make_uint4(0, 0, 0, 0);
#pragma unroll
            for (int g = 0; g < 8; ++g) *reinterpret_cast<uint4*>(dst + ((g ^ (r & 7)) * 16)) = v[g];
          }
        }
        fence_proxy_async_smem();  // generic-proxy writes, read by the tensor cores
        __syncwarp();
        if (lane == 0) mbar_arrive(&q_full[qb]);
      }
    }
  } else if (warp < 12) {
    regs_inc<kRegsSoftmaxP>();
    // -------------------------------------------------------------- softmax
    const int hw = (warp - 4) >> 2;  // softmax warpgroup: lanes 0-15 or 16-31 of the quarter
    const int q4 = warp & 3;         // TMEM lane quarter this warp may access
    const int sub = lane >> 4;       // which half of the row's scores this thread holds
    const int row = q4 * 32 + hw * 16 + (lane & 15);
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q4 * 32 + hw * 16) << 16);
    const int half = row >> 6;
    constexpr int HB = C::BS / 2;  // scores per thread per step
    int e = 0, jg = 0;
    bool ok = true;
    for (int i = 0;; ++i) {
      int w, e0, n, b, h, t;
      next_tile(i, w, e0, n, b, h, t);
      __syncwarp();
      if (lane == 0) mbar_arrive(&tile_free[i % kTileRing]);
      if (w < 0) break;
      if (n == 0) continue;  // the epilogue writes its zero rows
      const int ob = e & 1;
      float m_run = -INFINITY, l_run = 0.f;
      const int nsteps = (n + C::SUB - 1) / C::SUB;
      for (int j = 0; j < nsteps; ++j, ++jg) {
        const int sb = jg & 1;
        // after a failed wait every later wait returns at once (abort flag)
        if (!(ok = ok && __all_sync(0xffffffffu, mbar_wait(&s_full[sb], (jg >> 1) & 1, abort_flag, p.err, p.wait_ns))))
          continue;
        tc_fence_after();
        // S_jg complete: the tensor cores are done with K_jg's stage
        if (warp == 4 && lane == 0) mbar_arrive(&k_empty[jg % KS]);
        uint32_t sr[HB];
        tmem_ld16x2<HB, HB>(lane_base + sb * C::BS, sr);
        tmem_wait_ld();
        // Per plan entry of the step: whether this row's query block keeps it
        // (per-half flags at BN 64; a missing second entry is never kept) and
        // how many of its keys lie before N (TMA zero-filled the rest).  The
        // same for all rows of a warp (they share a 64-row query block).
        bool act[C::SUB];
        int kvalid[C::SUB];
        bool any = false, need_mask = false;
#pragma unroll
        for (int u = 0; u < C::SUB; ++u) {
          const int ei = j * C::SUB + u;
          const uint32_t entry = ei < n ? static_cast<uint32_t>(__ldg(&p.tile_col[e0 + ei])) : 0u;
          act[u] = ei < n && (BN == 128 || ((entry >> 24 >> half) & 1u) != 0);
          kvalid[u] = p.N - static_cast<int>(entry & 0xFFFFFFu) * BN;
          any = any || act[u];
          need_mask = need_mask || !act[u] || kvalid[u] < BN;
        }
        uint32_t pr[HB / 2];
        if (any) {
          // this thread's HB keys lie in one entry of the step (HB divides BN)
          const int u = sub * HB / BN;
          const bool act_u = C::SUB == 1 || u == 0 ? act[0] : act[C::SUB - 1];
          if (need_mask) {
            // keys at or past N of a kept entry (an entry this row's block
            // does not keep is handled whole by softmax_block_split)
            const int kvalid_u = C::SUB == 1 || u == 0 ? kvalid[0] : kvalid[C::SUB - 1];
            const int key0 = sub * HB - u * BN;  // key of sr[0] within that entry
            if (__any_sync(0xffffffffu, act_u && key0 + HB > kvalid_u)) {
#pragma unroll
              for (int i = 0; i < HB; ++i)
                if (key0 + i >= kvalid_u) sr[i] = __float_as_uint(-INFINITY);
            }
          }
          const float alpha = softmax_block_split<HB, BF16>(sr, pr, p.scale_log2, m_run, l_run, act_u);
          if (__any_sync(0xffffffffu, alpha != 1.f)) {
            // O holds the sum up to block j-1 of this tile: wait for that PV, rescale in TMEM.
            if (!(ok = __all_sync(0xffffffffu,
                                  mbar_wait(&step_done[(jg - 1) & 3], ((jg - 1) >> 2) & 1, abort_flag, p.err, p.wait_ns))))
              continue;
            tc_fence_after();
#pragma unroll
            for (int c = 0; c < D / 64; ++c) {
              uint32_t o[32];
              tmem_ld16x2<32, D / 2>(lane_base + C::O_COL0 + ob * D + c * 32, o);
              tmem_wait_ld();
#pragma unroll
              for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
              tmem_st16x2<32, D / 2>(lane_base + C::O_COL0 + ob * D + c * 32, o);
            }
          }
        } else {
#pragma unroll
          for (int i = 0; i < HB / 2; ++i) pr[i] = 0u;
        }
        // P_j into the first BS/2 columns of its S buffer (all of S is in registers)
        tmem_st16x2<HB / 2, HB / 2>(lane_base + sb * C::BS, pr);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0 && !(p.withhold_arrive && jg == 0 && q4 == 0 && hw == 0 && blockIdx.x == 0))
          mbar_arrive(&p_ready[sb]);
      }
      // hand the row's (m, l) to the epilogue warps
      if (e >= 2)
        ok = ok && __all_sync(0xffffffffu, mbar_wait(&stats_empty[ob], ((e >> 1) - 1) & 1, abort_flag, p.err, p.wait_ns));
      if (sub == 0) {
        stats[ob * 256 + row] = m_run;
        stats[ob * 256 + 128 + row] = l_run;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&stats_ready[ob]);
      ++e;
    }
  } else {
    regs_dec<kRegsEpilogueP>();
    // ------------------------------------------------------------- epilogue
    const int q4 = warp & 3;
    const int row = q4 * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q4 * 32) << 16);
    int e = 0;
    bool ok = true;
    for (int i = 0;; ++i) {
      int w, e0, n, b, h, t;
      next_tile(i, w, e0, n, b, h, t);
      __syncwarp();
      if (lane == 0) mbar_arrive(&tile_free[i % kTileRing]);
      if (w < 0) break;
      const int grow = t * 128 + row;
      // destination row: the permuted query's original row
      int64_t drow = grow;
      if (p.q_perm && grow < p.N) {
        drow = load_perm(p.q_perm, p.perm_dtype, grow);
        if (drow < 0 || drow >= p.N) {
          set_err(p.err, BSA_DEVERR_PERM_RANGE);
          drow = p.N;  // no store
        }
      }
      const bool store = grow < p.N && drow < p.N;
      uint8_t* orow = p.o + 2 * (b * p.os_b + h * p.os_h + drow * p.os_n);
      float* lrow = p.lse ? p.lse + (static_cast<int64_t>(b) * p.H + h) * p.N + drow : nullptr;
      if (n == 0) {
        // no kept block: O = 0 and lse = -inf for the tile's rows
        if (store) {
#pragma unroll
          for (int i = 0; i < D / 8; ++i) reinterpret_cast<uint4*>(orow)[i] = make_uint4(0, 0, 0, 0);
          if (lrow) *lrow = -INFINITY;
        }
        continue;
      }
      const int ob = e & 1;
      ok = ok && __all_sync(0xffffffffu, mbar_wait(&stats_ready[ob], (e >> 1) & 1, abort_flag, p.err, p.wait_ns));
      float m_run = 0.f, l_run = 0.f;
      if (ok) {
        m_run = stats[ob * 256 + row];
        l_run = stats[ob * 256 + 128 + row];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&stats_empty[ob]);
      ok = ok && __all_sync(0xffffffffu, mbar_wait(&o_final[ob], (e >> 1) & 1, abort_flag, p.err, p.wait_ns));
      if (ok) {
        tc_fence_after();
        const float inv_l = l_run > 0.f ? 1.f / l_run : 0.f;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(lane_base + C::O_COL0 + ob * D + c * 32, o);
          tmem_wait_ld();
          if (c == D / 32 - 1) {
            // every read of O_e is done: the MMA may start tile e+2 in this buffer
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&o_empty[ob]);
          }
          if (store) {
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              uint4 v;
              v.x = pack2<BF16>(__uint_as_float(o[8 * g + 0]) * inv_l, __uint_as_float(o[8 * g + 1]) * inv_l);
              v.y = pack2<BF16>(__uint_as_float(o[8 * g + 2]) * inv_l, __uint_as_float(o[8 * g + 3]) * inv_l);
              v.z = pack2<BF16>(__uint_as_float(o[8 * g + 4]) * inv_l, __uint_as_float(o[8 * g + 5]) * inv_l);
              v.w = pack2<BF16>(__uint_as_float(o[8 * g + 6]) * inv_l, __uint_as_float(o[8 * g + 7]) * inv_l);
              reinterpret_cast<uint4*>(orow)[c * 4 + g] = v;
            }
          }
        }
        if (lrow && store) *lrow = l_run > 0.f ? m_run + log2f(l_run) : -INFINITY;
      }
      ++e;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
  if (threadIdx.x == 0) {
    // every claim of this CTA is done; the last CTA resets the slot for the next launch
    __threadfence();
    if (atomicAdd(&g_work_done[p.slot], 1u) == gridDim.x - 1) {
      g_work_next[p.slot] = 0;
      g_work_done[p.slot] = 0;
      __threadfence();
    }
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

// The three tensor maps of a forward, encoded once per argument set: the
// encoding is host work that every call with the same tensors would repeat.
// A small per-thread cache keyed by everything the encoding reads.
struct MapKey {
  const void* q;
  const void* k;
  const void* v;
  int64_t s[9];
  int B, H, N, D, bf16, bn;
  bool operator==(const MapKey& o) const {
    if (q != o.q || k != o.k || v != o.v || B != o.B || H != o.H || N != o.N || D != o.D || bf16 != o.bf16 ||
        bn != o.bn)
      return false;
    for (int i = 0; i < 9; ++i)
      if (s[i] != o.s[i]) return false;
    return true;
  }
};
struct MapEntry {
  MapKey key;
  CUtensorMap mq, mk, mv;
  bool used;
};
constexpr int kMapCache = 8;

int tensor_maps(const bsa_fwd_args* a, int D, bool bf16, int bn, CUtensorMap* mq, CUtensorMap* mk, CUtensorMap* mv) {
  thread_local MapEntry cache[kMapCache] = {};
  thread_local int next = 0;
  MapKey key{a->q.data, a->k.data, a->v.data,
             {a->q.stride_b, a->q.stride_h, a->q.stride_n, a->k.stride_b, a->k.stride_h, a->k.stride_n, a->v.stride_b,
              a->v.stride_h, a->v.stride_n},
             a->B, a->H, a->N, D, bf16 ? 1 : 0, bn};
  for (int i = 0; i < kMapCache; ++i) {
    if (cache[i].used && cache[i].key == key) {
      *mq = cache[i].mq;
      *mk = cache[i].mk;
      *mv = cache[i].mv;
      return BSA_OK;
    }
  }
  int r;
  if ((r = make_tensor_map_4d(mq, a->q, a->B, a->H, a->N, D, bf16, 128))) return r;
  if ((r = make_tensor_map_4d(mk, a->k, a->B, a->H, a->N, D, bf16, bn))) return r;
  if ((r = make_tensor_map_4d(mv, a->v, a->B, a->H, a->N, D, bf16, bn))) return r;
  MapEntry& e = cache[next];
  next = (next + 1) % kMapCache;
  e.key = key;
  e.mq = *mq;
  e.mk = *mk;
  e.mv = *mv;
  e.used = true;
  return BSA_OK;
}

template <int D, int BN, bool BF16, bool PAIR>
int launch_p(const bsa_fwd_args* a, cudaStream_t st, const void* q_perm, int perm_dtype, int select,
             uint32_t test_wait_us) {
  using C = TcpCfg<D, BN, PAIR>;
  auto kern = attn_tcp_kernel<D, BN, BF16, PAIR>;
  // The setmaxnreg split needs the launch to hold at least the sum of the
  // three warpgroups' shares; with fewer the increase would never be granted.
  static std::atomic<int> checked{0};  // 1 ok, 2 too few registers
  if (!checked.load(std::memory_order_relaxed)) {
    cudaFuncAttributes fa;
    BSA_CUDA_CHECK(cudaFuncGetAttributes(&fa, kern));
    checked.store(fa.numRegs * kThreadsP >= 128 * kRegsSplitP ? 1 : 2);
  }
  if (checked.load(std::memory_order_relaxed) != 1) return BSA_ERR_UNSUPPORTED;
  // the shared-memory opt-in, once per device
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
  if ((r = tensor_maps(a, D, BF16, BN, &mq, &mk, &mv))) return r;
  TcpParams p;
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
  p.select = select;
  p.wait_ns = test_wait_us ? static_cast<uint64_t>(test_wait_us) * 1000ull : kWaitNs;
  p.withhold_arrive = test_wait_us ? 1 : 0;
  p.slot = static_cast<int>(g_launches.fetch_add(1, std::memory_order_relaxed) % kWorkSlots);
  int grid = sm_count();
  if (grid > p.total_tiles) grid = p.total_tiles;
  // programmatic stream serialization: the CTAs may start (barriers, TMEM)
  // while the previous kernel on the stream finishes; they wait for it in
  // grid_dependency_wait() before touching global memory
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreadsP);
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

int launch_attn_tcp(const bsa_fwd_args* a, cudaStream_t st, const void* q_perm, int perm_dtype) {
  const bool bf16 = a->dtype == BSA_DTYPE_BF16;
  const int bn = a->plan.block;
  // an armed timeout test applies to this forward (both BLOCK 64 launches)
  const uint32_t tw = g_test_wait_us.load(std::memory_order_relaxed) ? g_test_wait_us.exchange(0) : 0u;
  // BLOCK 64: both forms are launched back to back and the plan's density
  // (read on the device, no host synchronisation) picks the one that runs.
#define BSA_TCP_CASE(D_, BN_)                                                                     \
  if (a->D == D_ && bn == BN_) {                                                                  \
    if constexpr (BN_ == 128)                                                                     \
      return bf16 ? launch_p<D_, BN_, true, false>(a, st, q_perm, perm_dtype, 0, tw)                  \
                  : launch_p<D_, BN_, false, false>(a, st, q_perm, perm_dtype, 0, tw);                \
    else {                                                                                        \
      int r_ = bf16 ? launch_p<D_, BN_, true, true>(a, st, q_perm, perm_dtype, 1, tw)                 \
                    : launch_p<D_, BN_, false, true>(a, st, q_perm, perm_dtype, 1, tw);               \
      if (r_) return r_;                                                                          \
      return bf16 ? launch_p<D_, BN_, true, false>(a, st, q_perm, perm_dtype, 2, tw)                  \
                  : launch_p<D_, BN_, false, false>(a, st, q_perm, perm_dtype, 2, tw);                \
    }                                                                                             \
  }
  BSA_TCP_CASE(64, 64)
  BSA_TCP_CASE(64, 128)
  BSA_TCP_CASE(128, 64)
  BSA_TCP_CASE(128, 128)
#undef BSA_TCP_CASE
  return BSA_ERR_UNSUPPORTED;
}

int arm_test_wait_timeout(uint32_t wait_us) {
  g_test_wait_us.store(wait_us);
  return BSA_OK;
}

}  // namespace bsa
