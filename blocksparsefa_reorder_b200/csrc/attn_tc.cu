// tcgen05 block-sparse attention forward for sm_100a.
//
// Replaces the reference kernel _attn_fwd_block_sparse
// (triton_kernels/BlockSparse_Naive.py:68-125).  The reference scans every
// mask byte of its query block and branches; here each CTA owns one tile of
// 128 query rows of one (b, h) and walks only the kept key blocks listed in
// the plan (bsa_build_plan), so masked blocks cost nothing.
//
// Roles (192 threads):
//   warp 0      TMA producer: Q once, then K_j and V_j of each kept key block
//               into a STAGES-deep shared-memory ring (128-byte swizzle).
//   warp 1      TMEM allocator; one thread issues every tcgen05.mma:
//                 S_j = Q K_j^T   (A, B from shared memory) -> TMEM S[j % 2]
//                 O  += P_j V_j   (A = P from TMEM, B = V from shared memory)
//   warps 2..5  softmax warpgroup, one query row per thread (TMEM lane):
//               tcgen05.ld S_j, base-2 online softmax, P_j -> TMEM as 16-bit,
//               lazy rescale of O in TMEM, epilogue O / l -> smem -> TMA store.
//
// Pipeline: S is double-buffered, so S_{j+1} is computed on the tensor cores
// while the softmax warps work on S_j and PV_{j-1} drains.  The running max
// is only moved (and O rescaled) when it grows by more than 2^8, keeping the
// rescale off the common path; P <= 2^8 stays exact enough in 16 bits and the
// fp32 accumulators.  Results equal the reference's online softmax
// (BlockSparse_Naive.py:39-60, 119-125): rows with no kept block give O = 0
// and lse = -inf.
//
// Barrier phases.  Every parity wait below is on a barrier that can be at
// most one phase ahead of or behind the phase waited for, which the
// issue order guarantees: the MMA thread issues S_j, then PV_{j-1}; a
// tcgen05.commit arrives when all earlier MMAs of the thread are complete, so
// "S_j complete" implies "PV_{j-2} complete".  The epilogue uses its own
// single-phase barrier (o_final) because pv_done may lag two phases there.
//
// Every mbarrier wait is bounded (common.cuh: mbar_wait); a timeout sets
// BSA_DEVERR_TIMEOUT in the error word and the CTA drains and exits.
#include <cudaTypedefs.h>

#include "common.cuh"
#include "internal.h"
#include "softmax.cuh"

namespace bsa {

namespace {

struct TcParams {
  const int32_t* tile_ptr;
  const int32_t* tile_col;
  float* lse;
  int32_t* err;
  int H, N, nb, T, mask_b, mask_h;
  float scale_log2;
};

constexpr int kSmemLimit = 232448;  // 227 KB opt-in dynamic shared memory per block

template <int D, int BN>
struct TcCfg {
  static constexpr int BM = 128;
  static constexpr int NCHUNK = D / 64;      // 64-element (128-byte) column chunks
  static constexpr int Q_CHUNK = BM * 128;   // bytes of one Q column chunk
  static constexpr int KV_CHUNK = BN * 128;  // bytes of one K / V column chunk
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_BYTES = BN * D * 2;
  static constexpr int BAR_BYTES = 256;
  static constexpr int fit_stages() {
    int s = 4;
    while (s > 1 && 1024 + Q_BYTES + 2 * s * KV_BYTES + BAR_BYTES > kSmemLimit) --s;
    return s;
  }
  static constexpr int STAGES = fit_stages();
  static constexpr int SMEM = 1024 + Q_BYTES + 2 * STAGES * KV_BYTES + BAR_BYTES;
  // TMEM columns (32-bit each, 128 lanes)
  static constexpr int S_COL0 = 0;
  static constexpr int S_COL1 = BN;
  static constexpr int O_COL = 2 * BN;
  static constexpr int P_COL0 = 2 * BN + D;
  static constexpr int P_COL1 = 2 * BN + D + BN / 2;
  static constexpr int USED_COLS = 2 * BN + D + BN;
  static constexpr int TMEM_COLS = USED_COLS <= 256 ? 256 : 512;
  static_assert(USED_COLS <= 512, "TMEM budget");
  static_assert(D % 64 == 0 && (BN == 64 || BN == 128), "tile shape");
  static_assert(STAGES >= 2, "K_{j+1} must load while V_j is still in use");
  static_assert((1 + 3 * STAGES + 7) * 8 + 8 <= BAR_BYTES, "barrier area");
};

template <int D, int BN, bool BF16>
__global__ void __launch_bounds__(192, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmO,
                   const TcParams p) {
  using C = TcCfg<D, BN>;
  constexpr int STAGES = C::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + C::Q_BYTES;
  uint8_t* sV = sK + STAGES * C::KV_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + STAGES * C::KV_BYTES);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = k_full + STAGES;
  uint64_t* kv_empty = v_full + STAGES;
  uint64_t* s_full = kv_empty + STAGES;  // [2]
  uint64_t* p_ready = s_full + 2;        // [2]
  uint64_t* pv_done = p_ready + 2;       // one phase per PV_j (rescale waits: PV_{j-1})
  uint64_t* o_final = pv_done + 1;       // one phase: the last PV of the tile completed
  uint64_t* drain = o_final + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x;
  const int bh = blockIdx.y;
  const int b = bh / p.H, h = bh % p.H;
  const int s = (p.mask_b == 1 ? 0 : b) * p.mask_h + (p.mask_h == 1 ? 0 : h);
  const int e0 = p.tile_ptr[s * p.T + t];
  const int n = p.tile_ptr[s * p.T + t + 1] - e0;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_ready[i], 4);
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

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && n > 0) {
      tma_prefetch_desc(&tmQ);
      tma_prefetch_desc(&tmK);
      tma_prefetch_desc(&tmV);
      mbar_arrive_expect_tx(q_full, C::Q_BYTES);
      for (int c = 0; c < C::NCHUNK; ++c) tma_load_4d(sQ + c * C::Q_CHUNK, &tmQ, q_full, c * 64, t * 128, h, b);
      int issued = 0;
      for (int j = 0; j < n; ++j) {
        const int st = j % STAGES;
        if (j >= STAGES && !mbar_wait(&kv_empty[st], ((j / STAGES) - 1) & 1, abort_flag, p.err)) break;
        int kb = static_cast<int>(static_cast<uint32_t>(p.tile_col[e0 + j]) & 0xFFFFFFu);
        if (kb >= p.nb) {
          set_err(p.err, BSA_DEVERR_PLAN);
          kb = 0;
        }
        mbar_arrive_expect_tx(&k_full[st], C::KV_BYTES);
        for (int c = 0; c < C::NCHUNK; ++c)
          tma_load_4d(sK + st * C::KV_BYTES + c * C::KV_CHUNK, &tmK, &k_full[st], c * 64, kb * BN, h, b);
        mbar_arrive_expect_tx(&v_full[st], C::KV_BYTES);
        for (int c = 0; c < C::NCHUNK; ++c)
          tma_load_4d(sV + st * C::KV_BYTES + c * C::KV_CHUNK, &tmV, &v_full[st], c * 64, kb * BN, h, b);
        issued = j + 1;
      }
      if (*abort_flag) {
        // Let the loads still in flight land before the CTA's shared memory goes away.
        for (int j = issued > STAGES ? issued - STAGES : 0; j < issued; ++j) {
          mbar_wait(&k_full[j % STAGES], (j / STAGES) & 1, nullptr, nullptr);
          mbar_wait(&v_full[j % STAGES], (j / STAGES) & 1, nullptr, nullptr);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && n > 0) {
      constexpr uint32_t idesc_qk = make_idesc_f16(BF16, 128, BN, false, false);
      constexpr uint32_t idesc_pv = make_idesc_f16(BF16, 128, D, false, true);
      const uint32_t q_addr = smem_u32(sQ);
      const uint32_t k_addr = smem_u32(sK);
      const uint32_t v_addr = smem_u32(sV);
      bool ok = mbar_wait(q_full, 0, abort_flag, p.err);
      tc_fence_after();
      for (int j = 0; ok && j <= n; ++j) {
        if (j < n) {
          const int st = j % STAGES;
          if (!(ok = mbar_wait(&k_full[st], (j / STAGES) & 1, abort_flag, p.err))) break;
          tc_fence_after();
          const uint32_t d_tmem = tmem + ((j & 1) ? C::S_COL1 : C::S_COL0);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk & 3) * 32;  // 16 elements = 32 bytes inside the 128-byte swizzle row
            const uint64_t a = make_sw128_desc(q_addr + (kk >> 2) * C::Q_CHUNK + off, 16, 1024);
            const uint64_t bd = make_sw128_desc(k_addr + st * C::KV_BYTES + (kk >> 2) * C::KV_CHUNK + off, 16, 1024);
            tc_mma_ss(d_tmem, a, bd, idesc_qk, kk > 0 ? 1u : 0u);
          }
          tc_commit(&s_full[j & 1]);
        }
        if (j >= 1) {
          const int i = j - 1;
          const int st = i % STAGES;
          if (!(ok = mbar_wait(&p_ready[i & 1], (i >> 1) & 1, abort_flag, p.err))) break;
          if (!(ok = mbar_wait(&v_full[st], (i / STAGES) & 1, abort_flag, p.err))) break;
          tc_fence_after();
          const uint32_t p_tmem = tmem + ((i & 1) ? C::P_COL1 : C::P_COL0);
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {
            // V tile is [BN keys][D] (D contiguous): an MN-major B operand.
            // 16 keys per MMA = 16 rows of 128 bytes; D chunks LBO apart.
            const uint64_t bd = make_sw128_desc(v_addr + st * C::KV_BYTES + kk * 16 * 128, C::KV_CHUNK, 1024);
            tc_mma_ts(tmem + C::O_COL, p_tmem + kk * 8, bd, idesc_pv, (i > 0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(&kv_empty[st]);
          tc_commit(pv_done);
          if (i == n - 1) tc_commit(o_final);
        }
      }
      // Every MMA issued above completes before TMEM is released.
      tc_commit(drain);
      mbar_wait(drain, 0, nullptr, nullptr);
    }
  } else {
    // ------------------------------------------------------------ softmax warpgroup
    const int q4 = warp & 3;  // TMEM lane quarter this warp may access
    const int row = q4 * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q4 * 32) << 16);
    const int half = row >> 6;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      const int sb = j & 1;
      // Keep every decision warp-uniform: the tcgen05.ld / st below are .sync.aligned.
      if (!(ok = __all_sync(0xffffffffu, mbar_wait(&s_full[sb], (j >> 1) & 1, abort_flag, p.err)))) break;
      tc_fence_after();
      uint32_t sr[BN];
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) tmem_ld32(lane_base + (sb ? C::S_COL1 : C::S_COL0) + c * 32, &sr[c * 32]);
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
          // O holds the sum up to block j-1: wait for PV_{j-1}, rescale in TMEM.
          if (!(ok = __all_sync(0xffffffffu, mbar_wait(pv_done, (j - 1) & 1, abort_flag, p.err)))) break;
          tc_fence_after();
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            uint32_t o[32];
            tmem_ld32(lane_base + C::O_COL + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st32(lane_base + C::O_COL + c * 32, o);
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < BN / 2; ++i) pr[i] = 0u;
      }
      const uint32_t p_col = sb ? C::P_COL1 : C::P_COL0;
#pragma unroll
      for (int c = 0; c < BN / 64; ++c) tmem_st32(lane_base + p_col + c * 32, &pr[c * 32]);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_ready[sb]);
    }

    // ------------------------------------------------------------ epilogue
    if (ok && n > 0) ok = __all_sync(0xffffffffu, mbar_wait(o_final, 0, abort_flag, p.err));
    if (ok) {
      tc_fence_after();
      const float inv_l = l_run > 0.f ? 1.f / l_run : 0.f;
      uint8_t* orow = sQ + row * 128;  // Q's shared memory is free once the last MMA completed
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        if (n > 0) {
          tmem_ld32(lane_base + C::O_COL + c * 32, o);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = 0u;
        }
        uint8_t* chunk_row = orow + (c >> 1) * C::Q_CHUNK;
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          uint4 v;
          v.x = pack2<BF16>(__uint_as_float(o[8 * g + 0]) * inv_l, __uint_as_float(o[8 * g + 1]) * inv_l);
          v.y = pack2<BF16>(__uint_as_float(o[8 * g + 2]) * inv_l, __uint_as_float(o[8 * g + 3]) * inv_l);
          v.z = pack2<BF16>(__uint_as_float(o[8 * g + 4]) * inv_l, __uint_as_float(o[8 * g + 5]) * inv_l);
          v.w = pack2<BF16>(__uint_as_float(o[8 * g + 6]) * inv_l, __uint_as_float(o[8 * g + 7]) * inv_l);
          const int gran = ((c & 1) * 4 + g) ^ (row & 7);  // 128-byte swizzle
          *reinterpret_cast<uint4*>(chunk_row + gran * 16) = v;
        }
      }
      fence_proxy_async_smem();
      const int grow = t * 128 + row;
      if (p.lse && grow < p.N)
        p.lse[static_cast<int64_t>(bh) * p.N + grow] = l_run > 0.f ? m_run + log2f(l_run) : -INFINITY;
    }
    named_bar_sync(1, 128);
    if (warp == 2 && lane == 0 && !*abort_flag) {
      for (int c = 0; c < C::NCHUNK; ++c) tma_store_4d(&tmO, sQ + c * C::Q_CHUNK, c * 64, t * 128, h, b);
      tma_store_commit();
      tma_store_wait0();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
template <int D, int BN, bool BF16>
int launch_cfg(const bsa_fwd_args* a, cudaStream_t st) {
  using C = TcCfg<D, BN>;
  CUtensorMap mq, mk, mv, mo;
  int r;
  if ((r = make_tensor_map_4d(&mq, a->q, a->B, a->H, a->N, D, BF16, 128))) return r;
  if ((r = make_tensor_map_4d(&mk, a->k, a->B, a->H, a->N, D, BF16, BN))) return r;
  if ((r = make_tensor_map_4d(&mv, a->v, a->B, a->H, a->N, D, BF16, BN))) return r;
  if ((r = make_tensor_map_4d(&mo, a->o, a->B, a->H, a->N, D, BF16, 128))) return r;
  TcParams p;
  p.tile_ptr = a->plan.tile_ptr;
  p.tile_col = a->plan.tile_col;
  p.lse = a->lse;
  p.err = a->err_flag;
  p.H = a->H;
  p.N = a->N;
  p.nb = a->plan.nb;
  p.T = tiles_per_row(a->plan.nb, a->plan.block);
  p.mask_b = a->plan.mask_b;
  p.mask_h = a->plan.mask_h;
  p.scale_log2 = a->sm_scale * 1.4426950408889634f;
  auto kern = attn_tc_kernel<D, BN, BF16>;
  BSA_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
  dim3 grid(p.T, a->B * a->H);
  kern<<<grid, 192, C::SMEM, st>>>(mq, mk, mv, mo, p);
  return cudaGetLastError() == cudaSuccess ? BSA_OK : BSA_ERR_CUDA;
}

bool aligned16(const bsa_tensor4d& t) {
  return (reinterpret_cast<uintptr_t>(t.data) % 16) == 0 && (t.stride_n * 2) % 16 == 0 &&
         (t.stride_h * 2) % 16 == 0 && (t.stride_b * 2) % 16 == 0;
}

}  // namespace

namespace {
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

// 4-D map over [B, H, N, D] (TMA order: D, N, H, B), box = 64 x rows, 128B swizzle.
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

int launch_attn_tc(const bsa_fwd_args* a, cudaStream_t st) {
  const bool bf16 = a->dtype == BSA_DTYPE_BF16;
  const int bn = a->plan.block;
#define BSA_TC_CASE(D_, BN_) \
  if (a->D == D_ && bn == BN_) return bf16 ? launch_cfg<D_, BN_, true>(a, st) : launch_cfg<D_, BN_, false>(a, st);
  BSA_TC_CASE(64, 64)
  BSA_TC_CASE(64, 128)
  BSA_TC_CASE(128, 64)
  BSA_TC_CASE(128, 128)
#undef BSA_TC_CASE
  return BSA_ERR_UNSUPPORTED;
}

}  // namespace bsa
