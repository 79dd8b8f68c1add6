// Online softmax of one kept key block for one query row (one thread per
// row), shared by the tcgen05 attention kernels.
//
// The reference kernel (triton_kernels/BlockSparse_Naive.py:39-60) keeps the
// exact running row max m and, per block, computes p = 2^(s*scale - m), a
// correction 2^(m_old - m) for O and l, and l += sum(p).  The result
// O = sum(p v) / sum(p) does not depend on which reference point m is used,
// only that 2^(s*scale - m) stays finite: P is rounded to bf16 / fp16 relative
// to its own magnitude and O, l accumulate in fp32, both with 8-bit exponents.
// So here m_run is the exact max of the row's FIRST kept block only; later
// blocks reuse it, and only when a block's sum exceeds kRefSlack (a score more
// than ~32 above m_run in log2 units, or an overflow) is the block redone with
// the exact max and O, l scaled by 2^(m_old - m_new).  lse = m_run + log2(l)
// is exact either way.  This removes the per-block max (a 128-deep fmax
// chain) from the common path.
#pragma once

#include "common.cuh"

namespace bsa {

constexpr float kRefSlack = 4294967296.f;  // 2^32

// Max of a row's BN scores (fp32 bits), as a tree of 8 independent chains.
template <int BN>
__device__ __forceinline__ float row_max(const uint32_t (&sr)[BN]) {
  float m[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) m[k] = __uint_as_float(sr[k]);
#pragma unroll
  for (int i = 8; i < BN; i += 8) {
#pragma unroll
    for (int k = 0; k < 8; ++k) m[k] = fmaxf(m[k], __uint_as_float(sr[i + k]));
  }
  return fmaxf(fmaxf(fmaxf(m[0], m[1]), fmaxf(m[2], m[3])), fmaxf(fmaxf(m[4], m[5]), fmaxf(m[6], m[7])));
}

// p = 2^(s * scale - m) packed in pairs into pr; returns sum(p) (four
// independent partial sums).
template <int BN, bool BF16>
__device__ __forceinline__ float exp_block(const uint32_t (&sr)[BN], uint32_t (&pr)[BN / 2], float scale_log2,
                                           float neg_m) {
  float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
  for (int i = 0; i < BN / 2; i += 2) {
    const float p0 = ex2_approx(fmaf(__uint_as_float(sr[2 * i]), scale_log2, neg_m));
    const float p1 = ex2_approx(fmaf(__uint_as_float(sr[2 * i + 1]), scale_log2, neg_m));
    const float p2 = ex2_approx(fmaf(__uint_as_float(sr[2 * i + 2]), scale_log2, neg_m));
    const float p3 = ex2_approx(fmaf(__uint_as_float(sr[2 * i + 3]), scale_log2, neg_m));
    a0 += p0;
    a1 += p1;
    a2 += p2;
    a3 += p3;
    pr[i] = pack2<BF16>(p0, p1);
    pr[i + 1] = pack2<BF16>(p2, p3);
  }
  return (a0 + a1) + (a2 + a3);
}

// One block of the row's online softmax.  sr: raw scores (keys past the end
// already set to -inf); m_run = -inf before the row's first kept block.
// Writes P to pr, updates m_run / l_run and returns the factor by which the
// caller must scale the row of O accumulated so far (1 when unchanged).
template <int BN, bool BF16>
__device__ __forceinline__ float softmax_block(const uint32_t (&sr)[BN], uint32_t (&pr)[BN / 2], float scale_log2,
                                               float& m_run, float& l_run) {
  if (m_run == -INFINITY) m_run = row_max<BN>(sr) * scale_log2;
  float ls = exp_block<BN, BF16>(sr, pr, scale_log2, -m_run);
  float alpha = 1.f;
  if (!(ls <= kRefSlack)) {
    const float m_new = fmaxf(m_run, row_max<BN>(sr) * scale_log2);
    alpha = ex2_approx(m_run - m_new);
    l_run *= alpha;
    m_run = m_new;
    ls = exp_block<BN, BF16>(sr, pr, scale_log2, -m_run);
  }
  l_run += ls;
  return alpha;
}

}  // namespace bsa
