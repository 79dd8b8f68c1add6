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
// blocks reuse it, and only when a block's sum exceeds the slack is the block
// redone with the exact max and O, l scaled by 2^(m_old - m_new).  The slack
// bounds every single p as well: 2^32 for bf16 (8-bit exponent, like fp32);
// 2^15 for fp16, whose largest finite value is 65504, so no p of a kept
// block rounds to infinity.  lse = m_run + log2(l) is exact either way.  This
// removes the per-block max (a 128-deep fmax chain) from the common path.
#pragma once

#include "common.cuh"

namespace bsa {

template <bool BF16>
__host__ __device__ constexpr float ref_slack() {
  return BF16 ? 4294967296.f /* 2^32 */ : 32768.f /* 2^15 */;
}

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

// Two fp32 lanes in one 64-bit register, for the paired FP32 instructions of
// sm_100 (fma.rn.f32x2, add.rn.f32x2): one instruction issue per two values.
__device__ __forceinline__ uint64_t f32x2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f32x2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f32x2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t f32x2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// p = 2^(s * scale - m) packed in pairs into pr; returns sum(p) (four
// independent partial sums, two paired accumulators).
template <int BN, bool BF16>
__device__ __forceinline__ float exp_block(const uint32_t (&sr)[BN], uint32_t (&pr)[BN / 2], float scale_log2,
                                           float neg_m) {
  const uint64_t sc2 = f32x2_pack(scale_log2, scale_log2);
  const uint64_t nm2 = f32x2_pack(neg_m, neg_m);
  uint64_t a01 = f32x2_pack(0.f, 0.f), a23 = a01;
#pragma unroll
  for (int i = 0; i < BN / 2; i += 2) {
    const uint64_t x01 = f32x2_fma(f32x2_pack(__uint_as_float(sr[2 * i]), __uint_as_float(sr[2 * i + 1])), sc2, nm2);
    const uint64_t x23 =
        f32x2_fma(f32x2_pack(__uint_as_float(sr[2 * i + 2]), __uint_as_float(sr[2 * i + 3])), sc2, nm2);
    float x0, x1, x2, x3;
    f32x2_unpack(x01, x0, x1);
    f32x2_unpack(x23, x2, x3);
    const float p0 = ex2_approx(x0), p1 = ex2_approx(x1), p2 = ex2_approx(x2), p3 = ex2_approx(x3);
    a01 = f32x2_add(a01, f32x2_pack(p0, p1));
    a23 = f32x2_add(a23, f32x2_pack(p2, p3));
    pr[i] = pack2<BF16>(p0, p1);
    pr[i + 1] = pack2<BF16>(p2, p3);
  }
  float s0, s1, s2, s3;
  f32x2_unpack(a01, s0, s1);
  f32x2_unpack(a23, s2, s3);
  return (s0 + s2) + (s1 + s3);
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
  if (!(ls <= ref_slack<BF16>())) {
    const float m_new = fmaxf(m_run, row_max<BN>(sr) * scale_log2);
    alpha = ex2_approx(m_run - m_new);
    l_run *= alpha;
    m_run = m_new;
    ls = exp_block<BN, BF16>(sr, pr, scale_log2, -m_run);
  }
  l_run += ls;
  return alpha;
}

// The same for a row whose scores are split between two threads of a warp
// (lanes i and i ^ 16, BN scores each): the row max and the block sum are
// combined with one shuffle, so both threads take the same decisions and keep
// the same m_run / l_run.  Every thread of the warp calls it: the first-block
// max and the redo run warp-wide when any row of the warp needs them (a row
// redone without need gets the same reference point or a larger one, and
// alpha rescales its O and l either way).
// `active` false: none of this thread's scores is kept (at BLOCK 64, an
// entry the row's query block does not keep): its P is exactly 0 (the
// exponent's reference is -inf) and its scores take no part in the max,
// without masking each score.
template <int BN, bool BF16>
__device__ __forceinline__ float softmax_block_split(const uint32_t (&sr)[BN], uint32_t (&pr)[BN / 2],
                                                     float scale_log2, float& m_run, float& l_run,
                                                     bool active = true) {
  if (__any_sync(0xffffffffu, m_run == -INFINITY)) {
    float mx = active ? row_max<BN>(sr) : -INFINITY;
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
    if (m_run == -INFINITY) m_run = mx * scale_log2;
  }
  float ls = exp_block<BN, BF16>(sr, pr, scale_log2, active ? -m_run : -INFINITY);
  ls += __shfl_xor_sync(0xffffffffu, ls, 16);
  float alpha = 1.f;
  if (__any_sync(0xffffffffu, !(ls <= ref_slack<BF16>()))) {
    float mx = active ? row_max<BN>(sr) : -INFINITY;
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
    const float m_new = fmaxf(m_run, mx * scale_log2);
    alpha = ex2_approx(m_run - m_new);
    l_run *= alpha;
    m_run = m_new;
    ls = exp_block<BN, BF16>(sr, pr, scale_log2, active ? -m_run : -INFINITY);
    ls += __shfl_xor_sync(0xffffffffu, ls, 16);
  }
  l_run += ls;
  return alpha;
}

}  // namespace bsa
