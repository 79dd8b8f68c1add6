// SIMT (CUDA-core) block-sparse attention forward.
//
// The fp32 path (the reference's fp32 masked softmax at 1e-5) and the
// fallback for head dims the tcgen05 kernel does not take.  One CTA per query
// block of BLOCK rows and (b, h); one thread per query row.  Only the key
// blocks listed in the plan are visited, in ascending order, with the
// reference's base-2 online softmax (triton_kernels/BlockSparse_Naive.py:
// 39-60): running max m, running sum l, accumulator rescaled by
// exp2(m_old - m_new).  For 16-bit inputs P is rounded to the input type
// before the PV product, as the reference does (p.to(dtype), :54).
#include "common.cuh"
#include "internal.h"

namespace bsa {

namespace {

constexpr int kKeyChunk = 16;

struct SimtParams {
  const void* q;
  const void* k;
  const void* v;
  void* o;
  int64_t qs[3], ks[3], vs[3], os[3];  // b, h, n strides (elements)
  float* lse;
  const int32_t* tile_ptr;
  const int32_t* tile_col;
  int32_t* err;
  int B, H, N, nb, block, T, mask_b, mask_h;
  float qk_scale;  // sm_scale * log2(e)
};

template <typename T, int D>
__global__ void attn_simt_kernel(const SimtParams p) {
  extern __shared__ float sm[];
  const int BM = p.block;
  float* sq = sm;                  // [BM][D + 1]
  float* sk = sq + BM * (D + 1);   // [kKeyChunk][D]
  float* sv = sk + kKeyChunk * D;  // [kKeyChunk][D]

  const int m = blockIdx.x;  // query block
  const int bh = blockIdx.y;
  const int b = bh / p.H, h = bh % p.H;
  const int tid = threadIdx.x;
  const int row = m * BM + tid;
  const bool row_ok = row < p.N;

  const T* qb = static_cast<const T*>(p.q) + b * p.qs[0] + h * p.qs[1];
  const T* kb = static_cast<const T*>(p.k) + b * p.ks[0] + h * p.ks[1];
  const T* vb = static_cast<const T*>(p.v) + b * p.vs[0] + h * p.vs[1];
  T* ob = static_cast<T*>(p.o) + b * p.os[0] + h * p.os[1];

  for (int idx = tid; idx < BM * D; idx += blockDim.x) {  // stage this block's Q rows
    const int r = idx / D, c = idx % D;
    const int gr = m * BM + r;
    sq[r * (D + 1) + c] = gr < p.N ? to_f32(qb[gr * p.qs[2] + c]) : 0.f;
  }

  const int s = (p.mask_b == 1 ? 0 : b) * p.mask_h + (p.mask_h == 1 ? 0 : h);
  const int tile = (m * BM) / 128;
  const int bit = BM == 64 ? (m & 1) : 0;
  const int e0 = p.tile_ptr[s * p.T + tile], e1 = p.tile_ptr[s * p.T + tile + 1];

  float acc[D];
#pragma unroll
  for (int c = 0; c < D; ++c) acc[c] = 0.f;
  float m_i = -INFINITY, l_i = 0.f;

  for (int e = e0; e < e1; ++e) {
    const uint32_t ent = static_cast<uint32_t>(p.tile_col[e]);
    if (!((ent >> (24 + bit)) & 1u)) continue;
    const int kblk = static_cast<int>(ent & 0xFFFFFFu);
    if (kblk >= p.nb) {
      if (tid == 0) set_err(p.err, BSA_DEVERR_PLAN);
      continue;
    }
    for (int c0 = 0; c0 < BM; c0 += kKeyChunk) {
      __syncthreads();
      for (int idx = tid; idx < kKeyChunk * D; idx += blockDim.x) {
        const int r = idx / D, c = idx % D;
        const int gk = kblk * BM + c0 + r;
        const bool ok = gk < p.N;
        sk[idx] = ok ? to_f32(kb[gk * p.ks[2] + c]) : 0.f;
        sv[idx] = ok ? to_f32(vb[gk * p.vs[2] + c]) : 0.f;
      }
      __syncthreads();
      float sc[kKeyChunk];
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < kKeyChunk; ++j) {
        float dot = 0.f;
#pragma unroll
        for (int c = 0; c < D; ++c) dot = fmaf(sq[tid * (D + 1) + c], sk[j * D + c], dot);
        const bool key_ok = kblk * BM + c0 + j < p.N;
        sc[j] = key_ok ? dot * p.qk_scale : -INFINITY;
        mx = fmaxf(mx, sc[j]);
      }
      const float m_new = fmaxf(m_i, mx);
      if (m_new == -INFINITY) continue;  // no valid key in this chunk
      const float alpha = exp2f(m_i - m_new);
      float lsum = 0.f;
#pragma unroll
      for (int c = 0; c < D; ++c) acc[c] *= alpha;
#pragma unroll
      for (int j = 0; j < kKeyChunk; ++j) {
        const float pj = exp2f(sc[j] - m_new);
        lsum += pj;
        const float pr = to_f32(from_f32<T>(pj));
#pragma unroll
        for (int c = 0; c < D; ++c) acc[c] = fmaf(pr, sv[j * D + c], acc[c]);
      }
      l_i = l_i * alpha + lsum;
      m_i = m_new;
    }
  }

  if (row_ok) {
    const float inv = l_i > 0.f ? 1.f / l_i : 0.f;
#pragma unroll
    for (int c = 0; c < D; ++c) ob[row * p.os[2] + c] = from_f32<T>(acc[c] * inv);
    if (p.lse) p.lse[static_cast<int64_t>(bh) * p.N + row] = l_i > 0.f ? m_i + log2f(l_i) : -INFINITY;
  }
}

template <typename T, int D>
int launch_typed(const SimtParams& p, cudaStream_t st) {
  const size_t smem = (static_cast<size_t>(p.block) * (D + 1) + 2 * kKeyChunk * D) * sizeof(float);
  auto kern = attn_simt_kernel<T, D>;
  BSA_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  dim3 grid(p.nb, p.B * p.H);
  kern<<<grid, p.block, smem, st>>>(p);
  return cudaGetLastError() == cudaSuccess ? BSA_OK : BSA_ERR_CUDA;
}

template <typename T>
int launch_d(const SimtParams& p, int D, cudaStream_t st) {
  switch (D) {
    case 16: return launch_typed<T, 16>(p, st);
    case 32: return launch_typed<T, 32>(p, st);
    case 64: return launch_typed<T, 64>(p, st);
    case 128: return launch_typed<T, 128>(p, st);
    default: return BSA_ERR_UNSUPPORTED;
  }
}

}  // namespace

int launch_attn_simt(const bsa_fwd_args* a, cudaStream_t st) {
  SimtParams p;
  p.q = a->q.data;
  p.k = a->k.data;
  p.v = a->v.data;
  p.o = a->o.data;
  const bsa_tensor4d* ts[4] = {&a->q, &a->k, &a->v, &a->o};
  int64_t* ds[4] = {p.qs, p.ks, p.vs, p.os};
  for (int i = 0; i < 4; ++i) {
    ds[i][0] = ts[i]->stride_b;
    ds[i][1] = ts[i]->stride_h;
    ds[i][2] = ts[i]->stride_n;
  }
  p.lse = a->lse;
  p.tile_ptr = a->plan.tile_ptr;
  p.tile_col = a->plan.tile_col;
  p.err = a->err_flag;
  p.B = a->B;
  p.H = a->H;
  p.N = a->N;
  p.nb = a->plan.nb;
  p.block = a->plan.block;
  p.T = tiles_per_row(a->plan.nb, a->plan.block);
  p.mask_b = a->plan.mask_b;
  p.mask_h = a->plan.mask_h;
  p.qk_scale = a->sm_scale * 1.4426950408889634f;
  switch (a->dtype) {
    case BSA_DTYPE_F32: return launch_d<float>(p, a->D, st);
    case BSA_DTYPE_F16: return launch_d<__half>(p, a->D, st);
    case BSA_DTYPE_BF16: return launch_d<__nv_bfloat16>(p, a->D, st);
    default: return BSA_ERR_DTYPE;
  }
}

}  // namespace bsa
