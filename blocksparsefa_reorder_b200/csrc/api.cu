// C ABI entry points: argument validation, kernel choice, the unfused
// "with reordering" forward and library identity.  See include/bsattn_b200.h.
#include <math.h>

#include "common.cuh"
#include "internal.h"

using namespace bsa;

namespace {

int check_device() {
  static int cached[64];  // 0 unknown, 1 ok, 2 not sm_100
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return BSA_ERR_CUDA;
  if (dev < 0 || dev >= 64) return BSA_ERR_DEVICE;
  if (!cached[dev]) {
    int major = 0, minor = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess)
      return BSA_ERR_CUDA;
    cached[dev] = (major == 10 && minor == 0) ? 1 : 2;
  }
  return cached[dev] == 1 ? BSA_OK : BSA_ERR_DEVICE;
}

bool valid_tensor(const bsa_tensor4d& t) { return t.data && t.stride_b >= 0 && t.stride_h >= 0 && t.stride_n >= 0; }

int validate_fwd(const bsa_fwd_args* a) {
  if (!a) return BSA_ERR_INVALID_ARG;
  if (a->B <= 0 || a->H <= 0 || a->N <= 0 || a->D <= 0) return BSA_ERR_INVALID_ARG;
  if (!dtype_bytes(a->dtype)) return BSA_ERR_DTYPE;
  if (!valid_tensor(a->q) || !valid_tensor(a->k) || !valid_tensor(a->v) || !valid_tensor(a->o))
    return BSA_ERR_INVALID_ARG;
  if (!a->plan.tile_ptr || !a->plan.tile_col) return BSA_ERR_INVALID_ARG;
  if (a->plan.block != 64 && a->plan.block != 128) return BSA_ERR_UNSUPPORTED;
  if (a->plan.nb != (a->N + a->plan.block - 1) / a->plan.block) return BSA_ERR_SHAPE;
  if (!(a->plan.mask_b == 1 || a->plan.mask_b == a->B)) return BSA_ERR_SHAPE;
  if (!(a->plan.mask_h == 1 || a->plan.mask_h == a->H)) return BSA_ERR_SHAPE;
  if (!(a->sm_scale > 0.f) || !isfinite(a->sm_scale)) return BSA_ERR_UNSUPPORTED;
  if (a->kernel < BSA_KERNEL_AUTO || a->kernel > BSA_KERNEL_TCGEN05) return BSA_ERR_INVALID_ARG;
  return BSA_OK;
}

// The SIMT kernel's grid has one y index per (b, h).
bool simt_supported(const bsa_fwd_args* a) {
  return (a->D == 16 || a->D == 32 || a->D == 64 || a->D == 128) && static_cast<int64_t>(a->B) * a->H <= 65535;
}

size_t round256(size_t x) { return (x + 255) & ~size_t(255); }

int launch_tc(const bsa_fwd_args* a, cudaStream_t st) { return launch_attn_tcp(a, st); }

// The fused reordered forward: the tcgen05 kernel gathers Q rows and
// scatters O / lse rows through q_perm itself; only K and V are permuted
// beforehand.
bool fused_reorder(const bsa_fwd_args* a) { return a->kernel != BSA_KERNEL_SIMT && attn_tc_supported(a); }

// Workspace layout of bsa_fwd_reordered, 256-byte aligned regions:
//   [q'] [k' v'] [o' lse'] [check] -- k', v' when kv_perm is given; q', o',
//   lse' when q_perm is and the forward is not the fused one; the bits of the
//   permutation check when an error word is given.
struct ReorderLayout {
  size_t q, k, v, o, lse, check, total;
};

ReorderLayout reorder_layout(const bsa_fwd_args* a, bool has_q, bool has_kv, bool check) {
  const size_t tensor = round256(static_cast<size_t>(a->B) * a->H * a->N * a->D * dtype_bytes(a->dtype));
  const size_t lse = round256(static_cast<size_t>(a->B) * a->H * a->N * sizeof(float));
  ReorderLayout L{};
  size_t off = 0;
  if (has_q) {
    L.q = off;
    off += tensor;
  }
  if (has_kv) {
    L.k = off;
    off += tensor;
    L.v = off;
    off += tensor;
  }
  if (has_q) {
    L.o = off;
    off += tensor;
    if (a->lse) {
      L.lse = off;
      off += lse;
    }
  }
  if (check) {
    L.check = off;
    off += round256(perm_check_bytes(a->N));
  }
  L.total = off;
  return L;
}

bsa_tensor4d contiguous(void* base, const bsa_fwd_args* a) {
  bsa_tensor4d t;
  t.data = base;
  t.stride_n = a->D;
  t.stride_h = static_cast<int64_t>(a->N) * a->D;
  t.stride_b = static_cast<int64_t>(a->H) * a->N * a->D;
  return t;
}

}  // namespace

extern "C" int bsa_abi_version(void) { return BSA_ABI_VERSION; }

extern "C" const char* bsa_status_string(int status) {
  switch (status) {
    case BSA_OK: return "ok";
    case BSA_ERR_INVALID_ARG: return "invalid argument";
    case BSA_ERR_SHAPE: return "inconsistent shapes";
    case BSA_ERR_DTYPE: return "unsupported dtype";
    case BSA_ERR_ALIGNMENT: return "pointer or stride not 16-byte aligned";
    case BSA_ERR_UNSUPPORTED: return "unsupported configuration";
    case BSA_ERR_NOT_PERMUTATION: return "not a permutation";
    case BSA_ERR_TIMEOUT: return "device wait timed out";
    case BSA_ERR_CUDA: return "CUDA runtime error";
    case BSA_ERR_WORKSPACE: return "workspace missing or too small";
    case BSA_ERR_DEVICE: return "device is not sm_100 (B200)";
    default: return "unknown status";
  }
}

extern "C" int bsa_test_arm_wait_timeout(uint32_t wait_us) {
  if (wait_us < 100 || wait_us > 2000000) return BSA_ERR_INVALID_ARG;
  return arm_test_wait_timeout(wait_us);
}

extern "C" int bsa_device_supported(int device, int* supported) {
  if (!supported) return BSA_ERR_INVALID_ARG;
  int major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device) != cudaSuccess ||
      cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device) != cudaSuccess) {
    cudaGetLastError();
    *supported = 0;
    return BSA_ERR_CUDA;
  }
  *supported = (major == 10 && minor == 0) ? 1 : 0;
  return BSA_OK;
}

extern "C" int bsa_fwd(const bsa_fwd_args* a, void* stream) {
  int rc = validate_fwd(a);
  if (rc) return rc;
  if ((rc = check_device())) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool tc_ok = attn_tc_supported(a);
  switch (a->kernel) {
    case BSA_KERNEL_TCGEN05: return tc_ok ? launch_tc(a, st) : BSA_ERR_UNSUPPORTED;
    case BSA_KERNEL_SIMT: return simt_supported(a) ? launch_attn_simt(a, st) : BSA_ERR_UNSUPPORTED;
    default:
      if (tc_ok) return launch_tc(a, st);
      return simt_supported(a) ? launch_attn_simt(a, st) : BSA_ERR_UNSUPPORTED;
  }
}

extern "C" int bsa_bwd(const bsa_bwd_args* a, void* stream) {
  if (!a) return BSA_ERR_INVALID_ARG;
  if (a->B <= 0 || a->H <= 0 || a->N <= 0 || a->D <= 0) return BSA_ERR_INVALID_ARG;
  if (a->dtype != BSA_DTYPE_F16 && a->dtype != BSA_DTYPE_BF16) return BSA_ERR_DTYPE;
  const bsa_tensor4d* ts[] = {&a->q, &a->k, &a->v, &a->o, &a->dout, &a->dq, &a->dk, &a->dv};
  for (const bsa_tensor4d* t : ts)
    if (!valid_tensor(*t)) return BSA_ERR_INVALID_ARG;
  if (!a->lse || !a->delta) return BSA_ERR_INVALID_ARG;
  if (a->D != 64 && a->D != 128) return BSA_ERR_UNSUPPORTED;
  const bsa_plan* ps[] = {&a->plan, &a->plan_t};
  for (const bsa_plan* p : ps) {
    if (!p->tile_ptr || !p->tile_col) return BSA_ERR_INVALID_ARG;
    if (p->block != 64 && p->block != 128) return BSA_ERR_UNSUPPORTED;
    if (p->block != a->plan.block) return BSA_ERR_SHAPE;
    if (p->nb != (a->N + p->block - 1) / p->block) return BSA_ERR_SHAPE;
    if (!(p->mask_b == 1 || p->mask_b == a->B) || !(p->mask_h == 1 || p->mask_h == a->H)) return BSA_ERR_SHAPE;
  }
  if (!(a->sm_scale > 0.f) || !isfinite(a->sm_scale)) return BSA_ERR_UNSUPPORTED;
  for (const bsa_tensor4d* t : ts)
    if ((reinterpret_cast<uintptr_t>(t->data) % 16) || (t->stride_n * 2) % 16 || (t->stride_h * 2) % 16 ||
        (t->stride_b * 2) % 16)
      return BSA_ERR_ALIGNMENT;
  if (reinterpret_cast<uintptr_t>(a->delta) % 16) return BSA_ERR_ALIGNMENT;
  int rc = check_device();
  if (rc) return rc;
  return launch_attn_bwd(a, static_cast<cudaStream_t>(stream));
}

extern "C" int bsa_fwd_reordered_workspace_bytes(const bsa_fwd_args* a, size_t* bytes) {
  if (!a || !bytes) return BSA_ERR_INVALID_ARG;
  const int rc = validate_fwd(a);
  if (rc) return rc;
  *bytes = reorder_layout(a, !fused_reorder(a), true, a->err_flag != nullptr).total;
  return BSA_OK;
}

extern "C" int bsa_fwd_reordered(const bsa_fwd_args* a, const void* q_perm, const void* kv_perm, int32_t perm_dtype,
                                 void* workspace, size_t workspace_bytes, void* stream) {
  int rc = validate_fwd(a);
  if (rc) return rc;
  if ((q_perm || kv_perm) && perm_dtype != BSA_INDEX_I32 && perm_dtype != BSA_INDEX_I64) return BSA_ERR_DTYPE;
  const bool fused = fused_reorder(a);
  const bool check = a->err_flag && (q_perm || kv_perm);
  const ReorderLayout L = reorder_layout(a, !fused && q_perm != nullptr, kv_perm != nullptr, check);
  if (L.total && (!workspace || workspace_bytes < L.total)) return BSA_ERR_WORKSPACE;
  if ((rc = check_device())) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const int eb = dtype_bytes(a->dtype);
  bsa_fwd_args inner = *a;
  // With an error word, both permutations are checked first (range and
  // repeated values): a repeated q_perm value would make two rows write one
  // output row, which neither the fused gather / scatter nor the row-copy
  // kernels can see.
  if (check) {
    if (q_perm && (rc = launch_perm_check(q_perm, perm_dtype, a->N, ws + L.check, a->err_flag, st))) return rc;
    if (kv_perm && kv_perm != q_perm &&
        (rc = launch_perm_check(kv_perm, perm_dtype, a->N, ws + L.check, a->err_flag, st)))
      return rc;
  }
  if (fused) {
    if (kv_perm) {
      inner.k = contiguous(ws + L.k, a);
      inner.v = contiguous(ws + L.v, a);
      if ((rc = launch_permute_rows(inner.k, a->k, a->B, a->H, a->N, a->D, eb, kv_perm, perm_dtype, 0, a->err_flag,
                                    st)))
        return rc;
      if ((rc = launch_permute_rows(inner.v, a->v, a->B, a->H, a->N, a->D, eb, kv_perm, perm_dtype, 0, a->err_flag,
                                    st)))
        return rc;
    }
    return launch_attn_tcp(&inner, st, q_perm, perm_dtype);
  }
  if (q_perm) {
    inner.q = contiguous(ws + L.q, a);
    if ((rc = launch_permute_rows(inner.q, a->q, a->B, a->H, a->N, a->D, eb, q_perm, perm_dtype, 0, a->err_flag, st)))
      return rc;
    inner.o = contiguous(ws + L.o, a);
    if (a->lse) inner.lse = reinterpret_cast<float*>(ws + L.lse);
  }
  if (kv_perm) {
    inner.k = contiguous(ws + L.k, a);
    inner.v = contiguous(ws + L.v, a);
    if ((rc = launch_permute_rows(inner.k, a->k, a->B, a->H, a->N, a->D, eb, kv_perm, perm_dtype, 0, a->err_flag,
                                  st)))
      return rc;
    if ((rc = launch_permute_rows(inner.v, a->v, a->B, a->H, a->N, a->D, eb, kv_perm, perm_dtype, 0, a->err_flag,
                                  st)))
      return rc;
  }
  if ((rc = bsa_fwd(&inner, stream))) return rc;
  if (q_perm) {
    if ((rc = launch_permute_rows(a->o, inner.o, a->B, a->H, a->N, a->D, eb, q_perm, perm_dtype, 1, a->err_flag, st)))
      return rc;
    if (a->lse) {
      // lse is a contiguous [B, H, N] fp32 array: rows of one element.
      bsa_tensor4d dst{a->lse, static_cast<int64_t>(a->H) * a->N, a->N, 1};
      bsa_tensor4d src{inner.lse, static_cast<int64_t>(a->H) * a->N, a->N, 1};
      if ((rc = launch_permute_rows(dst, src, a->B, a->H, a->N, 1, 4, q_perm, perm_dtype, 1, a->err_flag, st)))
        return rc;
    }
  }
  return BSA_OK;
}
