// C ABI entry points (include/linearard_b200.h): argument validation that
// mirrors the assertions of LinearARD's wrappers (kernel_A.py:190-227,
// kernel_B.py:262-331, kernel_C.py:306-375), scratch layout, and dispatch to
// the sm_100a tensor-core kernels or the generic CUDA-core kernels.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <algorithm>
#include <atomic>
#include <vector>

#include "lkl_common.cuh"

namespace {

using lkl::Problem;

thread_local int32_t t_last_path = -1;
thread_local int32_t t_last_cuda_error = 0;
std::atomic<int32_t> g_force_generic{0};

inline bool head_dim_ok(int d) {
  return d == 8 || d == 16 || d == 32 || d == 64 || d == 128 || d == 256;
}

inline size_t round256(size_t x) { return (x + 255) & ~size_t(255); }

inline size_t bits_bytes(const lkl_problem* p) {
  return round256((size_t)p->B * (size_t)((p->T + 31) / 32) * sizeof(uint32_t));
}

inline size_t lsc_bytes(const lkl_problem* p) {
  return round256((size_t)p->B * p->Hq * p->T * 2 * sizeof(float));
}

Problem to_problem(const lkl_problem* p);

inline int max_partials(const Problem& q) {
  const int a = lkl::generic_num_partials(q), b = lkl::sm100_num_partials(q);
  return a > b ? a : b;
}

Problem to_problem(const lkl_problem* p) {
  Problem q;
  q.B = p->B;
  q.Hq = p->Hq;
  q.Hkv_s = p->Hkv_s;
  q.Hkv_t = p->Hkv_t;
  q.T = p->T;
  q.Ds = p->Ds;
  q.Dt = p->Dt;
  q.dtype_s = p->dtype_s;
  q.dtype_t = p->dtype_t;
  q.causal = p->causal ? 1 : 0;
  q.sc_s = p->sm_scale_s > 0.f ? p->sm_scale_s : 1.0f / sqrtf((float)p->Ds);
  q.sc_t = p->sm_scale_t > 0.f ? p->sm_scale_t : 1.0f / sqrtf((float)p->Dt);
  return q;
}

// Shape / dtype checks shared by every entry point.  `teacher` = the teacher
// pair (Hkv_t, Dt, dtype_t) is also used.
int32_t check_problem(const lkl_problem* p, bool teacher) {
  if (!p) return LKL_ERR_NULL_POINTER;
  if (p->B < 0 || p->T < 0 || p->Hq <= 0 || p->Hkv_s <= 0) return LKL_ERR_BAD_SHAPE;
  if (p->Hq % p->Hkv_s != 0) return LKL_ERR_BAD_SHAPE;
  if (!head_dim_ok(p->Ds)) return LKL_ERR_BAD_HEAD_DIM;
  if (p->dtype_s != LKL_F16 && p->dtype_s != LKL_BF16) return LKL_ERR_BAD_DTYPE;
  if (teacher) {
    if (p->Hkv_t <= 0 || p->Hq % p->Hkv_t != 0) return LKL_ERR_BAD_SHAPE;
    if (!head_dim_ok(p->Dt)) return LKL_ERR_BAD_HEAD_DIM;
    if (p->dtype_t != LKL_F16 && p->dtype_t != LKL_BF16) return LKL_ERR_BAD_DTYPE;
  }
  if (p->mask_dtype < LKL_MASK_BOOL || p->mask_dtype > LKL_MASK_I64) return LKL_ERR_BAD_DTYPE;
  // grid / index limits
  const long long rows = (long long)p->B * p->Hq * (((long long)p->T + 31) / 32);
  if (rows > (1ll << 31) - 1) return LKL_ERR_TOO_LARGE;
  return LKL_OK;
}

inline bool aligned(const void* ptr, size_t a) { return (reinterpret_cast<uintptr_t>(ptr) % a) == 0; }

int32_t check_mask(const void* mask, int mdt) {
  if (!mask) return LKL_OK;
  const size_t es = mdt == LKL_MASK_I64 ? 8 : (mdt == LKL_MASK_I32 ? 4 : 1);
  return aligned(mask, es) ? LKL_OK : LKL_ERR_MISALIGNED;
}

// `need` is lkl_forward_workspace_size for the forward entry points and
// lkl_workspace_size (which adds the backward's per-row offsets) for lkl_backward.
int32_t check_workspace(size_t need, void* ws, size_t ws_bytes) {
  if (need == 0) return LKL_OK;
  if (!ws || ws_bytes < need || !aligned(ws, 256)) return LKL_ERR_WORKSPACE;
  return LKL_OK;
}

// Makes the device that owns `ptr` current on this host thread (which also
// makes its primary context current: callers such as PyTorch's autograd
// worker threads may enter without one, and the TMA descriptor encoder needs
// it).  Returns false if `ptr` is not device memory.
bool bind_device_of(const void* ptr) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, ptr) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  if (a.type != cudaMemoryTypeDevice && a.type != cudaMemoryTypeManaged) return false;
  return cudaSetDevice(a.device) == cudaSuccess;
}

bool device_is_sm100() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  int major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
    return false;
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  return major == 10 && minor == 0;
}

bool use_tensor_cores(const Problem& q, const void* a, const void* b, const void* c,
                      const void* d) {
  if (g_force_generic.load()) return false;
  if (!(aligned(a, 16) && aligned(b, 16) && aligned(c, 16) && aligned(d, 16))) return false;
  return lkl::sm100_supports(q);
}

inline int32_t launch_status(cudaError_t e) {
  if (e != cudaSuccess) t_last_cuda_error = (int32_t)e;
  return e == cudaSuccess ? LKL_OK : LKL_ERR_LAUNCH;
}

// Packs the mask (if any) into the workspace; returns the bits pointer via *bits.
int32_t prepare_mask(const lkl_problem* p, const void* mask, void* ws, uint32_t** bits,
                     cudaStream_t st) {
  *bits = nullptr;
  if (!mask || p->B == 0 || p->T == 0) return LKL_OK;
  *bits = static_cast<uint32_t*>(ws);
  return launch_status(lkl::launch_pack_mask(mask, p->mask_dtype, p->B, p->T, *bits, st));
}

inline float* partials_ptr(const lkl_problem* p, const void* mask, void* ws) {
  return reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + (mask ? bits_bytes(p) : 0));
}

// Backward scratch: per-row exponent offsets (float2) after the bits and partials.
inline float2* lsc_ptr(const lkl_problem* p, const void* mask, void* ws) {
  const size_t off = (mask ? bits_bytes(p) : 0) +
                     round256((size_t)max_partials(to_problem(p)) * sizeof(float));
  return reinterpret_cast<float2*>(static_cast<uint8_t*>(ws) + off);
}

}  // namespace

extern "C" {

int32_t lkl_abi_version(void) { return LKL_ABI_VERSION; }

const char* lkl_status_string(int32_t s) {
  switch (s) {
    case LKL_OK: return "ok";
    case LKL_ERR_NULL_POINTER: return "a required pointer is NULL";
    case LKL_ERR_BAD_SHAPE: return "bad shape (B/T/H mismatch or Hq not divisible by Hkv)";
    case LKL_ERR_BAD_HEAD_DIM: return "head dim is not in the supported set {8,16,32,64,128,256}";
    case LKL_ERR_BAD_DTYPE: return "unsupported dtype";
    case LKL_ERR_MISALIGNED: return "pointer not aligned to its element size";
    case LKL_ERR_WORKSPACE: return "workspace missing, misaligned or too small";
    case LKL_ERR_LAUNCH: return "CUDA kernel launch failed";
    case LKL_ERR_NO_DEVICE: return "no sm_100 CUDA device is current";
    case LKL_ERR_DEVICE_TIMEOUT: return "a device-side bounded wait expired";
    case LKL_ERR_BAD_ALIAS: return "dq == dk requires qs == ks and Hkv_s == Hq";
    case LKL_ERR_TOO_LARGE: return "problem exceeds the supported size";
    case LKL_ERR_UNSUPPORTED:
      return "strided or grouped inputs need the tensor-core path (sm_100, Ds and Dt in "
             "{8, 16, 32, 64, 128}, 16-byte aligned)";
    default: return "unknown status";
  }
}

size_t lkl_forward_workspace_size(const lkl_problem* p, int32_t has_mask) {
  if (!p || p->B <= 0 || p->T <= 0 || p->Hq <= 0) return 0;
  const Problem q = to_problem(p);
  size_t n = round256((size_t)max_partials(q) * sizeof(float));
  if (has_mask) n += bits_bytes(p);
  return n;
}

size_t lkl_workspace_size(const lkl_problem* p, int32_t has_mask) {
  const size_t n = lkl_forward_workspace_size(p, has_mask);
  return n == 0 ? 0 : n + lsc_bytes(p);
}

size_t lkl_backward_workspace_size(const lkl_problem* p, int32_t has_mask) {
  const size_t base = lkl_workspace_size(p, has_mask);
  if (base == 0 || check_problem(p, true) != LKL_OK) return base;
  return base + round256(lkl::sm100_dbuf_bytes(to_problem(p)));
}

int32_t lkl_lse(const void* q, const void* k, const void* mask, const lkl_problem* p, float* lse,
                void* ws, size_t ws_bytes, void* stream) {
  int32_t s = check_problem(p, false);
  if (s) return s;
  if (!q || !k || !lse) return LKL_ERR_NULL_POINTER;
  if (!aligned(q, 2) || !aligned(k, 2) || !aligned(lse, 4)) return LKL_ERR_MISALIGNED;
  if ((s = check_mask(mask, p->mask_dtype))) return s;
  if (p->B == 0 || p->T == 0) return LKL_OK;
  if ((s = check_workspace(lkl_forward_workspace_size(p, mask != nullptr), ws, ws_bytes))) return s;
  if (!bind_device_of(q) || !device_is_sm100()) return LKL_ERR_NO_DEVICE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint32_t* bits;
  if ((s = prepare_mask(p, mask, ws, &bits, st))) return s;
  lkl_problem pp = *p;
  pp.Hkv_t = p->Hkv_s;
  pp.Dt = p->Ds;
  pp.dtype_t = p->dtype_s;
  pp.sm_scale_t = p->sm_scale_s;
  const Problem qq = to_problem(&pp);
  if (use_tensor_cores(qq, q, k, q, k)) {
    t_last_path = 1;
    return launch_status(lkl::launch_sm100_forward(qq, q, k, q, k, nullptr, bits, lse, nullptr,
                                                   nullptr, nullptr, st, 0));
  }
  t_last_path = 0;
  return launch_status(lkl::launch_generic_forward(0, qq, q, k, q, k, bits, lse, nullptr,
                                                   nullptr, nullptr, st));
}

int32_t lkl_kl_forward(const void* qs, const void* ks, const float* lse_s, const void* qt,
                       const void* kt, const float* lse_t, const void* mask,
                       const lkl_problem* p, float* loss, void* ws, size_t ws_bytes,
                       void* stream) {
  int32_t s = check_problem(p, true);
  if (s) return s;
  if (!qs || !ks || !qt || !kt || !lse_s || !lse_t || !loss) return LKL_ERR_NULL_POINTER;
  if (!aligned(qs, 2) || !aligned(ks, 2) || !aligned(qt, 2) || !aligned(kt, 2) ||
      !aligned(lse_s, 4) || !aligned(lse_t, 4) || !aligned(loss, 4))
    return LKL_ERR_MISALIGNED;
  if ((s = check_mask(mask, p->mask_dtype))) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (p->B == 0 || p->T == 0) return launch_status(cudaMemsetAsync(loss, 0, sizeof(float), st));
  if ((s = check_workspace(lkl_forward_workspace_size(p, mask != nullptr), ws, ws_bytes))) return s;
  if (!bind_device_of(qs) || !device_is_sm100()) return LKL_ERR_NO_DEVICE;
  uint32_t* bits;
  if ((s = prepare_mask(p, mask, ws, &bits, st))) return s;
  const Problem q = to_problem(p);
  float* part = partials_ptr(p, mask, ws);
  int np = 0;
  cudaError_t e;
  if (use_tensor_cores(q, qs, ks, qt, kt)) {
    t_last_path = 1;
    e = lkl::launch_sm100_forward(q, qs, ks, qt, kt, nullptr, bits, const_cast<float*>(lse_s),
                                  const_cast<float*>(lse_t), part, &np, st, 2);
  } else {
    t_last_path = 0;
    e = lkl::launch_generic_forward(2, q, qs, ks, qt, kt, bits, const_cast<float*>(lse_s),
                                    const_cast<float*>(lse_t), part, &np, st);
  }
  if (e != cudaSuccess) return launch_status(e);
  return launch_status(lkl::launch_reduce_partials(part, np, loss, st));
}

}  // extern "C"

namespace {

// Strided inputs: every stride a positive multiple of 8 elements (16 bytes,
// the TMA rule), base pointers 16-byte aligned.
int32_t check_strides(const lkl_strides* s, const void* const ptrs[4]) {
  if (!s) return LKL_ERR_NULL_POINTER;
  for (int i = 0; i < 4; ++i) {
    if (s[i].b <= 0 || s[i].h <= 0 || s[i].t <= 0) return LKL_ERR_BAD_SHAPE;
    if (s[i].b % 8 || s[i].h % 8 || s[i].t % 8 || !aligned(ptrs[i], 16)) return LKL_ERR_MISALIGNED;
  }
  return LKL_OK;
}

void to_strides(const lkl_strides* s, lkl::TensorStrides out[4]) {
  for (int i = 0; i < 4; ++i) out[i] = lkl::TensorStrides{s[i].b, s[i].h, s[i].t};
}

// lkl_forward with optional strides (nullptr = contiguous inputs).
int32_t forward_impl(const void* qs, const void* ks, const void* qt, const void* kt,
                     const lkl_strides* strides, const void* mask, const lkl_problem* p,
                     float* lse_s, float* lse_t, float* loss, void* ws, size_t ws_bytes,
                     void* stream) {
  int32_t s = check_problem(p, true);
  if (s) return s;
  if (!qs || !ks || !qt || !kt || !lse_s || !lse_t || !loss) return LKL_ERR_NULL_POINTER;
  if (!aligned(qs, 2) || !aligned(ks, 2) || !aligned(qt, 2) || !aligned(kt, 2) ||
      !aligned(lse_s, 4) || !aligned(lse_t, 4) || !aligned(loss, 4))
    return LKL_ERR_MISALIGNED;
  if ((s = check_mask(mask, p->mask_dtype))) return s;
  const void* const ptrs[4] = {qs, ks, qt, kt};
  if (strides && (s = check_strides(strides, ptrs))) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (p->B == 0 || p->T == 0) return launch_status(cudaMemsetAsync(loss, 0, sizeof(float), st));
  if ((s = check_workspace(lkl_forward_workspace_size(p, mask != nullptr), ws, ws_bytes))) return s;
  if (!bind_device_of(qs) || !device_is_sm100()) return LKL_ERR_NO_DEVICE;
  const Problem q = to_problem(p);
  const bool tc = use_tensor_cores(q, qs, ks, qt, kt);
  if (strides && !tc) return LKL_ERR_UNSUPPORTED;
  uint32_t* bits;
  if ((s = prepare_mask(p, mask, ws, &bits, st))) return s;
  float* part = partials_ptr(p, mask, ws);
  int np = 0;
  cudaError_t e;
  if (tc) {
    t_last_path = 1;
    lkl::TensorStrides ts[4];
    if (strides) to_strides(strides, ts);
    e = lkl::launch_sm100_forward(q, qs, ks, qt, kt, strides ? ts : nullptr, bits, lse_s, lse_t,
                                  part, &np, st);
  } else {
    t_last_path = 0;
    e = lkl::launch_generic_forward(1, q, qs, ks, qt, kt, bits, lse_s, lse_t, part, &np, st);
  }
  if (e != cudaSuccess) return launch_status(e);
  return launch_status(lkl::launch_reduce_partials(part, np, loss, st));
}

// lkl_backward with optional strides (nullptr = contiguous inputs).
int32_t backward_impl(const void* qs, const void* ks, const float* lse_s, const void* qt,
                      const void* kt, const float* lse_t, const lkl_strides* strides,
                      const void* mask, const lkl_problem* p, const float* dloss, float* dq,
                      float* dk, void* ws, size_t ws_bytes, void* stream) {
  int32_t s = check_problem(p, true);
  if (s) return s;
  if (!qs || !ks || !qt || !kt || !lse_s || !lse_t || !dq || !dk) return LKL_ERR_NULL_POINTER;
  if (!aligned(qs, 2) || !aligned(ks, 2) || !aligned(qt, 2) || !aligned(kt, 2) ||
      !aligned(lse_s, 4) || !aligned(lse_t, 4) || !aligned(dq, 16) || !aligned(dk, 16) ||
      (dloss && !aligned(dloss, 4)))
    return LKL_ERR_MISALIGNED;
  if ((s = check_mask(mask, p->mask_dtype))) return s;
  const void* const ptrs[4] = {qs, ks, qt, kt};
  if (strides && (s = check_strides(strides, ptrs))) return s;
  const bool alias = dq == dk;
  if (alias && (qs != ks || p->Hkv_s != p->Hq)) return LKL_ERR_BAD_ALIAS;
  if (alias && strides && (strides[0].b != strides[1].b || strides[0].h != strides[1].h ||
                           strides[0].t != strides[1].t))
    return LKL_ERR_BAD_ALIAS;
  if (p->B == 0 || p->T == 0) return LKL_OK;
  const size_t base = lkl_workspace_size(p, mask != nullptr);
  if ((s = check_workspace(base, ws, ws_bytes))) return s;
  const Problem q = to_problem(p);
  // the tensor-core backward needs room for at least one chunk of D tiles
  // beyond the common scratch (more room means fewer, larger chunks); the
  // CUDA-core backward needs none.  Decided from shape, alignment and the
  // force flag alone, so it is checked before any device work.
  const bool tc_shape = !g_force_generic.load() && aligned(qs, 16) && aligned(ks, 16) &&
                        aligned(qt, 16) && aligned(kt, 16) && lkl::sm100_shape_ok(q);
  if (tc_shape && ws_bytes < base + lkl::sm100_dbuf_min_bytes(q)) return LKL_ERR_WORKSPACE;
  if (!bind_device_of(qs) || !device_is_sm100()) return LKL_ERR_NO_DEVICE;
  const bool tc = tc_shape && use_tensor_cores(q, qs, ks, qt, kt) &&
                  lkl::sm100_backward_supports(q);
  if (strides && !tc) return LKL_ERR_UNSUPPORTED;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint32_t* bits;
  if ((s = prepare_mask(p, mask, ws, &bits, st))) return s;
  cudaError_t e;
  if (tc) {
    // every gradient row is written by exactly one CTA per chunk: no clearing needed
    t_last_path = 1;
    lkl::TensorStrides ts[4];
    if (strides) to_strides(strides, ts);
    e = lkl::launch_sm100_backward(q, qs, ks, lse_s, qt, kt, lse_t, strides ? ts : nullptr, bits,
                                   dloss, dq, dk, alias, lsc_ptr(p, mask, ws),
                                   static_cast<uint8_t*>(ws) + base, ws_bytes - base, st);
  } else {
    t_last_path = 0;
    e = lkl::launch_generic_backward(q, qs, ks, lse_s, qt, kt, lse_t, bits, dloss, dq, dk, alias,
                                     st);
  }
  return launch_status(e);
}

// ---------------------------------------------------------------- grouped calls
// Problem of item i of a grouped call (shared fields + the item's heads).
lkl_problem item_problem(const lkl_problem* shared, const lkl_group_item& it) {
  lkl_problem q = *shared;
  q.Hq = it.Hq;
  q.Hkv_s = it.Hkv_s;
  q.Hkv_t = it.Hkv_t;
  return q;
}

// Validation of a grouped call; fills `specs` (and `strides`, 4 per item).
// backward: also the gradient rules.
int32_t check_group(int32_t n, const lkl_group_item* items, const lkl_problem* shared,
                    bool backward, std::vector<lkl::GroupSpec>& specs,
                    std::vector<lkl::TensorStrides>& strides) {
  if (!items || !shared) return LKL_ERR_NULL_POINTER;
  if (n <= 0) return LKL_ERR_BAD_SHAPE;
  if (n > LKL_MAX_GROUP_ITEMS) return LKL_ERR_TOO_LARGE;
  specs.clear();
  strides.assign((size_t)n * 4, lkl::TensorStrides{0, 0, 0});
  for (int i = 0; i < n; ++i) {
    const lkl_group_item& it = items[i];
    const lkl_problem q = item_problem(shared, it);
    int32_t s = check_problem(&q, true);
    if (s) return s;
    if (!it.qs || !it.ks || !it.qt || !it.kt || !it.lse_s || !it.lse_t) return LKL_ERR_NULL_POINTER;
    if (!aligned(it.lse_s, 4) || !aligned(it.lse_t, 4)) return LKL_ERR_MISALIGNED;
    const Problem pp = to_problem(&q);
    if (!lkl::sm100_shape_ok(pp) || !aligned(it.qs, 16) || !aligned(it.ks, 16) ||
        !aligned(it.qt, 16) || !aligned(it.kt, 16))
      return LKL_ERR_UNSUPPORTED;
    if (it.strided != 0 && it.strided != 1) return LKL_ERR_BAD_SHAPE;
    if (it.strided) {
      const void* const ptrs[4] = {it.qs, it.ks, it.qt, it.kt};
      if ((s = check_strides(it.strides, ptrs))) return s;
      if (backward && it.dq == it.dk &&
          (it.strides[0].b != it.strides[1].b || it.strides[0].h != it.strides[1].h ||
           it.strides[0].t != it.strides[1].t))
        return LKL_ERR_BAD_ALIAS;
      to_strides(it.strides, &strides[(size_t)i * 4]);
    }
    if (backward) {
      if (!it.dq || !it.dk) return LKL_ERR_NULL_POINTER;
      if (!aligned(it.dq, 16) || !aligned(it.dk, 16)) return LKL_ERR_MISALIGNED;
      if (it.dq == it.dk && (it.qs != it.ks || it.Hkv_s != it.Hq)) return LKL_ERR_BAD_ALIAS;
    }
    lkl::GroupSpec g{};
    g.qs = it.qs;
    g.ks = it.ks;
    g.qt = it.qt;
    g.kt = it.kt;
    g.Hq = it.Hq;
    g.Hkv_s = it.Hkv_s;
    g.Hkv_t = it.Hkv_t;
    g.lse_s = it.lse_s;
    g.lse_t = it.lse_t;
    g.dq = it.dq;
    g.dk = it.dk;
    g.strides = it.strided ? &strides[(size_t)i * 4] : nullptr;
    specs.push_back(g);
  }
  return LKL_OK;
}

// Grouped workspace: [mask bits][partials][lse offsets][item table][D tiles].
struct GroupLayout {
  size_t bits, partials, lsc, desc, dbuf, total;
};

GroupLayout group_layout(int32_t n, const lkl_group_item* items, const lkl_problem* shared,
                         bool has_mask, bool backward, const std::vector<lkl::GroupSpec>& specs) {
  long long heads = 0;
  for (int i = 0; i < n; ++i) heads += (long long)shared->B * items[i].Hq;
  const long long n_t = (shared->T + 127) / 128;
  GroupLayout l{};
  l.bits = has_mask ? bits_bytes(shared) : 0;
  l.partials = round256((size_t)(heads * n_t) * sizeof(float));
  l.lsc = round256((size_t)heads * shared->T * 2 * sizeof(float));
  const Problem base = to_problem(shared);
  l.desc = lkl::sm100_group_desc_bytes(base, specs.data(), n);
  l.dbuf = backward ? round256(lkl::sm100_group_dbuf_bytes(base, specs.data(), n)) : 0;
  l.total = l.bits + l.partials + l.lsc + l.desc + l.dbuf;
  return l;
}

}  // namespace

extern "C" {

size_t lkl_grouped_workspace_size(int32_t n, const lkl_group_item* items,
                                  const lkl_problem* shared, int32_t has_mask,
                                  int32_t backward) {
  std::vector<lkl::GroupSpec> specs;
  std::vector<lkl::TensorStrides> strides;
  if (check_group(n, items, shared, backward != 0, specs, strides) != LKL_OK) return 0;
  if (shared->B <= 0 || shared->T <= 0) return 0;
  return group_layout(n, items, shared, has_mask != 0, backward != 0, specs).total;
}

int32_t lkl_forward_grouped(int32_t n, const lkl_group_item* items, const void* mask,
                            const lkl_problem* shared, float* losses, void* ws, size_t ws_bytes,
                            void* stream) {
  std::vector<lkl::GroupSpec> specs;
  std::vector<lkl::TensorStrides> strides;
  int32_t s = check_group(n, items, shared, false, specs, strides);
  if (s) return s;
  if (!losses) return LKL_ERR_NULL_POINTER;
  if (!aligned(losses, 4)) return LKL_ERR_MISALIGNED;
  if ((s = check_mask(mask, shared->mask_dtype))) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (shared->B == 0 || shared->T == 0)
    return launch_status(cudaMemsetAsync(losses, 0, sizeof(float) * n, st));
  const GroupLayout l = group_layout(n, items, shared, mask != nullptr, false, specs);
  if (!ws || ws_bytes < l.total || !aligned(ws, 256)) return LKL_ERR_WORKSPACE;
  if (!bind_device_of(items[0].qs) || !device_is_sm100()) return LKL_ERR_NO_DEVICE;
  if (g_force_generic.load() || !lkl::sm100_supports(to_problem(shared))) return LKL_ERR_UNSUPPORTED;
  uint32_t* bits;
  if ((s = prepare_mask(shared, mask, ws, &bits, st))) return s;
  uint8_t* w = static_cast<uint8_t*>(ws);
  float* part = reinterpret_cast<float*>(w + l.bits);
  void* desc = w + l.bits + l.partials + l.lsc;
  t_last_path = 1;
  return launch_status(lkl::launch_sm100_forward_grouped(to_problem(shared), specs.data(), n,
                                                         bits, desc, part, losses, st));
}

int32_t lkl_backward_grouped(int32_t n, const lkl_group_item* items, const void* mask,
                             const lkl_problem* shared, const float* dlosses, void* ws,
                             size_t ws_bytes, void* stream) {
  std::vector<lkl::GroupSpec> specs;
  std::vector<lkl::TensorStrides> strides;
  int32_t s = check_group(n, items, shared, true, specs, strides);
  if (s) return s;
  if (dlosses && !aligned(dlosses, 4)) return LKL_ERR_MISALIGNED;
  if ((s = check_mask(mask, shared->mask_dtype))) return s;
  if (shared->B == 0 || shared->T == 0) return LKL_OK;
  for (int i = 0; i < n; ++i) specs[i].dloss = dlosses ? dlosses + i : nullptr;
  const GroupLayout l = group_layout(n, items, shared, mask != nullptr, true, specs);
  if (!ws || !aligned(ws, 256)) return LKL_ERR_WORKSPACE;
  // a smaller D buffer runs in more chunks, down to one kv group of the largest item
  const size_t min_dbuf = lkl::sm100_group_dbuf_min_bytes(to_problem(shared), specs.data(), n);
  const size_t fixed = l.total - l.dbuf;
  if (ws_bytes < fixed + min_dbuf) return LKL_ERR_WORKSPACE;
  if (!bind_device_of(items[0].qs) || !device_is_sm100()) return LKL_ERR_NO_DEVICE;
  if (g_force_generic.load() || !lkl::sm100_supports(to_problem(shared))) return LKL_ERR_UNSUPPORTED;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint32_t* bits;
  if ((s = prepare_mask(shared, mask, ws, &bits, st))) return s;
  uint8_t* w = static_cast<uint8_t*>(ws);
  float2* lsc = reinterpret_cast<float2*>(w + l.bits + l.partials);
  void* desc = w + l.bits + l.partials + l.lsc;
  void* dbuf = w + fixed;
  t_last_path = 1;
  return launch_status(lkl::launch_sm100_backward_grouped(to_problem(shared), specs.data(), n,
                                                          bits, desc, lsc, dbuf,
                                                          ws_bytes - fixed, st));
}

int32_t lkl_forward(const void* qs, const void* ks, const void* qt, const void* kt,
                    const void* mask, const lkl_problem* p, float* lse_s, float* lse_t,
                    float* loss, void* ws, size_t ws_bytes, void* stream) {
  return forward_impl(qs, ks, qt, kt, nullptr, mask, p, lse_s, lse_t, loss, ws, ws_bytes, stream);
}

int32_t lkl_forward_strided(const void* qs, const void* ks, const void* qt, const void* kt,
                            const lkl_strides* strides, const void* mask, const lkl_problem* p,
                            float* lse_s, float* lse_t, float* loss, void* ws, size_t ws_bytes,
                            void* stream) {
  if (!strides) return LKL_ERR_NULL_POINTER;
  return forward_impl(qs, ks, qt, kt, strides, mask, p, lse_s, lse_t, loss, ws, ws_bytes, stream);
}

int32_t lkl_backward(const void* qs, const void* ks, const float* lse_s, const void* qt,
                     const void* kt, const float* lse_t, const void* mask, const lkl_problem* p,
                     const float* dloss, float* dq, float* dk, void* ws, size_t ws_bytes,
                     void* stream) {
  return backward_impl(qs, ks, lse_s, qt, kt, lse_t, nullptr, mask, p, dloss, dq, dk, ws,
                       ws_bytes, stream);
}

int32_t lkl_backward_strided(const void* qs, const void* ks, const float* lse_s, const void* qt,
                             const void* kt, const float* lse_t, const lkl_strides* strides,
                             const void* mask, const lkl_problem* p, const float* dloss,
                             float* dq, float* dk, void* ws, size_t ws_bytes, void* stream) {
  if (!strides) return LKL_ERR_NULL_POINTER;
  return backward_impl(qs, ks, lse_s, qt, kt, lse_t, strides, mask, p, dloss, dq, dk, ws,
                       ws_bytes, stream);
}

int32_t lkl_backward_plan(const lkl_problem* p, int32_t has_mask, size_t ws_bytes, int32_t fused,
                          int32_t* n_chunks) {
  if (!n_chunks) return LKL_ERR_NULL_POINTER;
  int32_t s = check_problem(p, true);
  if (s) return s;
  *n_chunks = 0;
  const Problem q = to_problem(p);
  if (p->B == 0 || p->T == 0 || lkl::sm100_dbuf_bytes(q) == 0) return LKL_OK;
  const size_t base = lkl_workspace_size(p, has_mask);
  if (ws_bytes < base + lkl::sm100_dbuf_min_bytes(q)) return LKL_ERR_WORKSPACE;
  const int n = lkl::sm100_backward_chunks(q, ws_bytes - base, fused != 0);
  if (n < 0) return LKL_ERR_WORKSPACE;
  *n_chunks = n;
  return LKL_OK;
}

int32_t lkl_device_status(void) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, lkl::g_device_error, sizeof(int)) != cudaSuccess)
    return LKL_ERR_LAUNCH;
  if (v != 0) {
    const int zero = 0;
    cudaMemcpyToSymbol(lkl::g_device_error, &zero, sizeof(int));
    return LKL_ERR_DEVICE_TIMEOUT;
  }
  return LKL_OK;
}

int32_t lkl_selftest_bounded_wait(uint32_t limit_us, void* stream) {
  if (limit_us == 0 || limit_us > 2000000u) return LKL_ERR_BAD_SHAPE;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || !device_is_sm100()) return LKL_ERR_NO_DEVICE;
  return launch_status(lkl::launch_bounded_wait_probe((uint64_t)limit_us * 1000u,
                                                      static_cast<cudaStream_t>(stream)));
}

int32_t lkl_last_path(void) { return t_last_path; }

int32_t lkl_last_cuda_error(void) { return t_last_cuda_error; }

void lkl_set_force_generic(int32_t force) { g_force_generic.store(force ? 1 : 0); }

}  // extern "C"
