// Generic CUDA-core kernels for the attention-relation KL loss.
//
// These cover every head dim the reference accepts (8..256, Ds != Dt) and any
// alignment; the sm_100a tensor-core kernels (lkl_sm100.cu) take the shapes
// they support.  Both compute the same quantities:
//   forward  -- row LSEs (kernel_A.py:146-158) and the KL sum (kernel_B.py:206-218),
//   backward -- dq = sc*D.Ks (row-stationary launch), dk = sc*D^T.Qs
//               (column-stationary launch that recomputes D), with D = ps - pt
//               rounded to the input dtype (kernel_C.py:224-253); each
//               gradient row has one writer, so results are bit-reproducible.
//
// Tiling: a 256-thread block owns 32 rows of one (batch, head) and walks
// 32-column tiles (only those at or below the diagonal when causal).  Thread t
// handles row t/8 and columns (t%8) + 8k, k = 0..3; each row's statistics are
// merged across its 8 lanes with shuffles at the end.
#include <math_constants.h>

#include "lkl_common.cuh"

namespace lkl {
namespace {

constexpr int kGBM = 32;
constexpr int kGBN = 32;
constexpr int kGThreads = 256;

// ---------------------------------------------------------------- mask / reduce
__global__ void pack_mask_kernel(const void* mask, int mdt, int B, int T, uint32_t* bits) {
  const int words = (T + 31) / 32;
  const int total = B * words;
  for (int w = blockIdx.x * blockDim.x + threadIdx.x; w < total; w += gridDim.x * blockDim.x) {
    const int b = w / words, t0 = (w % words) * 32;
    uint32_t v = 0;
    for (int t = 0; t < 32 && t0 + t < T; ++t)
      if (mask_elem(mask, (size_t)b * T + t0 + t, mdt)) v |= 1u << t;
    bits[w] = v;
  }
}

// Block k sums partials [begins[k], begins[k + 1]) (all n when begins is
// null) into out[k], in the same fixed order for every range.
__global__ void reduce_partials_kernel(const float* partials, int n, const int* begins,
                                       float* out) {
  __shared__ double red[32];
  int lo = 0, hi = n;
  if (begins) {
    lo = begins[blockIdx.x];
    hi = begins[blockIdx.x + 1];
  }
  double s = 0.0;
  for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) s += (double)partials[i];
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    s = (threadIdx.x < (blockDim.x >> 5)) ? red[threadIdx.x] : 0.0;
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (threadIdx.x == 0) out[blockIdx.x] = (float)s;
  }
}

// Loads a [kGBN rows][D] tile starting at row r0 of a [T][D] slab into padded
// fp32 shared memory; rows past T read as zero.
__device__ __forceinline__ void load_tile(float* dst, const void* src, size_t slab_off, int r0,
                                          int T, int D, int dtype) {
  const int ld = D + 1;
  for (int e = threadIdx.x; e < kGBN * D; e += kGThreads) {
    const int r = e / D, d = e % D;
    float v = 0.f;
    if (r0 + r < T) v = load_elem(src, slab_off + (size_t)(r0 + r) * D + d, dtype);
    dst[r * ld + d] = v;
  }
}

__device__ __forceinline__ float dot_rows(const float* a, const float* b, int D) {
  float acc0 = 0.f, acc1 = 0.f;
  int d = 0;
  for (; d + 1 < D; d += 2) {
    acc0 = fmaf(a[d], b[d], acc0);
    acc1 = fmaf(a[d + 1], b[d + 1], acc1);
  }
  if (d < D) acc0 = fmaf(a[d], b[d], acc0);
  return acc0 + acc1;
}

// Online (max, sum) state merge: (m, l) absorbs (m2, l2); natural-log domain.
__device__ __forceinline__ void merge_ml(float& m, float& l, float& a, float m2, float l2,
                                         float a2) {
  const float mn = fmaxf(m, m2);
  if (mn == -CUDART_INF_F) return;
  const float f1 = (m == -CUDART_INF_F) ? 0.f : __expf(m - mn);
  const float f2 = (m2 == -CUDART_INF_F) ? 0.f : __expf(m2 - mn);
  l = l * f1 + l2 * f2;
  a = a * f1 + a2 * f2;
  m = mn;
}

// ---------------------------------------------------------------- forward
// mode 0: lse of (qs, ks) -> lse_s.  mode 1: lse_s, lse_t and KL partials.
// mode 2: KL partials from the given lse_s / lse_t (kernel_B.py semantics).
template <int MODE>
__global__ void __launch_bounds__(kGThreads)
generic_forward_kernel(Problem p, const void* __restrict__ qs, const void* __restrict__ ks,
                       const void* __restrict__ qt, const void* __restrict__ kt,
                       const uint32_t* __restrict__ bits, float* __restrict__ lse_s,
                       float* __restrict__ lse_t, float* __restrict__ partials) {
  extern __shared__ float smem[];
  const int Ds = p.Ds, Dt = p.Dt, T = p.T;
  const bool need_t = MODE != 0;
  float* sQs = smem;
  float* sKs = sQs + kGBM * (Ds + 1);
  float* sQt = sKs + kGBN * (Ds + 1);
  float* sKt = sQt + (need_t ? kGBM * (Dt + 1) : 0);
  __shared__ float red[kGThreads / 32];

  const int n_mt = (T + kGBM - 1) / kGBM;
  const int bh = blockIdx.x / n_mt;
  // heavy (late) row tiles first
  const int mt = n_mt - 1 - (blockIdx.x % n_mt);
  const int b = bh / p.Hq, h = bh % p.Hq;
  const int hs = h / (p.Hq / p.Hkv_s), ht = h / (p.Hq / p.Hkv_t);
  const int words = (T + 31) / 32;
  const size_t q_off_s = ((size_t)b * p.Hq + h) * T * Ds;
  const size_t k_off_s = ((size_t)b * p.Hkv_s + hs) * T * Ds;
  const size_t q_off_t = ((size_t)b * p.Hq + h) * T * Dt;
  const size_t k_off_t = ((size_t)b * p.Hkv_t + ht) * T * Dt;
  const size_t row_off = (size_t)bh * T;

  const int r = threadIdx.x >> 3, sub = threadIdx.x & 7;
  const int i = mt * kGBM + r;
  const bool row_in = i < T;
  const bool row_valid = row_in && token_valid(bits, words, b, i);

  load_tile(sQs, qs, q_off_s, mt * kGBM, T, Ds, p.dtype_s);
  if (need_t) load_tile(sQt, qt, q_off_t, mt * kGBM, T, Dt, p.dtype_t);

  // mode 2 inputs
  float Ls = 0.f, Lt = 0.f;
  bool row_ok = row_valid;
  if (MODE == 2 && row_in) {
    Ls = lse_s[row_off + i];
    Lt = lse_t[row_off + i];
    row_ok = row_ok && (Ls != -CUDART_INF_F) && (Lt != -CUDART_INF_F);
    if (Ls == -CUDART_INF_F) Ls = 0.f;
    if (Lt == -CUDART_INF_F) Lt = 0.f;
  }

  float m_s = -CUDART_INF_F, l_s = 0.f, dummy = 0.f;
  float m_t = -CUDART_INF_F, l_t = 0.f, acc = 0.f;

  const int last_row = min(T - 1, mt * kGBM + kGBM - 1);
  const int n_ct = p.causal ? (last_row / kGBN + 1) : (T + kGBN - 1) / kGBN;
  for (int ct = 0; ct < n_ct; ++ct) {
    const int j0 = ct * kGBN;
    __syncthreads();
    load_tile(sKs, ks, k_off_s, j0, T, Ds, p.dtype_s);
    if (need_t) load_tile(sKt, kt, k_off_t, j0, T, Dt, p.dtype_t);
    __syncthreads();
    float xs[4], xt[4];
    bool ok[4];
    float mx_s = -CUDART_INF_F, mx_t = -CUDART_INF_F;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int c = sub + 8 * k, j = j0 + c;
      ok[k] = row_valid && j < T && (!p.causal || j <= i) && token_valid(bits, words, b, j);
      xs[k] = dot_rows(sQs + r * (Ds + 1), sKs + c * (Ds + 1), Ds) * p.sc_s;
      xt[k] = need_t ? dot_rows(sQt + r * (Dt + 1), sKt + c * (Dt + 1), Dt) * p.sc_t : 0.f;
      if (ok[k]) {
        mx_s = fmaxf(mx_s, xs[k]);
        mx_t = fmaxf(mx_t, xt[k]);
      }
    }
    if (MODE == 2) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (ok[k] && row_ok) {
          const float lps = xs[k] - Ls, lpt = xt[k] - Lt;
          acc += __expf(lpt) * (lpt - lps);
        }
      }
      continue;
    }
    if (mx_s != -CUDART_INF_F) {
      const float mn = fmaxf(m_s, mx_s);
      l_s *= (m_s == -CUDART_INF_F) ? 0.f : __expf(m_s - mn);
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (ok[k]) l_s += __expf(xs[k] - mn);
      m_s = mn;
    }
    if (MODE == 1 && mx_t != -CUDART_INF_F) {
      const float mn = fmaxf(m_t, mx_t);
      const float f = (m_t == -CUDART_INF_F) ? 0.f : __expf(m_t - mn);
      l_t *= f;
      acc *= f;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (ok[k]) {
          const float e = __expf(xt[k] - mn);
          l_t += e;
          acc = fmaf(e, xt[k] - xs[k], acc);
        }
      }
      m_t = mn;
    }
  }

  // merge the 8 lanes that share a row
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) {
    if (MODE == 2) {
      acc += __shfl_xor_sync(0xffffffffu, acc, o);
    } else {
      const float m2 = __shfl_xor_sync(0xffffffffu, m_s, o);
      const float l2 = __shfl_xor_sync(0xffffffffu, l_s, o);
      merge_ml(m_s, l_s, dummy, m2, l2, 0.f);
      if (MODE == 1) {
        const float mt2 = __shfl_xor_sync(0xffffffffu, m_t, o);
        const float lt2 = __shfl_xor_sync(0xffffffffu, l_t, o);
        const float a2 = __shfl_xor_sync(0xffffffffu, acc, o);
        merge_ml(m_t, l_t, acc, mt2, lt2, a2);
      }
    }
  }

  float kl = 0.f;
  if (MODE == 2) {
    kl = row_ok ? acc : 0.f;
  } else {
    const float ls = (l_s > 0.f) ? m_s + __logf(l_s) : -CUDART_INF_F;
    float lt = 0.f;
    if (MODE == 1) lt = (l_t > 0.f) ? m_t + __logf(l_t) : -CUDART_INF_F;
    if (sub == 0 && row_in) {
      lse_s[row_off + i] = row_valid ? ls : 0.f;
      if (MODE == 1) lse_t[row_off + i] = row_valid ? lt : 0.f;
    }
    if (MODE == 1 && row_valid && l_s > 0.f && l_t > 0.f) kl = acc / l_t + ls - lt;
  }
  if (MODE != 0) {
    float v = (sub == 0) ? kl : 0.f;
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
      float s = 0.f;
      for (int w = 0; w < kGThreads / 32; ++w) s += red[w];
      partials[blockIdx.x] = s;
    }
  }
}

// ---------------------------------------------------------------- backward
__global__ void __launch_bounds__(kGThreads)
generic_dq_kernel(Problem p, const void* __restrict__ qs, const void* __restrict__ ks,
                        const float* __restrict__ lse_s, const void* __restrict__ qt,
                        const void* __restrict__ kt, const float* __restrict__ lse_t,
                        const uint32_t* __restrict__ bits, const float* __restrict__ dloss,
                        float* dq) {
  extern __shared__ float smem[];
  const int Ds = p.Ds, Dt = p.Dt, T = p.T;
  float* sQs = smem;
  float* sKs = sQs + kGBM * (Ds + 1);
  float* sQt = sKs + kGBN * (Ds + 1);
  float* sKt = sQt + kGBM * (Dt + 1);
  float* sD = sKt + kGBN * (Dt + 1);  // [kGBM][kGBN + 1]

  const int n_mt = (T + kGBM - 1) / kGBM;
  const int bh = blockIdx.x / n_mt;
  const int mt = n_mt - 1 - (blockIdx.x % n_mt);
  const int b = bh / p.Hq, h = bh % p.Hq;
  const int hs = h / (p.Hq / p.Hkv_s), ht = h / (p.Hq / p.Hkv_t);
  const int words = (T + 31) / 32;
  const size_t q_off_s = ((size_t)b * p.Hq + h) * T * Ds;
  const size_t k_off_s = ((size_t)b * p.Hkv_s + hs) * T * Ds;
  const size_t q_off_t = ((size_t)b * p.Hq + h) * T * Dt;
  const size_t k_off_t = ((size_t)b * p.Hkv_t + ht) * T * Dt;
  const size_t row_off = (size_t)bh * T;
  const float gscale = p.sc_s * (dloss ? *dloss : 1.f);

  const int r = threadIdx.x >> 3, sub = threadIdx.x & 7;
  const int i = mt * kGBM + r;
  const bool row_in = i < T;
  float Ls = 0.f, Lt = 0.f;
  bool row_ok = row_in && token_valid(bits, words, b, i);
  if (row_in) {
    Ls = lse_s[row_off + i];
    Lt = lse_t[row_off + i];
    row_ok = row_ok && isfinite(Ls) && isfinite(Lt);
  }

  load_tile(sQs, qs, q_off_s, mt * kGBM, T, Ds, p.dtype_s);
  load_tile(sQt, qt, q_off_t, mt * kGBM, T, Dt, p.dtype_t);

  float dqacc[32];
#pragma unroll
  for (int k = 0; k < 32; ++k) dqacc[k] = 0.f;
  const int nd = Ds / 8 > 0 ? Ds / 8 : 1;  // d = sub + 8*kk, kk < nd (Ds >= 8)

  const int last_row = min(T - 1, mt * kGBM + kGBM - 1);
  const int n_ct = p.causal ? (last_row / kGBN + 1) : (T + kGBN - 1) / kGBN;
  for (int ct = 0; ct < n_ct; ++ct) {
    const int j0 = ct * kGBN;
    __syncthreads();
    load_tile(sKs, ks, k_off_s, j0, T, Ds, p.dtype_s);
    load_tile(sKt, kt, k_off_t, j0, T, Dt, p.dtype_t);
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int c = sub + 8 * k, j = j0 + c;
      const bool ok = row_ok && j < T && (!p.causal || j <= i) && token_valid(bits, words, b, j);
      float dv = 0.f;
      if (ok) {
        const float xs = dot_rows(sQs + r * (Ds + 1), sKs + c * (Ds + 1), Ds) * p.sc_s;
        const float xt = dot_rows(sQt + r * (Dt + 1), sKt + c * (Dt + 1), Dt) * p.sc_t;
        dv = round_to_dtype(__expf(xs - Ls) - __expf(xt - Lt), p.dtype_s);
      }
      sD[r * (kGBN + 1) + c] = dv;
    }
    __syncthreads();
    // dq[i][d] += sum_c D[r][c] * Ks[c][d]
#pragma unroll
    for (int kk = 0; kk < 32; ++kk) {
      if (kk < nd) {
        const int d = sub + 8 * kk;
        float a = 0.f;
        for (int c = 0; c < kGBN; ++c) a = fmaf(sD[r * (kGBN + 1) + c], sKs[c * (Ds + 1) + d], a);
        dqacc[kk] += a;
      }
    }
  }
  if (row_in) {
    float* dst = dq + (((size_t)b * p.Hq + h) * T + i) * Ds;
#pragma unroll
    for (int kk = 0; kk < 32; ++kk)
      if (kk < nd) dst[sub + 8 * kk] = row_ok ? dqacc[kk] * gscale : 0.f;
  }
}

// dk launch (column-stationary, deterministic): a block owns 32 key columns j
// of one (batch, student kv head) and walks the query rows of every query
// head of that kv group (rows i >= j when causal), recomputing D for its
// columns; dk[j][d] = sc * sum_i D[i][j] Qs[i][d] is written once by its
// owner block (added to what the dq launch wrote when dq and dk share a
// buffer), so no float atomics are involved.
__global__ void __launch_bounds__(kGThreads)
generic_dk_kernel(Problem p, const void* __restrict__ qs, const void* __restrict__ ks,
                  const float* __restrict__ lse_s, const void* __restrict__ qt,
                  const void* __restrict__ kt, const float* __restrict__ lse_t,
                  const uint32_t* __restrict__ bits, const float* __restrict__ dloss, float* dk,
                  int alias) {
  extern __shared__ float smem[];
  const int Ds = p.Ds, Dt = p.Dt, T = p.T;
  float* sQs = smem;
  float* sKs = sQs + kGBM * (Ds + 1);
  float* sQt = sKs + kGBN * (Ds + 1);
  float* sKt = sQt + kGBM * (Dt + 1);
  float* sD = sKt + kGBN * (Dt + 1);  // [kGBM][kGBN + 1]
  __shared__ float sLs[kGBM], sLt[kGBM];
  __shared__ int sOk[kGBM];

  const int n_ct = (T + kGBN - 1) / kGBN;
  const int bg = blockIdx.x / n_ct;             // b * Hkv_s + hs
  const int ct = n_ct - 1 - (int)(blockIdx.x % n_ct);
  const int b = bg / p.Hkv_s, hs = bg % p.Hkv_s;
  const int G = p.Hq / p.Hkv_s;
  const int words = (T + 31) / 32;
  const int j0 = ct * kGBN;
  const float gscale = p.sc_s * (dloss ? *dloss : 1.f);
  const size_t k_off_s = ((size_t)b * p.Hkv_s + hs) * T * Ds;
  load_tile(sKs, ks, k_off_s, j0, T, Ds, p.dtype_s);

  const int r = threadIdx.x >> 3, sub = threadIdx.x & 7;  // D: row r, columns sub + 8k
  const int cc = threadIdx.x >> 3;                          // dk: column cc, d = sub + 8kk
  const int nd = Ds / 8 > 0 ? Ds / 8 : 1;
  float dkacc[32];
#pragma unroll
  for (int k = 0; k < 32; ++k) dkacc[k] = 0.f;

  const int n_mt = (T + kGBM - 1) / kGBM;
  const int mt0 = p.causal ? j0 / kGBM : 0;
  int ht_loaded = -1;
  for (int g = 0; g < G; ++g) {
    const int h = hs * G + g;
    const int ht = h / (p.Hq / p.Hkv_t);
    const size_t q_off_s = ((size_t)b * p.Hq + h) * T * Ds;
    const size_t q_off_t = ((size_t)b * p.Hq + h) * T * Dt;
    const size_t row_off = ((size_t)b * p.Hq + h) * T;
    for (int mt = mt0; mt < n_mt; ++mt) {
      __syncthreads();
      if (ht != ht_loaded) load_tile(sKt, kt, ((size_t)b * p.Hkv_t + ht) * T * Dt, j0, T, Dt,
                                     p.dtype_t);
      load_tile(sQs, qs, q_off_s, mt * kGBM, T, Ds, p.dtype_s);
      load_tile(sQt, qt, q_off_t, mt * kGBM, T, Dt, p.dtype_t);
      if (threadIdx.x < kGBM) {
        const int i = mt * kGBM + threadIdx.x;
        float Ls = 0.f, Lt = 0.f;
        bool ok = i < T && token_valid(bits, words, b, i);
        if (i < T) {
          Ls = lse_s[row_off + i];
          Lt = lse_t[row_off + i];
          ok = ok && isfinite(Ls) && isfinite(Lt);
        }
        sLs[threadIdx.x] = Ls;
        sLt[threadIdx.x] = Lt;
        sOk[threadIdx.x] = ok ? 1 : 0;
      }
      __syncthreads();
      ht_loaded = ht;
      const int i = mt * kGBM + r;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int c = sub + 8 * k, j = j0 + c;
        const bool ok = sOk[r] && j < T && (!p.causal || j <= i) && token_valid(bits, words, b, j);
        float dv = 0.f;
        if (ok) {
          const float xs = dot_rows(sQs + r * (Ds + 1), sKs + c * (Ds + 1), Ds) * p.sc_s;
          const float xt = dot_rows(sQt + r * (Dt + 1), sKt + c * (Dt + 1), Dt) * p.sc_t;
          dv = round_to_dtype(__expf(xs - sLs[r]) - __expf(xt - sLt[r]), p.dtype_s);
        }
        sD[r * (kGBN + 1) + c] = dv;
      }
      __syncthreads();
#pragma unroll
      for (int kk = 0; kk < 32; ++kk) {
        if (kk < nd) {
          const int d = sub + 8 * kk;
          float a = 0.f;
          for (int rr = 0; rr < kGBM; ++rr)
            a = fmaf(sD[rr * (kGBN + 1) + cc], sQs[rr * (Ds + 1) + d], a);
          dkacc[kk] += a;
        }
      }
    }
  }
  const int j = j0 + cc;
  if (j < T) {
    float* dst = dk + (((size_t)b * p.Hkv_s + hs) * T + j) * Ds;
#pragma unroll
    for (int kk = 0; kk < 32; ++kk) {
      if (kk < nd) {
        const float v = dkacc[kk] * gscale;
        dst[sub + 8 * kk] = alias ? dst[sub + 8 * kk] + v : v;
      }
    }
  }
}

size_t fwd_smem(const Problem& p, int mode) {
  size_t f = (size_t)kGBM * (p.Ds + 1) + (size_t)kGBN * (p.Ds + 1);
  if (mode != 0) f += (size_t)kGBM * (p.Dt + 1) + (size_t)kGBN * (p.Dt + 1);
  return f * sizeof(float);
}

size_t bwd_smem(const Problem& p) {
  return ((size_t)kGBM * (p.Ds + 1) * 2 + (size_t)kGBN * (p.Dt + 1) * 2 + kGBM * (kGBN + 1)) *
         sizeof(float);
}

template <typename K>
cudaError_t set_smem(K kernel, size_t bytes) {
  if (bytes <= 48 * 1024) return cudaSuccess;
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
}

}  // namespace

cudaError_t launch_pack_mask(const void* mask, int mdt, int B, int T, uint32_t* bits,
                             cudaStream_t st) {
  const int total = B * ((T + 31) / 32);
  const int grid = (total + 255) / 256;
  pack_mask_kernel<<<grid > 0 ? grid : 1, 256, 0, st>>>(mask, mdt, B, T, bits);
  return cudaGetLastError();
}

cudaError_t launch_reduce_partials(const float* partials, int n, float* out, cudaStream_t st) {
  reduce_partials_kernel<<<1, 1024, 0, st>>>(partials, n, nullptr, out);
  return cudaGetLastError();
}

cudaError_t launch_reduce_partial_ranges(const float* partials, const int* begins, int n_ranges,
                                         float* out, cudaStream_t st) {
  if (n_ranges <= 0) return cudaSuccess;
  reduce_partials_kernel<<<n_ranges, 1024, 0, st>>>(partials, 0, begins, out);
  return cudaGetLastError();
}

int generic_num_partials(const Problem& p) {
  return p.B * p.Hq * ((p.T + kGBM - 1) / kGBM);
}

cudaError_t launch_generic_forward(int mode, const Problem& p, const void* qs, const void* ks,
                                   const void* qt, const void* kt, const uint32_t* bits,
                                   float* lse_s, float* lse_t, float* partials,
                                   int* num_partials, cudaStream_t st) {
  const int grid = generic_num_partials(p);
  const size_t smem = fwd_smem(p, mode);
  cudaError_t e;
  switch (mode) {
    case 0:
      if ((e = set_smem(generic_forward_kernel<0>, smem)) != cudaSuccess) return e;
      generic_forward_kernel<0><<<grid, kGThreads, smem, st>>>(p, qs, ks, qt, kt, bits, lse_s,
                                                               lse_t, partials);
      break;
    case 1:
      if ((e = set_smem(generic_forward_kernel<1>, smem)) != cudaSuccess) return e;
      generic_forward_kernel<1><<<grid, kGThreads, smem, st>>>(p, qs, ks, qt, kt, bits, lse_s,
                                                               lse_t, partials);
      break;
    default:
      if ((e = set_smem(generic_forward_kernel<2>, smem)) != cudaSuccess) return e;
      generic_forward_kernel<2><<<grid, kGThreads, smem, st>>>(p, qs, ks, qt, kt, bits, lse_s,
                                                               lse_t, partials);
      break;
  }
  if (num_partials) *num_partials = grid;
  return cudaGetLastError();
}

cudaError_t launch_generic_backward(const Problem& p, const void* qs, const void* ks,
                                    const float* lse_s, const void* qt, const void* kt,
                                    const float* lse_t, const uint32_t* bits,
                                    const float* dloss, float* dq, float* dk, bool alias,
                                    cudaStream_t st) {
  // dq rows first (plain stores), then dk rows (stored, or added to the dq
  // rows when both are one buffer): every row has one writer per launch
  const size_t smem = bwd_smem(p);
  cudaError_t e = set_smem(generic_dq_kernel, smem);
  if (e == cudaSuccess) e = set_smem(generic_dk_kernel, smem);
  if (e != cudaSuccess) return e;
  generic_dq_kernel<<<generic_num_partials(p), kGThreads, smem, st>>>(p, qs, ks, lse_s, qt, kt,
                                                                      lse_t, bits, dloss, dq);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  const int grid_k = p.B * p.Hkv_s * ((p.T + kGBN - 1) / kGBN);
  generic_dk_kernel<<<grid_k, kGThreads, smem, st>>>(p, qs, ks, lse_s, qt, kt, lse_t, bits, dloss,
                                                     dk, alias ? 1 : 0);
  return cudaGetLastError();
}

}  // namespace lkl
