// sm_100a tensor-core kernels for the attention-relation KL loss.
//
// The forward and dq kernels are row-stationary: one CTA owns a 128-row tile
// i of one (batch, query head) and walks the 128-column tiles j <= i (all j
// when not causal); the dk kernel is a persistent GEMM over the D tiles.  Operand tiles are staged by TMA (128-byte swizzle, no multicast),
// scores are computed by tcgen05.mma into TMEM, and sixteen "row" warps (four
// warpgroups, each owning 32 of the 128 columns of a tile for all 128 rows)
// read them back with tcgen05.ld.
//
// Forward (replaces kernel_A x2 + kernel_B, kernel_A.py:42-159 / kernel_B.py:57-218):
//   ss = Qs_i Ks_j^T, st = Qt_i Kt_j^T into a double-buffered TMEM pair; the
//   row warps keep online (max, sum) for both and the teacher-weighted sum
//   A = sum_j e^{st_j - m_t} (st_j - ss_j), so that
//   KL_i = A / l_t + lse_s - lse_t   (exact: sum_j pt_j = 1).
//
// Backward (replaces kernel_C, kernel_C.py:63-261), per chunk of the D-tile
// buffer, two launches and no reductions:
//   dq launch (row-stationary, same shape as the forward): recompute ss, st;
//   D = e^{ss - lse_s} - e^{st - lse_t} rounded to the input dtype (as
//   kernel_C.py:233), written to TMEM as the A operand of dq_i += D Ks_j and
//   to the D buffer in HBM (no-swizzle core-matrix layout, 32 KB per tile);
//   dk launch (persistent GEMM): dk_j = sum_i D_ij^T Qs_i, streaming D back.
// Every gradient row is written by one CTA per chunk: bit-reproducible.
//
// Warp roles of the forward and dq kernels (576 threads): warps 0-15 = row warps in four warpgroups (warp
// w reads TMEM lanes 32*(w%4) .. +31; warpgroup g owns 32 of each tile's 128
// columns), warp 16 = TMA producer, warp 17 = MMA issuer and TMEM owner.
#include <math_constants.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <vector>

#include "lkl_common.cuh"
#include "sm100_ptx.cuh"

namespace lkl {
namespace {

using namespace sm100;

constexpr int kBM = 128;          // rows per tile (= TMEM lanes)
constexpr int kBN = 128;          // columns per tile
constexpr int kChunk = 128 * 64 * 2;  // one [128 rows][64 elems] 16-bit swizzled chunk
// Warp roles: warps 0-15 = four row warpgroups (warp w reads TMEM lanes
// 32*(w%4) and owns 32 of each tile's 128 columns), warp 16 = TMA producer,
// warp 17 = MMA issuer and TMEM owner.
constexpr int kRowWarps = 16;
constexpr int kProducerWarp = 16;
constexpr int kMmaWarp = 17;
constexpr int kThreads = 32 * (kRowWarps + 2);
constexpr int kMaxDynSmem = 232448;
constexpr int kMisc = 1024;
constexpr uint32_t kTmemCols = 512;
// Upper bound of the D buffer (the backward's bf16/fp16 D tiles of one chunk).
constexpr long long kDBufCapBytes = 8ll << 30;

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float lg2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void named_bar(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

__device__ __forceinline__ uint8_t* align1024(uint8_t* p) {
  return reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

template <int DS, int DT>
struct FwdLayout {
  static constexpr int QS = kBM * DS * 2, QT = kBM * DT * 2;
  static constexpr int STAGE = kBN * (DS + DT) * 2;
  static constexpr int STAT = 3 * 5 * kBM * 4;  // row statistics of warpgroups 1-3
  static constexpr int AVAIL = kMaxDynSmem - 1024 - kMisc - STAT - QS - QT;
  static constexpr int NS = (AVAIL / STAGE) >= 4 ? 4 : (AVAIL / STAGE);
  static constexpr int OFF_QS = 0, OFF_QT = QS, OFF_K = QS + QT;
  static constexpr int OFF_MISC = OFF_K + NS * STAGE;
  static constexpr int OFF_STAT = OFF_MISC + kMisc;
  static constexpr int BYTES = 1024 + OFF_STAT + STAT;
  static_assert(NS >= 2, "forward needs two K stages");
};


// Gradient kernels: the stationary student tile passes through shared memory
// only once (it is copied into TMEM), so it borrows the last stage slot; the
// stationary teacher tile stays in shared memory; D lives in TMEM.
template <int DS, int DT>
struct GradLayout {
  static constexpr int QS = kBM * DS * 2, QT = kBM * DT * 2;
  static constexpr int STAGE = kBN * (DS + DT) * 2;
  static constexpr int AVAIL = kMaxDynSmem - 1024 - kMisc - QT;
  static constexpr int NS = (AVAIL / STAGE) >= 4 ? 4 : (AVAIL / STAGE);
  static constexpr int OFF_QT = 0, OFF_K = QT;
  static constexpr int OFF_QS = OFF_K + (NS - 1) * STAGE;
  static constexpr int OFF_MISC = OFF_K + NS * STAGE;
  static constexpr int BYTES = 1024 + OFF_MISC + kMisc;
  static_assert(NS >= 3, "gradient kernels need three K stages");
  static_assert(QS <= STAGE, "stationary student tile must fit one stage");
};

struct Misc {
  uint64_t q_full;
  uint64_t k_full[4];
  uint64_t k_empty[4];
  uint64_t s_full[2];
  uint64_t s_empty[2];
  uint64_t d_full;
  uint64_t d_empty;
  uint64_t a_ready;  // gradient kernels: stationary tile copied into TMEM
  uint32_t tmem_base;
  int abort;
  float red[8];
};
static_assert(sizeof(Misc) <= kMisc, "misc region too small");

struct Tile {
  int b, h, hs, ht, mt, n_ct, bh;
};

// One item of a grouped call (several relations / layers of one sequence in
// one launch), in device memory: everything that differs between items.  The
// items share B, T, the head dims, dtypes, causal flag, scales and mask.
// Global query heads (and kv groups) number the items' heads one item after
// the other: item k owns heads [head_begin, head_begin + B*Hq).
struct alignas(64) GroupItem {
  CUtensorMap qs, ks, qt, kt;
  int Hq, Hkv_s, Hkv_t;
  int head_begin;  // first global query head
  int grp_begin;   // first global kv group (B * Hkv_s per item)
  int alias;       // dq == dk (qs is ks)
  float* lse_s;
  float* lse_t;
  float* dq;
  float* dk;
  const float* dloss;
};

// Device view of a grouped call: the items and, per global query head and
// per global kv group, the index of its item (one load per lookup).  items ==
// nullptr: a single problem passed by value.
struct GroupRef {
  const GroupItem* items;
  const int* head_item;
  const int* group_item;
};

__device__ __forceinline__ const GroupItem* item_of_head(const GroupRef& g, int head) {
  return g.items ? g.items + g.head_item[head] : nullptr;
}

__device__ __forceinline__ const GroupItem* item_of_group(const GroupRef& g, int grp) {
  return g.items ? g.items + g.group_item[grp] : nullptr;
}

// Problem of one item: the shared fields of `p` with the item's head counts.
__device__ __forceinline__ Problem item_problem(const Problem& p, const GroupItem* it) {
  Problem q = p;
  if (it) {
    q.Hq = it->Hq;
    q.Hkv_s = it->Hkv_s;
    q.Hkv_t = it->Hkv_t;
  }
  return q;
}

// Tile of CTA `blk` (counted from the first CTA of its item).
__device__ __forceinline__ Tile tile_of(const Problem& p, int blk) {
  Tile t;
  const int n_mt = (p.T + kBM - 1) / kBM;
  // Head-major order, longest (latest) row tiles of each head first: the CTAs
  // resident at any time work on one or two heads, so those heads' K tiles and
  // gradient rows stay in L2 instead of every head's at once.
  t.bh = blk / n_mt;
  t.mt = n_mt - 1 - blk % n_mt;
  t.b = t.bh / p.Hq;
  t.h = t.bh % p.Hq;
  t.hs = t.h / (p.Hq / p.Hkv_s);
  t.ht = t.h / (p.Hq / p.Hkv_t);
  const int n_ct_all = (p.T + kBN - 1) / kBN;
  t.n_ct = p.causal ? min(t.mt + 1, n_ct_all) : n_ct_all;
  return t;
}

// K-major SW128 operand: K-step kk (16 elements) of a tile stored as
// [rows][64]-element chunks of 16 KB.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int kk) {
  return desc_sw128(base + (uint32_t)((kk >> 2) * kChunk + (kk & 3) * 32), 16, 1024);
}
// MN-major SW128 operand: K-step kk = 16 rows of 128 B; MN chunks 16 KB apart.
__device__ __forceinline__ uint64_t mnmajor_desc(uint32_t base, int kk) {
  return desc_sw128(base + (uint32_t)(kk * 16 * 128), kChunk, 1024);
}

// Rows [row, row + 128) of head h, batch b of a {D, T, H, B} tensor map, as
// D / 64 swizzled [128][64] chunks.
__device__ __forceinline__ void issue_tile_loads(void* dst, const CUtensorMap* map,
                                                 uint64_t* bar, int D, int row, int h, int b) {
  for (int c = 0; c < D / 64; ++c)
    tma_load_4d(static_cast<uint8_t*>(dst) + c * kChunk, map, bar, c * 64, row, h, b);
}

template <typename Layout>
__device__ __forceinline__ void setup_cta(Misc* misc, int warp, int lane) {
  if (threadIdx.x == 0) {
    mbar_init(&misc->q_full, 1);
    for (int s = 0; s < 4; ++s) {
      mbar_init(&misc->k_full[s], 1);
      mbar_init(&misc->k_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&misc->s_full[s], 1);
      mbar_init(&misc->s_empty[s], kRowWarps);
    }
    mbar_init(&misc->d_full, kRowWarps);
    mbar_init(&misc->d_empty, 1);
    mbar_init(&misc->a_ready, 4);
    misc->abort = 0;
    fence_barrier_init();
  }
  if (warp == kMmaWarp) {
    tmem_alloc(&misc->tmem_base, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
}

// ============================================================== forward
// Row warps of the LSE-only forward (MODE 0): online (max, sum) of the
// student scores, merged across the four warpgroups; rows removed by the mask
// get 0, rows with no valid column -inf (kernel_A.py:146-158).
template <typename L>
__device__ __forceinline__ void forward_rows_lse(Misc* misc, float* stat, const Problem& p,
                                                 const Tile& t, const uint32_t* bits,
                                                 float* lse_s, uint32_t tmem, int warp, int lane,
                                                 volatile int* abort, int* err) {
  const int wg = warp >> 2, q = warp & 3;
  const int r = q * 32 + lane;
  const int i = t.mt * kBM + r;
  const int words = (p.T + 31) >> 5;
  const bool row_in = i < p.T;
  const bool row_valid = row_in && token_valid(bits, words, t.b, i);
  const int lim = p.causal ? min(i, p.T - 1) : p.T - 1;
  const float cs = p.sc_s * kLog2e;
  float m_s = -CUDART_INF_F, l_s = 0.f;
  const uint32_t lane_addr = tmem + ((uint32_t)(q * 32) << 16);
  const uint64_t cs2 = f2pack(cs, cs);
  for (int j = 0; j < t.n_ct; ++j) {
    const int bf = j & 1;
    if (!mbar_wait(&misc->s_full[bf], (j >> 1) & 1, abort, err)) break;
    tc_fence_after();
    float x[32];
    tmem_ld32(lane_addr + bf * 256 + wg * 32, x);
    tmem_wait_ld_dep(x);
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&misc->s_empty[bf]);
    if (!row_valid) continue;
    const int c0 = (t.n_ct - 1 - j) * kBN + wg * 32;
    if (!((c0 + 31 <= lim) && (bits == nullptr))) {
#pragma unroll
      for (int k = 0; k < 32; ++k)
        if (!((c0 + k <= lim) && token_valid(bits, words, t.b, c0 + k))) x[k] = -1.0e30f;
    }
    float mx = x[0];
#pragma unroll
    for (int k = 1; k < 31; k += 2) mx = fmax3(mx, x[k], x[k + 1]);
    mx = fmaxf(mx, x[31]);
    if (mx < -1.0e29f) continue;
    const float ms_new = fmaxf(m_s, mx * cs);
    if (__any_sync(__activemask(), ms_new > m_s)) l_s *= ex2(m_s - ms_new);
    const uint64_t nms2 = f2pack(-ms_new, -ms_new);
    uint64_t ls2 = 0;
#pragma unroll
    for (int k = 0; k < 32; k += 2) {
      float a0, a1;
      f2unpack(ffma2(f2pack(x[k], x[k + 1]), cs2, nms2), a0, a1);
      ls2 = fadd2(ls2, f2pack(ex2(a0), ex2(a1)));
    }
    float s0, s1;
    f2unpack(ls2, s0, s1);
    l_s += s0 + s1;
    m_s = ms_new;
  }
  if (wg > 0) {
    stat[(wg - 1) * 2 * kBM + r] = m_s;
    stat[((wg - 1) * 2 + 1) * kBM + r] = l_s;
  }
  named_bar(1, 32 * kRowWarps);
  if (wg == 0 && row_in) {
    float M = m_s;
#pragma unroll
    for (int g = 0; g < 3; ++g) M = fmaxf(M, stat[g * 2 * kBM + r]);
    float Ls = 0.f;
    if (M != -CUDART_INF_F) {
      Ls = l_s * ex2(m_s - M);
#pragma unroll
      for (int g = 0; g < 3; ++g) Ls += stat[(g * 2 + 1) * kBM + r] * ex2(stat[g * 2 * kBM + r] - M);
    }
    const float v = (Ls > 0.f) ? (M + lg2(Ls)) * kLn2 : -CUDART_INF_F;
    lse_s[(size_t)t.bh * p.T + i] = row_valid ? v : 0.f;
  }
}

// Row warps of the KL forward given both LSEs (MODE 2): sum over valid j of
// pt (log pt - log ps) with log p = s - lse, as kernel_B.py:57-218; rows that
// the mask removes or whose LSE is -inf give 0.  Base-2 exponents
// b = st log2e - lse_t log2e, a = ss log2e - lse_s log2e: the term is
// 2^b (b - a) ln 2.
template <typename L>
__device__ __forceinline__ void forward_rows_kl_given_lse(
    Misc* misc, float* stat, const Problem& p, const Tile& t, const uint32_t* bits,
    const float* lse_s, const float* lse_t, float* partials, uint32_t tmem, int warp, int lane,
    volatile int* abort, int* err) {
  const int wg = warp >> 2, q = warp & 3;
  const int r = q * 32 + lane;
  const int i = t.mt * kBM + r;
  const int words = (p.T + 31) >> 5;
  const bool row_in = i < p.T;
  bool row_ok = row_in && token_valid(bits, words, t.b, i);
  float Ls = 0.f, Lt = 0.f;
  if (row_in) {
    Ls = lse_s[(size_t)t.bh * p.T + i];
    Lt = lse_t[(size_t)t.bh * p.T + i];
  }
  row_ok = row_ok && Ls != -CUDART_INF_F && Lt != -CUDART_INF_F;
  const int lim = p.causal ? min(i, p.T - 1) : p.T - 1;
  const float cs = p.sc_s * kLog2e, ct = p.sc_t * kLog2e;
  const uint64_t cs2 = f2pack(cs, cs), ct2 = f2pack(ct, ct);
  const uint64_t nls2 = f2pack(-Ls * kLog2e, -Ls * kLog2e);
  const uint64_t nlt2 = f2pack(-Lt * kLog2e, -Lt * kLog2e);
  const uint32_t lane_addr = tmem + ((uint32_t)(q * 32) << 16);
  float acc = 0.f;
  for (int j = 0; j < t.n_ct; ++j) {
    const int bf = j & 1;
    if (!mbar_wait(&misc->s_full[bf], (j >> 1) & 1, abort, err)) break;
    tc_fence_after();
    float x[32], y[32];
    const uint32_t col = bf * 256 + wg * 32;
    tmem_ld32(lane_addr + col, x);
    tmem_ld32(lane_addr + col + 128, y);
    tmem_wait_ld_dep(x);
    tmem_wait_ld_dep(y);
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&misc->s_empty[bf]);
    if (!row_ok) continue;
    const int c0 = (t.n_ct - 1 - j) * kBN + wg * 32;
    const bool full = (c0 + 31 <= lim) && (bits == nullptr);
    uint64_t acc2 = 0;
#pragma unroll
    for (int k = 0; k < 32; k += 2) {
      const uint64_t aa = ffma2(f2pack(x[k], x[k + 1]), cs2, nls2);
      const uint64_t bb = ffma2(f2pack(y[k], y[k + 1]), ct2, nlt2);
      float b0, b1;
      f2unpack(bb, b0, b1);
      float pt0 = ex2(b0), pt1 = ex2(b1);
      if (!full) {
        if (!((c0 + k <= lim) && token_valid(bits, words, t.b, c0 + k))) pt0 = 0.f;
        if (!((c0 + k + 1 <= lim) && token_valid(bits, words, t.b, c0 + k + 1))) pt1 = 0.f;
      }
      acc2 = ffma2(f2pack(pt0, pt1), fsub2(bb, aa), acc2);
    }
    float a0, a1;
    f2unpack(acc2, a0, a1);
    acc += a0 + a1;
  }
  if (wg > 0) stat[(wg - 1) * kBM + r] = acc;
  named_bar(1, 32 * kRowWarps);
  if (wg == 0) {
    float kl = acc;
#pragma unroll
    for (int g = 0; g < 3; ++g) kl += stat[g * kBM + r];
    kl = row_ok ? kl * kLn2 : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) kl += __shfl_xor_sync(0xffffffffu, kl, o);
    if (lane == 0) misc->red[q] = kl;
    named_bar(2, 128);
    if (q == 0 && lane == 0)
      partials[blockIdx.x] = (misc->red[0] + misc->red[1]) + (misc->red[2] + misc->red[3]);
  }
}

// MODE 1: the fused forward (both LSEs and the KL partials).  MODE 0: the
// LSE of the student pair only (lkl_lse, kernel_A.py:42-159): one score GEMM
// and one exponential per element.  MODE 2: the KL partials given both LSEs
// (lkl_kl_forward, kernel_B.py:57-218): two score GEMMs, one exponential per
// element and no running maxima.
template <int DS, int DT, int MODE>
__global__ void __launch_bounds__(kThreads, 1)
sm100_forward_kernel(const __grid_constant__ CUtensorMap tm_qs0,
                     const __grid_constant__ CUtensorMap tm_ks0,
                     const __grid_constant__ CUtensorMap tm_qt0,
                     const __grid_constant__ CUtensorMap tm_kt0, const Problem p0,
                     const uint32_t* __restrict__ bits, float* __restrict__ lse_s0,
                     float* __restrict__ lse_t0, float* __restrict__ partials,
                     const GroupRef gref) {
  using L = FwdLayout<DS, DT>;
  constexpr bool kTeacher = MODE != 0;   // the teacher pair takes part
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  Misc* misc = reinterpret_cast<Misc*>(smem + L::OFF_MISC);
  float* stat = reinterpret_cast<float*>(smem + L::OFF_STAT);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // grouped call: this CTA's item (its tensors, head counts and outputs)
  const int n_mt = (p0.T + kBM - 1) / kBM;
  const GroupItem* it = item_of_head(gref, (int)(blockIdx.x / n_mt));
  const Problem p = item_problem(p0, it);
  const CUtensorMap& tm_qs = it ? it->qs : tm_qs0;
  const CUtensorMap& tm_ks = it ? it->ks : tm_ks0;
  const CUtensorMap& tm_qt = it ? it->qt : tm_qt0;
  const CUtensorMap& tm_kt = it ? it->kt : tm_kt0;
  float* lse_s = it ? it->lse_s : lse_s0;
  float* lse_t = it ? it->lse_t : lse_t0;
  const Tile t = tile_of(p, (int)blockIdx.x - (it ? it->head_begin * n_mt : 0));
  int* err = &g_device_error;
  volatile int* abort = &misc->abort;

  if (warp == kProducerWarp && lane == 0) {
    tma_prefetch_desc(&tm_qs);
    tma_prefetch_desc(&tm_ks);
    tma_prefetch_desc(&tm_qt);
    tma_prefetch_desc(&tm_kt);
  }
  setup_cta<L>(misc, warp, lane);
  const uint32_t tmem = misc->tmem_base;

  if (warp == kProducerWarp) {
    if (lane == 0) {
      // ---------------- TMA producer
      mbar_arrive_expect_tx(&misc->q_full, L::QS + (kTeacher ? L::QT : 0));
      issue_tile_loads(smem + L::OFF_QS, &tm_qs, &misc->q_full, DS, t.mt * kBM, t.h, t.b);
      if (kTeacher)
        issue_tile_loads(smem + L::OFF_QT, &tm_qt, &misc->q_full, DT, t.mt * kBM, t.h, t.b);
      for (int j = 0; j < t.n_ct; ++j) {
        const int s = j % L::NS;
        if (j >= L::NS && !mbar_wait(&misc->k_empty[s], ((j / L::NS) - 1) & 1, abort, err)) break;
        uint8_t* st = smem + L::OFF_K + s * L::STAGE;
        mbar_arrive_expect_tx(&misc->k_full[s], kBN * DS * 2 + (kTeacher ? kBN * DT * 2 : 0));
        issue_tile_loads(st, &tm_ks, &misc->k_full[s], DS, (t.n_ct - 1 - j) * kBN, t.hs, t.b);
        if (kTeacher)
          issue_tile_loads(st + kBN * DS * 2, &tm_kt, &misc->k_full[s], DT, (t.n_ct - 1 - j) * kBN,
                           t.ht, t.b);
      }
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      // ---------------- MMA issuer
      const uint32_t id_s = idesc_f16(kBM, kBN, p.dtype_s, p.dtype_s, 0, 0);
      const uint32_t id_t = idesc_f16(kBM, kBN, p.dtype_t, p.dtype_t, 0, 0);
      const uint32_t a_s = smem_u32(smem + L::OFF_QS), a_t = smem_u32(smem + L::OFF_QT);
      if (mbar_wait(&misc->q_full, 0, abort, err)) {
        for (int j = 0; j < t.n_ct; ++j) {
          const int s = j % L::NS, bf = j & 1;
          if (!mbar_wait(&misc->k_full[s], (j / L::NS) & 1, abort, err)) break;
          if (j >= 2 && !mbar_wait(&misc->s_empty[bf], ((j >> 1) - 1) & 1, abort, err)) break;
          tc_fence_after();
          const uint32_t b_s = smem_u32(smem + L::OFF_K + s * L::STAGE);
          const uint32_t b_t = b_s + kBN * DS * 2;
          const uint32_t d = tmem + bf * 256;
#pragma unroll
          for (int kk = 0; kk < DS / 16; ++kk)
            umma_f16_ss(d, kmajor_desc(a_s, kk), kmajor_desc(b_s, kk), id_s, kk > 0);
          if (kTeacher) {
#pragma unroll
            for (int kk = 0; kk < DT / 16; ++kk)
              umma_f16_ss(d + 128, kmajor_desc(a_t, kk), kmajor_desc(b_t, kk), id_t, kk > 0);
          }
          umma_commit(&misc->k_empty[s]);
          umma_commit(&misc->s_full[bf]);
        }
      }
    }
  } else if (warp < kRowWarps && MODE == 0) {
    forward_rows_lse<L>(misc, stat, p, t, bits, lse_s, tmem, warp, lane, abort, err);
  } else if (warp < kRowWarps && MODE == 2) {
    forward_rows_kl_given_lse<L>(misc, stat, p, t, bits, lse_s, lse_t, partials, tmem, warp,
                                 lane, abort, err);
  } else if (warp < kRowWarps) {
    // ---------------- row warps: warpgroup wg owns columns [32 wg, 32 wg + 32) of each tile
    const int wg = warp >> 2, q = warp & 3;
    const int r = q * 32 + lane;
    const int i = t.mt * kBM + r;
    const int words = (p.T + 31) >> 5;
    const bool row_in = i < p.T;
    const bool row_valid = row_in && token_valid(bits, words, t.b, i);
    const int lim = p.causal ? min(i, p.T - 1) : p.T - 1;
    const float cs = p.sc_s * kLog2e, ct = p.sc_t * kLog2e;
    float m_s = -CUDART_INF_F, l_s = 0.f, m_t = -CUDART_INF_F, l_t = 0.f, ay = 0.f, ax = 0.f;
    const uint32_t lane_addr = tmem + ((uint32_t)(q * 32) << 16);

    for (int j = 0; j < t.n_ct; ++j) {
      const int bf = j & 1;
      if (!mbar_wait(&misc->s_full[bf], (j >> 1) & 1, abort, err)) break;
      tc_fence_after();
#pragma unroll
      for (int chunk = 0; chunk < 1; ++chunk) {
        float x[32], y[32];
        const uint32_t col = bf * 256 + wg * 32;
        tmem_ld32(lane_addr + col, x);
        tmem_ld32(lane_addr + col + 128, y);
        tmem_wait_ld_dep(x);
        tmem_wait_ld_dep(y);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&misc->s_empty[bf]);
        if (!row_valid) continue;
        const int c0 = (t.n_ct - 1 - j) * kBN + wg * 32;
        const bool full = (c0 + 31 <= lim) && (bits == nullptr);
        if (!full) {
          // masked columns get a large finite negative score: e^(s - m) = 0 and
          // every product below stays finite
#pragma unroll
          for (int k = 0; k < 32; ++k) {
            const int c = c0 + k;
            const bool ok = (c <= lim) && token_valid(bits, words, t.b, c);
            if (!ok) {
              x[k] = -1.0e30f;
              y[k] = -1.0e30f;
            }
          }
        }
        float mx = x[0], my = y[0];
#pragma unroll
        for (int k = 1; k < 31; k += 2) {
          mx = fmax3(mx, x[k], x[k + 1]);
          my = fmax3(my, y[k], y[k + 1]);
        }
        mx = fmaxf(mx, x[31]);
        my = fmaxf(my, y[31]);
        if (my < -1.0e29f) continue;  // no valid column in this chunk
        const float ms_new = fmaxf(m_s, mx * cs);
        const float mt_new = fmaxf(m_t, my * ct);
        // key tiles run from the diagonal down, so the row maxima are mostly
        // found in the first tile and later tiles skip the rescale
        if (__any_sync(__activemask(), ms_new > m_s || mt_new > m_t)) {
          l_s *= ex2(m_s - ms_new);
          const float beta = ex2(m_t - mt_new);
          l_t *= beta;
          ay *= beta;
          ax *= beta;
        }
        // packed pairs: l_s += e^(ss - m_s); l_t += e^(st - m_t);
        // ay += e^(st - m_t) * st_raw; ax += e^(st - m_t) * ss_raw
        const uint64_t cs2 = f2pack(cs, cs), ct2 = f2pack(ct, ct);
        const uint64_t nms2 = f2pack(-ms_new, -ms_new), nmt2 = f2pack(-mt_new, -mt_new);
        uint64_t ls2 = 0, lt2 = 0, ay2 = 0, ax2 = 0;
#pragma unroll
        for (int k = 0; k < 32; k += 2) {
          const uint64_t xx = f2pack(x[k], x[k + 1]), yy = f2pack(y[k], y[k + 1]);
          float a0, a1, b0, b1;
          f2unpack(ffma2(xx, cs2, nms2), a0, a1);
          f2unpack(ffma2(yy, ct2, nmt2), b0, b1);
          const float ps0 = ex2(a0), ps1 = ex2(a1), pt0 = ex2(b0), pt1 = ex2(b1);
          const uint64_t ps = f2pack(ps0, ps1), pt = f2pack(pt0, pt1);
          ls2 = fadd2(ls2, ps);
          lt2 = fadd2(lt2, pt);
          ay2 = ffma2(pt, yy, ay2);
          ax2 = ffma2(pt, xx, ax2);
        }
        float ls0, ls1, lt0, lt1, ay0, ay1, ax0, ax1;
        f2unpack(ls2, ls0, ls1);
        f2unpack(lt2, lt0, lt1);
        f2unpack(ay2, ay0, ay1);
        f2unpack(ax2, ax0, ax1);
        l_s += ls0 + ls1;
        l_t += lt0 + lt1;
        ay += ay0 + ay1;
        ax += ax0 + ax1;
        m_s = ms_new;
        m_t = mt_new;
      }
    }
    // sum_j pt_j (st_j - ss_j) = sc_t * ay - sc_s * ax (pt not yet normalised)
    const float acc = fmaf(p.sc_t, ay, -p.sc_s * ax);

    // combine the four warpgroups' statistics of each row
    if (wg > 0) {
      float* st5 = stat + (wg - 1) * 5 * kBM;
      st5[0 * kBM + r] = m_s;
      st5[1 * kBM + r] = l_s;
      st5[2 * kBM + r] = m_t;
      st5[3 * kBM + r] = l_t;
      st5[4 * kBM + r] = acc;
    }
    named_bar(1, 32 * kRowWarps);
    if (wg == 0) {
      float Ms = m_s, Mt = m_t;
#pragma unroll
      for (int g = 0; g < 3; ++g) {
        Ms = fmaxf(Ms, stat[(g * 5 + 0) * kBM + r]);
        Mt = fmaxf(Mt, stat[(g * 5 + 2) * kBM + r]);
      }
      float Ls = 0.f, Lt = 0.f, A = 0.f;
      if (Ms != -CUDART_INF_F) {
        Ls = l_s * ex2(m_s - Ms);
#pragma unroll
        for (int g = 0; g < 3; ++g)
          Ls += stat[(g * 5 + 1) * kBM + r] * ex2(stat[(g * 5 + 0) * kBM + r] - Ms);
      }
      if (Mt != -CUDART_INF_F) {
        const float f0 = ex2(m_t - Mt);
        Lt = l_t * f0;
        A = acc * f0;
#pragma unroll
        for (int g = 0; g < 3; ++g) {
          const float f = ex2(stat[(g * 5 + 2) * kBM + r] - Mt);
          Lt += stat[(g * 5 + 3) * kBM + r] * f;
          A += stat[(g * 5 + 4) * kBM + r] * f;
        }
      }
      const float lse_sv = (Ls > 0.f) ? (Ms + lg2(Ls)) * kLn2 : -CUDART_INF_F;
      const float lse_tv = (Lt > 0.f) ? (Mt + lg2(Lt)) * kLn2 : -CUDART_INF_F;
      float kl = 0.f;
      if (row_valid && Ls > 0.f && Lt > 0.f) kl = A / Lt + lse_sv - lse_tv;
      if (row_in) {
        const size_t o = (size_t)t.bh * p.T + i;
        lse_s[o] = row_valid ? lse_sv : 0.f;
        lse_t[o] = row_valid ? lse_tv : 0.f;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) kl += __shfl_xor_sync(0xffffffffu, kl, o);
      if (lane == 0) misc->red[q] = kl;
      named_bar(2, 128);
      if (q == 0 && lane == 0)
        partials[blockIdx.x] = (misc->red[0] + misc->red[1]) + (misc->red[2] + misc->red[3]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ============================================================== backward
// The gradient takes two reduction-free launches per chunk of the D buffer:
//   dq launch (row-stationary: query tile i, key tiles j <= i):
//     recompute ss, st; D = e^{ss - lse_s} - e^{st - lse_t} rounded to the
//     input dtype (kernel_C.py:224-233); dq_i = sc * sum_j D_ij Ks_j; D
//     stored to HBM;
//   dk launch (persistent GEMM over (kv head, key tile j)):
//     dk_j = sc * sum_i D_ij^T Qs_i, reading the stored D tiles.
// Each output row is owned by one CTA per chunk and written once (later
// chunks add in a fixed order), so no fp32 partials go through L2 reductions
// and the gradients are reproducible bit for bit (the reference adds dk with
// float atomics, kernel_C.py:242-253).  Exponentials are computed once per
// tile pair; the D hand-off costs 32 KB of HBM writes and reads per pair.
template <bool BF16>
__device__ __forceinline__ uint32_t pack2t(float a, float b) {
  if (BF16) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ uint32_t pack2(float a, float b, int bf16) {
  if (bf16) {
    __nv_bfloat162 v = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  __half2 v = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Per-row exponent offsets -(lse_s, lse_t) * log2(e), or -inf for rows that
// take no gradient (padding mask, non-finite LSE): e^{s - inf} = 0 removes
// them without a branch.
__global__ void scale_lse_kernel(const float* __restrict__ lse_s, const float* __restrict__ lse_t,
                                 const uint32_t* __restrict__ bits, int B, int Hq, int T,
                                 float2* __restrict__ out) {
  const size_t total = (size_t)B * Hq * T;
  const int words = (T + 31) >> 5;
  for (size_t idx = blockIdx.x * (size_t)blockDim.x + threadIdx.x; idx < total;
       idx += (size_t)gridDim.x * blockDim.x) {
    const int i = (int)(idx % T);
    const int b = (int)(idx / T) / Hq;
    const float ls = lse_s[idx], lt = lse_t[idx];
    const bool ok = token_valid(bits, words, b, i) && isfinite(ls) && isfinite(lt);
    out[idx] = ok ? make_float2(-ls * kLog2e, -lt * kLog2e)
                  : make_float2(-CUDART_INF_F, -CUDART_INF_F);
  }
}

// NC fp32 columns of this thread's TMEM lane, times `scale`, into
// row_ptr[0 .. NC): stored, or added to what is there (read-modify-write by
// the row's only owner).
template <int NC>
__device__ __forceinline__ void store_rows(uint32_t taddr, float* row_ptr, float scale,
                                           bool do_store, bool accumulate, int n_valid = NC) {
  constexpr int W = NC < 32 ? NC : 32;
#pragma unroll
  for (int c = 0; c < NC; c += W) {
    float v[32];
    if (W == 32) tmem_ld32(taddr + c, v);
    else tmem_ld16(taddr + c, v);
    tmem_wait_ld_dep(v);
    if (do_store) {
#pragma unroll
      for (int k = 0; k < W; k += 4) {
        // head dims below 64 run zero-padded to 64: only the real columns exist
        if (c + k >= n_valid) break;
        float4* dst = reinterpret_cast<float4*>(row_ptr + c + k);
        float4 f = make_float4(v[k] * scale, v[k + 1] * scale, v[k + 2] * scale, v[k + 3] * scale);
        if (accumulate) {
          const float4 o = *dst;
          f.x += o.x;
          f.y += o.y;
          f.z += o.z;
          f.w += o.w;
        }
        *dst = f;
      }
    }
  }
}

// Row r of a [128][D] 16-bit tile stored as 128B-swizzled [128][64] chunks
// -> TMEM lane r, D/2 columns, two elements per column in K order: the
// layout tcgen05.mma reads an A operand from.
template <int D>
__device__ __forceinline__ void tile_row_to_tmem(const uint8_t* tile, int r, uint32_t taddr) {
#pragma unroll
  for (int c = 0; c < D / 64; ++c) {
    uint32_t v[32];
    const uint8_t* row = tile + c * kChunk + r * 128;
#pragma unroll
    for (int pc = 0; pc < 8; ++pc) {
      const uint4 q = *reinterpret_cast<const uint4*>(row + ((pc ^ (r & 7)) << 4));
      v[pc * 4 + 0] = q.x;
      v[pc * 4 + 1] = q.y;
      v[pc * 4 + 2] = q.z;
      v[pc * 4 + 3] = q.w;
    }
    tmem_st32(taddr + c * 32, v);
  }
}

// One backward chunk: kv groups [bk0, bk0 + nk) (query heads bk0*G ..), query
// tiles [i0, i1) of each; their D tiles are stored in the D buffer,
// head-major, row tile by row tile (tiles j <= i per row when causal).
// One backward chunk: global query heads [h0, h1) = the heads of global kv
// groups [g0, g1), query tiles [i0, i1) of each.  Their D tiles are stored in
// the D buffer head after head, row tile by row tile (tiles j <= i per row
// when causal).  Without grouping, global heads and groups are the problem's
// own (b * H + h).
struct Chunk {
  int h0, h1, g0, g1, i0, i1;
  int dq_acc;            // dq adds into the output (alias, non-causal, split rows)
  int band;              // dk: kv groups per band of work items (their Qs tiles fit L2)
  long long tph;         // D tiles per query head in this chunk
};

__host__ __device__ __forceinline__ long long d_row_offset(const Problem& p, const Chunk& c,
                                                           int i, int n_t) {
  return p.causal ? ((long long)i * (i + 1) / 2 - (long long)c.i0 * (c.i0 + 1) / 2)
                  : (long long)(i - c.i0) * n_t;
}

constexpr int kDTileElems = kBM * kBN;  // one D tile: [128 query rows][128 key columns]

// dq launch: one CTA per (query head, query tile i).  Recomputes both score
// tiles against every key tile j, forms D = e^{ss - lse_s} - e^{st - lse_t}
// (masked, rounded to the input dtype), accumulates dq_i += D Ks_j in TMEM and
// stores D to the D buffer for the dk launch.
template <int DS, int DT, bool BF16>
__global__ void __launch_bounds__(kThreads, 1)
sm100_dq_kernel(const __grid_constant__ CUtensorMap tm_qs0,
                const __grid_constant__ CUtensorMap tm_ks0,
                const __grid_constant__ CUtensorMap tm_qt0,
                const __grid_constant__ CUtensorMap tm_kt0, const Problem p0, const Chunk c,
                const float2* __restrict__ lsc, const uint32_t* __restrict__ bits,
                const float* __restrict__ dloss0, float* out0, uint16_t* __restrict__ dbuf,
                const GroupRef gref) {
  using L = GradLayout<DS, DT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  Misc* misc = reinterpret_cast<Misc*>(smem + L::OFF_MISC);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* err = &g_device_error;
  volatile int* abort = &misc->abort;
  constexpr uint32_t kColAcc = 256;
  // TMEM: scores [0, 256), accumulator, the stationary student tile (A of the
  // student score GEMM) and D (A of the gradient GEMM, written by the row warps)
  constexpr uint32_t kColAs = kColAcc + DS, kColD = kColAs + DS / 2;
  static_assert(kColD + kBN / 2 <= kTmemCols, "TMEM budget");

  // ---- work of this CTA (head-major, longest first)
  const int n_i = c.i1 - c.i0;
  const int local = (int)(blockIdx.x / n_i);               // head within the chunk
  const int st_tile = c.i1 - 1 - (int)(blockIdx.x % n_i);  // descending = longest first
  const int gh = c.h0 + local;                             // global query head
  const GroupItem* it = item_of_head(gref, gh);
  const Problem p = item_problem(p0, it);
  const CUtensorMap& tm_qs = it ? it->qs : tm_qs0;
  const CUtensorMap& tm_ks = it ? it->ks : tm_ks0;
  const CUtensorMap& tm_qt = it ? it->qt : tm_qt0;
  const CUtensorMap& tm_kt = it ? it->kt : tm_kt0;
  const float* dloss = it ? it->dloss : dloss0;
  float* out = it ? it->dq : out0;
  const int n_t = (p.T + kBM - 1) / kBM;
  const int G = p.Hq / p.Hkv_s;
  const int bh = gh - (it ? it->head_begin : 0);           // b * Hq + h within the item
  const int b = bh / p.Hq, h = bh % p.Hq;
  const int hs = h / G, ht = h / (p.Hq / p.Hkv_t);
  const int n_steps = p.causal ? st_tile + 1 : n_t;
  uint16_t* const drow = dbuf + ((long long)local * c.tph + d_row_offset(p, c, st_tile, n_t)) *
                                    (long long)kDTileElems;

  if (warp == kProducerWarp && lane == 0) {
    tma_prefetch_desc(&tm_qs);
    tma_prefetch_desc(&tm_ks);
    tma_prefetch_desc(&tm_qt);
    tma_prefetch_desc(&tm_kt);
  }
  setup_cta<L>(misc, warp, lane);
  const uint32_t tmem = misc->tmem_base;

  if (warp == kProducerWarp) {
    if (lane == 0) {
      // ---------------- TMA producer
      mbar_arrive_expect_tx(&misc->q_full, L::QS + L::QT);
      issue_tile_loads(smem + L::OFF_QS, &tm_qs, &misc->q_full, DS, st_tile * kBM, h, b);
      issue_tile_loads(smem + L::OFF_QT, &tm_qt, &misc->q_full, DT, st_tile * kBM, h, b);
      for (int j = 0; j < n_steps; ++j) {
        const int s = j % L::NS;
        if (j >= L::NS && !mbar_wait(&misc->k_empty[s], ((j / L::NS) - 1) & 1, abort, err)) break;
        // the last slot first holds the stationary tiles until they are in TMEM
        if (j == L::NS - 1 && !mbar_wait(&misc->a_ready, 0, abort, err)) break;
        uint8_t* stg = smem + L::OFF_K + s * L::STAGE;
        mbar_arrive_expect_tx(&misc->k_full[s], L::STAGE);
        issue_tile_loads(stg, &tm_ks, &misc->k_full[s], DS, j * kBN, hs, b);
        issue_tile_loads(stg + kBN * DS * 2, &tm_kt, &misc->k_full[s], DT, j * kBN, ht, b);
      }
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      // ---------------- MMA issuer: scores of step j+1 ahead of the gradient GEMM of j
      const uint32_t id_s = idesc_f16(kBM, kBN, p.dtype_s, p.dtype_s, 0, 0);
      const uint32_t id_t = idesc_f16(kBM, kBN, p.dtype_t, p.dtype_t, 0, 0);
      const uint32_t id_g = idesc_f16(kBM, DS, p.dtype_s, p.dtype_s, 0, 1);
      const uint32_t a_t = smem_u32(smem + L::OFF_QT);
      auto issue_scores = [&](int j) {
        const int s = j % L::NS;
        const uint32_t b_s = smem_u32(smem + L::OFF_K + s * L::STAGE);
        const uint32_t b_t = b_s + kBN * DS * 2;
#pragma unroll
        for (int kk = 0; kk < DS / 16; ++kk)
          umma_f16_ts(tmem, tmem + kColAs + kk * 8, kmajor_desc(b_s, kk), id_s, kk > 0);
#pragma unroll
        for (int kk = 0; kk < DT / 16; ++kk)
          umma_f16_ss(tmem + 128, kmajor_desc(a_t, kk), kmajor_desc(b_t, kk), id_t, kk > 0);
        umma_commit(&misc->s_full[0]);
      };
      bool ok = mbar_wait(&misc->a_ready, 0, abort, err) &&
                mbar_wait(&misc->k_full[0], 0, abort, err);
      if (ok) {
        tc_fence_after();
        issue_scores(0);
      }
      for (int j = 0; ok && j < n_steps; ++j) {
        if (j + 1 < n_steps) {
          const int s1 = (j + 1) % L::NS;
          if (!mbar_wait(&misc->k_full[s1], ((j + 1) / L::NS) & 1, abort, err)) break;
          if (!mbar_wait(&misc->s_empty[0], j & 1, abort, err)) break;
          tc_fence_after();
          issue_scores(j + 1);
        }
        if (!mbar_wait(&misc->d_full, j & 1, abort, err)) break;
        tc_fence_after();
        const int s = j % L::NS;
        const uint32_t b_s = smem_u32(smem + L::OFF_K + s * L::STAGE);
        // acc += D . X  with D from TMEM and X = the streamed student tile, MN-major
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk)
          umma_f16_ts(tmem + kColAcc, tmem + kColD + kk * 8, mnmajor_desc(b_s, kk), id_g,
                      (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&misc->d_empty);
        umma_commit(&misc->k_empty[s]);
      }
    }
  } else if (warp < kRowWarps) {
    // ---------------- row warps: lane r of the stationary tile, 32 streamed
    // columns (of each 128) per warpgroup
    const int wg = warp >> 2, q = warp & 3;
    const int r = q * 32 + lane;
    const int words = (p.T + 31) >> 5;
    const int own = st_tile * kBM + r;  // query row of this lane
    const bool own_in = own < p.T;
    const float cs = p.sc_s * kLog2e, ct = p.sc_t * kLog2e;
    const float gscale = p.sc_s * (dloss ? *dloss : 1.f);
    const uint32_t lane_addr = tmem + ((uint32_t)(q * 32) << 16);
    // this row's exponent offsets (-inf for rows that take no gradient)
    float2 Lrow = make_float2(-CUDART_INF_F, -CUDART_INF_F);
    if (own_in) Lrow = lsc[(size_t)gh * p.T + own];
    const bool row_live = Lrow.x != -CUDART_INF_F;
    if (wg == 0) {
      // warpgroup 0 moves the stationary tiles (all 128 rows) into TMEM
      if (mbar_wait(&misc->q_full, 0, abort, err)) {
        tile_row_to_tmem<DS>(smem + L::OFF_QS, r, lane_addr + kColAs);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&misc->a_ready);
    }
    const uint64_t cs2 = f2pack(cs, cs), ct2 = f2pack(ct, ct);
    const uint64_t nls2 = f2pack(Lrow.x, Lrow.x), nlt2 = f2pack(Lrow.y, Lrow.y);
    // D tiles are stored as 16 groups of 8 key columns, each [128 query rows]
    // x 16 bytes (the no-swizzle core-matrix layout the dk GEMM reads): this
    // thread's 32 columns are groups 4 wg .. 4 wg + 3 of row r, so a warp's
    // store covers 512 contiguous bytes
    uint4* dst = reinterpret_cast<uint4*>(drow) + (wg * 4) * kBM + r;

    for (int j = 0; j < n_steps; ++j) {
      if (!mbar_wait(&misc->s_full[0], j & 1, abort, err)) break;
      tc_fence_after();
      uint32_t packed[16];
      // load this thread's 32 ss and 32 st values and release the (single)
      // score buffer at once, so the next tile's score GEMMs run under this
      // tile's exponentials
      float x[32], y[32];
      tmem_ld32(lane_addr + wg * 32, x);
      tmem_ld32(lane_addr + 128 + wg * 32, y);
      tmem_wait_ld_dep(x);
      tmem_wait_ld_dep(y);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&misc->s_empty[0]);
      {
        const int c0 = j * kBN + wg * 32;  // first key column of this thread
        float d[32];
#pragma unroll
        for (int k = 0; k < 32; k += 2) {
          float a0, a1, b0, b1;
          f2unpack(ffma2(f2pack(x[k], x[k + 1]), cs2, nls2), a0, a1);
          f2unpack(ffma2(f2pack(y[k], y[k + 1]), ct2, nlt2), b0, b1);
          f2unpack(fsub2(f2pack(ex2(a0), ex2(a1)), f2pack(ex2(b0), ex2(b1))), d[k], d[k + 1]);
        }
        // columns are keys c: valid iff c <= i (causal), c < T, key not padded
        const int lim = p.causal ? min(own, p.T - 1) : p.T - 1;
        const bool full = (c0 + 31 <= lim) && (bits == nullptr);
        if (!full) {
#pragma unroll
          for (int k = 0; k < 32; ++k)
            if (!((c0 + k <= lim) && token_valid(bits, words, b, c0 + k))) d[k] = 0.f;
        }
        if (!row_live) {
#pragma unroll
          for (int k = 0; k < 32; ++k) d[k] = 0.f;
        }
#pragma unroll
        for (int k = 0; k < 32; k += 2) packed[k >> 1] = pack2t<BF16>(d[k], d[k + 1]);
      }
      // D to the buffer read by the dk launch (64 contiguous bytes per thread)
      uint4* dj = dst + (size_t)j * (kDTileElems / 8);
#pragma unroll
      for (int k = 0; k < 4; ++k)
        dj[k * kBM] =
            make_uint4(packed[4 * k], packed[4 * k + 1], packed[4 * k + 2], packed[4 * k + 3]);
      if (j > 0) {
        if (!mbar_wait(&misc->d_empty, (j - 1) & 1, abort, err)) break;
        tc_fence_after();
      }
      // D row r, this warpgroup's 32 columns -> TMEM columns [16 wg, 16 wg + 16) of D
      tmem_st16(lane_addr + kColD + wg * 16, packed);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&misc->d_full);
    }
    if (n_steps > 0 && mbar_wait(&misc->d_empty, (n_steps - 1) & 1, abort, err)) {
      tc_fence_after();
      float* row = out + ((size_t)bh * p.T + own) * p.Ds;
      store_rows<DS / 4>(lane_addr + kColAcc + wg * (DS / 4), row + wg * (DS / 4), gscale,
                         own_in && wg * (DS / 4) < p.Ds, c.dq_acc != 0, p.Ds - wg * (DS / 4));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// dk launch: a plain pipelined GEMM, persistent.  Work item = (kv head, key
// tile j): dk_j = sum over the group's query heads and query tiles i of
// D_ij^T Qs_i, both operands MN-major in shared memory (D: one bulk copy of a
// tile stored in the no-swizzle core-matrix layout; Qs: TMA, 128-byte
// swizzle), the accumulator in TMEM (two buffers, so that the epilogue of one
// item overlaps the GEMM of the next).  One CTA per SM; HBM-bound.
// Warp 0 = TMA producer, warp 1 = MMA issuer and TMEM owner, warps 2-5 =
// epilogue (TMEM lanes 32 (w % 4)).
constexpr int kDkThreads = 192;
constexpr uint32_t kDkTmemCols = 256;

template <int DS>
struct DkLayout {
  static constexpr int DT_BYTES = kDTileElems * 2, Q_BYTES = kBM * DS * 2;
  static constexpr int STAGE = DT_BYTES + Q_BYTES;
  static constexpr int AVAIL = kMaxDynSmem - 1024 - kMisc;
  static constexpr int NS = (AVAIL / STAGE) >= 4 ? 4 : (AVAIL / STAGE);
  static constexpr int OFF_MISC = NS * STAGE;
  static constexpr int BYTES = 1024 + OFF_MISC + kMisc;
  static_assert(NS >= 2, "dk GEMM needs two stages");
};

// Items of one dk launch per kv head: the key tiles that meet the chunk's query tiles.
__host__ __device__ __forceinline__ int dk_tiles_per_head(const Problem& p, const Chunk& c) {
  return p.causal ? c.i1 : (p.T + kBM - 1) / kBM;
}

template <int DS>
__global__ void __launch_bounds__(kDkThreads, 1)
sm100_dk_kernel(const __grid_constant__ CUtensorMap tm_qs0, const Problem p0, const Chunk c,
                const uint16_t* __restrict__ dbuf, const float* __restrict__ dloss0, float* out0,
                int alias0, const GroupRef gref) {
  using L = DkLayout<DS>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  Misc* misc = reinterpret_cast<Misc*>(smem + L::OFF_MISC);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* err = &g_device_error;
  volatile int* abort = &misc->abort;

  const int n_t = (p0.T + kBM - 1) / kBM;
  const int n_groups = c.g1 - c.g0;
  const int n_j = dk_tiles_per_head(p0, c);
  const int n_work = n_groups * n_j;
  // Round rd of this CTA takes work item rd * grid + b, or rd * grid + grid -
  // 1 - b in odd rounds ("snake" order).  Work items come in bands of
  // c.band kv groups, key-tile major inside a band (j ascending = longest first
  // when causal, which the snake evens out across CTAs); the CTAs at work at
  // any time read the Qs tiles of one or two bands, which stay in L2.
  auto work_at = [&](int rd) {
    const int g = (int)gridDim.x, b = (int)blockIdx.x;
    return rd * g + ((rd & 1) ? g - 1 - b : b);
  };
  // work item -> (kv group, key tile j, first query tile, query tiles) and the
  // group's item (its head counts, tensors and outputs)
  struct Work {
    const GroupItem* it;
    Problem p;
    int G, b, hs, j, i_first, n_i;
    long long head0;  // global query head of the group's first head
  };
  const int band = min(max(c.band, 1), n_groups);
  const int full_bands = n_groups / band, rest = n_groups - full_bands * band;
  auto work_of = [&](int w) {
    Work k;
    int lg0 = 0, r = w, size = band;
    if (w < full_bands * band * n_j) {
      lg0 = (w / (band * n_j)) * band;
      r = w % (band * n_j);
    } else {
      lg0 = full_bands * band;
      r = w - full_bands * band * n_j;
      size = rest;
    }
    k.j = r / size;
    const int g = c.g0 + lg0 + r % size;  // global kv group
    k.it = item_of_group(gref, g);
    k.p = item_problem(p0, k.it);
    k.G = k.p.Hq / k.p.Hkv_s;
    const int lg = g - (k.it ? k.it->grp_begin : 0);  // b * Hkv_s + hs within the item
    k.b = lg / k.p.Hkv_s;
    k.hs = lg % k.p.Hkv_s;
    k.head0 = (long long)(k.it ? k.it->head_begin : 0) + (long long)k.b * k.p.Hq + k.hs * k.G;
    k.i_first = k.p.causal ? max(c.i0, k.j) : c.i0;
    k.n_i = c.i1 - k.i_first;
    return k;
  };

  if (warp == 0 && lane == 0 && !gref.items) tma_prefetch_desc(&tm_qs0);
  if (threadIdx.x == 0) {
    for (int s = 0; s < 4; ++s) {
      mbar_init(&misc->k_full[s], 1);
      mbar_init(&misc->k_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&misc->s_full[b], 1);   // accumulator b complete
      mbar_init(&misc->s_empty[b], 4);  // accumulator b drained by the epilogue warps
    }
    misc->abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&misc->tmem_base, kDkTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = misc->tmem_base;

  if (warp == 0) {
    if (lane == 0) {
      int gs = 0;  // running stage counter over all work items of this CTA
      bool ok = true;
      for (int rd = 0, w = work_at(0); ok && w < n_work; w = work_at(++rd)) {
        const Work k = work_of(w);
        const CUtensorMap* tm_qs = k.it ? &k.it->qs : &tm_qs0;
        for (int s = 0; s < k.G * k.n_i; ++s, ++gs) {
          const int slot = gs % L::NS;
          if (gs >= L::NS &&
              !mbar_wait(&misc->k_empty[slot], ((gs / L::NS) - 1) & 1, abort, err)) {
            ok = false;
            break;
          }
          const int g = s / k.n_i, i = k.i_first + s % k.n_i;
          const long long tile = (k.head0 + g - c.h0) * c.tph + d_row_offset(k.p, c, i, n_t) + k.j;
          uint8_t* stg = smem + slot * L::STAGE;
          mbar_arrive_expect_tx(&misc->k_full[slot], L::STAGE);
          bulk_load(stg, dbuf + tile * kDTileElems, L::DT_BYTES, &misc->k_full[slot]);
          issue_tile_loads(stg + L::DT_BYTES, tm_qs, &misc->k_full[slot], DS, i * kBM,
                           k.hs * k.G + g, k.b);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // acc[key j][feature] += sum over query rows of D[query][key] Qs[query][feature]:
      // A = D^T (no swizzle, MN-major) and B = Qs (128B swizzle, MN-major)
      const uint32_t id = idesc_f16(kBN, DS, p0.dtype_s, p0.dtype_s, 1, 1);
      int gs = 0, it = 0;
      bool ok = true;
      for (int rd = 0, w = work_at(0); ok && w < n_work; w = work_at(++rd), ++it) {
        const Work k = work_of(w);
        const int ab = it & 1;
        if (it >= 2 && !mbar_wait(&misc->s_empty[ab], ((it >> 1) - 1) & 1, abort, err)) break;
        tc_fence_after();
        const uint32_t acc = tmem + ab * 128;
        for (int s = 0; s < k.G * k.n_i; ++s, ++gs) {
          const int slot = gs % L::NS;
          if (!mbar_wait(&misc->k_full[slot], (gs / L::NS) & 1, abort, err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(smem + slot * L::STAGE), bq = a + L::DT_BYTES;
#pragma unroll
          for (int kk = 0; kk < kBM / 16; ++kk)
            umma_f16_ss(acc, desc_interleave(a + kk * 2 * 128, 128, kBM * 16),
                        mnmajor_desc(bq, kk), id, (s > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&misc->k_empty[slot]);
        }
        if (ok) umma_commit(&misc->s_full[ab]);
      }
    }
  } else {
    const int q = warp & 3;
    const int r = q * 32 + lane;
    int it = 0;
    for (int rd = 0, w = work_at(0); w < n_work; w = work_at(++rd), ++it) {
      const Work k = work_of(w);
      const int ab = it & 1;
      if (!mbar_wait(&misc->s_full[ab], (it >> 1) & 1, abort, err)) break;
      tc_fence_after();
      const int own = k.j * kBN + r;  // key row of this lane
      const int alias = k.it ? k.it->alias : alias0;
      const float* dloss = k.it ? k.it->dloss : dloss0;
      float* out = k.it ? (alias ? k.it->dq : k.it->dk) : out0;
      const float gscale = k.p.sc_s * (dloss ? *dloss : 1.f);
      // the first chunk that reaches key tile j stores, later ones add
      const bool accumulate = alias != 0 || (k.p.causal ? k.j < c.i0 : c.i0 > 0);
      float* row = out + (((size_t)k.b * k.p.Hkv_s + k.hs) * k.p.T + own) * k.p.Ds;
      store_rows<DS>(tmem + ab * 128 + ((uint32_t)(q * 32) << 16), row, gscale, own < k.p.T,
                     accumulate, k.p.Ds);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&misc->s_empty[ab]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kDkTmemCols);
  }
}

// ============================================================== host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encoder() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// A [B][H][T][D] 16-bit tensor with element strides (sb, sh, st; d stride 1)
// viewed as a 4-D map {D, T, H, B} with a {64, 128, 1, 1} box.  Rows past T
// read as zeros.
// Head dim the tensor-core kernels are instantiated for: 64 for 8..64, else 128.
int tc_dim(int d) { return d <= 64 ? 64 : 128; }

bool make_map(CUtensorMap* m, const void* ptr, int dtype, int D, int T, int H, int B,
              const TensorStrides& s) {
  EncodeTiledFn enc = get_encoder();
  if (!enc) return false;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)T, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)s.t * 2, (cuuint64_t)s.h * 2, (cuuint64_t)s.b * 2};
  cuuint32_t box[4] = {64, 128, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(m, dtype == LKL_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                        : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                   4, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <typename K>
cudaError_t prep(K kernel, int bytes) {
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
}

struct Maps {
  CUtensorMap qs, ks, qt, kt;
};

TensorStrides contiguous_strides(int H, int T, int D) {
  return TensorStrides{(long long)H * T * D, (long long)T * D, (long long)D};
}

// `strides` = qs, ks, qt, kt element strides, or nullptr for contiguous tensors.
bool build_maps(Maps& m, const Problem& p, const void* qs, const void* ks, const void* qt,
                const void* kt, const TensorStrides* strides) {
  const TensorStrides s0 = strides ? strides[0] : contiguous_strides(p.Hq, p.T, p.Ds);
  const TensorStrides s1 = strides ? strides[1] : contiguous_strides(p.Hkv_s, p.T, p.Ds);
  const TensorStrides s2 = strides ? strides[2] : contiguous_strides(p.Hq, p.T, p.Dt);
  const TensorStrides s3 = strides ? strides[3] : contiguous_strides(p.Hkv_t, p.T, p.Dt);
  return make_map(&m.qs, qs, p.dtype_s, p.Ds, p.T, p.Hq, p.B, s0) &&
         make_map(&m.ks, ks, p.dtype_s, p.Ds, p.T, p.Hkv_s, p.B, s1) &&
         make_map(&m.qt, qt, p.dtype_t, p.Dt, p.T, p.Hq, p.B, s2) &&
         make_map(&m.kt, kt, p.dtype_t, p.Dt, p.T, p.Hkv_t, p.B, s3);
}

template <int DS, int DT, int MODE = 1>
cudaError_t run_forward(const Problem& p, const Maps& m, const uint32_t* bits, float* lse_s,
                        float* lse_t, float* partials, int grid, const GroupRef& gref,
                        cudaStream_t st) {
  using L = FwdLayout<DS, DT>;
  auto k = sm100_forward_kernel<DS, DT, MODE>;
  cudaError_t e = prep(k, L::BYTES);
  if (e != cudaSuccess) return e;
  k<<<grid, kThreads, L::BYTES, st>>>(m.qs, m.ks, m.qt, m.kt, p, bits, lse_s, lse_t, partials,
                                      gref);
  return cudaGetLastError();
}

template <int DS, int DT>
cudaError_t run_grad(const Problem& p, const Maps& m, const std::vector<Chunk>& plan,
                     const float2* lsc, const uint32_t* bits, const float* dloss, float* dq,
                     float* dk, bool alias, uint16_t* dbuf, const GroupRef& gref,
                     cudaStream_t st) {
  using L = GradLayout<DS, DT>;
  using LK = DkLayout<DS>;
  const bool bf = p.dtype_s == LKL_BF16;
  auto kq = bf ? sm100_dq_kernel<DS, DT, true> : sm100_dq_kernel<DS, DT, false>;
  auto kk = sm100_dk_kernel<DS>;
  cudaError_t e = prep(kq, L::BYTES);
  if (e == cudaSuccess) e = prep(kk, LK::BYTES);
  if (e != cudaSuccess) return e;
  int dev = 0, num_sms = 0;
  if ((e = cudaGetDevice(&dev)) != cudaSuccess ||
      (e = cudaDeviceGetAttribute(&num_sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
    return e;
  for (const Chunk& c : plan) {
    // dq rows of the chunk (stores D); then dk, which in the fused case adds
    // into rows that dq has already written.  (Running the HBM-bound dk
    // launch beside the next chunk's dq launch was measured: no gain, the
    // chip is at its power limit either way.)
    kq<<<(c.h1 - c.h0) * (c.i1 - c.i0), kThreads, L::BYTES, st>>>(
        m.qs, m.ks, m.qt, m.kt, p, c, lsc, bits, dloss, dq, dbuf, gref);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    const int grid = std::min((c.g1 - c.g0) * dk_tiles_per_head(p, c), num_sms);
    kk<<<grid, kDkThreads, LK::BYTES, st>>>(m.qs, p, c, dbuf, dloss, alias ? dq : dk,
                                            alias ? 1 : 0, gref);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  return cudaSuccess;
}

constexpr long long kDTileBytes = (long long)kDTileElems * 2;

// kv groups per band of dk work items: the bands' Qs tiles (G heads of T rows
// each) stay within half of the 126 MB L2.
int dk_band(const Problem& p, int G) {
  const long long per_group = (long long)G * p.T * p.Ds * 2;
  return (int)std::max<long long>(1, (64ll << 20) / std::max<long long>(per_group, 1));
}

long long d_tiles_per_head(const Problem& p) {
  const long long n_t = (p.T + kBM - 1) / kBM;
  return p.causal ? n_t * (n_t + 1) / 2 : n_t * n_t;
}

// Splits the backward of one problem into chunks whose D tiles fit
// `cap_tiles`: whole kv groups when one group fits, otherwise one group at a
// time in ranges of query tiles.  Returns false when not even one query-tile
// row of a group fits.
bool plan_chunks(const Problem& p, long long cap_tiles, bool alias, std::vector<Chunk>& out,
                 bool& zero_dq) {
  const int n_t = (p.T + kBM - 1) / kBM;
  const int G = p.Hq / p.Hkv_s;
  const int groups = p.B * p.Hkv_s;
  const long long group_tiles = (long long)G * d_tiles_per_head(p);
  out.clear();
  zero_dq = false;
  auto add = [&](int g0, int g1, int i0, int i1, long long tph, int acc) {
    Chunk c{};
    c.g0 = g0;
    c.g1 = g1;
    c.h0 = g0 * G;
    c.h1 = g1 * G;
    c.i0 = i0;
    c.i1 = i1;
    c.tph = tph;
    c.dq_acc = acc;
    c.band = dk_band(p, G);
    out.push_back(c);
  };
  if (group_tiles <= cap_tiles) {
    // as few chunks as fit, of near-equal size (a small last chunk would
    // leave most SMs idle)
    const int per = (int)std::min<long long>(groups, cap_tiles / group_tiles);
    const int n_chunks = (groups + per - 1) / per;
    for (int k = 0; k < n_chunks; ++k)
      add((int)((long long)k * groups / n_chunks), (int)((long long)(k + 1) * groups / n_chunks),
          0, n_t, d_tiles_per_head(p), 0);
    return true;
  }
  const bool acc = alias && !p.causal;
  for (int g0 = 0; g0 < groups; ++g0) {
    for (int i0 = 0; i0 < n_t;) {
      long long tiles = 0;
      int i1 = i0;
      for (; i1 < n_t; ++i1) {
        const long long row_tiles = p.causal ? i1 + 1 : n_t;
        if ((long long)G * (tiles + row_tiles) > cap_tiles) break;
        tiles += row_tiles;
      }
      if (i1 == i0) return false;
      add(g0, g0 + 1, i0, i1, tiles, acc ? 1 : 0);
      i0 = i1;
    }
  }
  zero_dq = acc;
  return true;
}

// ---------------------------------------------------------------- grouped calls
// Device image of a grouped call, written into the workspace: the items, the
// partial-sum range of each item (n + 1 ints), then the item index of every
// global query head and of every global kv group.
size_t group_desc_bytes(int n, long long heads, long long groups) {
  const size_t bytes = (size_t)n * sizeof(GroupItem) + (size_t)(n + 1 + heads + groups) * 4;
  return (bytes + 255) & ~size_t(255);
}

// Pinned staging for the item tables.  A copy from pageable memory would
// make cudaMemcpyAsync wait for the stream, so that the host could not queue
// the launches behind it; from pinned memory it is asynchronous.  A ring of
// slots per process; a slot is reused once the event recorded after its copy
// has completed (it waits only when kSlots calls are still in flight).
class PinnedRing {
 public:
  static constexpr int kSlots = 8;
  static constexpr size_t kSlotBytes = 1u << 20;

  // Queues a copy of `image` to `dst` on `st`.
  cudaError_t copy(void* dst, const std::vector<uint8_t>& image, cudaStream_t st) {
    if (image.size() > kSlotBytes) return cudaErrorInvalidValue;
    std::lock_guard<std::mutex> lock(mu_);
    if (!host_) {
      cudaError_t e = cudaHostAlloc(reinterpret_cast<void**>(&host_), kSlots * kSlotBytes,
                                    cudaHostAllocPortable);
      if (e != cudaSuccess) {
        host_ = nullptr;
        return e;
      }
    }
    Slot& slot = slots_[next_];
    next_ = (next_ + 1) % kSlots;
    cudaError_t e;
    if (slot.event && (e = cudaEventSynchronize(slot.event)) != cudaSuccess) return e;
    uint8_t* h = host_ + (&slot - slots_) * kSlotBytes;
    std::memcpy(h, image.data(), image.size());
    if ((e = cudaMemcpyAsync(dst, h, image.size(), cudaMemcpyHostToDevice, st)) != cudaSuccess)
      return e;
    // events are tied to the device current when they are created
    int dev = 0;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
    if (slot.event && slot.device != dev) {
      cudaEventDestroy(slot.event);
      slot.event = nullptr;
    }
    if (!slot.event &&
        (e = cudaEventCreateWithFlags(&slot.event, cudaEventDisableTiming)) != cudaSuccess)
      return e;
    slot.device = dev;
    return cudaEventRecord(slot.event, st);
  }

 private:
  struct Slot {
    cudaEvent_t event = nullptr;
    int device = -1;
  };
  std::mutex mu_;
  uint8_t* host_ = nullptr;
  Slot slots_[kSlots];
  int next_ = 0;
};

PinnedRing& pinned_ring() {
  static PinnedRing ring;
  return ring;
}

// Host image of a grouped call for device address `desc`; *ref_dev gets the
// device view.  group_heads (optional): query heads of every global kv group.
bool build_group(const Problem& base, const GroupSpec* g, int n, std::vector<uint8_t>& image,
                 GroupRef* ref_dev, const void* desc, int* total_heads,
                 std::vector<int>* group_heads) {
  const int n_t = (base.T + kBM - 1) / kBM;
  long long heads = 0, groups = 0;
  for (int i = 0; i < n; ++i) {
    heads += (long long)base.B * g[i].Hq;
    groups += (long long)base.B * g[i].Hkv_s;
  }
  if (heads * n_t > INT32_MAX) return false;
  image.assign(group_desc_bytes(n, heads, groups), 0);
  GroupItem* items = reinterpret_cast<GroupItem*>(image.data());
  int* begins = reinterpret_cast<int*>(image.data() + (size_t)n * sizeof(GroupItem));
  int* head_item = begins + n + 1;
  int* group_item = head_item + heads;
  int head = 0, grp = 0;
  for (int i = 0; i < n; ++i) {
    Problem p = base;
    p.Hq = g[i].Hq;
    p.Hkv_s = g[i].Hkv_s;
    p.Hkv_t = g[i].Hkv_t;
    Maps m;
    if (!build_maps(m, p, g[i].qs, g[i].ks, g[i].qt, g[i].kt, g[i].strides)) return false;
    GroupItem& it = items[i];
    it.qs = m.qs;
    it.ks = m.ks;
    it.qt = m.qt;
    it.kt = m.kt;
    it.Hq = p.Hq;
    it.Hkv_s = p.Hkv_s;
    it.Hkv_t = p.Hkv_t;
    it.head_begin = head;
    it.grp_begin = grp;
    it.alias = g[i].dq != nullptr && g[i].dq == g[i].dk;
    it.lse_s = g[i].lse_s;
    it.lse_t = g[i].lse_t;
    it.dq = g[i].dq;
    it.dk = g[i].dk;
    it.dloss = g[i].dloss;
    begins[i] = head * n_t;
    for (int k = 0; k < base.B * p.Hq; ++k) head_item[head + k] = i;
    for (int k = 0; k < base.B * p.Hkv_s; ++k) {
      group_item[grp + k] = i;
      if (group_heads) group_heads->push_back(p.Hq / p.Hkv_s);
    }
    head += base.B * p.Hq;
    grp += base.B * p.Hkv_s;
  }
  begins[n] = head * n_t;
  *total_heads = head;
  const uint8_t* d = static_cast<const uint8_t*>(desc);
  ref_dev->items = reinterpret_cast<const GroupItem*>(d);
  ref_dev->head_item = reinterpret_cast<const int*>(
      d + (reinterpret_cast<uint8_t*>(head_item) - image.data()));
  ref_dev->group_item = reinterpret_cast<const int*>(
      d + (reinterpret_cast<uint8_t*>(group_item) - image.data()));
  return true;
}

template <int MODE>
cudaError_t dispatch_forward_mode(const Problem& p, const Maps& m, const uint32_t* bits,
                                  float* lse_s, float* lse_t, float* partials, int grid,
                                  const GroupRef& g, cudaStream_t st) {
  if (MODE == 0) {  // the student pair only
    if (tc_dim(p.Ds) == 128) return run_forward<128, 128, 0>(p, m, bits, lse_s, lse_t, partials, grid, g, st);
    return run_forward<64, 64, 0>(p, m, bits, lse_s, lse_t, partials, grid, g, st);
  }
  if (tc_dim(p.Ds) == 128 && tc_dim(p.Dt) == 128)
    return run_forward<128, 128, MODE>(p, m, bits, lse_s, lse_t, partials, grid, g, st);
  if (tc_dim(p.Ds) == 64 && tc_dim(p.Dt) == 64)
    return run_forward<64, 64, MODE>(p, m, bits, lse_s, lse_t, partials, grid, g, st);
  if (tc_dim(p.Ds) == 128 && tc_dim(p.Dt) == 64)
    return run_forward<128, 64, MODE>(p, m, bits, lse_s, lse_t, partials, grid, g, st);
  return run_forward<64, 128, MODE>(p, m, bits, lse_s, lse_t, partials, grid, g, st);
}

cudaError_t dispatch_forward(const Problem& p, const Maps& m, const uint32_t* bits, float* lse_s,
                             float* lse_t, float* partials, int grid, const GroupRef& g,
                             cudaStream_t st, int mode = 1) {
  if (mode == 0) return dispatch_forward_mode<0>(p, m, bits, lse_s, lse_t, partials, grid, g, st);
  if (mode == 2) return dispatch_forward_mode<2>(p, m, bits, lse_s, lse_t, partials, grid, g, st);
  return dispatch_forward_mode<1>(p, m, bits, lse_s, lse_t, partials, grid, g, st);
}

cudaError_t dispatch_grad(const Problem& p, const Maps& m, const std::vector<Chunk>& plan,
                          const float2* lsc, const uint32_t* bits, const float* dloss, float* dq,
                          float* dk, bool alias, uint16_t* dbuf, const GroupRef& g,
                          cudaStream_t st) {
  if (tc_dim(p.Ds) == 128 && tc_dim(p.Dt) == 128)
    return run_grad<128, 128>(p, m, plan, lsc, bits, dloss, dq, dk, alias, dbuf, g, st);
  if (tc_dim(p.Ds) == 64 && tc_dim(p.Dt) == 64)
    return run_grad<64, 64>(p, m, plan, lsc, bits, dloss, dq, dk, alias, dbuf, g, st);
  if (tc_dim(p.Ds) == 128 && tc_dim(p.Dt) == 64)
    return run_grad<128, 64>(p, m, plan, lsc, bits, dloss, dq, dk, alias, dbuf, g, st);
  return run_grad<64, 128>(p, m, plan, lsc, bits, dloss, dq, dk, alias, dbuf, g, st);
}

}  // namespace

bool sm100_shape_ok(const Problem& p) {
  // 8, 16 and 32 run as 64 with the tensor maps' zero fill beyond D (the
  // padded columns add nothing to the scores and are never stored)
  auto ok = [](int d) { return d == 8 || d == 16 || d == 32 || d == 64 || d == 128; };
  const bool ds_ok = ok(p.Ds);
  const bool dt_ok = ok(p.Dt);
  return ds_ok && dt_ok && p.sc_s > 0.f && p.sc_t > 0.f && p.T >= 1;
}

bool sm100_supports(const Problem& p) { return sm100_shape_ok(p) && get_encoder() != nullptr; }

int sm100_num_partials(const Problem& p) { return p.B * p.Hq * ((p.T + kBM - 1) / kBM); }

cudaError_t launch_sm100_forward(const Problem& p, const void* qs, const void* ks,
                                 const void* qt, const void* kt, const TensorStrides* strides,
                                 const uint32_t* bits, float* lse_s, float* lse_t,
                                 float* partials, int* num_partials, cudaStream_t st, int mode) {
  Maps m;
  if (!build_maps(m, p, qs, ks, qt, kt, strides)) return cudaErrorInvalidValue;
  const int grid = sm100_num_partials(p);
  if (num_partials) *num_partials = grid;
  return dispatch_forward(p, m, bits, lse_s, lse_t, partials, grid, GroupRef{}, st, mode);
}

bool sm100_backward_supports(const Problem& p) {
  // the teacher's kv grouping only enters the dq launch (its score GEMM);
  // D and the dk launch depend on the student's grouping alone
  return sm100_supports(p);
}

size_t sm100_dbuf_bytes(const Problem& p) {
  if (p.B <= 0 || p.T <= 0 || !sm100_shape_ok(p)) return 0;
  const long long all = (long long)p.B * p.Hq * d_tiles_per_head(p);
  const long long cap = kDBufCapBytes / kDTileBytes;
  const long long row = (long long)(p.Hq / p.Hkv_s) * ((p.T + kBM - 1) / kBM);
  return (size_t)(std::max(std::min(all, cap), row) * kDTileBytes);
}

int sm100_backward_chunks(const Problem& p, size_t dbuf_bytes, bool alias) {
  std::vector<Chunk> plan;
  bool zero_dq = false;
  if (!plan_chunks(p, (long long)(dbuf_bytes / kDTileBytes), alias, plan, zero_dq)) return -1;
  return (int)plan.size();
}

size_t sm100_dbuf_min_bytes(const Problem& p) {
  if (sm100_dbuf_bytes(p) == 0) return 0;
  return (size_t)((long long)(p.Hq / p.Hkv_s) * ((p.T + kBM - 1) / kBM) * kDTileBytes);
}

cudaError_t launch_sm100_backward(const Problem& p, const void* qs, const void* ks,
                                  const float* lse_s, const void* qt, const void* kt,
                                  const float* lse_t, const TensorStrides* strides,
                                  const uint32_t* bits, const float* dloss, float* dq, float* dk,
                                  bool alias, float2* lsc, void* dbuf, size_t dbuf_bytes,
                                  cudaStream_t st) {
  std::vector<Chunk> plan;
  bool zero_dq = false;
  if (!plan_chunks(p, (long long)(dbuf_bytes / kDTileBytes), alias, plan, zero_dq))
    return cudaErrorInvalidValue;
  Maps m;
  if (!build_maps(m, p, qs, ks, qt, kt, strides)) return cudaErrorInvalidValue;
  const size_t rows = (size_t)p.B * p.Hq * p.T;
  const int grid = (int)((rows + 255) / 256 < 4096 ? (rows + 255) / 256 : 4096);
  scale_lse_kernel<<<grid, 256, 0, st>>>(lse_s, lse_t, bits, p.B, p.Hq, p.T, lsc);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  if (zero_dq && (e = cudaMemsetAsync(dq, 0, rows * p.Ds * sizeof(float), st)) != cudaSuccess)
    return e;
  return dispatch_grad(p, m, plan, lsc, bits, dloss, dq, dk, alias,
                       static_cast<uint16_t*>(dbuf), GroupRef{}, st);
}

size_t sm100_group_desc_bytes(const Problem& base, const GroupSpec* g, int n) {
  long long heads = 0, groups = 0;
  for (int i = 0; i < n; ++i) {
    heads += (long long)base.B * g[i].Hq;
    groups += (long long)base.B * g[i].Hkv_s;
  }
  return group_desc_bytes(n, heads, groups);
}

size_t sm100_group_dbuf_bytes(const Problem& base, const GroupSpec* g, int n) {
  long long all = 0, largest = 0;
  for (int i = 0; i < n; ++i) {
    const long long group = (long long)(g[i].Hq / g[i].Hkv_s) * d_tiles_per_head(base);
    all += (long long)base.B * g[i].Hkv_s * group;
    largest = std::max(largest, group);
  }
  return (size_t)(std::max(std::min(all, kDBufCapBytes / kDTileBytes), largest) * kDTileBytes);
}

size_t sm100_group_dbuf_min_bytes(const Problem& base, const GroupSpec* g, int n) {
  long long largest = 0;
  for (int i = 0; i < n; ++i)
    largest = std::max(largest, (long long)(g[i].Hq / g[i].Hkv_s) * d_tiles_per_head(base));
  return (size_t)(largest * kDTileBytes);
}

cudaError_t launch_sm100_forward_grouped(const Problem& base, const GroupSpec* g, int n,
                                         const uint32_t* bits, void* desc, float* partials,
                                         float* losses, cudaStream_t st) {
  std::vector<uint8_t> image;
  GroupRef ref{};
  int heads = 0;
  if (n <= 0 || !build_group(base, g, n, image, &ref, desc, &heads, nullptr))
    return cudaErrorInvalidValue;
  cudaError_t e = pinned_ring().copy(desc, image, st);
  if (e != cudaSuccess) return e;
  const int* begins = reinterpret_cast<const int*>(static_cast<const uint8_t*>(desc) +
                                                   (size_t)n * sizeof(GroupItem));
  // the kernel reads every item's maps from `items`; the by-value maps of
  // the first item only fill the parameters
  const GroupItem& first = *reinterpret_cast<const GroupItem*>(image.data());
  Maps m{first.qs, first.ks, first.qt, first.kt};
  const int grid = heads * ((base.T + kBM - 1) / kBM);
  e = dispatch_forward(base, m, bits, nullptr, nullptr, partials, grid, ref, st);
  if (e != cudaSuccess) return e;
  return launch_reduce_partial_ranges(partials, begins, n, losses, st);
}

cudaError_t launch_sm100_backward_grouped(const Problem& base, const GroupSpec* g, int n,
                                          const uint32_t* bits, void* desc, float2* lsc,
                                          void* dbuf, size_t dbuf_bytes, cudaStream_t st) {
  std::vector<uint8_t> image;
  std::vector<int> group_heads;
  GroupRef ref{};
  int heads = 0;
  if (n <= 0 || !build_group(base, g, n, image, &ref, desc, &heads, &group_heads))
    return cudaErrorInvalidValue;
  // chunks of whole kv groups (in item order) whose D tiles fit the buffer
  const int n_t = (base.T + kBM - 1) / kBM;
  const long long tph = d_tiles_per_head(base), cap = (long long)(dbuf_bytes / kDTileBytes);
  std::vector<Chunk> plan;
  for (int g0 = 0, h0 = 0; g0 < (int)group_heads.size();) {
    int g1 = g0, h1 = h0;
    while (g1 < (int)group_heads.size() && (long long)(h1 - h0 + group_heads[g1]) * tph <= cap)
      h1 += group_heads[g1++];
    if (g1 == g0) return cudaErrorInvalidValue;  // one kv group does not fit
    Chunk c{};
    c.g0 = g0;
    c.g1 = g1;
    c.h0 = h0;
    c.h1 = h1;
    c.i0 = 0;
    c.i1 = n_t;
    c.tph = tph;
    c.band = dk_band(base, *std::max_element(group_heads.begin() + g0, group_heads.begin() + g1));
    plan.push_back(c);
    g0 = g1;
    h0 = h1;
  }
  cudaError_t e = pinned_ring().copy(desc, image, st);
  if (e != cudaSuccess) return e;
  const GroupItem* host_items = reinterpret_cast<const GroupItem*>(image.data());
  for (int i = 0; i < n; ++i) {
    const size_t rows = (size_t)base.B * g[i].Hq * base.T;
    const int grid = (int)((rows + 255) / 256 < 4096 ? (rows + 255) / 256 : 4096);
    scale_lse_kernel<<<grid, 256, 0, st>>>(g[i].lse_s, g[i].lse_t, bits, base.B, g[i].Hq, base.T,
                                           lsc + (size_t)host_items[i].head_begin * base.T);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
  }
  Maps m{host_items[0].qs, host_items[0].ks, host_items[0].qt, host_items[0].kt};
  return dispatch_grad(base, m, plan, lsc, bits, nullptr, nullptr, nullptr, false,
                       static_cast<uint16_t*>(dbuf), ref, st);
}

// Diagnostic: one CTA whose mbarrier never completes (nothing arrives on it).
// Two waiters in different warps run the kernels' own bounded wait with a
// short limit: the first to run out sets the CTA abort flag and the device
// error word, the other sees the flag, and the kernel returns -- the path a
// stalled pipeline takes instead of hanging the GPU.
__global__ void __launch_bounds__(64, 1) bounded_wait_probe_kernel(uint64_t limit_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0)
    mbar_wait_for(&bar, 0, &abort_flag, &g_device_error, limit_ns);
  __syncthreads();
}

cudaError_t launch_bounded_wait_probe(uint64_t limit_ns, cudaStream_t st) {
  bounded_wait_probe_kernel<<<1, 64, 0, st>>>(limit_ns);
  return cudaGetLastError();
}

}  // namespace lkl
