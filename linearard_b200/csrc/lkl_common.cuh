// Shared device helpers for the attention-relation KL kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "linearard_b200.h"

namespace lkl {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// Device-side error word, one per device that loads the library.  The bounded
// waits of the tensor-core kernels set it instead of spinning forever.  The
// library is one translation unit (liblinearard_b200.cu), so it is defined here.
__device__ int g_device_error = 0;

// Loads element `idx` of a fp16 / bf16 tensor as float.
__device__ __forceinline__ float load_elem(const void* base, size_t idx, int dtype) {
  if (dtype == LKL_BF16) {
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[idx]);
  }
  return __half2float(reinterpret_cast<const __half*>(base)[idx]);
}

// Rounds a float through the tensor dtype (the reference casts the score
// difference to the input dtype before the gradient dot, kernel_C.py:233).
__device__ __forceinline__ float round_to_dtype(float v, int dtype) {
  if (dtype == LKL_BF16) return __bfloat162float(__float2bfloat16_rn(v));
  return __half2float(__float2half_rn(v));
}

// Nonzero test of one padding-mask element of any supported mask dtype.
__device__ __forceinline__ bool mask_elem(const void* mask, size_t idx, int mdt) {
  switch (mdt) {
    case LKL_MASK_I32: return reinterpret_cast<const int32_t*>(mask)[idx] != 0;
    case LKL_MASK_I64: return reinterpret_cast<const int64_t*>(mask)[idx] != 0;
    default: return reinterpret_cast<const uint8_t*>(mask)[idx] != 0;
  }
}

// Validity bit of token t of batch b in the packed [B][words] mask
// (bit t%32 of word t/32).  `bits == nullptr` means every token is valid.
__device__ __forceinline__ bool token_valid(const uint32_t* bits, int words, int b, int t) {
  if (bits == nullptr) return true;
  return (bits[(size_t)b * words + (t >> 5)] >> (t & 31)) & 1u;
}

}  // namespace lkl

// Host-side launchers implemented in the .cu files.
namespace lkl {

struct Problem {
  int B, Hq, Hkv_s, Hkv_t, T, Ds, Dt;
  int dtype_s, dtype_t, causal;
  float sc_s, sc_t;
};

// Packs a [B, T] mask into bit words; words = ceil(T/32).
cudaError_t launch_pack_mask(const void* mask, int mdt, int B, int T, uint32_t* bits,
                             cudaStream_t st);
// Sums n partials in a fixed order into *out.
cudaError_t launch_reduce_partials(const float* partials, int n, float* out, cudaStream_t st);
// out[k] = sum of partials [begins[k], begins[k + 1]), k < n_ranges (device begins).
cudaError_t launch_reduce_partial_ranges(const float* partials, const int* begins, int n_ranges,
                                         float* out, cudaStream_t st);

// Generic CUDA-core kernels (any supported head dim).
// mode 0: lse of the student pair only; 1: fused lse_s, lse_t, KL partials;
// 2: KL partials from given lse_s/lse_t.
cudaError_t launch_generic_forward(int mode, const Problem& p, const void* qs, const void* ks,
                                   const void* qt, const void* kt, const uint32_t* bits,
                                   float* lse_s, float* lse_t, float* partials,
                                   int* num_partials, cudaStream_t st);
cudaError_t launch_generic_backward(const Problem& p, const void* qs, const void* ks,
                                    const float* lse_s, const void* qt, const void* kt,
                                    const float* lse_t, const uint32_t* bits,
                                    const float* dloss, float* dq, float* dk, bool alias,
                                    cudaStream_t st);
int generic_num_partials(const Problem& p);

// sm_100a tensor-core kernels.
bool sm100_supports(const Problem& p);
int sm100_num_partials(const Problem& p);
// One item of a grouped call (relations / layers of one sequence): the
// per-item tensors, head counts and outputs.  Items share B, T, the head
// dims, dtypes, causal flag, scales and mask (the Problem passed beside them).
struct TensorStrides;
struct GroupSpec {
  const void *qs, *ks, *qt, *kt;
  int Hq, Hkv_s, Hkv_t;
  float *lse_s, *lse_t;          // forward outputs, backward inputs
  float *dq, *dk;                // backward outputs; dq == dk = fused (qs == ks)
  const float* dloss;            // backward: device scalar or nullptr (= 1)
  const TensorStrides* strides;  // qs, ks, qt, kt strides, or nullptr (contiguous)
};

// Element strides of a [B][H][T][D] input (the d stride is 1).
struct TensorStrides {
  long long b, h, t;
};

// `strides`: qs, ks, qt, kt strides, or nullptr for contiguous inputs.
// mode 1: fused forward (lse_s, lse_t and KL partials); mode 0: lse_s of the
// student pair only (the teacher fields of `p` must repeat the student's);
// mode 2: KL partials from the given lse_s / lse_t.
cudaError_t launch_sm100_forward(const Problem& p, const void* qs, const void* ks,
                                 const void* qt, const void* kt, const TensorStrides* strides,
                                 const uint32_t* bits, float* lse_s, float* lse_t,
                                 float* partials, int* num_partials, cudaStream_t st,
                                 int mode = 1);
// Backward: per chunk, a dq launch that also stores the rounded D tiles into
// `dbuf`, then a dk GEMM launch over them; no reductions.  `lsc` is B*Hq*T
// float2 of scratch, `dbuf` at least
// sm100_dbuf_bytes(p) bytes (smaller buffers give more, smaller chunks; too
// small for one query-tile row of a kv group -> cudaErrorInvalidValue).
bool sm100_backward_supports(const Problem& p);
size_t sm100_dbuf_bytes(const Problem& p);
// Smallest D buffer the backward runs with (one query-tile row of a kv group).
size_t sm100_dbuf_min_bytes(const Problem& p);
// Chunks (dq + dk launch pairs) of the backward with a D buffer of dbuf_bytes,
// or -1 when it is too small (host-only).
int sm100_backward_chunks(const Problem& p, size_t dbuf_bytes, bool alias);

// Grouped calls (all items on the tensor-core path; `base` holds the shared
// fields).  `desc` is sm100_group_desc_bytes(n) of device scratch for the
// item table; the forward writes each item's LSEs and losses[i]; the backward
// needs a D buffer of at least one kv group of the largest item
// (sm100_group_dbuf_bytes gives the preferred size).
size_t sm100_group_desc_bytes(const Problem& base, const GroupSpec* items, int n);
size_t sm100_group_dbuf_bytes(const Problem& base, const GroupSpec* items, int n);
size_t sm100_group_dbuf_min_bytes(const Problem& base, const GroupSpec* items, int n);
cudaError_t launch_sm100_forward_grouped(const Problem& base, const GroupSpec* items, int n,
                                         const uint32_t* bits, void* desc, float* partials,
                                         float* losses, cudaStream_t st);
cudaError_t launch_sm100_backward_grouped(const Problem& base, const GroupSpec* items, int n,
                                          const uint32_t* bits, void* desc, float2* lsc,
                                          void* dbuf, size_t dbuf_bytes, cudaStream_t st);
cudaError_t launch_sm100_backward(const Problem& p, const void* qs, const void* ks,
                                  const float* lse_s, const void* qt, const void* kt,
                                  const float* lse_t, const TensorStrides* strides,
                                  const uint32_t* bits, const float* dloss, float* dq, float* dk,
                                  bool alias, float2* lsc, void* dbuf, size_t dbuf_bytes,
                                  cudaStream_t st);

// Diagnostic launch of a bounded wait that cannot complete (limit in ns).
cudaError_t launch_bounded_wait_probe(uint64_t limit_ns, cudaStream_t st);

}  // namespace lkl
