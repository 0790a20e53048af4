/* The C ABI on a GPU from plain C (CUDA runtime only, no Python, no torch):
 * seeded bf16 inputs -> lkl_forward and lkl_backward through
 * include/linearard_b200.h.  Checks that the tensor-core loss matches the
 * CUDA-core kernels' loss (lkl_set_force_generic) within 1e-3 relative, that
 * two backward calls give bit-identical gradients, and that the gradients are
 * finite.  Built and run by tests/test_c_abi_gpu.py; prints "ok <loss>". */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <cuda_runtime.h>

#include "linearard_b200.h"

#define CK(x)                                                                   \
  do {                                                                          \
    cudaError_t e_ = (x);                                                       \
    if (e_ != cudaSuccess) {                                                    \
      fprintf(stderr, "%s: %s (line %d)\n", #x, cudaGetErrorString(e_), __LINE__); \
      return 1;                                                                 \
    }                                                                           \
  } while (0)
#define LK(x)                                                                   \
  do {                                                                          \
    int32_t s_ = (x);                                                           \
    if (s_ != LKL_OK) {                                                         \
      fprintf(stderr, "%s: %s (line %d)\n", #x, lkl_status_string(s_), __LINE__); \
      return 1;                                                                 \
    }                                                                           \
  } while (0)

static uint64_t rng = 88172645463325252ull;
static float uniform(void) {  /* xorshift64 -> [0, 1) */
  rng ^= rng << 13; rng ^= rng >> 7; rng ^= rng << 17;
  return (float)((rng >> 11) * (1.0 / 9007199254740992.0));
}
static float normal(void) {  /* Box-Muller */
  float u = uniform() + 1e-7f, v = uniform();
  return sqrtf(-2.f * logf(u)) * cosf(6.2831853f * v);
}
static uint16_t to_bf16(float f) {  /* round to nearest even */
  uint32_t u;
  memcpy(&u, &f, 4);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

int main(void) {
  const int B = 1, H = 2, T = 300, D = 128;
  const size_t n = (size_t)B * H * T * D;
  uint16_t* hs = malloc(n * 2);
  uint16_t* ht = malloc(n * 2);
  for (size_t i = 0; i < n; ++i) {
    const float x = normal();
    ht[i] = to_bf16(x);
    hs[i] = to_bf16(x + 0.2f * normal());
  }
  void *s, *t, *ws_f, *ws_b;
  float *lse_s, *lse_t, *loss, *g1, *g2;
  CK(cudaMalloc(&s, n * 2));
  CK(cudaMalloc(&t, n * 2));
  CK(cudaMemcpy(s, hs, n * 2, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(t, ht, n * 2, cudaMemcpyHostToDevice));
  CK(cudaMalloc((void**)&lse_s, (size_t)B * H * T * 4));
  CK(cudaMalloc((void**)&lse_t, (size_t)B * H * T * 4));
  CK(cudaMalloc((void**)&loss, 4));
  CK(cudaMalloc((void**)&g1, n * 4));
  CK(cudaMalloc((void**)&g2, n * 4));

  lkl_problem p;
  memset(&p, 0, sizeof p);
  p.B = B; p.Hq = H; p.Hkv_s = H; p.Hkv_t = H; p.T = T; p.Ds = D; p.Dt = D;
  p.dtype_s = LKL_BF16; p.dtype_t = LKL_BF16; p.causal = 1; p.mask_dtype = LKL_MASK_U8;
  const size_t nf = lkl_workspace_size(&p, 0), nb = lkl_backward_workspace_size(&p, 0);
  CK(cudaMalloc(&ws_f, nf));
  CK(cudaMalloc(&ws_b, nb));

  /* forward: tensor cores, then the CUDA-core kernels */
  float l_tc, l_gen;
  LK(lkl_forward(s, s, t, t, NULL, &p, lse_s, lse_t, loss, ws_f, nf, NULL));
  if (lkl_last_path() != 1) { fprintf(stderr, "not the tensor-core path\n"); return 1; }
  CK(cudaMemcpy(&l_tc, loss, 4, cudaMemcpyDeviceToHost));
  lkl_set_force_generic(1);
  LK(lkl_forward(s, s, t, t, NULL, &p, lse_s, lse_t, loss, ws_f, nf, NULL));
  lkl_set_force_generic(0);
  CK(cudaMemcpy(&l_gen, loss, 4, cudaMemcpyDeviceToHost));
  if (!(fabsf(l_tc - l_gen) <= 1e-3f * fabsf(l_gen)) || !(l_tc > 0.f)) {
    fprintf(stderr, "loss %g vs %g\n", l_tc, l_gen);
    return 1;
  }
  /* LSEs of the tensor-core forward for the backward */
  LK(lkl_forward(s, s, t, t, NULL, &p, lse_s, lse_t, loss, ws_f, nf, NULL));

  /* backward twice into the fused dq + dk buffer (qs == ks): bit-identical */
  LK(lkl_backward(s, s, lse_s, t, t, lse_t, NULL, &p, NULL, g1, g1, ws_b, nb, NULL));
  LK(lkl_backward(s, s, lse_s, t, t, lse_t, NULL, &p, NULL, g2, g2, ws_b, nb, NULL));
  CK(cudaDeviceSynchronize());
  LK(lkl_device_status());
  float* a = malloc(n * 4);
  float* b = malloc(n * 4);
  CK(cudaMemcpy(a, g1, n * 4, cudaMemcpyDeviceToHost));
  CK(cudaMemcpy(b, g2, n * 4, cudaMemcpyDeviceToHost));
  double norm = 0.0;
  for (size_t i = 0; i < n; ++i) {
    if (!isfinite(a[i]) || memcmp(&a[i], &b[i], 4) != 0) {
      fprintf(stderr, "gradient mismatch at %zu: %g %g\n", i, a[i], b[i]);
      return 1;
    }
    norm += (double)a[i] * a[i];
  }
  if (!(norm > 0.0)) { fprintf(stderr, "zero gradient\n"); return 1; }
  printf("ok %.6f\n", l_tc);
  return 0;
}
