/* Host-only check of the C ABI from plain C (no Python, no torch): compiled
 * with gcc against include/linearard_b200.h and linked to
 * liblinearard_b200.so by tests/test_c_abi_cpu.py.  Exercises only calls that
 * return before touching a device: version, status strings, workspace sizes
 * and argument validation.  Prints "ok" and exits 0 on success. */
#include <stdint.h>
#include <stdio.h>
#include <string.h>

#include "linearard_b200.h"

#define CHECK(cond)                                                  \
  do {                                                               \
    if (!(cond)) {                                                   \
      fprintf(stderr, "check failed: %s (line %d)\n", #cond, __LINE__); \
      return 1;                                                      \
    }                                                                \
  } while (0)

int main(void) {
  CHECK(lkl_abi_version() == LKL_ABI_VERSION);
  CHECK(strcmp(lkl_status_string(LKL_OK), "ok") == 0);
  for (int s = 0; s <= LKL_ERR_UNSUPPORTED; ++s) CHECK(lkl_status_string(s) != NULL);

  lkl_problem p;
  memset(&p, 0, sizeof p);
  p.B = 1; p.Hq = 4; p.Hkv_s = 2; p.Hkv_t = 2; p.T = 300; p.Ds = 128; p.Dt = 128;
  p.dtype_s = LKL_BF16; p.dtype_t = LKL_BF16; p.causal = 1; p.mask_dtype = LKL_MASK_I32;

  const size_t fwd = lkl_workspace_size(&p, 0);
  const size_t bwd = lkl_backward_workspace_size(&p, 0);
  const size_t n_t = (300 + 127) / 128;
  CHECK(fwd > 0 && fwd % 256 == 0);
  CHECK(bwd == fwd + 4 * (n_t * (n_t + 1) / 2) * 32768);  /* one 32 KB D tile per pair */
  /* the forward entry points need less: no per-row backward offsets */
  CHECK(lkl_forward_workspace_size(&p, 0) + 256 * ((8 * 4 * 300 + 255) / 256) == fwd);
  CHECK(lkl_selftest_bounded_wait(0, NULL) == LKL_ERR_BAD_SHAPE);

  void* fake = (void*)(uintptr_t)0x10000;
  float* ff = (float*)fake;
  /* null input, misaligned gradient, too-small backward workspace */
  CHECK(lkl_forward(NULL, fake, fake, fake, NULL, &p, ff, ff, ff, fake, 1 << 20, NULL) ==
        LKL_ERR_NULL_POINTER);
  CHECK(lkl_backward(fake, fake, ff, fake, fake, ff, NULL, &p, NULL, (float*)0x10004,
                     (float*)0x20000, fake, 1 << 20, NULL) == LKL_ERR_MISALIGNED);
  CHECK(lkl_backward(fake, fake, ff, fake, fake, ff, NULL, &p, NULL, ff, (float*)0x20000, fake,
                     fwd, NULL) == LKL_ERR_WORKSPACE);
  /* bad head dim, bad Hq / Hkv */
  lkl_problem q = p;
  q.Ds = 96;
  CHECK(lkl_forward(fake, fake, fake, fake, NULL, &q, ff, ff, ff, fake, 1 << 20, NULL) ==
        LKL_ERR_BAD_HEAD_DIM);
  q = p;
  q.Hkv_s = 3;
  CHECK(lkl_forward(fake, fake, fake, fake, NULL, &q, ff, ff, ff, fake, 1 << 20, NULL) ==
        LKL_ERR_BAD_SHAPE);

  /* strided: a stride that is not a multiple of 8 elements */
  lkl_strides st[4];
  for (int i = 0; i < 4; ++i) {
    st[i].b = 300 * 4 * 128; st[i].h = 128; st[i].t = 4 * 128 + 4;
  }
  CHECK(lkl_forward_strided(fake, fake, fake, fake, st, NULL, &p, ff, ff, ff, fake, 1 << 20,
                            NULL) == LKL_ERR_MISALIGNED);

  /* grouped: sizes grow with items; dq == dk needs qs == ks */
  lkl_group_item it[2];
  memset(it, 0, sizeof it);
  for (int i = 0; i < 2; ++i) {
    it[i].qs = fake; it[i].ks = (char*)fake + 0x1000; it[i].qt = fake; it[i].kt = fake;
    it[i].Hq = 4; it[i].Hkv_s = 2; it[i].Hkv_t = 2;
    it[i].lse_s = ff; it[i].lse_t = ff; it[i].dq = ff; it[i].dk = ff;
  }
  const size_t g1 = lkl_grouped_workspace_size(1, it, &p, 0, 0);
  const size_t g2 = lkl_grouped_workspace_size(2, it, &p, 0, 0);
  CHECK(g1 > 0 && g2 > g1);
  CHECK(lkl_backward_grouped(2, it, NULL, &p, NULL, fake, 1 << 20, NULL) == LKL_ERR_BAD_ALIAS);
  CHECK(lkl_forward_grouped(LKL_MAX_GROUP_ITEMS + 1, it, NULL, &p, ff, fake, 1 << 20, NULL) ==
        LKL_ERR_TOO_LARGE);

  printf("ok\n");
  return 0;
}
