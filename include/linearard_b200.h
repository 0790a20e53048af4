/*
 * linearard_b200.h -- C ABI of the B200 (sm_100a) attention-relation KL loss.
 *
 * The loss, for every (batch b, query head h, row i):
 *   KL_i = sum_j pt_ij * (log pt_ij - log ps_ij),
 *   ps_ij = softmax_j(sc_s * qs_i . ks_j),  pt_ij = softmax_j(sc_t * qt_i . kt_j),
 * over the columns j that are valid for row i (padding mask on row and column,
 * and j <= i when causal).  The kv head of query head h is h / (Hq / Hkv).
 * Every function returns the sum over rows, never an n x n map.
 *
 * Each entry point replaces one operator of LinearARD's
 * kernels/attention_KL package (paths are inside that project):
 *   lkl_lse          <- lse_stats_triton    kernels/attention_KL/kernel_A.py:190-265
 *   lkl_kl_forward   <- kl_forward_triton   kernels/attention_KL/kernel_B.py:249-391
 *   lkl_forward      <- AttnKLAlignFn.forward (A, A, B chained)
 *                                           kernels/attention_KL/integration.py:8-45
 *   lkl_backward     <- kl_backward_triton + the dloss chain rule of
 *                       AttnKLAlignFn.backward
 *                                           kernels/attention_KL/kernel_C.py:293-449,
 *                                           kernels/attention_KL/integration.py:48-67
 *
 * Conventions
 *  - Plain device pointers.  q/k tensors are contiguous [B, H, T, D] fp16 or
 *    bf16 (last stride 1), lse tensors contiguous fp32 [B, Hq, T].
 *  - mask: NULL (no padding) or a device pointer to a contiguous [B, T] array
 *    of LKL_MASK_* elements, nonzero = valid token.
 *  - Each entry point makes the device that owns its first q pointer current
 *    on the calling thread (cudaSetDevice) before any work; `stream` must
 *    belong to that device.  All work is enqueued on `stream`; nothing
 *    synchronises the host.
 *  - Scratch memory is caller-provided (`workspace`, `workspace_bytes`); query
 *    the size with lkl_workspace_size().  The library never allocates.
 *  - Return value: LKL_OK or an LKL_ERR_* code; lkl_status_string() names it.
 *    Validation mirrors the reference wrappers' assertions.
 */
#ifndef LINEARARD_B200_H_
#define LINEARARD_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define LKL_ABI_VERSION 6

/* element types of q/k tensors */
enum lkl_dtype { LKL_F16 = 0, LKL_BF16 = 1 };

/* element types accepted for the [B, T] padding mask (kernel_A.py:215-217) */
enum lkl_mask_dtype { LKL_MASK_BOOL = 0, LKL_MASK_U8 = 1, LKL_MASK_I32 = 2, LKL_MASK_I64 = 3 };

/* status codes */
enum lkl_status {
  LKL_OK = 0,
  LKL_ERR_NULL_POINTER = 1,     /* a required pointer is NULL                        */
  LKL_ERR_BAD_SHAPE = 2,        /* B/T/H mismatch, Hq % Hkv != 0, non-positive sizes */
  LKL_ERR_BAD_HEAD_DIM = 3,     /* D not in {8,16,32,64,128,256}                     */
  LKL_ERR_BAD_DTYPE = 4,        /* unknown lkl_dtype / lkl_mask_dtype                */
  LKL_ERR_MISALIGNED = 5,       /* pointer not aligned to its element size           */
  LKL_ERR_WORKSPACE = 6,        /* workspace NULL or smaller than *_workspace_size  */
  LKL_ERR_LAUNCH = 7,           /* a kernel launch or driver call failed             */
  LKL_ERR_NO_DEVICE = 8,        /* current device is not sm_100 / no CUDA device     */
  LKL_ERR_DEVICE_TIMEOUT = 9,   /* a device-side bounded wait expired (see below)    */
  LKL_ERR_BAD_ALIAS = 10,       /* dq == dk requires qs == ks and Hkv_s == Hq        */
  LKL_ERR_TOO_LARGE = 11,       /* a size exceeds what the entry point supports      */
  LKL_ERR_UNSUPPORTED = 12      /* strided inputs on a shape the tensor-core path
                                   does not cover (ABI version 3)                     */
};

/* Shape / option block shared by every entry point. */
typedef struct lkl_problem {
  int32_t B;          /* batch                                               */
  int32_t Hq;         /* query heads (student and teacher)                   */
  int32_t Hkv_s;      /* student key heads, Hq % Hkv_s == 0                   */
  int32_t Hkv_t;      /* teacher key heads, Hq % Hkv_t == 0                   */
  int32_t T;          /* sequence length                                     */
  int32_t Ds;         /* student head dim                                    */
  int32_t Dt;         /* teacher head dim                                    */
  int32_t dtype_s;    /* lkl_dtype of qs/ks                                  */
  int32_t dtype_t;    /* lkl_dtype of qt/kt                                  */
  int32_t causal;     /* nonzero: keep j <= i                                */
  int32_t mask_dtype; /* lkl_mask_dtype, ignored when mask == NULL           */
  float sm_scale_s;   /* <= 0 selects 1/sqrt(Ds)                              */
  float sm_scale_t;   /* <= 0 selects 1/sqrt(Dt)                              */
} lkl_problem;

/* ABI version (LKL_ABI_VERSION) and a static status description. */
int32_t lkl_abi_version(void);
const char* lkl_status_string(int32_t status);

/* Bytes of scratch the forward entry points (lkl_lse, lkl_kl_forward,
 * lkl_forward, lkl_forward_strided) need for problem `p` (has_mask != 0 when a
 * padding mask will be passed): one fp32 partial per 32 query rows of each
 * (batch, head) and, with a mask, the mask packed to one bit per token.
 * Always a multiple of 256.  Added in ABI version 6. */
size_t lkl_forward_workspace_size(const lkl_problem* p, int32_t has_mask);

/* lkl_forward_workspace_size plus the backward's per-row scratch (8 bytes per
 * (batch, head, row)): enough for every single-problem entry point except the
 * backward's D tiles (lkl_backward_workspace_size).  A multiple of 256. */
size_t lkl_workspace_size(const lkl_problem* p, int32_t has_mask);

/* Bytes of scratch lkl_backward needs: lkl_workspace_size plus, for the
 * tensor-core path (Ds, Dt in {8, 16, 32, 64, 128}), a buffer for the
 * 16-bit D tiles (p_s - p_t) that the dq pass hands to the dk pass: all of
 * them up to 8 GiB, beyond that the backward runs in chunks of kv heads or of
 * query-tile ranges (so the buffer stays bounded for any T).  A multiple of
 * 256.  Added in ABI version 2. */
size_t lkl_backward_workspace_size(const lkl_problem* p, int32_t has_mask);

/* Row log-sum-exp of one (q, k) pair -> lse [B, Hq, T] fp32.
 * Uses (Hkv_s, Ds, dtype_s, sm_scale_s) of `p`; rows removed by the mask get 0,
 * rows with no valid column get -inf (kernel_A.py:146-158).
 * Replaces lse_stats_triton, kernels/attention_KL/kernel_A.py:190-265. */
int32_t lkl_lse(const void* q, const void* k, const void* mask, const lkl_problem* p,
                float* lse, void* workspace, size_t workspace_bytes, void* stream);

/* KL sum given precomputed row LSEs -> *loss (fp32 device scalar, overwritten).
 * Replaces kl_forward_triton, kernels/attention_KL/kernel_B.py:249-391. */
int32_t lkl_kl_forward(const void* qs, const void* ks, const float* lse_s,
                       const void* qt, const void* kt, const float* lse_t,
                       const void* mask, const lkl_problem* p, float* loss,
                       void* workspace, size_t workspace_bytes, void* stream);

/* Fused forward: writes lse_s, lse_t [B, Hq, T] and *loss (sum of row KLs)
 * in one pass over the causal column tiles.  The loss is reduced
 * deterministically (fixed order).
 * Replaces AttnKLAlignFn.forward, kernels/attention_KL/integration.py:8-45. */
int32_t lkl_forward(const void* qs, const void* ks, const void* qt, const void* kt,
                    const void* mask, const lkl_problem* p,
                    float* lse_s, float* lse_t, float* loss,
                    void* workspace, size_t workspace_bytes, void* stream);

/* Backward: dq [B, Hq, T, Ds] and dk [B, Hkv_s, T, Ds], fp32, both multiplied
 * by *dloss (a device fp32 scalar; NULL means 1).  dq and dk are overwritten.
 * If dk == dq (allowed only when qs == ks and Hkv_s == Hq, the symmetric call
 * attn_kl_align(qs, qs, qt, qt) made by train.py:380-402), the buffer receives
 * dq + dk, the gradient of the shared tensor.
 * Replaces kl_backward_triton (kernels/attention_KL/kernel_C.py:293-449) and
 * the chain rule in AttnKLAlignFn.backward (integration.py:48-67).
 * Workspace: lkl_backward_workspace_size(p, mask != NULL) bytes give the
 * fastest plan.  Less also works, down to lkl_workspace_size plus one
 * query-tile row of D tiles of one kv group ((Hq / Hkv_s) * ceil(T / 128)
 * tiles of 32 KB) for the tensor-core shapes, in more and smaller chunks;
 * below that LKL_ERR_WORKSPACE. */
int32_t lkl_backward(const void* qs, const void* ks, const float* lse_s,
                     const void* qt, const void* kt, const float* lse_t,
                     const void* mask, const lkl_problem* p, const float* dloss,
                     float* dq, float* dk, void* workspace, size_t workspace_bytes,
                     void* stream);

/* ---- Strided inputs (ABI version 3) ----
 * The hot-path entry points above take contiguous [B, H, T, D] tensors, as the
 * reference wrappers require (kernel_B.py:289-290).  These two take each of
 * qs, ks, qt, kt as a [B, H, T, D] view with element strides (b, h, t) and a
 * d stride of 1, e.g. the transposed [B, T, H, D] projections that an
 * attention hook sees before it calls .contiguous() (train.py:133-142).  The
 * tensors are read in place through TMA, so no copy is made.
 * Requirements: every stride a positive multiple of 8 elements and every base
 * pointer 16-byte aligned (LKL_ERR_MISALIGNED otherwise); the tensor-core path
 * (sm_100, Ds and Dt in {8, 16, 32, 64, 128}), LKL_ERR_UNSUPPORTED otherwise.  Outputs (lse, loss, dq, dk) are contiguous,
 * as in lkl_forward / lkl_backward; everything else is the same.
 * `strides` points to 4 entries: qs, ks, qt, kt. */
typedef struct lkl_strides {
  int64_t b, h, t;    /* element strides of the batch, head and token dims */
} lkl_strides;

int32_t lkl_forward_strided(const void* qs, const void* ks, const void* qt, const void* kt,
                            const lkl_strides* strides, const void* mask,
                            const lkl_problem* p, float* lse_s, float* lse_t, float* loss,
                            void* workspace, size_t workspace_bytes, void* stream);

int32_t lkl_backward_strided(const void* qs, const void* ks, const float* lse_s,
                             const void* qt, const void* kt, const float* lse_t,
                             const lkl_strides* strides, const void* mask,
                             const lkl_problem* p, const float* dloss, float* dq, float* dk,
                             void* workspace, size_t workspace_bytes, void* stream);

/* ---- Grouped calls (ABI version 4) ----
 * One call for many (relation, layer) items of one sequence, as the training
 * loop issues them (train.py:369-402: 3 relations x L layers per
 * micro-batch).  The forward is ONE launch over every item's row tiles and the
 * backward one dq and one dk launch per chunk of kv groups across items, so
 * there is one tail per call instead of one per item.
 * `shared` gives what the items have in common (B, T, Ds, Dt, dtypes, causal,
 * mask dtype, scales; its Hq / Hkv_s / Hkv_t are ignored); the mask is shared.
 * Every item must be on the tensor-core path (16-byte-aligned inputs,
 * contiguous or strided, Ds and Dt in {8, 16, 32, 64, 128}), else LKL_ERR_UNSUPPORTED.  At most LKL_MAX_GROUP_ITEMS items (LKL_ERR_TOO_LARGE).
 * The item table (tensor maps and pointers, 576 B per item) goes to the device
 * inside the call through a pinned host ring that the library allocates once
 * (8 MiB, the only host allocation it makes), so the call does not wait for
 * the stream.  Because the table is read from that ring when the copy runs,
 * grouped calls must not be captured into CUDA graphs (the single-problem
 * entry points have no such restriction).
 * Results equal the per-item calls: lkl_forward_grouped writes each item's
 * lse_s, lse_t and losses[i] (device fp32 [n], the row-KL sum of item i);
 * lkl_backward_grouped reads them and writes each item's dq and dk (dq == dk:
 * fused, needs qs == ks and Hkv_s == Hq), each multiplied by dlosses[i]
 * (device fp32 [n]; NULL = 1). */
#define LKL_MAX_GROUP_ITEMS 1024

typedef struct lkl_group_item {
  const void* qs;      /* [B, Hq, T, Ds]     */
  const void* ks;      /* [B, Hkv_s, T, Ds]  */
  const void* qt;      /* [B, Hq, T, Dt]     */
  const void* kt;      /* [B, Hkv_t, T, Dt]  */
  int32_t Hq, Hkv_s, Hkv_t;
  int32_t strided;     /* 0: contiguous inputs; 1: use `strides` (ABI version 5) */
  float* lse_s;        /* [B, Hq, T] fp32    */
  float* lse_t;
  float* dq;           /* [B, Hq, T, Ds] fp32 (backward) */
  float* dk;           /* [B, Hkv_s, T, Ds] fp32 (backward) */
  lkl_strides strides[4];  /* qs, ks, qt, kt element strides when `strided`, as
                              for lkl_forward_strided (multiples of 8 elements) */
} lkl_group_item;

/* Scratch for a grouped forward (backward = 0) or backward (backward = 1):
 * partials, packed mask, LSE offsets, the item table and, for the backward,
 * the D-tile buffer (all tiles up to 8 GiB; at least one kv group). */
size_t lkl_grouped_workspace_size(int32_t n, const lkl_group_item* items,
                                  const lkl_problem* shared, int32_t has_mask,
                                  int32_t backward);

int32_t lkl_forward_grouped(int32_t n, const lkl_group_item* items, const void* mask,
                            const lkl_problem* shared, float* losses, void* workspace,
                            size_t workspace_bytes, void* stream);

int32_t lkl_backward_grouped(int32_t n, const lkl_group_item* items, const void* mask,
                             const lkl_problem* shared, const float* dlosses, void* workspace,
                             size_t workspace_bytes, void* stream);

/* Host-only query (no device work): how many chunks (one dq and one dk launch
 * each) lkl_backward splits problem `p` into with `workspace_bytes` of scratch
 * (fused != 0: dq == dk).  *n_chunks = 0 for shapes the CUDA-core kernels
 * serve (one launch, no D buffer).  LKL_ERR_WORKSPACE below the minimum.
 * Added in ABI version 5. */
int32_t lkl_backward_plan(const lkl_problem* p, int32_t has_mask, size_t workspace_bytes,
                          int32_t fused, int32_t* n_chunks);

/* Device-side error word of the CURRENT device: the bounded waits inside the
 * tensor-core kernels set it instead of hanging.  Reads (synchronously) and
 * clears it; returns LKL_OK or LKL_ERR_DEVICE_TIMEOUT.  The word is per
 * device: a process that drives several GPUs calls this once with each of
 * them current (cudaSetDevice). */
int32_t lkl_device_status(void);

/* Diagnostic (ABI version 6; no counterpart in the reference): launches, on
 * `stream` of the current device, one CTA whose mbarrier wait can never
 * complete, using the same bounded wait as the tensor-core kernels but with a
 * limit of `limit_us` microseconds (1 .. 2,000,000; LKL_ERR_BAD_SHAPE
 * otherwise).  The wait gives up, sets the device error word and the kernel
 * returns, so after the stream is synchronised lkl_device_status() reports
 * LKL_ERR_DEVICE_TIMEOUT (and clears it) and the context stays usable.  For
 * tests of the failure path; it touches no other state. */
int32_t lkl_selftest_bounded_wait(uint32_t limit_us, void* stream);

/* Which implementation the last lkl_forward / lkl_backward call on this host
 * thread dispatched to: 1 = sm_100a tensor-core kernels, 0 = generic CUDA-core
 * kernels (head dims or alignments the tensor-core kernels do not cover). */
int32_t lkl_last_path(void);

/* cudaError_t value (as int) of the last CUDA call that made an entry point on
 * this host thread return LKL_ERR_LAUNCH; 0 if none.  Diagnostic only. */
int32_t lkl_last_cuda_error(void);

/* Force the generic CUDA-core kernels (nonzero) or allow the tensor-core path
 * (0, the default); process-wide.  For parity tests that cross-check paths. */
void lkl_set_force_generic(int32_t force);

/* Size of the scratch array that lkl_forward_noalloc uses on each device. */
#define LKL_NOALLOC_SCRATCH_BYTES (1u << 20)

/* lkl_forward without a workspace argument and without any device allocation.
 * No counterpart in the reference: LinearARD's wrappers always allocate their
 * outputs and scratch through PyTorch.  This is for callers that cannot
 * allocate device memory -- a C/Go/Java binding that only receives pointers
 * from a framework owning the memory pool, or code that must not call
 * cudaMalloc mid-step because it can synchronise the device.  The caller still
 * passes every input and output (lse_s, lse_t, loss) exactly as for
 * lkl_forward; the scratch comes from a fixed LKL_NOALLOC_SCRATCH_BYTES array
 * inside the library, which every GPU that loads the library keeps until the
 * process exits.
 *  - Limit: problems whose lkl_forward_workspace_size() exceeds
 *    LKL_NOALLOC_SCRATCH_BYTES are refused with LKL_ERR_TOO_LARGE (use
 *    lkl_forward with a workspace).  That size is 4 bytes per 32 query rows of
 *    each (batch, head), rounded up to 256, plus with a mask 4 bytes per 32
 *    tokens of each sequence, rounded up to 256: e.g. 8 sequences x 32 heads x
 *    32K tokens without a mask (exactly 1 MiB), or one sequence of 32 heads x
 *    248K tokens with a mask.
 *  - The first call on each device looks up the array's device address
 *    (cudaGetSymbolAddress, with that device current); make that first call
 *    before any stream capture.
 *  - All calls on a device share the one array: calls that can overlap on the
 *    GPU (different streams, or host threads without ordering) race on it and
 *    must be serialised by the caller.  Each call rewrites every byte it
 *    reads, so nothing needs clearing in between. */
int32_t lkl_forward_noalloc(const void* qs, const void* ks, const void* qt, const void* kt,
                            const void* mask, const lkl_problem* p,
                            float* lse_s, float* lse_t, float* loss, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LINEARARD_B200_H_ */
