// lkl_forward_noalloc: the fused forward for callers that cannot allocate
// device memory.
//
// Who needs it: a host that only ever receives device pointers from someone
// else (a C, Go or Java binding sitting under a framework that owns the memory
// pool) has no allocator to hand a workspace from, and a caller in the middle
// of a latency-critical step may not call cudaMalloc either, because it can
// synchronise the device and break a memory budget reserved up front.
// lkl_forward needs a small workspace (per-tile KL partial sums and the packed
// padding mask); this variant takes that scratch from a fixed array compiled
// into the library instead, so the caller passes only inputs and outputs.
//
// The array is a file-scope __device__ object: every GPU that loads the
// library holds kNoAllocScratchBytes of it until the process exits.  Host code
// may not pass the array's name to a kernel (on the host it is only a stand-in
// symbol, not a device address), so the first call on each device looks up
// its device address with cudaGetSymbolAddress while that device is current
// and caches it.
#include <mutex>

#include "lkl_common.cuh"

namespace {

// LKL_NOALLOC_SCRATCH_BYTES (1 MiB) holds what the forward needs
// (lkl_forward_workspace_size): per-tile partials (4 B per 32 query rows of
// each batch x head, rounded up to 256 B) plus, with a mask, the packed mask
// (4 B per 32 tokens of each sequence, rounded up to 256 B).  That is enough
// for 8 sequences x 32 heads x 32K tokens without a mask (exactly 1 MiB), or
// one sequence of 32 heads x 248K tokens with a mask.
constexpr size_t kNoAllocScratchBytes = LKL_NOALLOC_SCRATCH_BYTES;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mutex;
void* g_noalloc_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device (looked up once
// per device, with that device current), or nullptr on failure.
void* noalloc_scratch_for_current_device(int32_t* status) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    *status = LKL_ERR_NO_DEVICE;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      *status = LKL_ERR_LAUNCH;
      return nullptr;
    }
    g_noalloc_ptr[dev] = p;
  }
  *status = LKL_OK;
  return g_noalloc_ptr[dev];
}

}  // namespace

extern "C" {

int32_t lkl_forward_noalloc(const void* qs, const void* ks, const void* qt, const void* kt,
                            const void* mask, const lkl_problem* p, float* lse_s, float* lse_t,
                            float* loss, void* stream) {
  if (!p) return LKL_ERR_NULL_POINTER;
  // Size limit first, so an oversized problem is refused before any CUDA call.
  const size_t need = lkl_forward_workspace_size(p, mask != nullptr);
  if (need > kNoAllocScratchBytes) return LKL_ERR_TOO_LARGE;
  int32_t status = LKL_OK;
  void* scratch = nullptr;
  // the scratch address is per device: look it up on the device of the inputs
  if (need > 0 && qs && !bind_device_of(qs)) return LKL_ERR_NO_DEVICE;
  if (need > 0) {
    scratch = noalloc_scratch_for_current_device(&status);
    if (!scratch) return status;
  }
  // Every region of the scratch that the forward reads is written earlier in
  // the same call (mask words by the packing kernel, one partial per CTA by
  // the forward kernel), so nothing needs clearing between calls.
  return lkl_forward(qs, ks, qt, kt, mask, p, lse_s, lse_t, loss, scratch,
                     kNoAllocScratchBytes, stream);
}

}  // extern "C"
