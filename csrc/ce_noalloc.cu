// Allocation-free entry point for the fused lm_head + cross-entropy forward.
//
// This entry point has no counterpart in the reference project; it exists for
// callers of this library that cannot allocate device memory on their own:
// for example a host runtime that reserves all of its device memory up front
// and forbids further cudaMalloc, or a caller that must not let cudaMalloc /
// cudaFree synchronise the device in the middle of its work.  Such a caller
// passes only its inputs and outputs; the scratch the kernels need lives in a
// file-scope device array of fixed size instead of a per-call allocation.
// The interface, limits, return codes and sharing rules are declared in
// ce_noalloc.h.
//
// Set-up: the first call on a device looks up the device address of the
// scratch array (cudaGetSymbolAddress, with that device current) and caches
// it together with the id of the current CUDA context; a call under a new
// context (after cudaDeviceReset) looks it up again.  Make the first call on
// each device before any stream capture.
//
// Nothing here calls cudaMalloc, cudaFree or an allocating library routine.
#include <cuda.h>

#include <atomic>
#include <cstdio>
#include <cstring>
#include <exception>
#include <mutex>

#include "ce_noalloc.h"
#include "gemm_kernel.cuh"
#include "kernels.h"
#include "kernels_ew.h"

namespace {

struct CeScratch {
  float part_max[OXI_CE_NOALLOC_MAX_PARTIALS];
  float part_sum[OXI_CE_NOALLOC_MAX_PARTIALS];
  float tgt_logit[OXI_CE_NOALLOC_MAX_ROWS];
  int status[4];
};

static __device__ __align__(256) CeScratch g_ce_scratch;

constexpr int kMaxDevices = 128;

// Per device: the scratch address and the id of the context it was looked up in.
struct ScratchSlot {
  CeScratch* addr = nullptr;
  unsigned long long ctx_id = 0;
};
ScratchSlot g_slots[kMaxDevices];
std::mutex g_slots_mu;

thread_local char g_last_error[512];

// Driver calls through the runtime's entry-point query, so the library does
// not link libcuda directly (it still imports on a machine without a driver).
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
using CtxGetIdFn = CUresult (*)(CUcontext, unsigned long long*);

template <typename F>
F driver_fn(const char* name, int version) {
  void* ptr = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPointByVersion(name, &ptr, version, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess)
    return nullptr;
  return reinterpret_cast<F>(ptr);
}

int set_error(int code, const char* msg) {
  std::snprintf(g_last_error, sizeof(g_last_error), "%s", msg);
  return code;
}

// Device address of the scratch array on the current device (host code may
// not use the symbol itself as a device pointer).
int scratch_for_current_device(CeScratch** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(OXI_CE_NOALLOC_CUDA_ERROR, cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return set_error(OXI_CE_NOALLOC_BAD_ARGUMENT, "device ordinal out of range");
  // make the device's primary context current (CUDA 12 initialises it here), then identify it
  e = cudaSetDevice(dev);
  if (e != cudaSuccess) return set_error(OXI_CE_NOALLOC_CUDA_ERROR, cudaGetErrorString(e));
  std::lock_guard<std::mutex> lk(g_slots_mu);
  static const CtxGetCurrentFn get_current = driver_fn<CtxGetCurrentFn>("cuCtxGetCurrent", 4000);
  static const CtxGetIdFn get_id = driver_fn<CtxGetIdFn>("cuCtxGetId", 12000);
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr ||
      get_id(ctx, &id) != CUDA_SUCCESS)
    return set_error(OXI_CE_NOALLOC_CUDA_ERROR, "no current CUDA context");
  ScratchSlot& slot = g_slots[dev];
  if (slot.addr == nullptr || slot.ctx_id != id) {
    void* addr = nullptr;
    e = cudaGetSymbolAddress(&addr, g_ce_scratch);
    if (e != cudaSuccess || addr == nullptr)
      return set_error(OXI_CE_NOALLOC_CUDA_ERROR, e != cudaSuccess ? cudaGetErrorString(e) : "null symbol address");
    slot.addr = static_cast<CeScratch*>(addr);
    slot.ctx_id = id;
  }
  *out = slot.addr;
  return OXI_CE_NOALLOC_OK;
}

}  // namespace

extern "C" {

__attribute__((visibility("default"))) const char* oxi_linear_ce_noalloc_last_error(void) { return g_last_error; }

__attribute__((visibility("default"))) void oxi_linear_ce_noalloc_limits(int64_t* max_rows, int64_t* max_partials) {
  if (max_rows) *max_rows = OXI_CE_NOALLOC_MAX_ROWS;
  if (max_partials) *max_partials = OXI_CE_NOALLOC_MAX_PARTIALS;
}

__attribute__((visibility("default"))) int oxi_linear_ce_fwd_noalloc(const void* x, int64_t M, int64_t K,
                                                                     int64_t ldx, const void* w, int64_t V,
                                                                     int64_t ldw, const int64_t* targets,
                                                                     float* loss, float* lse, cudaStream_t stream) {
  g_last_error[0] = '\0';
  if (M < 0 || K <= 0 || V <= 0 || !x || !w || !targets || !loss || !lse || ldx < K || ldw < K)
    return set_error(OXI_CE_NOALLOC_BAD_ARGUMENT, "invalid pointer or size argument");
  if (M == 0) return OXI_CE_NOALLOC_OK;
  const int64_t tiles_n = (V + oxi::BN - 1) / oxi::BN;
  if (M > OXI_CE_NOALLOC_MAX_ROWS || M * tiles_n > OXI_CE_NOALLOC_MAX_PARTIALS) {
    char buf[256];
    std::snprintf(buf, sizeof(buf),
                  "problem too large for the fixed scratch: M=%lld rows, M*ceil(V/256)=%lld partials "
                  "(limits %d rows, %d partials); split the rows into smaller blocks",
                  (long long)M, (long long)(M * tiles_n), OXI_CE_NOALLOC_MAX_ROWS, OXI_CE_NOALLOC_MAX_PARTIALS);
    return set_error(OXI_CE_NOALLOC_TOO_LARGE, buf);
  }
  CeScratch* s = nullptr;
  int rc = scratch_for_current_device(&s);
  if (rc) return rc;
  try {
    // Target logits of rows whose target falls in no tile are never written by
    // the GEMM epilogue: clear them (and the status word) first.
    cudaError_t e = cudaMemsetAsync(s->tgt_logit, 0, M * sizeof(float), stream);
    if (e == cudaSuccess) e = cudaMemsetAsync(s->status, 0, sizeof(s->status), stream);
    if (e != cudaSuccess) return set_error(OXI_CE_NOALLOC_CUDA_ERROR, cudaGetErrorString(e));
    oxi::Mat mx{x, M, K, ldx}, mw{w, V, K, ldw};
    oxi::launch_gemm_ce(mx, mw, targets, s->part_max, s->part_sum, s->tgt_logit, nullptr, 0, 1.0f, s->status,
                        stream);
    oxi::launch_ce_finish(s->part_max, s->part_sum, (int)tiles_n, s->tgt_logit, targets, lse, loss, M, stream);
  } catch (const std::exception& ex) {
    // a failed launch or runtime call leaves a CUDA error behind; a failed
    // shape / stride / alignment check does not
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
      char buf[512];
      std::snprintf(buf, sizeof(buf), "%s (%s)", cudaGetErrorString(e), ex.what());
      return set_error(OXI_CE_NOALLOC_CUDA_ERROR, buf);
    }
    return set_error(OXI_CE_NOALLOC_BAD_ARGUMENT, ex.what());
  }
  return OXI_CE_NOALLOC_OK;
}

__attribute__((visibility("default"))) int oxi_linear_ce_noalloc_status(int* status_out) {
  g_last_error[0] = '\0';
  CeScratch* s = nullptr;
  int rc = scratch_for_current_device(&s);
  if (rc) return rc;
  int word = 0;
  // a blocking device-to-host copy of one int from the fixed array (no allocation)
  const cudaError_t e = cudaMemcpy(&word, s->status, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return set_error(OXI_CE_NOALLOC_CUDA_ERROR, cudaGetErrorString(e));
  if (status_out) *status_out = word;
  if (word != 0) {
    char buf[128];
    std::snprintf(buf, sizeof(buf), "the kernels of the last call recorded error code %d", word);
    return set_error(OXI_CE_NOALLOC_KERNEL_ERROR, buf);
  }
  return OXI_CE_NOALLOC_OK;
}

}  // extern "C"
