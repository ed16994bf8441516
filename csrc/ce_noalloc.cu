// Allocation-free entry point for the fused lm_head + cross-entropy forward.
//
// This entry point has no counterpart in the reference project; it exists for
// callers of this library that cannot allocate device memory on their own:
// for example a host runtime that reserves all of its device memory up front
// and forbids further cudaMalloc, or a caller that must not let cudaMalloc /
// cudaFree synchronise the device in the middle of its work.  Such a caller
// passes only its inputs and outputs; the scratch the kernels need lives in a
// file-scope device array of fixed size instead of a per-call allocation.
//
//   int oxi_linear_ce_fwd_noalloc(x, M, K, ldx, w, V, ldw, targets,
//                                 loss, lse, stream)
//
//   x       bf16 [M, K] row stride ldx (elements)     hidden states
//   w       bf16 [V, K] row stride ldw                lm_head weight
//   targets int64 [M]; a negative target marks an ignored row (loss 0)
//   loss    f32 [M] per-row cross-entropy (output)
//   lse     f32 [M] per-row log-sum-exp of the logits (output)
//
// Limits: M <= OXI_CE_NOALLOC_MAX_ROWS and M * ceil(V / 256) <=
// OXI_CE_NOALLOC_MAX_PARTIALS.  Larger problems are rejected with
// OXI_CE_NOALLOC_TOO_LARGE before anything is launched; split them into row
// blocks.  The scratch array takes about 8.3 MB on every GPU that loads this
// library and stays there until the process exits.
//
// Set-up: the first call on a device looks up the device address of the
// scratch array (cudaGetSymbolAddress, with that device current) and caches
// it; make that first call on each device before any stream capture.
//
// Sharing: every call uses the same scratch array, which keeps the contents
// of the last call (this entry point clears what must start at zero).  Calls
// whose kernels overlap on the GPU (different streams, no ordering between
// them) race on the scratch array and give wrong results; order them.
//
// Nothing here calls cudaMalloc, cudaFree or an allocating library routine.
#include <atomic>
#include <cstdio>
#include <cstring>
#include <exception>

#include "gemm_kernel.cuh"
#include "kernels.h"
#include "kernels_ew.h"

#define OXI_CE_NOALLOC_MAX_ROWS (1 << 16)
#define OXI_CE_NOALLOC_MAX_PARTIALS (1 << 20)

enum : int {
  OXI_CE_NOALLOC_OK = 0,
  OXI_CE_NOALLOC_TOO_LARGE = 1,
  OXI_CE_NOALLOC_BAD_ARGUMENT = 2,
  OXI_CE_NOALLOC_CUDA_ERROR = 3,
};

namespace {

struct CeScratch {
  float part_max[OXI_CE_NOALLOC_MAX_PARTIALS];
  float part_sum[OXI_CE_NOALLOC_MAX_PARTIALS];
  float tgt_logit[OXI_CE_NOALLOC_MAX_ROWS];
  int status[4];
};

static __device__ __align__(256) CeScratch g_ce_scratch;

constexpr int kMaxDevices = 128;
std::atomic<CeScratch*> g_scratch_addr[kMaxDevices];

thread_local char g_last_error[512];

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
  CeScratch* p = g_scratch_addr[dev].load(std::memory_order_acquire);
  if (!p) {
    void* addr = nullptr;
    e = cudaGetSymbolAddress(&addr, g_ce_scratch);
    if (e != cudaSuccess || addr == nullptr)
      return set_error(OXI_CE_NOALLOC_CUDA_ERROR, e != cudaSuccess ? cudaGetErrorString(e) : "null symbol address");
    p = static_cast<CeScratch*>(addr);
    g_scratch_addr[dev].store(p, std::memory_order_release);
  }
  *out = p;
  return OXI_CE_NOALLOC_OK;
}

}  // namespace

extern "C" {

// Message for the last non-zero return code of this thread.
__attribute__((visibility("default"))) const char* oxi_linear_ce_noalloc_last_error() { return g_last_error; }

// Largest supported sizes (for callers that split their problem).
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
    return set_error(OXI_CE_NOALLOC_BAD_ARGUMENT, ex.what());
  }
  return OXI_CE_NOALLOC_OK;
}

}  // extern "C"
