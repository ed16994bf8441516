// Allocation-free entry point for the fused lm_head + cross-entropy forward:
// the C interface.  It has no counterpart in the reference project.
//
// Who it is for: callers that cannot allocate device memory themselves, such
// as a host runtime that reserves all of its device memory up front and
// forbids further cudaMalloc, or code that must not let cudaMalloc / cudaFree
// synchronise the device in the middle of its work.  The caller passes only
// inputs and outputs; the scratch the kernels need is one fixed file-scope
// device array inside the library (about 8.3 MB on every GPU that loads it,
// held until the process exits).
//
// Limits: M <= OXI_CE_NOALLOC_MAX_ROWS rows and
// M * ceil(V / 256) <= OXI_CE_NOALLOC_MAX_PARTIALS per-tile partials.  Larger
// calls return OXI_CE_NOALLOC_TOO_LARGE before anything is launched; split the
// rows into blocks.
//
// Set-up: the first call on a device (per CUDA context) looks up the device
// address of the scratch array with that device current and caches it; make
// that first call before any stream capture.  A context that is destroyed and
// recreated (cudaDeviceReset) is noticed through its context id and the
// address is looked up again.
//
// Sharing: every call uses the same scratch array, which keeps the contents of
// the last call (the entry point clears what must start at zero).  Calls whose
// kernels overlap on the GPU (different streams without ordering between them)
// race on the array and give wrong results: order them.
//
// Kernel errors: the kernels run asynchronously, so a bounded pipeline wait
// that ran out of time inside them cannot be reported by the return code of
// the call that launched them.  After synchronising the stream, call
// oxi_linear_ce_noalloc_status(): it returns OXI_CE_NOALLOC_KERNEL_ERROR (and
// the device status word) when the last call's kernels recorded an error, in
// which case loss and lse are not valid.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#define OXI_CE_NOALLOC_MAX_ROWS (1 << 16)
#define OXI_CE_NOALLOC_MAX_PARTIALS (1 << 20)

enum {
  OXI_CE_NOALLOC_OK = 0,
  OXI_CE_NOALLOC_TOO_LARGE = 1,     // sizes beyond the fixed scratch
  OXI_CE_NOALLOC_BAD_ARGUMENT = 2,  // null pointer, bad size, stride or alignment
  OXI_CE_NOALLOC_CUDA_ERROR = 3,    // a CUDA runtime call or launch failed
  OXI_CE_NOALLOC_KERNEL_ERROR = 4,  // (status query) the kernels recorded an error
};

#ifdef __cplusplus
extern "C" {
#endif

// x bf16 [M, K] (row stride ldx elements), w bf16 [V, K] (row stride ldw),
// targets int64 [M] (negative = ignored row, loss 0); outputs loss f32 [M]
// (per-row cross-entropy) and lse f32 [M] (per-row log-sum-exp of the logits).
// Work is queued on `stream`; the return code covers argument checks and
// launches only (see oxi_linear_ce_noalloc_status).
int oxi_linear_ce_fwd_noalloc(const void* x, int64_t M, int64_t K, int64_t ldx, const void* w, int64_t V,
                              int64_t ldw, const int64_t* targets, float* loss, float* lse, cudaStream_t stream);

// Reads the device status word the last call on the current device left in
// the scratch array (a blocking copy: synchronise the call's stream first).
// Returns OXI_CE_NOALLOC_OK when it is zero, OXI_CE_NOALLOC_KERNEL_ERROR when
// the kernels recorded an error (its code in *status_out when non-null), or
// OXI_CE_NOALLOC_CUDA_ERROR when the copy failed.
int oxi_linear_ce_noalloc_status(int* status_out);

// Message for the last non-zero return code of the calling thread.
const char* oxi_linear_ce_noalloc_last_error(void);

// Largest supported sizes, for callers that split their problem.
void oxi_linear_ce_noalloc_limits(int64_t* max_rows, int64_t* max_partials);

#ifdef __cplusplus
}
#endif
