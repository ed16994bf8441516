// NVLink data-parallel runtime (comm.cu): IPC buffers and fused collectives.
#pragma once
#include <cstdint>
#include <string>
#include <cuda_runtime.h>

namespace oxi {

// Peer waits give up after wait_ns nanoseconds, record OXI_ERR_TIMEOUT_PEER in
// the status word, skip their work and return.

// Signal pad layout (int32 words; PAD_NORMV holds f32 values).
constexpr int PAD_MAXW = 16;
constexpr int PAD_MAXB = 512;
constexpr int PAD_READY = 0;                                // [PAD_MAXB][PAD_MAXW]
constexpr int PAD_NORMF = PAD_READY + PAD_MAXB * PAD_MAXW;  // [PAD_MAXW]
constexpr int PAD_NORMV = PAD_NORMF + PAD_MAXW;             // [PAD_MAXW] f32
constexpr int PAD_AGF = PAD_NORMV + PAD_MAXW;               // [PAD_MAXB][PAD_MAXW]
constexpr int PAD_WORDS = PAD_AGF + PAD_MAXB * PAD_MAXW;

void* ipc_alloc(size_t nbytes, std::string* handle);
void ipc_free(void* p);
void* ipc_open(const std::string& handle);
void ipc_close(void* p);

// bf16 copy of an f32 gradient range; `zero` clears the source in the same pass.
void launch_grad_to_bf16(float* g, void* out, int64_t n, bool zero, cudaStream_t st);
// f32 copy of a bf16 shard and its sum of squares (added to *sumsq).
void launch_bf16_to_f32_sumsq(const void* src, float* dst, int64_t n, float* sumsq, cudaStream_t st);
// Reduce-scatter of one bucket.  mode 0 (pull): cast grad into this rank's
// send buffer `my_buf`, then read the owned shard from every peer's send
// buffer.  mode 1 (push): cast + store each owner's part into the owner's
// receive buffer, then reduce locally.  mode 2 (NVLS): cast into `my_buf`,
// then read the owned shard through the multicast address `mc_buf` with
// multimem.ld_reduce.  `peers_buf` holds the peers' send (pull) or receive
// (push) buffers.  done_ctr: int [PAD_MAXB].  zero_grad clears the f32
// gradient range as it is read.
void launch_rs_bucket(int mode, float* grad, bool zero_grad, const uint64_t* peers_buf, void* my_buf, void* mc_buf,
                      const uint64_t* peer_pads, int* my_pad, int* done_ctr, int rank, int W, int bucket, int epoch,
                      int64_t lo, int64_t len, float* rgrad, float* sumsq, int ctas, int* status, int64_t wait_ns,
                      cudaStream_t st);
// skip (nullable): a non-zero word skips the update (NaN coefficient), the norm stays as measured.
void launch_norm_exchange(const uint64_t* peer_pads, int* my_pad, int rank, int W, int epoch, const float* sumsq,
                          float max_norm, float* coef, float* norm_out, int* status, int64_t wait_ns, const int* skip,
                          cudaStream_t st);
// AdamW on this rank's shard of bucket [lo, lo + len) (shard state at offset
// `so`) and the bf16 all-gather of the result: mode 0/1 bulk-stores it into the
// first `ndst` parameter buffers of `peers_param` (ndst = 1: only this rank's,
// for a library all-gather afterwards), mode 2 multicasts it through
// `mc_param`.  With peer_pads the last CTA publishes the bucket's epoch in
// every peer's pad (ag[bucket][rank]).
void launch_adamw_ag_bucket(int mode, int64_t lo, int64_t len, int64_t so, int W, int rank, int ndst,
                            const float* rgrad, float* master, float* m, float* v, const uint64_t* peers_param,
                            void* mc_param, const uint64_t* peer_pads, int bucket, int epoch, float lr, float b1,
                            float b2, float eps, float wd, float bc1, float bc2, const float* coef, int* done_ctr,
                            int* status, int ctas, cudaStream_t st);
// One thread waits (bounded) until ag[bucket][*] >= epoch in this rank's pad.
void launch_ag_wait(int* my_pad, int W, int bucket, int epoch, int* status, int64_t wait_ns, cudaStream_t st);

}  // namespace oxi
