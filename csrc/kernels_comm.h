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
constexpr int PAD_AGF = PAD_NORMV + PAD_MAXW;               // [PAD_MAXW]
constexpr int PAD_WORDS = PAD_AGF + PAD_MAXW;

void* ipc_alloc(size_t nbytes, std::string* handle);
void ipc_free(void* p);
void* ipc_open(const std::string& handle);
void ipc_close(void* p);

void launch_grad_to_bf16(const float* g, void* out, int64_t n, cudaStream_t st);
// Reduce-scatter of one bucket.  mode 0 (pull): cast grad into this rank's
// send buffer `my_buf`, then read the owned shard from every peer's send
// buffer with TMA bulk copies.  mode 1 (push): cast + store each owner's part
// into the owner's receive buffer, then reduce locally.  `peers_buf` holds the
// peers' send (pull) or receive (push) buffers.  done_ctr: int [PAD_MAXB].
void launch_rs_bucket(int mode, const float* grad, const uint64_t* peers_buf, void* my_buf, const uint64_t* peer_pads,
                      int* my_pad, int* done_ctr, int rank, int W, int bucket, int epoch, int64_t lo, int64_t len,
                      float* rgrad, float* sumsq, int ctas, int* status, int64_t wait_ns, cudaStream_t st);
void launch_norm_exchange(const uint64_t* peer_pads, int* my_pad, int rank, int W, int epoch, const float* sumsq,
                          float max_norm, float* coef, float* norm_out, int* status, int64_t wait_ns,
                          cudaStream_t st);
void launch_adamw_allgather(const int64_t* buckets, int nb, int rank, int W, const float* rgrad, float* master,
                            float* m, float* v, const uint64_t* peers_param, const uint64_t* peer_pads, int* my_pad,
                            int epoch, float lr, float b1, float b2, float eps, float wd, float bc1, float bc2,
                            const float* coef, int* done_ctr, int* status, int64_t wait_ns, cudaStream_t st);

// NVLink microbenchmark kernels (p2pbench.cu): move `bytes` bytes from/to a
// (peer) buffer with SM loads / stores or bulk copies; nothing waits on a peer.
void launch_p2p_read(const void* src, int64_t bytes, void* sink, int ctas, int threads, int unr, cudaStream_t st);
void launch_p2p_write(void* dst, int64_t bytes, int ctas, int threads, int unr, cudaStream_t st);
void launch_p2p_bulk(bool write, void* peer, int64_t bytes, int ctas, int chunk, int stages, int* status,
                     cudaStream_t st);
}  // namespace oxi
