// NVLink microbenchmark kernels (p2pbench.cu): move `bytes` bytes from/to a
// (peer) buffer with SM loads / stores or bulk copies; nothing waits on a peer.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace oxi {
void launch_p2p_read(const void* src, int64_t bytes, void* sink, int ctas, int threads, int unr, cudaStream_t st);
void launch_p2p_write(void* dst, int64_t bytes, int ctas, int threads, int unr, cudaStream_t st);
void launch_p2p_bulk(bool write, void* peer, int64_t bytes, int ctas, int chunk, int stages, int* status,
                     cudaStream_t st);
}  // namespace oxi
