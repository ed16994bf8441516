// NVLink peer-access microbenchmark kernels: how fast can one GPU's SMs read
// or write another GPU's memory, as a function of CTAs, bytes in flight per
// thread, and thread loads/stores versus bulk (TMA engine) copies.  Used to
// size the reduce-scatter / all-gather / expert-dispatch kernels.  No kernel
// here waits on another GPU; each just moves `bytes` bytes.  Built as its own
// extension (oxidizr_b200_tools), not part of the training library.
#include <cuda_runtime.h>
#include <cstdint>

#include "host_util.h"
#include "p2pbench.h"
#include "ptx.cuh"

namespace oxi {
namespace {

template <int UNR>
__global__ void __launch_bounds__(512) p2p_read_kernel(const uint4* __restrict__ src, int64_t nvec,
                                                       uint4* __restrict__ sink) {
  uint4 acc = make_uint4(0u, 0u, 0u, 0u);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t base = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; base < nvec; base += stride * UNR) {
    uint4 u[UNR];
#pragma unroll
    for (int r = 0; r < UNR; ++r) {
      const int64_t v = base + r * stride;
      u[r] = v < nvec ? src[v] : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int r = 0; r < UNR; ++r) {
      acc.x ^= u[r].x; acc.y ^= u[r].y; acc.z ^= u[r].z; acc.w ^= u[r].w;
    }
  }
  if ((acc.x | acc.y | acc.z | acc.w) == 0x9e3779b9u) sink[0] = acc;  // keeps the loads alive
}

template <int UNR>
__global__ void __launch_bounds__(512) p2p_write_kernel(uint4* __restrict__ dst, int64_t nvec) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t base = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; base < nvec; base += stride * UNR) {
#pragma unroll
    for (int r = 0; r < UNR; ++r) {
      const int64_t v = base + r * stride;
      if (v < nvec) dst[v] = make_uint4((uint32_t)v, 1u, 2u, 3u);
    }
  }
}

// bulk read: one thread per CTA streams `chunk`-byte pieces into a STAGES-deep
// ring of shared buffers; the other warps only release the buffers.
constexpr int PB_MAX_SMEM = 96 * 1024;

__global__ void __launch_bounds__(128) p2p_bulk_read_kernel(const uint8_t* __restrict__ src, int64_t bytes,
                                                            int chunk, int stages, int* status) {
  extern __shared__ __align__(128) uint8_t sm[];
  __shared__ uint64_t full[16];
  const int64_t nch = bytes / chunk;
  if (threadIdx.x == 0) {
    for (int i = 0; i < stages; ++i) mbar_init(&full[i], 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int64_t it = 0;
    for (int64_t c = blockIdx.x; c < nch; c += gridDim.x, ++it) {
      const int st = (int)(it % stages);
      if (it >= stages) {  // reuse: the copy issued `stages` iterations ago has landed
        if (!mbar_wait(&full[st], (uint32_t)(((it - stages) / stages) & 1), nullptr, status)) return;
      }
      mbar_arrive_expect_tx(&full[st], (uint32_t)chunk);
      bulk_load(sm + (size_t)st * chunk, src + c * chunk, (uint32_t)chunk, &full[st]);
    }
    for (int64_t j = (it > stages ? it - stages : 0); j < it; ++j)
      mbar_wait(&full[j % stages], (uint32_t)((j / stages) & 1), nullptr, status);
  }
}

// bulk write: shared -> peer global, `stages` bulk groups in flight per CTA
__global__ void __launch_bounds__(128) p2p_bulk_write_kernel(uint8_t* __restrict__ dst, int64_t bytes, int chunk,
                                                             int stages) {
  extern __shared__ __align__(128) uint8_t sm[];
  for (int i = threadIdx.x; i < chunk / 16; i += blockDim.x) reinterpret_cast<uint4*>(sm)[i] = make_uint4(1, 2, 3, 4);
  fence_proxy_async_smem();
  __syncthreads();
  if (threadIdx.x != 0) return;
  const int64_t nch = bytes / chunk;
  int64_t it = 0;
  for (int64_t c = blockIdx.x; c < nch; c += gridDim.x, ++it) {
    bulk_store(dst + c * chunk, sm, (uint32_t)chunk);
    bulk_commit();
    if (stages <= 2) bulk_wait_read<1>();
    else if (stages <= 4) bulk_wait_read<3>();
    else bulk_wait_read<7>();
  }
  bulk_wait<0>();
}

}  // namespace

void launch_p2p_read(const void* src, int64_t bytes, void* sink, int ctas, int threads, int unr, cudaStream_t st) {
  const int64_t nvec = bytes / 16;
  const uint4* s = reinterpret_cast<const uint4*>(src);
  uint4* k = reinterpret_cast<uint4*>(sink);
  switch (unr) {
    case 1: p2p_read_kernel<1><<<ctas, threads, 0, st>>>(s, nvec, k); break;
    case 4: p2p_read_kernel<4><<<ctas, threads, 0, st>>>(s, nvec, k); break;
    case 8: p2p_read_kernel<8><<<ctas, threads, 0, st>>>(s, nvec, k); break;
    case 16: p2p_read_kernel<16><<<ctas, threads, 0, st>>>(s, nvec, k); break;
    default: OXI_CHECK(false, "unroll must be 1, 4, 8 or 16");
  }
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_p2p_write(void* dst, int64_t bytes, int ctas, int threads, int unr, cudaStream_t st) {
  const int64_t nvec = bytes / 16;
  uint4* d = reinterpret_cast<uint4*>(dst);
  switch (unr) {
    case 1: p2p_write_kernel<1><<<ctas, threads, 0, st>>>(d, nvec); break;
    case 4: p2p_write_kernel<4><<<ctas, threads, 0, st>>>(d, nvec); break;
    case 8: p2p_write_kernel<8><<<ctas, threads, 0, st>>>(d, nvec); break;
    case 16: p2p_write_kernel<16><<<ctas, threads, 0, st>>>(d, nvec); break;
    default: OXI_CHECK(false, "unroll must be 1, 4, 8 or 16");
  }
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_p2p_bulk(bool write, void* peer, int64_t bytes, int ctas, int chunk, int stages, int* status,
                     cudaStream_t st) {
  OXI_CHECK(chunk % 16 == 0 && bytes % chunk == 0 && stages >= 1 && stages <= 16 &&
                (int64_t)chunk * stages <= PB_MAX_SMEM, "bulk: chunk multiple of 16, bytes multiple of chunk");
  const int smem = chunk * (write ? 1 : stages);
  if (write) {
    OXI_CUDA_CHECK(cudaFuncSetAttribute(p2p_bulk_write_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    p2p_bulk_write_kernel<<<ctas, 128, smem, st>>>(reinterpret_cast<uint8_t*>(peer), bytes, chunk, stages);
  } else {
    OXI_CUDA_CHECK(cudaFuncSetAttribute(p2p_bulk_read_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    p2p_bulk_read_kernel<<<ctas, 128, smem, st>>>(reinterpret_cast<const uint8_t*>(peer), bytes, chunk, stages,
                                                  status);
  }
  OXI_CUDA_CHECK(cudaGetLastError());
}

}  // namespace oxi
