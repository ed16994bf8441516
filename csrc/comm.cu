// NVLink data-parallel runtime: CUDA-IPC symmetric buffers and the fused
// gradient reduce-scatter / clip / AdamW / parameter all-gather kernels.
//
// Every rank owns, in device memory mapped by all peers:
//   recv  bf16 [N]   per bucket, W slots of this rank's shard: peers push
//                    their bf16-rounded gradient of the shard into slot r
//   param bf16 [N]   the model parameters (flat)
//   pad   signal pad: epoch flags written by peers, partial norms
// and privately: the reduced f32 gradient of its shards, and f32 master
// weights / AdamW moments of its shards only (optimizer state sharded W ways).
//
// Bucket b covers flat range [lo, lo + len), len a multiple of W * 64; rank r
// owns [lo + r*len/W, lo + (r+1)*len/W).  Per step (epoch e, monotonic):
//   1. bucket ready in backward: push kernel casts grad f32 -> bf16 and
//      stores each owner's part into the owner's recv slot (P2P 16-byte
//      stores); its last CTA posts epoch into every peer's ready[b][r]
//   2. reduce kernel: wait until ready[b][*] >= e in the local pad; sum the W
//      slots of the owned shard (local loads), f32 -> rgrad; sum(g^2)
//   3. norm kernel: exchange partial sum(g^2) through the pads -> clip coef
//   4. per bucket, on the communication stream: AdamW on the owned shard (f32
//      master), bf16 result sent to every peer's param buffer (bulk stores, or
//      one multicast store through NVSwitch); post epoch into every peer's
//      ag[b][r].  The next forward waits (bounded, one thread on the compute
//      stream) for ag[b][*] >= e just before it first uses bucket b, so the
//      all-gather of later buckets overlaps the forward of earlier layers.
// The f32 gradient of a bucket is cleared by the cast that reads it (step 1),
// so no separate zeroing pass follows the step.
// NVLS variant (multicast object over the send and param buffers): the
// reduce-scatter reads the owned shard with multimem.ld_reduce (the switch
// sums the W copies, f32 accumulation) and the all-gather writes it once with
// multimem.st (the switch replicates it to every GPU).
// Cross-GPU ordering: data stores, then a system-scope fence, then a release
// store of the flag; the waiter acquires the flag before reading data.  All
// waits are bounded (OXI_WAIT_LIMIT_NS); on timeout the kernel records
// OXI_ERR_TIMEOUT_PEER in the status word, skips its work and returns.
// Upstream: gradient synchronisation distributed/nccl.rs:153-184 and
// distributed/cpu_staging.rs:146-172; AdamW distributed/optimizer.rs:126-192; clipping trainer.rs:560-574.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>
#include <algorithm>
#include <cstring>
#include <string>
#include <vector>

#include "host_util.h"
#include "kernels_comm.h"
#include "ptx.cuh"

namespace oxi {
namespace {

// The reduce-scatter kernels run next to backward's persistent GEMMs: 128-thread
// CTAs (about 16K registers each) fit on an SM beside a GEMM CTA (192 threads, up
// to 202 registers), so a GEMM launched meanwhile does not wait for them.
constexpr int RS_THREADS = 128;

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Wait until flags[i*stride] >= epoch for i in [0, W) (local pad).  One thread.
__device__ bool wait_flags(const int* flags, int W, int stride, int epoch, int* status, uint64_t limit_ns) {
  const uint64_t t0 = globaltimer();
  for (int i = 0; i < W; ++i) {
    uint32_t spins = 0;
    while (ld_acquire_sys(flags + (int64_t)i * stride) < epoch) {
      if ((++spins & 255u) == 0) {
        if (globaltimer() - t0 > limit_ns) {
          record_error(status, OXI_ERR_TIMEOUT_PEER);
          return false;
        }
      }
    }
  }
  return true;
}

__device__ __forceinline__ void add8(float* acc, uint4 u) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    acc[2 * i] += f.x;
    acc[2 * i + 1] += f.y;
  }
}

// bf16 copy of the f32 gradient; with `zero` the f32 source is cleared in the
// same pass (the next backward accumulates into it from zero).
__global__ void grad_to_bf16_kernel(float* __restrict__ g, __nv_bfloat16* __restrict__ out, int64_t n, bool zero) {
  const int64_t nv = n / 8;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
    const float4 a = reinterpret_cast<const float4*>(g)[2 * i];
    const float4 b = reinterpret_cast<const float4*>(g)[2 * i + 1];
    reinterpret_cast<uint4*>(out)[i] =
        make_uint4(pack_bf16(a.x, a.y), pack_bf16(a.z, a.w), pack_bf16(b.x, b.y), pack_bf16(b.z, b.w));
    if (zero) {
      const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
      reinterpret_cast<float4*>(g)[2 * i] = z;
      reinterpret_cast<float4*>(g)[2 * i + 1] = z;
    }
  }
}

// f32 copy of a bf16 shard (the NCCL reduce-scatter result) plus its sum of squares.
__global__ void __launch_bounds__(512) bf16_to_f32_sumsq_kernel(const __nv_bfloat16* __restrict__ src,
                                                                float* __restrict__ dst, int64_t n,
                                                                float* __restrict__ sumsq) {
  __shared__ float red[32];
  float ss = 0.f;
  const int64_t nv = n / 8;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    add8(acc, reinterpret_cast<const uint4*>(src)[i]);
    reinterpret_cast<float4*>(dst)[2 * i] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    reinterpret_cast<float4*>(dst)[2 * i + 1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
#pragma unroll
    for (int k = 0; k < 8; ++k) ss += acc[k] * acc[k];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) atomicAdd(sumsq, t);
  }
}

// Reduce-scatter of one bucket, push then reduce.
//
// push: every rank casts its f32 gradient of the bucket to bf16 and stores the
// part owned by rank s straight into rank s's receive buffer, in the slot of
// the sender: recv_s[lo + r*shard + i] = bf16(grad_r[lo + s*shard + i]).
// NVLink stores are posted writes, so no thread waits on a round trip.  The
// last CTA to finish publishes the bucket's epoch in every peer's pad.
template <int W>
__global__ void __launch_bounds__(RS_THREADS) push_bucket_kernel(float* __restrict__ grad, bool zero, int64_t lo, int64_t len,
                                                          int rank, const uint64_t* __restrict__ peers_recv,
                                                          const uint64_t* __restrict__ peer_pads, int bucket,
                                                          int epoch, int* __restrict__ done_ctr) {
  constexpr int UNR = 8;  // 8-element vectors per thread in flight (256 B of f32 loads)
  const int64_t shard = len / W;
  const int64_t nv = len / 8;
  const int64_t sv = shard / 8;  // 8-element vectors per shard
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  float4* g4 = reinterpret_cast<float4*>(grad + lo);
  for (int64_t base = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; base < nv; base += stride * UNR) {
    float4 a[UNR], b[UNR];
#pragma unroll
    for (int r = 0; r < UNR; ++r) {
      const int64_t v = base + r * stride;
      if (v < nv) {
        a[r] = g4[2 * v];
        b[r] = g4[2 * v + 1];
        if (zero) g4[2 * v] = g4[2 * v + 1] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
#pragma unroll
    for (int r = 0; r < UNR; ++r) {
      const int64_t v = base + r * stride;
      if (v < nv) {
        const int owner = (int)(v / sv);
        const int64_t i = v - (int64_t)owner * sv;
        __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(peers_recv[owner]) + lo + (int64_t)rank * shard;
        reinterpret_cast<uint4*>(dst)[i] = make_uint4(pack_bf16(a[r].x, a[r].y), pack_bf16(a[r].z, a[r].w),
                                                      pack_bf16(b[r].x, b[r].y), pack_bf16(b[r].z, b[r].w));
      }
    }
  }
  __threadfence_system();
  __syncthreads();
  __shared__ int last;
  if (threadIdx.x == 0) last = (atomicAdd(done_ctr + bucket, 1) == (int)gridDim.x - 1);
  __syncthreads();
  if (last && threadIdx.x == 0) {
    done_ctr[bucket] = 0;
    __threadfence_system();
    for (int i = 0; i < W; ++i)
      st_release_sys(reinterpret_cast<int*>(peer_pads[i]) + PAD_READY + bucket * PAD_MAXW + rank, epoch);
  }
}

// reduce: wait until every rank has pushed the bucket, then sum the W slots of
// this rank's shard from local memory (f32), store the reduced shard and add
// its sum of squares.
template <int W>
__global__ void __launch_bounds__(RS_THREADS) reduce_bucket_kernel(const __nv_bfloat16* __restrict__ recv,
                                                            int* __restrict__ my_pad, int bucket, int epoch,
                                                            int64_t lo, int64_t len, float* __restrict__ rgrad,
                                                            float* __restrict__ sumsq, int* status,
                                                            uint64_t wait_ns) {
  __shared__ int ok_s;
  __shared__ float red[32];
  const int64_t shard = len / W;
  if (threadIdx.x == 0)
    ok_s = wait_flags(my_pad + PAD_READY + bucket * PAD_MAXW, W, 1, epoch, status, wait_ns) ? 1 : 0;
  __syncthreads();
  float ss = 0.f;
  if (ok_s) {
    constexpr int UNR = (16 / W) < 1 ? 1 : ((16 / W) > 4 ? 4 : 16 / W);
    const uint4* src = reinterpret_cast<const uint4*>(recv + lo);
    const int64_t sv = shard / 8;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t base = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; base < sv; base += stride * UNR) {
      uint4 u[UNR][W];
#pragma unroll
      for (int q = 0; q < UNR; ++q) {
        const int64_t v = base + q * stride;
#pragma unroll
        for (int r = 0; r < W; ++r) u[q][r] = v < sv ? src[r * sv + v] : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int q = 0; q < UNR; ++q) {
        const int64_t v = base + q * stride;
        if (v >= sv) break;
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int r = 0; r < W; ++r) add8(acc, u[q][r]);
        float4* o = reinterpret_cast<float4*>(rgrad + v * 8);  // rgrad points at this bucket's shard
        o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
#pragma unroll
        for (int k = 0; k < 8; ++k) ss += acc[k] * acc[k];
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) atomicAdd(sumsq, t);
  }
}

// One thread: make this rank's send buffer of the bucket visible, post the
// bucket's epoch in every peer's pad and wait (bounded) for every peer's post.
__global__ void rs_flags_kernel(const uint64_t* __restrict__ peer_pads, int* __restrict__ my_pad, int rank, int W,
                                int bucket, int epoch, int* status, uint64_t wait_ns) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  __threadfence_system();
  for (int i = 0; i < W; ++i)
    st_release_sys(reinterpret_cast<int*>(peer_pads[i]) + PAD_READY + bucket * PAD_MAXW + rank, epoch);
  wait_flags(my_pad + PAD_READY + bucket * PAD_MAXW, W, 1, epoch, status, wait_ns);
}

// Reduce-scatter of one bucket, pull: every rank has cast its gradient of the
// bucket to bf16 in its own send buffer (grad_to_bf16) and posts the bucket's
// epoch (CTA 0); the owner of each shard then reads the W slices with 16-byte
// loads and sums them in f32.  NVLink reads take microseconds, so each thread
// keeps UNR vectors of every peer in flight (measured on B200: about 2 MB in
// flight per GPU saturates a peer link).
// Posting and waiting for the bucket's flags is done by rs_flags_kernel (one
// thread) just before this kernel on the same stream, so no SM spins here
// while peers are still in their backward pass.
template <int W>
__global__ void __launch_bounds__(RS_THREADS) rs_pull_kernel(const uint64_t* __restrict__ peers_send, int rank, int64_t lo,
                                                      int64_t len, float* __restrict__ rgrad,
                                                      float* __restrict__ sumsq, const int* status) {
  constexpr int UNR = (16 / W) < 1 ? 1 : ((16 / W) > 8 ? 8 : 16 / W);
  __shared__ float red[32];
  const int64_t shard = len / W;
  const int64_t s0 = lo + rank * shard;
  const int ok_s = (status == nullptr || *reinterpret_cast<const volatile int*>(status) == 0) ? 1 : 0;
  float ss = 0.f;
  if (ok_s) {
    const uint4* src[W];
#pragma unroll
    for (int i = 0; i < W; ++i) {
      const int peer = (rank + i) % W;  // stagger peers so ranks do not all hit the same one
      src[i] = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(peers_send[peer]) + s0);
    }
    const int64_t nv = shard / 8;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t base = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; base < nv; base += stride * UNR) {
      uint4 u[UNR][W];
#pragma unroll
      for (int r = 0; r < UNR; ++r) {
        const int64_t v = base + r * stride;
#pragma unroll
        for (int i = 0; i < W; ++i) u[r][i] = v < nv ? src[i][v] : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int r = 0; r < UNR; ++r) {
        const int64_t v = base + r * stride;
        if (v >= nv) break;
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int i = 0; i < W; ++i) add8(acc, u[r][i]);
        float4* o = reinterpret_cast<float4*>(rgrad + v * 8);  // rgrad points at this bucket's shard
        o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
#pragma unroll
        for (int k = 0; k < 8; ++k) ss += acc[k] * acc[k];
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) atomicAdd(sumsq, t);
  }
}

// Exchange partial sums of squares; coef = min(1, max_norm / (norm + 1e-6)) / W.
// skip (nullable): a non-zero word skips the update (NaN coefficient) with the norm as measured.
__global__ void norm_exchange_kernel(const uint64_t* __restrict__ peer_pads, int* __restrict__ my_pad, int rank,
                                     int W, int epoch, const float* __restrict__ sumsq, float max_norm,
                                     float* __restrict__ coef, float* __restrict__ norm_out, int* status,
                                     uint64_t wait_ns, const int* __restrict__ skip) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const float mine = *sumsq;
  for (int i = 0; i < W; ++i) {
    int* pad = reinterpret_cast<int*>(peer_pads[i]);
    reinterpret_cast<volatile float*>(pad + PAD_NORMV)[rank] = mine;
  }
  __threadfence_system();
  for (int i = 0; i < W; ++i) st_release_sys(reinterpret_cast<int*>(peer_pads[i]) + PAD_NORMF + rank, epoch);
  if (!wait_flags(my_pad + PAD_NORMF, W, 1, epoch, status, wait_ns)) {
    *coef = 0.f;  // no update on a failed exchange
    *norm_out = NAN;
    return;
  }
  float tot = 0.f;
  for (int i = 0; i < W; ++i) tot += reinterpret_cast<volatile float*>(my_pad + PAD_NORMV)[i];
  const float nrm = sqrtf(tot) / W;  // norm of the averaged gradient
  *norm_out = nrm;
  float c = 1.f / W;
  if (max_norm > 0.f && nrm > max_norm) c *= max_norm / (nrm + 1e-6f);
  // a non-finite norm skips the update on every rank: the AdamW kernels take a
  // NaN coefficient as "leave p, m, v as they are" (parameters are still sent)
  *coef = (isfinite(nrm) && !(skip && *skip)) ? c : __int_as_float(0x7fc00000);
}

// ---------------------------------------------------------------- NVLS (multicast) reduce-scatter
__device__ __forceinline__ uint4 multimem_ld_reduce_bf16x8(const void* mc) {
  uint4 r;
  asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(mc)
               : "memory");
  return r;
}
__device__ __forceinline__ void multimem_st_16(void* mc, uint4 v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(mc), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void fence_proxy_alias() { asm volatile("fence.proxy.alias;" ::: "memory"); }

// Reduce-scatter of one bucket through the switch: every rank has cast its
// gradient of the bucket into its send buffer and the flags say all have; the
// owner reads its shard through the multicast address with
// multimem.ld_reduce (NVSwitch fetches the W copies and sums them, f32
// accumulation) and keeps the f32 result.  UNR 16-byte reductions per thread
// are in flight.
__global__ void __launch_bounds__(RS_THREADS) rs_nvls_kernel(const __nv_bfloat16* __restrict__ mc_send, int rank, int W,
                                                      int64_t lo, int64_t len, float* __restrict__ rgrad,
                                                      float* __restrict__ sumsq, const int* status) {
  constexpr int UNR = 4;
  __shared__ float red[32];
  const int64_t shard = len / W;
  const uint4* src = reinterpret_cast<const uint4*>(mc_send + lo + rank * shard);
  const bool ok = status == nullptr || *reinterpret_cast<const volatile int*>(status) == 0;
  float ss = 0.f;
  if (ok) {
    const int64_t nv = shard / 8;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t base = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; base < nv; base += stride * UNR) {
      uint4 u[UNR];
#pragma unroll
      for (int r = 0; r < UNR; ++r) {
        const int64_t v = base + r * stride;
        u[r] = v < nv ? multimem_ld_reduce_bf16x8(src + v) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int r = 0; r < UNR; ++r) {
        const int64_t v = base + r * stride;
        if (v >= nv) break;
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        add8(acc, u[r]);
        float4* o = reinterpret_cast<float4*>(rgrad + v * 8);
        o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
#pragma unroll
        for (int k = 0; k < 8; ++k) ss += acc[k] * acc[k];
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x / 32] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) atomicAdd(sumsq, t);
  }
}

// ---------------------------------------------------------------- AdamW + all-gather, one bucket
__device__ __forceinline__ float adamw_one(float g, float& m, float& v, float& p, float b1, float b2, float rb1,
                                           float rb2, float lr, float eps, float wd) {
  m = b1 * m + (1.f - b1) * g;
  v = b2 * v + (1.f - b2) * g * g;
  p = p - lr * ((m * rb1) / (sqrtf(v * rb2) + eps)) - lr * wd * p;
  return p;
}

// AdamW on 8 consecutive shard elements at offset e (16-byte aligned) of the
// sharded state; returns the 8 new parameters as bf16.  gs is the clip
// coefficient (1/W included); a non-finite gs leaves p, m, v as they are.
__device__ __forceinline__ uint4 adamw8(int64_t e, const float* __restrict__ rgrad, float* __restrict__ master,
                                       float* __restrict__ m, float* __restrict__ v, float gs, bool apply, float b1,
                                       float b2, float rb1, float rb2, float lr, float eps, float wd) {
  float4 g4[2], m4[2], v4[2], p4[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    p4[h] = reinterpret_cast<const float4*>(master + e)[h];
    if (apply) {
      g4[h] = reinterpret_cast<const float4*>(rgrad + e)[h];
      m4[h] = reinterpret_cast<const float4*>(m + e)[h];
      v4[h] = reinterpret_cast<const float4*>(v + e)[h];
    }
  }
  if (apply) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      adamw_one(g4[h].x * gs, m4[h].x, v4[h].x, p4[h].x, b1, b2, rb1, rb2, lr, eps, wd);
      adamw_one(g4[h].y * gs, m4[h].y, v4[h].y, p4[h].y, b1, b2, rb1, rb2, lr, eps, wd);
      adamw_one(g4[h].z * gs, m4[h].z, v4[h].z, p4[h].z, b1, b2, rb1, rb2, lr, eps, wd);
      adamw_one(g4[h].w * gs, m4[h].w, v4[h].w, p4[h].w, b1, b2, rb1, rb2, lr, eps, wd);
      reinterpret_cast<float4*>(m + e)[h] = m4[h];
      reinterpret_cast<float4*>(v + e)[h] = v4[h];
      reinterpret_cast<float4*>(master + e)[h] = p4[h];
    }
  }
  return make_uint4(pack_bf16(p4[0].x, p4[0].y), pack_bf16(p4[0].z, p4[0].w), pack_bf16(p4[1].x, p4[1].y),
                    pack_bf16(p4[1].z, p4[1].w));
}

// Last CTA of a bucket's all-gather: publish this rank's epoch for the bucket
// in every peer's pad (after every CTA's stores are performed).
__device__ __forceinline__ void ag_publish(const uint64_t* __restrict__ peer_pads, int W, int rank, int bucket,
                                           int epoch, int* __restrict__ done_ctr) {
  __threadfence_system();
  __syncthreads();
  __shared__ int last;
  if (threadIdx.x == 0) last = (atomicAdd(done_ctr, 1) == (int)gridDim.x - 1);
  __syncthreads();
  if (last && threadIdx.x == 0) {
    *done_ctr = 0;
    __threadfence_system();
    if (peer_pads)
      for (int i = 0; i < W; ++i)
        st_release_sys(reinterpret_cast<int*>(peer_pads[i]) + PAD_AGF + bucket * PAD_MAXW + rank, epoch);
  }
}

// P2P / local all-gather: each thread updates 8 consecutive elements of the
// owned shard of bucket [lo, lo + len) and stores the 16 bytes of new bf16
// parameters straight into the `ndst` parameter buffers of the table (every
// rank, itself included; ndst = 1: only its own buffer, the NCCL baseline
// gathers afterwards).  No shared memory, so its CTAs can sit on an SM next to
// a GEMM's CTA while the forward runs.
__global__ void __launch_bounds__(256) adamw_ag_bucket_kernel(
    int64_t lo, int64_t len, int64_t so, int W, int rank, int ndst, const float* __restrict__ rgrad,
    float* __restrict__ master, float* __restrict__ m, float* __restrict__ v, const uint64_t* __restrict__ peers_param,
    const uint64_t* __restrict__ peer_pads, int bucket, int epoch, float lr, float b1, float b2, float eps, float wd,
    float bc1, float bc2, const float* __restrict__ coef, int* __restrict__ done_ctr, const int* status) {
  const float gs = *coef;
  const bool apply = isfinite(gs);
  const float rb1 = 1.f / bc1, rb2 = 1.f / bc2;
  const bool failed = status && *reinterpret_cast<const volatile int*>(status) != 0;
  if (!failed) {
    const int64_t shard = len / W;
    const int64_t p0 = lo + rank * shard;
    const int64_t nv = shard / 8;
    uint4* dst[PAD_MAXW];
    for (int j = 0; j < ndst; ++j)
      dst[j] = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(peers_param[(rank + j) % ndst]) + p0);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
      const uint4 u = adamw8(so + i * 8, rgrad, master, m, v, gs, apply, b1, b2, rb1, rb2, lr, eps, wd);
      for (int j = 0; j < ndst; ++j) dst[j][i] = u;
    }
  }
  ag_publish(peer_pads, W, rank, bucket, epoch, done_ctr);
}

// NVLS all-gather: each thread multicasts its 16 bytes of new parameters to
// every GPU's param buffer with one multimem.st.
__global__ void __launch_bounds__(256) adamw_ag_nvls_kernel(
    int64_t lo, int64_t len, int64_t so, int W, int rank, const float* __restrict__ rgrad, float* __restrict__ master,
    float* __restrict__ m, float* __restrict__ v, __nv_bfloat16* __restrict__ mc_param,
    const uint64_t* __restrict__ peer_pads, int bucket, int epoch, float lr, float b1, float b2, float eps, float wd,
    float bc1, float bc2, const float* __restrict__ coef, int* __restrict__ done_ctr, const int* status) {
  const float gs = *coef;
  const bool apply = isfinite(gs);
  const float rb1 = 1.f / bc1, rb2 = 1.f / bc2;
  const bool failed = status && *reinterpret_cast<const volatile int*>(status) != 0;
  if (!failed) {
    const int64_t shard = len / W;
    const int64_t p0 = lo + rank * shard;
    const int64_t nv = shard / 8;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
      const uint4 u = adamw8(so + i * 8, rgrad, master, m, v, gs, apply, b1, b2, rb1, rb2, lr, eps, wd);
      multimem_st_16(mc_param + p0 + i * 8, u);
    }
  }
  fence_proxy_alias();  // multicast stores before the unicast flag stores
  ag_publish(peer_pads, W, rank, bucket, epoch, done_ctr);
}

// One thread on the compute stream: wait (bounded) until every rank has
// published bucket b's parameters for this epoch.
__global__ void ag_wait_kernel(int* __restrict__ my_pad, int W, int bucket, int epoch, int* status, uint64_t wait_ns) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  wait_flags(my_pad + PAD_AGF + bucket * PAD_MAXW, W, 1, epoch, status, wait_ns);
}

int sms() {
  static int n = 0;
  if (!n) {
    int d;
    cudaGetDevice(&d);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d);
  }
  return n;
}

}  // namespace

// ------------------------------------------------------------- host side
void* ipc_alloc(size_t nbytes, std::string* handle) {
  void* p = nullptr;
  OXI_CUDA_CHECK(cudaMalloc(&p, nbytes));
  OXI_CUDA_CHECK(cudaMemset(p, 0, nbytes));
  cudaIpcMemHandle_t h;
  OXI_CUDA_CHECK(cudaIpcGetMemHandle(&h, p));
  handle->assign(reinterpret_cast<const char*>(&h), sizeof(h));
  return p;
}

void ipc_free(void* p) { OXI_CUDA_CHECK(cudaFree(p)); }

void* ipc_open(const std::string& handle) {
  OXI_CHECK(handle.size() == sizeof(cudaIpcMemHandle_t), "bad IPC handle size");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.data(), sizeof(h));
  void* p = nullptr;
  OXI_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return p;
}

void ipc_close(void* p) { OXI_CUDA_CHECK(cudaIpcCloseMemHandle(p)); }

void launch_grad_to_bf16(float* g, void* out, int64_t n, bool zero, cudaStream_t st) {
  OXI_CHECK(n % 8 == 0, "bucket length must be a multiple of 8");
  if (!n) return;
  const unsigned grid = (unsigned)std::min<int64_t>((n / 8 + 255) / 256, (int64_t)sms() * 4);
  grad_to_bf16_kernel<<<grid, 256, 0, st>>>(g, reinterpret_cast<__nv_bfloat16*>(out), n, zero);
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_bf16_to_f32_sumsq(const void* src, float* dst, int64_t n, float* sumsq, cudaStream_t st) {
  OXI_CHECK(n % 8 == 0, "shard length must be a multiple of 8");
  if (!n) return;
  const unsigned grid = (unsigned)std::min<int64_t>((n / 8 + 511) / 512, (int64_t)sms() * 2);
  bf16_to_f32_sumsq_kernel<<<grid, 512, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(src), dst, n, sumsq);
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_rs_bucket(int mode, float* grad, bool zero_grad, const uint64_t* peers_buf, void* my_buf, void* mc_buf,
                      const uint64_t* peer_pads, int* my_pad, int* done_ctr, int rank, int W, int bucket, int epoch,
                      int64_t lo, int64_t len, float* rgrad, float* sumsq, int ctas, int* status, int64_t wait_ns,
                      cudaStream_t st) {
  OXI_CHECK(W <= PAD_MAXW && bucket < PAD_MAXB, "too many ranks or buckets");
  OXI_CHECK(len % (W * 64) == 0, "bucket length must divide into 64-element shards");
  OXI_CHECK(W >= 1 && W <= 8, "fused data parallelism supports 1..8 ranks per node, got ", W);
  if (mode == 2) {
    // NVLS: local cast into the send buffer, then the owner reads its shard through the switch
    OXI_CHECK(mc_buf != nullptr, "NVLS reduce-scatter needs the multicast address of the send buffer");
    launch_grad_to_bf16(grad + lo, reinterpret_cast<__nv_bfloat16*>(my_buf) + lo, len, zero_grad, st);
    rs_flags_kernel<<<1, 32, 0, st>>>(peer_pads, my_pad, rank, W, bucket, epoch, status, (uint64_t)wait_ns);
    const int g = (int)std::max<int64_t>(1, std::min<int64_t>((len / W / 8 + RS_THREADS - 1) / RS_THREADS,
                                                               (int64_t)ctas));
    rs_nvls_kernel<<<g, RS_THREADS, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(mc_buf), rank, W, lo, len, rgrad, sumsq,
                                      status);
  } else if (mode == 0) {
    // pull: local cast into the send buffer, then the owner sums the W slices of its shard
    launch_grad_to_bf16(grad + lo, reinterpret_cast<__nv_bfloat16*>(my_buf) + lo, len, zero_grad, st);
    rs_flags_kernel<<<1, 32, 0, st>>>(peer_pads, my_pad, rank, W, bucket, epoch, status, (uint64_t)wait_ns);
    const int g = (int)std::max<int64_t>(1, std::min<int64_t>((len / W / 8 + RS_THREADS - 1) / RS_THREADS,
                                                               (int64_t)ctas));
    switch (W) {
#define OXI_RS(N)                                                                                                \
  case N:                                                                                                        \
    rs_pull_kernel<N><<<g, RS_THREADS, 0, st>>>(peers_buf, rank, lo, len, rgrad, sumsq, status);                 \
    break;
      OXI_RS(1) OXI_RS(2) OXI_RS(3) OXI_RS(4) OXI_RS(5) OXI_RS(6) OXI_RS(7) OXI_RS(8)
#undef OXI_RS
    }
  } else {
    // push: cast + NVLink stores into the owners' receive slots, then a local reduction
    const int push_ctas =
        (int)std::min<int64_t>(std::max<int64_t>((len / 8 + RS_THREADS - 1) / RS_THREADS, 1), (int64_t)ctas);
    const int red_ctas =
        (int)std::min<int64_t>(std::max<int64_t>((len / W / 8 + RS_THREADS - 1) / RS_THREADS, 1), (int64_t)ctas);
    const __nv_bfloat16* rv = reinterpret_cast<const __nv_bfloat16*>(my_buf);
    switch (W) {
#define OXI_RS(N)                                                                                                \
  case N:                                                                                                        \
    push_bucket_kernel<N><<<push_ctas, RS_THREADS, 0, st>>>(grad, zero_grad, lo, len, rank, peers_buf, peer_pads,       \
                                                     bucket, epoch, done_ctr);                                   \
    reduce_bucket_kernel<N><<<red_ctas, RS_THREADS, 0, st>>>(rv, my_pad, bucket, epoch, lo, len, rgrad, sumsq, status, \
                                                      (uint64_t)wait_ns);                                        \
    break;
      OXI_RS(1) OXI_RS(2) OXI_RS(3) OXI_RS(4) OXI_RS(5) OXI_RS(6) OXI_RS(7) OXI_RS(8)
#undef OXI_RS
    }
  }
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_norm_exchange(const uint64_t* peer_pads, int* my_pad, int rank, int W, int epoch, const float* sumsq,
                          float max_norm, float* coef, float* norm_out, int* status, int64_t wait_ns, const int* skip,
                          cudaStream_t st) {
  norm_exchange_kernel<<<1, 32, 0, st>>>(peer_pads, my_pad, rank, W, epoch, sumsq, max_norm, coef, norm_out, status,
                                         (uint64_t)wait_ns, skip);
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_adamw_ag_bucket(int mode, int64_t lo, int64_t len, int64_t so, int W, int rank, int ndst,
                            const float* rgrad, float* master, float* m, float* v, const uint64_t* peers_param,
                            void* mc_param, const uint64_t* peer_pads, int bucket, int epoch, float lr, float b1,
                            float b2, float eps, float wd, float bc1, float bc2, const float* coef, int* done_ctr,
                            int* status, int ctas, cudaStream_t st) {
  OXI_CHECK(W >= 1 && W <= PAD_MAXW && bucket >= 0 && bucket < PAD_MAXB, "bad rank count or bucket index");
  OXI_CHECK(len % (W * 64) == 0 && so % 8 == 0, "bucket length must divide into 64-element shards");
  const int64_t shard = len / W;
  if (mode == 2) {
    OXI_CHECK(mc_param != nullptr, "NVLS all-gather needs the multicast address of the parameter buffer");
    const int g = (int)std::max<int64_t>(1, std::min<int64_t>((shard / 8 + 255) / 256, (int64_t)ctas));
    adamw_ag_nvls_kernel<<<g, 256, 0, st>>>(lo, len, so, W, rank, rgrad, master, m, v,
                                            reinterpret_cast<__nv_bfloat16*>(mc_param), peer_pads, bucket, epoch, lr,
                                            b1, b2, eps, wd, bc1, bc2, coef, done_ctr, status);
  } else {
    OXI_CHECK(ndst >= 1 && ndst <= PAD_MAXW, "bad destination count");
    const int g = (int)std::max<int64_t>(1, std::min<int64_t>((shard / 8 + 255) / 256, (int64_t)ctas));
    adamw_ag_bucket_kernel<<<g, 256, 0, st>>>(lo, len, so, W, rank, ndst, rgrad, master, m, v, peers_param,
                                              peer_pads, bucket, epoch, lr, b1, b2, eps, wd, bc1, bc2, coef, done_ctr,
                                              status);
  }
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_ag_wait(int* my_pad, int W, int bucket, int epoch, int* status, int64_t wait_ns, cudaStream_t st) {
  OXI_CHECK(W >= 1 && W <= PAD_MAXW && bucket >= 0 && bucket < PAD_MAXB, "bad rank count or bucket index");
  ag_wait_kernel<<<1, 32, 0, st>>>(my_pad, W, bucket, epoch, status, (uint64_t)wait_ns);
  OXI_CUDA_CHECK(cudaGetLastError());
}

}  // namespace oxi
