// MoE router: softmax over the expert logits, top-k by logit, softmax over the
// k selected logits, and the per-expert mean routing probability (for the
// load-balancing loss) -- one warp per token, logits held in registers.
//
// Upstream (model.rs:541-556, 604-687): probs = softmax(logits); the top-k
// are found by k rounds of argmax with masking (the first index wins a tie);
// weights = softmax(selected logits); aux uses mean_t(probs) (model.rs:585-590).
//
// Backward, per token t (p = probs[t], s = top-k selection, w = weights):
//   d logits[s_j] += w_j * (dw_j - sum_i w_i dw_i)                (weights)
//   d logits      += p * (g - sum_e p_e g_e),  g_e = d_usage[e] / T   (usage)
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "host_util.h"
#include "kernels_moe.h"

namespace oxi {
namespace {

constexpr int RT_MAXE = 256;  // experts per router (8 per lane)
constexpr int RT_MAXK = 16;

template <typename T>
__device__ __forceinline__ float to_f(T v);
template <>
__device__ __forceinline__ float to_f<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename LT, int EPL>
__global__ void __launch_bounds__(256) router_fwd_kernel(const LT* __restrict__ logits, int64_t ld, int64_t T, int E,
                                                         int k, int64_t* __restrict__ topi, float* __restrict__ topw,
                                                         float* __restrict__ usage, int* __restrict__ counts) {
  __shared__ float s_usage[RT_MAXE];
  __shared__ int s_count[RT_MAXE];
  for (int e = threadIdx.x; e < E; e += blockDim.x) { s_usage[e] = 0.f; s_count[e] = 0; }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x / 32);
  float u_acc[EPL];
#pragma unroll
  for (int i = 0; i < EPL; ++i) u_acc[i] = 0.f;
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; t < T; t += warps) {
    float v[EPL];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const int e = lane + 32 * i;
      v[i] = e < E ? to_f(logits[t * ld + e]) : -INFINITY;
      mx = fmaxf(mx, v[i]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float se = 0.f, p[EPL];
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      p[i] = (lane + 32 * i < E) ? __expf(v[i] - mx) : 0.f;
      se += p[i];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) se += __shfl_xor_sync(0xffffffffu, se, o);
    const float inv = 1.f / se;
#pragma unroll
    for (int i = 0; i < EPL; ++i) u_acc[i] += p[i] * inv;
    // top-k by repeated argmax (lowest index wins a tie)
    float sel_v[RT_MAXK];
    int sel_i[RT_MAXK];
    bool taken[EPL];
#pragma unroll
    for (int i = 0; i < EPL; ++i) taken[i] = false;
    for (int j = 0; j < k; ++j) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
#pragma unroll
      for (int i = 0; i < EPL; ++i) {
        const int e = lane + 32 * i;
        if (e < E && !taken[i] && (v[i] > bv || (v[i] == bv && e < bi))) { bv = v[i]; bi = e; }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
      }
#pragma unroll
      for (int i = 0; i < EPL; ++i)
        if (i == (bi >> 5) && (bi & 31) == lane) taken[i] = true;  // bi < E always (E >= k)
      sel_v[j] = bv;
      sel_i[j] = bi;
    }
    if (lane == 0) {
      float smx = sel_v[0], ss = 0.f;  // sel_v[0] is the largest
      for (int j = 0; j < k; ++j) ss += __expf(sel_v[j] - smx);
      const float sinv = 1.f / ss;
      for (int j = 0; j < k; ++j) {
        topi[t * k + j] = sel_i[j];
        topw[t * k + j] = __expf(sel_v[j] - smx) * sinv;
        if (counts) atomicAdd(&s_count[sel_i[j]], 1);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int e = lane + 32 * i;
    if (e < E) atomicAdd(&s_usage[e], u_acc[i]);
  }
  __syncthreads();
  const float invT = 1.f / (float)T;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    atomicAdd(&usage[e], s_usage[e] * invT);
    if (counts) atomicAdd(&counts[e], s_count[e]);
  }
}

template <typename LT, int EPL>
__global__ void __launch_bounds__(256) router_bwd_kernel(const LT* __restrict__ logits, int64_t ld, int64_t T, int E,
                                                         int k, const int64_t* __restrict__ topi,
                                                         const float* __restrict__ topw,
                                                         const float* __restrict__ dtopw,
                                                         const float* __restrict__ dusage, LT* __restrict__ dlogits,
                                                         int64_t ldd) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x / 32);
  const float invT = 1.f / (float)T;
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; t < T; t += warps) {
    float v[EPL], g[EPL];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const int e = lane + 32 * i;
      v[i] = e < E ? to_f(logits[t * ld + e]) : -INFINITY;
      g[i] = (e < E && dusage) ? dusage[e] * invT : 0.f;
      mx = fmaxf(mx, v[i]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float se = 0.f, p[EPL];
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      p[i] = (lane + 32 * i < E) ? __expf(v[i] - mx) : 0.f;
      se += p[i];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) se += __shfl_xor_sync(0xffffffffu, se, o);
    const float inv = 1.f / se;
    float pg = 0.f;
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      p[i] *= inv;
      pg += p[i] * g[i];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) pg += __shfl_xor_sync(0xffffffffu, pg, o);
    float d[EPL];
#pragma unroll
    for (int i = 0; i < EPL; ++i) d[i] = p[i] * (g[i] - pg);
    // selected-logit softmax
    float wdw = 0.f;
    for (int j = 0; j < k; ++j) wdw += topw[t * k + j] * dtopw[t * k + j];
    for (int j = 0; j < k; ++j) {
      const int e = (int)topi[t * k + j];
      if ((e & 31) == lane) {
        const float w = topw[t * k + j];
#pragma unroll
        for (int i = 0; i < EPL; ++i)
          if (i == (e >> 5)) d[i] += w * (dtopw[t * k + j] - wdw);
      }
    }
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const int e = lane + 32 * i;
      if (e < E) {
        if constexpr (sizeof(LT) == 4) dlogits[t * ldd + e] = d[i];
        else dlogits[t * ldd + e] = __float2bfloat16(d[i]);
      }
    }
  }
}

int grid_for(int64_t T) {
  const int64_t blocks = (T + 7) / 8;
  return (int)(blocks < 148 * 8 ? (blocks > 0 ? blocks : 1) : 148 * 8);
}

}  // namespace

void launch_router_fwd(const void* logits, bool bf16, int64_t ld, int64_t T, int E, int k, int64_t* topi, float* topw,
                       float* usage, int* counts, cudaStream_t st) {
  OXI_CHECK(E >= 1 && E <= RT_MAXE && k >= 1 && k <= RT_MAXK && k <= E, "router supports E <= 256 experts and k <= 16");
  OXI_CUDA_CHECK(cudaMemsetAsync(usage, 0, sizeof(float) * E, st));
  if (counts) OXI_CUDA_CHECK(cudaMemsetAsync(counts, 0, sizeof(int) * E, st));
  if (T == 0) return;
  const int epl = (E + 31) / 32;
#define OXI_RF(N)                                                                                               \
  if (epl <= N) {                                                                                              \
    if (bf16)                                                                                                  \
      router_fwd_kernel<__nv_bfloat16, N><<<grid_for(T), 256, 0, st>>>(                                       \
          reinterpret_cast<const __nv_bfloat16*>(logits), ld, T, E, k, topi, topw, usage, counts);             \
    else                                                                                                       \
      router_fwd_kernel<float, N><<<grid_for(T), 256, 0, st>>>(reinterpret_cast<const float*>(logits), ld, T, E, \
                                                                 k, topi, topw, usage, counts);                \
    OXI_CUDA_CHECK(cudaGetLastError());                                                                        \
    return;                                                                                                    \
  }
  OXI_RF(1) OXI_RF(2) OXI_RF(4) OXI_RF(8)
#undef OXI_RF
}

void launch_router_bwd(const void* logits, bool bf16, int64_t ld, int64_t T, int E, int k, const int64_t* topi,
                       const float* topw, const float* dtopw, const float* dusage, void* dlogits, int64_t ldd,
                       cudaStream_t st) {
  OXI_CHECK(E >= 1 && E <= RT_MAXE && k >= 1 && k <= RT_MAXK, "router supports E <= 256 experts and k <= 16");
  if (T == 0) return;
  const int epl = (E + 31) / 32;
#define OXI_RB(N)                                                                                              \
  if (epl <= N) {                                                                                             \
    if (bf16)                                                                                                 \
      router_bwd_kernel<__nv_bfloat16, N><<<grid_for(T), 256, 0, st>>>(                                      \
          reinterpret_cast<const __nv_bfloat16*>(logits), ld, T, E, k, topi, topw, dtopw, dusage,             \
          reinterpret_cast<__nv_bfloat16*>(dlogits), ldd);                                                    \
    else                                                                                                      \
      router_bwd_kernel<float, N><<<grid_for(T), 256, 0, st>>>(reinterpret_cast<const float*>(logits), ld, T, \
                                                                 E, k, topi, topw, dtopw, dusage,             \
                                                                 reinterpret_cast<float*>(dlogits), ldd);     \
    OXI_CUDA_CHECK(cudaGetLastError());                                                                       \
    return;                                                                                                   \
  }
  OXI_RB(1) OXI_RB(2) OXI_RB(4) OXI_RB(8)
#undef OXI_RB
}

}  // namespace oxi
