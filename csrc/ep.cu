// Expert parallelism over NVLink: token dispatch / combine written and read
// directly in peers' memory (CUDA-IPC symmetric buffers), no NCCL.
//
// E experts are split over W ranks (El = E / W local experts each).  Every
// rank holds, mapped by all peers:
//   xrecv  bf16 [cap, H]  token rows routed to its experts, one MOE_SEG_ALIGN-aligned
//                         segment per local expert (sources in rank order)
//   srcidx int32 [cap]    source of each received row: rank * T*k + pair, -1 = padding
//   yret   bf16 [T*k, H]  this rank's own (token, slot) pairs: the expert output
//                         rows (forward), then their input gradients (backward),
//                         written by the owners' expert GEMM epilogues
//   dyrecv bf16 [cap, H]  output gradients pushed back by the sources (one
//                         buffer shared by all layers)
//   metaw  f32  [cap]     routing weight of each received row
//   pad    int32          flags [EP_NKIND][EP_MAXW] + counts [EP_MAXW][EP_MAXE]
//
// One step of a MoE layer (seq = a number that grows by one per exchange, the
// same on every rank because every rank runs the layers in the same order):
//   counts   : all-gather the per-expert selection counts through the pads
//              (-> every rank knows every segment of every peer)
//   dispatch : warp per (token, slot): P2P 16-byte stores of the token row
//              into the owner's xrecv (+ its srcidx, metaw); last CTA posts DISPATCHED
//   wait(DISPATCHED) ; gate/up grouped GEMM ; down-projection grouped GEMM
//              whose epilogue stores every output row straight into its
//              source's yret (P2P, overlapping the remaining tiles) and whose
//              last CTA posts YREADY
//   wait(YREADY) ; combine locally: y = resid + sum_j w_j yret[t k + j]
// backward:
//   push_dy  : warp per (token, slot): P2P stores of dy into the owner's dyrecv
//              and dw_j = <dy_t, yret[t k + j]> (local); last CTA posts DYPUSHED
//   wait(DYPUSHED) ; scale_rows: dyrecv *= metaw, pad rows zeroed ; grouped
//              backward GEMMs, the last one scattering the input-gradient rows
//              into the sources' yret and posting DXREADY
//   wait(DXREADY) ; gather locally: dx_t = sum_j yret[t k + j]
// Every wait is bounded; a timeout records OXI_ERR_TIMEOUT_PEER in the status
// word and the kernel skips its remote accesses.  No TMA is used here.
// Upstream: the MoE layer model.rs:541-593 (dense on one GPU in the reference; expert
// parallelism over NVLink is new here).
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <algorithm>
#include <cstdint>

#include "host_util.h"
#include "kernels_ep.h"
#include "kernels_moe.h"
#include "ptx.cuh"

namespace oxi {
namespace {

__device__ __forceinline__ void st_release_sys(int* p, int v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int* p) {
  int v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ bool ep_wait_all(const int* my_pad, int kind, int W, int seq, int* status, uint64_t wait_ns) {
  const int* f = my_pad + EP_FLAGS + kind * EP_MAXW;
  const uint64_t t0 = globaltimer();
  for (int i = 0; i < W; ++i) {
    uint32_t spins = 0;
    while (ld_acquire_sys(f + i) < seq) {
      if ((++spins & 255u) == 0 && globaltimer() - t0 > wait_ns) {
        record_error(status, OXI_ERR_TIMEOUT_PEER);
        return false;
      }
    }
  }
  return true;
}

__device__ void ep_post_all(const uint64_t* peer_pads, int kind, int rank, int W, int seq) {
  __threadfence_system();
  for (int i = 0; i < W; ++i)
    st_release_sys(reinterpret_cast<int*>(peer_pads[i]) + EP_FLAGS + kind * EP_MAXW + rank, seq);
}

// "last CTA out" helper: every thread fences its own stores, the last CTA to
// arrive resets the counter and posts `kind` to every peer.
__device__ void ep_last_cta_post(int* ctr, const uint64_t* peer_pads, int kind, int rank, int W, int seq) {
  __threadfence_system();
  __syncthreads();
  __shared__ int last;
  if (threadIdx.x == 0) last = (atomicAdd(ctr, 1) == (int)gridDim.x - 1);
  __syncthreads();
  if (last && threadIdx.x == 0) {
    *ctr = 0;
    ep_post_all(peer_pads, kind, rank, W, seq);
  }
}

// expert segments of a receive buffer start on MOE_SEG_ALIGN-row boundaries (CTA-pair tiles)
__device__ __forceinline__ int align_seg(int n) { return (n + MOE_SEG_ALIGN - 1) / MOE_SEG_ALIGN * MOE_SEG_ALIGN; }

// ------------------------------------------------------------------ counts
__global__ void ep_counts_kernel(const int* __restrict__ local_counts, const uint64_t* __restrict__ peer_pads,
                                 int* __restrict__ my_pad, int rank, int W, int E, int seq,
                                 int* __restrict__ all_counts, int* __restrict__ seg_off, int* __restrict__ recv_counts,
                                 int cap, int* __restrict__ overflow, int* __restrict__ need_max, int* status,
                                 uint64_t wait_ns) {
  __shared__ int ok_s;
  const int El = E / W;
  for (int i = 0; i < W; ++i) {
    int* pc = reinterpret_cast<int*>(peer_pads[i]) + EP_COUNTS + rank * EP_MAXE;
    for (int e = threadIdx.x; e < E; e += blockDim.x) reinterpret_cast<volatile int*>(pc)[e] = local_counts[e];
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    ep_post_all(peer_pads, EP_K_COUNTS, rank, W, seq);
    ok_s = ep_wait_all(my_pad, EP_K_COUNTS, W, seq, status, wait_ns) ? 1 : 0;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < W * E; i += blockDim.x) {
    const int s = i / E, e = i % E;
    all_counts[i] = ok_s ? reinterpret_cast<volatile int*>(my_pad + EP_COUNTS + s * EP_MAXE)[e] : 0;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // capacity check: every rank sees the same counts, so every rank reaches the
    // same verdict for every owner's receive buffer (all have `cap` rows)
    int need = 0;
    for (int d = 0; d < W; ++d) {
      int off = 0;
      for (int le = 0; le < El; ++le) {
        int c = 0;
        for (int s = 0; s < W; ++s) c += all_counts[s * E + d * El + le];
        off += align_seg(c);
      }
      need = max(need, off);
    }
    const bool skip = need > cap;
    if (skip) {
      // nothing of this layer is exchanged or computed: empty segments, and a
      // sticky flag that makes the optimizer skip this step's update
      atomicMax(need_max, need);
      atomicExch(overflow, 1);
    }
    int off = 0;
    for (int le = 0; le < El; ++le) {
      int c = 0;
      for (int s = 0; s < W; ++s) c += all_counts[s * E + rank * El + le];
      recv_counts[le] = skip ? 0 : c;
      seg_off[le] = off;
      if (!skip) off += align_seg(c);
    }
    seg_off[El] = off;
    seg_off[El + 1] = skip ? 1 : 0;
  }
}

// Start row (in the owner's buffers) of the rows this rank sends to expert e.
__device__ int dest_base(const int* __restrict__ all_counts, int rank, int W, int E, int e) {
  const int El = E / W;
  const int dest = e / El, le = e % El;
  int off = 0;
  for (int l = 0; l < le; ++l) {
    int c = 0;
    for (int s = 0; s < W; ++s) c += all_counts[s * E + dest * El + l];
    off += align_seg(c);
  }
  for (int s = 0; s < rank; ++s) off += all_counts[s * E + e];
  return off;
}

// ------------------------------------------------------------------ dispatch
__global__ void __launch_bounds__(256) ep_dispatch_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t ldx, const int64_t* __restrict__ topi,
    const float* __restrict__ topw, int64_t T, int k, int H, const int* __restrict__ all_counts, int rank, int W,
    int E, int* __restrict__ cursor, const uint64_t* __restrict__ peers_xrecv, const uint64_t* __restrict__ peers_metaw,
    const uint64_t* __restrict__ peers_srcidx, int* __restrict__ pos_out, int* __restrict__ done_ctr,
    const uint64_t* __restrict__ peer_pads, int seq, const int* __restrict__ seg_off, const int* status) {
  __shared__ int s_base[EP_MAXE];
  for (int e = threadIdx.x; e < E; e += blockDim.x) s_base[e] = dest_base(all_counts, rank, W, E, e);
  __syncthreads();
  const int El = E / W;
  // a layer over capacity (seg_off[El + 1]) sends nothing
  const bool failed = (status && *reinterpret_cast<const volatile int*>(status) != 0) || seg_off[El + 1] != 0;
  const int lane = threadIdx.x & 31;
  const int64_t pairs = T * k;
  const int nvec = H / 8;
  if (!failed) {
    for (int64_t p = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; p < pairs;
         p += (int64_t)gridDim.x * (blockDim.x / 32)) {
      const int e = (int)topi[p];
      int slot = 0;
      if (lane == 0) slot = atomicAdd(&cursor[e], 1);
      slot = __shfl_sync(0xffffffffu, slot, 0);
      const int pos = s_base[e] + slot;
      const int dest = e / El;
      const uint4* src = reinterpret_cast<const uint4*>(x + (p / k) * ldx);
      uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(peers_xrecv[dest]) + (int64_t)pos * H);
      for (int v = lane; v < nvec; v += 32) dst[v] = src[v];
      if (lane == 0) {
        pos_out[p] = pos;
        reinterpret_cast<float*>(peers_metaw[dest])[pos] = topw[p];
        reinterpret_cast<int*>(peers_srcidx[dest])[pos] = rank * (int)pairs + (int)p;
      }
    }
  }
  ep_last_cta_post(done_ctr, peer_pads, EP_K_DISPATCHED, rank, W, seq);
}

// srcidx of the padding rows of every local expert segment = -1 (peers write
// only real rows, so this never races with a dispatch)
__global__ void ep_mark_pad_kernel(const int* __restrict__ seg_off, const int* __restrict__ recv_counts, int El,
                                   int* __restrict__ srcidx) {
  const int e = blockIdx.x;
  for (int r = seg_off[e] + recv_counts[e] + threadIdx.x; r < seg_off[e + 1]; r += blockDim.x) srcidx[r] = -1;
}

__global__ void ep_wait_kernel(const int* my_pad, int kind, int W, int seq, int* status, uint64_t wait_ns) {
  if (threadIdx.x == 0 && blockIdx.x == 0) ep_wait_all(my_pad, kind, W, seq, status, wait_ns);
}

__global__ void ep_signal_kernel(const uint64_t* peer_pads, int kind, int rank, int W, int seq) {
  if (threadIdx.x == 0 && blockIdx.x == 0) ep_post_all(peer_pads, kind, rank, W, seq);
}

// warp per (token, slot) pair p: dy row -> owner's dyrecv (P2P stores) and
// dw[p] = <dy_t, yret[p]> from this rank's copy of the expert output row
__global__ void __launch_bounds__(256) ep_push_dy_kernel(
    const __nv_bfloat16* __restrict__ dy, const int64_t* __restrict__ topi, const int* __restrict__ pos, int64_t T,
    int k, int H, int El, const uint64_t* __restrict__ peers_dyrecv, const __nv_bfloat16* __restrict__ yret,
    float* __restrict__ dw, int* __restrict__ done_ctr, const uint64_t* __restrict__ peer_pads, int rank, int W,
    int seq, const int* __restrict__ seg_off, const int* status) {
  // a layer over capacity (seg_off[El + 1]) sent nothing forward: nothing goes back
  const bool failed = (status && *reinterpret_cast<const volatile int*>(status) != 0) || seg_off[El + 1] != 0;
  const int lane = threadIdx.x & 31;
  const int nvec = H / 8;
  if (!failed) {
    for (int64_t p = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; p < T * k;
         p += (int64_t)gridDim.x * (blockDim.x / 32)) {
      const int e = (int)topi[p];
      const uint4* src = reinterpret_cast<const uint4*>(dy + (p / k) * H);
      const uint4* yr = reinterpret_cast<const uint4*>(yret + p * H);
      uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(peers_dyrecv[e / El]) +
                                            (int64_t)pos[p] * H);
      float dot = 0.f;
      for (int v = lane; v < nvec; v += 32) {
        const uint4 a = src[v];
        dst[v] = a;
        const uint4 b = yr[v];
        const __nv_bfloat162* ha = reinterpret_cast<const __nv_bfloat162*>(&a);
        const __nv_bfloat162* hb = reinterpret_cast<const __nv_bfloat162*>(&b);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 fa = __bfloat1622float2(ha[q]), fb = __bfloat1622float2(hb[q]);
          dot += fa.x * fb.x + fa.y * fb.y;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
      if (lane == 0) dw[p] = dot;
    }
  }
  ep_last_cta_post(done_ctr, peer_pads, EP_K_DYPUSHED, rank, W, seq);
}

// Owner side, local: dyrecv[r] *= metaw[r]; padding rows of dyrecv are zeroed.
// Warp per row.
__global__ void __launch_bounds__(256) ep_scale_rows_kernel(__nv_bfloat16* __restrict__ dyrecv,
                                                            const float* __restrict__ metaw,
                                                            const int* __restrict__ seg_off,
                                                            const int* __restrict__ recv_counts, int El, int H) {
  const int lane = threadIdx.x & 31;
  const int rows = seg_off[El];
  const int nvec = H / 8;
  for (int r = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; r < rows; r += gridDim.x * (blockDim.x / 32)) {
    int lo = 0, hi = El - 1;  // segment of row r: largest le with seg_off[le] <= r
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (seg_off[mid] <= r) lo = mid; else hi = mid - 1;
    }
    const bool real = r < seg_off[lo] + recv_counts[lo];
    uint4* d = reinterpret_cast<uint4*>(dyrecv + (int64_t)r * H);
    if (!real) {
      for (int v = lane; v < nvec; v += 32) d[v] = make_uint4(0u, 0u, 0u, 0u);
      continue;
    }
    const float w = metaw[r];
    for (int v = lane; v < nvec; v += 32) {
      uint4 a = d[v];
      __nv_bfloat162* ha = reinterpret_cast<__nv_bfloat162*>(&a);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 fa = __bfloat1622float2(ha[q]);
        ha[q] = __floats2bfloat162_rn(fa.x * w, fa.y * w);
      }
      d[v] = a;
    }
  }
}

// local combine / gather over this rank's own pairs: out[t] = (resid[t]) +
// sum_j (w ? w[t k + j] : 1) * rows[t k + j]  (warp per token, f32 accumulate)
__global__ void __launch_bounds__(256) ep_sum_pairs_kernel(const __nv_bfloat16* __restrict__ rows,
                                                           const float* __restrict__ w, int64_t T, int k, int H,
                                                           const __nv_bfloat16* __restrict__ resid,
                                                           __nv_bfloat16* __restrict__ out, const int* status) {
  const bool ok_s = status == nullptr || *reinterpret_cast<const volatile int*>(status) == 0;
  const int lane = threadIdx.x & 31;
  const int nvec = H / 8;
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32; t < T;
       t += (int64_t)gridDim.x * (blockDim.x / 32)) {
    for (int v = lane; v < nvec; v += 32) {
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (resid) {
        const uint4 r = reinterpret_cast<const uint4*>(resid + t * H)[v];
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&r);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = __bfloat1622float2(h[q]);
          acc[2 * q] = f.x;
          acc[2 * q + 1] = f.y;
        }
      }
      if (ok_s) {
        for (int j = 0; j < k; ++j) {
          const uint4 u = reinterpret_cast<const uint4*>(rows + (t * k + j) * H)[v];
          const float wj = w ? w[t * k + j] : 1.f;
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 f = __bfloat1622float2(h[q]);
            acc[2 * q] += wj * f.x;
            acc[2 * q + 1] += wj * f.y;
          }
        }
      }
      reinterpret_cast<uint4*>(out + t * H)[v] =
          make_uint4(pack_bf16(acc[0], acc[1]), pack_bf16(acc[2], acc[3]), pack_bf16(acc[4], acc[5]),
                     pack_bf16(acc[6], acc[7]));
    }
  }
}

int sm_count() {
  static int n = 0;
  if (!n) {
    int d;
    cudaGetDevice(&d);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, d);
  }
  return n;
}

unsigned warp_grid(int64_t items) {
  const int64_t blocks = (items + 7) / 8;  // 8 warps per 256-thread CTA
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>(blocks, (int64_t)sm_count() * 8));
}

}  // namespace

void launch_ep_counts(const int* local_counts, const uint64_t* peer_pads, int* my_pad, int rank, int W, int E, int seq,
                      int* all_counts, int* seg_off, int* recv_counts, int cap, int* overflow, int* need_max,
                      int* status, int64_t wait_ns, cudaStream_t st) {
  OXI_CHECK(W >= 1 && W <= EP_MAXW && E <= EP_MAXE && E % W == 0, "expert parallelism: W <= 8, E <= 256, W | E");
  ep_counts_kernel<<<1, 256, 0, st>>>(local_counts, peer_pads, my_pad, rank, W, E, seq, all_counts, seg_off,
                                      recv_counts, cap, overflow, need_max, status, (uint64_t)wait_ns);
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_ep_dispatch(const void* x, int64_t ldx, const int64_t* topi, const float* topw, int64_t T, int k, int H,
                        const int* all_counts, int rank, int W, int E, int* cursor, const uint64_t* peers_xrecv,
                        const uint64_t* peers_metaw, const uint64_t* peers_srcidx, int* pos_out, int* done_ctr,
                        const uint64_t* peer_pads, int seq, const int* seg_off, const int* status, cudaStream_t st) {
  OXI_CHECK(H % 8 == 0 && ldx % 8 == 0, "hidden size must be a multiple of 8");
  OXI_CHECK((int64_t)W * T * k < (1ll << 31), "source index must fit int32");
  OXI_CUDA_CHECK(cudaMemsetAsync(cursor, 0, sizeof(int) * E, st));
  ep_dispatch_kernel<<<warp_grid(T * k), 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(x), ldx, topi, topw, T,
                                                       k, H, all_counts, rank, W, E, cursor, peers_xrecv, peers_metaw,
                                                       peers_srcidx, pos_out, done_ctr, peer_pads, seq, seg_off,
                                                       status);
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_ep_mark_pad(const int* seg_off, const int* recv_counts, int El, int* srcidx, cudaStream_t st) {
  ep_mark_pad_kernel<<<El, 128, 0, st>>>(seg_off, recv_counts, El, srcidx);
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_ep_wait(const int* my_pad, int kind, int W, int seq, int* status, int64_t wait_ns, cudaStream_t st) {
  ep_wait_kernel<<<1, 32, 0, st>>>(my_pad, kind, W, seq, status, (uint64_t)wait_ns);
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_ep_signal(const uint64_t* peer_pads, int kind, int rank, int W, int seq, cudaStream_t st) {
  ep_signal_kernel<<<1, 32, 0, st>>>(peer_pads, kind, rank, W, seq);
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_ep_sum_pairs(const void* rows, const float* w, int64_t T, int k, int H, const void* resid, void* out,
                         const int* my_pad, int wait_kind, int W, int seq, int* status, int64_t wait_ns,
                         cudaStream_t st) {
  OXI_CHECK(H % 8 == 0, "hidden size must be a multiple of 8");
  // one thread waits for every owner's rows (the grid does not spin)
  ep_wait_kernel<<<1, 32, 0, st>>>(my_pad, wait_kind, W, seq, status, (uint64_t)wait_ns);
  ep_sum_pairs_kernel<<<warp_grid(T), 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(rows), w, T, k, H,
                                                    reinterpret_cast<const __nv_bfloat16*>(resid),
                                                    reinterpret_cast<__nv_bfloat16*>(out), status);
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_ep_push_dy(const void* dy, const int64_t* topi, const int* pos, int64_t T, int k, int H, int El,
                       const uint64_t* peers_dyrecv, const void* yret, float* dw, int* done_ctr,
                       const uint64_t* peer_pads, int rank, int W, int seq, const int* seg_off, const int* status,
                       cudaStream_t st) {
  ep_push_dy_kernel<<<warp_grid(T * k), 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(dy), topi, pos, T, k, H,
                                                      El, peers_dyrecv, reinterpret_cast<const __nv_bfloat16*>(yret),
                                                      dw, done_ctr, peer_pads, rank, W, seq, seg_off, status);
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_ep_scale_rows(void* dyrecv, const float* metaw, const int* seg_off, const int* recv_counts, int El, int H,
                          int64_t cap_rows, cudaStream_t st) {
  ep_scale_rows_kernel<<<warp_grid(cap_rows), 256, 0, st>>>(reinterpret_cast<__nv_bfloat16*>(dyrecv), metaw, seg_off,
                                                            recv_counts, El, H);
  OXI_CUDA_CHECK(cudaGetLastError());
}

}  // namespace oxi
