// Mixture-of-experts token permutation (counting sort into MOE_SEG_ALIGN-row-aligned
// expert segments), weighted combine, their backward passes, and the grouped
// GEMM launchers that run every expert's GEMM in one persistent launch.
//
// Layout: for T tokens with top-k routing, the permuted matrix X_perm has
// rows seg_off[e] .. seg_off[e] + count[e] for expert e, where seg_off is the
// prefix sum of counts rounded up to MOE_SEG_ALIGN = 256 (rows past count[e]
// are zero), so no GEMM tile - one CTA's 128 rows or a CTA pair's 256 - straddles
// two experts and the grouped weight-gradient GEMMs can reduce over whole
// 64-row k-blocks.  pos[t, j] is the row of token t's j-th
// expert.  Upstream computes every expert on every token (model.rs:561-565);
// the sparse result is the same for the same routing.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

#include "gemm_kernel.cuh"
#include "kernels.h"
#include "kernels_moe.h"

namespace oxi {
namespace {

__global__ void moe_count_kernel(const int64_t* __restrict__ topi, int64_t n, int E, int* __restrict__ counts) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int e = (int)topi[i];
    if (e >= 0 && e < E) atomicAdd(&counts[e], 1);
  }
}

// single block: seg_off[e] = sum_{e' < e} roundup(count[e'], MOE_SEG_ALIGN); cursor = seg_off
__global__ void moe_offsets_kernel(const int* __restrict__ counts, int E, int* __restrict__ seg_off,
                                   int* __restrict__ cursor) {
  if (threadIdx.x == 0) {
    int o = 0;
    for (int e = 0; e < E; ++e) {
      seg_off[e] = o;
      cursor[e] = o;
      o += (counts[e] + MOE_SEG_ALIGN - 1) / MOE_SEG_ALIGN * MOE_SEG_ALIGN;
    }
    seg_off[E] = o;
  }
}

// one warp per (token, slot): claim a row in the expert segment, copy the token row
__global__ void moe_scatter_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, const int64_t* __restrict__ topi,
                                   int64_t T, int k, int H, int* __restrict__ cursor, int* __restrict__ pos,
                                   __nv_bfloat16* __restrict__ xp) {
  const int64_t w = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (w >= T * k) return;
  const int e = (int)topi[w];
  int r = 0;
  if (lane == 0) r = atomicAdd(&cursor[e], 1);
  r = __shfl_sync(0xffffffffu, r, 0);
  if (lane == 0) pos[w] = r;
  const int64_t t = w / k;
  const uint4* src = reinterpret_cast<const uint4*>(x + t * ldx);
  uint4* dst = reinterpret_cast<uint4*>(xp + (int64_t)r * H);
  for (int i = lane; i < H / 8; i += 32) dst[i] = src[i];
}

// zero rows [seg_off[e] + count[e], seg_off[e+1]) of a [rows, H] matrix
__global__ void moe_zero_pad_kernel(const int* __restrict__ seg_off, const int* __restrict__ counts, int E,
                                    __nv_bfloat16* __restrict__ m, int H) {
  const int e = blockIdx.y;
  const int r0 = seg_off[e] + counts[e], r1 = seg_off[e + 1];
  const int64_t n = (int64_t)(r1 - r0) * (H / 8);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    reinterpret_cast<uint4*>(m + (int64_t)r0 * H)[i] = make_uint4(0, 0, 0, 0);
}

// y[t] = (resid[t]) + sum_j w[t,j] * yp[pos[t,j]]   (one warp per token)
__global__ void moe_combine_kernel(const __nv_bfloat16* __restrict__ yp, const int* __restrict__ pos,
                                   const float* __restrict__ w, int64_t T, int k, int H,
                                   const __nv_bfloat16* __restrict__ resid, __nv_bfloat16* __restrict__ y) {
  const int64_t t = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  for (int i = lane; i < H / 8; i += 32) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (resid) {
      const uint4 u = reinterpret_cast<const uint4*>(resid + t * H)[i];
      const __nv_bfloat162* hh = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __bfloat1622float2(hh[q]);
        acc[2 * q] = f.x;
        acc[2 * q + 1] = f.y;
      }
    }
    for (int j = 0; j < k; ++j) {
      const float wj = w[t * k + j];
      const uint4 u = reinterpret_cast<const uint4*>(yp + (int64_t)pos[t * k + j] * H)[i];
      const __nv_bfloat162* hh = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __bfloat1622float2(hh[q]);
        acc[2 * q] += wj * f.x;
        acc[2 * q + 1] += wj * f.y;
      }
    }
    reinterpret_cast<uint4*>(y + t * H)[i] = make_uint4(pack_bf16(acc[0], acc[1]), pack_bf16(acc[2], acc[3]),
                                                        pack_bf16(acc[4], acc[5]), pack_bf16(acc[6], acc[7]));
  }
}

// backward of the combine: dyp[pos[t,j]] = w[t,j] dy[t]; dw[t,j] = <dy[t], yp[pos[t,j]]>
// one warp per (token, slot)
__global__ void moe_combine_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ yp,
                                       const int* __restrict__ pos, const float* __restrict__ w, int64_t T, int k,
                                       int H, __nv_bfloat16* __restrict__ dyp, float* __restrict__ dw) {
  const int64_t q = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (q >= T * k) return;
  const int64_t t = q / k;
  const int r = pos[q];
  const float wj = w[q];
  float dot = 0.f;
  for (int i = lane; i < H / 8; i += 32) {
    const uint4 g = reinterpret_cast<const uint4*>(dy + t * H)[i];
    const uint4 v = reinterpret_cast<const uint4*>(yp + (int64_t)r * H)[i];
    const __nv_bfloat162* gh = reinterpret_cast<const __nv_bfloat162*>(&g);
    const __nv_bfloat162* vh = reinterpret_cast<const __nv_bfloat162*>(&v);
    float o[8];
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      const float2 gf = __bfloat1622float2(gh[s]), vf = __bfloat1622float2(vh[s]);
      dot += gf.x * vf.x + gf.y * vf.y;
      o[2 * s] = wj * gf.x;
      o[2 * s + 1] = wj * gf.y;
    }
    reinterpret_cast<uint4*>(dyp + (int64_t)r * H)[i] =
        make_uint4(pack_bf16(o[0], o[1]), pack_bf16(o[2], o[3]), pack_bf16(o[4], o[5]), pack_bf16(o[6], o[7]));
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
  if (lane == 0) dw[q] = dot;
}

// dx[t] = sum_j dxp[pos[t,j]]   (one warp per token)
__global__ void moe_gather_sum_kernel(const __nv_bfloat16* __restrict__ dxp, const int* __restrict__ pos, int64_t T,
                                      int k, int H, __nv_bfloat16* __restrict__ dx) {
  const int64_t t = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (t >= T) return;
  for (int i = lane; i < H / 8; i += 32) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < k; ++j) {
      const uint4 u = reinterpret_cast<const uint4*>(dxp + (int64_t)pos[t * k + j] * H)[i];
      const __nv_bfloat162* hh = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __bfloat1622float2(hh[q]);
        acc[2 * q] += f.x;
        acc[2 * q + 1] += f.y;
      }
    }
    reinterpret_cast<uint4*>(dx + t * H)[i] = make_uint4(pack_bf16(acc[0], acc[1]), pack_bf16(acc[2], acc[3]),
                                                         pack_bf16(acc[4], acc[5]), pack_bf16(acc[6], acc[7]));
  }
}

unsigned warps_grid(int64_t n) { return (unsigned)((n + 7) / 8); }

Operand op_of(const Mat& m, bool mn) {
  Operand o;
  o.ptr = m.ptr;
  o.ld = m.ld;
  o.mn = mn;
  if (!mn) { o.rows = m.rows; o.k = m.cols; }
  else { o.rows = m.cols; o.k = m.rows; }
  return o;
}

}  // namespace

void launch_moe_permute(const void* x, int64_t ldx, const int64_t* topi, int64_t T, int k, int E, int H, int* counts,
                        int* seg_off, int* cursor, int* pos, void* xp, cudaStream_t st) {
  OXI_CHECK(H % 8 == 0 && ldx % 8 == 0, "MoE hidden size must be a multiple of 8");
  OXI_CUDA_CHECK(cudaMemsetAsync(counts, 0, E * sizeof(int), st));
  if (T * k > 0) {
    moe_count_kernel<<<(unsigned)std::min<int64_t>((T * k + 255) / 256, 1024), 256, 0, st>>>(topi, T * k, E, counts);
  }
  moe_offsets_kernel<<<1, 32, 0, st>>>(counts, E, seg_off, cursor);
  if (T * k > 0)
    moe_scatter_kernel<<<warps_grid(T * k), 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(x), ldx, topi, T, k,
                                                          H, cursor, pos, reinterpret_cast<__nv_bfloat16*>(xp));
  moe_zero_pad_kernel<<<dim3(4, E), 256, 0, st>>>(seg_off, counts, E, reinterpret_cast<__nv_bfloat16*>(xp), H);
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_moe_zero_pad(const int* seg_off, const int* counts, int E, void* m, int H, cudaStream_t st) {
  moe_zero_pad_kernel<<<dim3(4, E), 256, 0, st>>>(seg_off, counts, E, reinterpret_cast<__nv_bfloat16*>(m), H);
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_moe_combine(const void* yp, const int* pos, const float* w, int64_t T, int k, int H, const void* resid,
                        void* y, cudaStream_t st) {
  if (!T) return;
  moe_combine_kernel<<<warps_grid(T), 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(yp), pos, w, T, k, H,
                                                    reinterpret_cast<const __nv_bfloat16*>(resid),
                                                    reinterpret_cast<__nv_bfloat16*>(y));
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_moe_combine_bwd(const void* dy, const void* yp, const int* pos, const float* w, int64_t T, int k, int H,
                            void* dyp, float* dw, cudaStream_t st) {
  if (!T) return;
  moe_combine_bwd_kernel<<<warps_grid(T * k), 256, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(dy), reinterpret_cast<const __nv_bfloat16*>(yp), pos, w, T, k, H,
      reinterpret_cast<__nv_bfloat16*>(dyp), dw);
  OXI_CUDA_CHECK(cudaGetLastError());
}

void launch_moe_gather_sum(const void* dxp, const int* pos, int64_t T, int k, int H, void* dx, cudaStream_t st) {
  if (!T) return;
  moe_gather_sum_kernel<<<warps_grid(T), 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(dxp), pos, T, k, H,
                                                       reinterpret_cast<__nv_bfloat16*>(dx));
  OXI_CUDA_CHECK(cudaGetLastError());
}

// Grouped GEMM.  mode 1 (group-M): a = permuted rows [rows, K] (K-major), b =
// stacked expert weights (K-major [E*N, K] or MN-major [E*K, N]); mode 2
// (group-K): a, b MN-major [rows, M] / [rows, N]; out = [E, M, N] f32 (+=).
// epi: 0 bf16, 1 f32 (+= out), 2 SwiGLU (out = h [rows, N/2], out2 = gu),
//      3 SwiGLU backward (out = dgu [rows, 2N], aux = gu).
void launch_gemm_grouped(int mode, int epi, const Mat& a, bool a_mn, const Mat& b, bool b_mn, int n_groups,
                         const int* seg_off, int64_t group_rows_b, void* out, int64_t ldo, void* out2, int64_t ldo2,
                         const void* aux, int64_t ldaux, int* status, cudaStream_t st,
                         const GroupedScatter* scatter) {
  Operand oa = op_of(a, a_mn), ob = op_of(b, b_mn);
  GemmParams p{};
  gemm_tuning(p);
  p.group_mode = mode;
  p.n_groups = n_groups;
  p.seg_off = seg_off;
  p.status = status;
  p.alpha = 1.f;
  p.splits = 1;
  if (mode == 1) {
    // per-expert N x K weights; the tensor map spans all experts
    p.M = (int)oa.rows;
    p.K = (int)oa.k;
    p.N = (int)(b_mn ? ob.rows : group_rows_b);
    OXI_CHECK(ob.k == (b_mn ? (int64_t)n_groups * oa.k : oa.k), "grouped GEMM: B/K mismatch");
    p.b_group_stride = group_rows_b;
    p.tiles_m = (p.M + BM - 1) / BM;
    p.tiles_n = (p.N + BN - 1) / BN;
    p.num_tiles = p.tiles_m * p.tiles_n;
  } else {
    OXI_CHECK(a_mn && b_mn && epi == 1, "group-K GEMM: MN-major operands, f32 accumulate");
    p.M = (int)oa.rows;
    p.N = (int)ob.rows;
    p.K = (int)oa.k;
    p.b_group_stride = 0;
    p.d_group_stride = (int64_t)p.M * ldo;
    p.tiles_m = (p.M + BM - 1) / BM;
    p.tiles_n = (p.N + BN - 1) / BN;
    p.num_tiles = n_groups * p.tiles_m * p.tiles_n;
  }
  p.kb_per_split = (p.K + BK - 1) / BK;
  if (p.M == 0 || p.num_tiles == 0) return;
  // CTA pairs (256 x 256 tiles, each CTA loading its own half of A and of B's
  // rows): group-M needs segments aligned to the pair's 256 rows; group-K tiles
  // the weight rows (the segments are its K range), so any alignment works.
  use_pairs_grouped(p, MOE_SEG_ALIGN);
  CUtensorMap ta = operand_tmap(oa, BM), tb = operand_tmap(ob, b_tile_rows(p));
  p.D = out;
  p.ldd = ldo;
  if (scatter) {
    OXI_CHECK(mode == 1 && epi == 0 && scatter->rows_per_peer > 0, "row scatter: group-M bf16 epilogue only");
    p.scatter_idx = scatter->idx;
    p.scatter_ptrs = scatter->ptrs;
    p.scatter_rows = scatter->rows_per_peer;
    p.post_ctr = scatter->post_ctr;
    p.post_pads = scatter->post_pads;
    p.post_kind = scatter->post_kind;
    p.post_rank = scatter->post_rank;
    p.post_W = scatter->post_W;
    p.post_seq = scatter->post_seq;
  }
  switch (epi) {
    case 0: {
      p.vec_ok = aligned16(out, ldo, 2);
      // rows stay in the concatenated segment order, so one 2-D map covers every expert;
      // scattered rows (expert parallelism) keep per-thread stores
      CUtensorMap td;
      const bool tma = !scatter && gemm_tma_epilogue() && aligned16(out, ldo, 2);
      if (tma) {
        td = make_tmap_out(out, p.M, p.N, ldo, false);
        p.tma_out = 1;
      }
      if (!b_mn) launch_t<false, false, EPI_BF16>(ta, tb, p, st, tma ? &td : nullptr);
      else launch_t<false, true, EPI_BF16>(ta, tb, p, st, tma ? &td : nullptr);
      break;
    }
    case 1: {
      p.vec_ok = aligned16(out, ldo, 4);
      p.beta = 1.f;
      CUtensorMap td;
      const bool tma = gemm_tma_epilogue() && aligned16(out, ldo, 4) && (p.d_group_stride * 4) % 16 == 0;
      if (tma) {
        td = make_tmap_out3_f32(out, n_groups, p.M, p.N, ldo, p.d_group_stride);
        p.tma_out = 4;
      }
      launch_t<true, true, EPI_F32>(ta, tb, p, st, tma ? &td : nullptr);
      break;
    }
    case 2:
      OXI_CHECK(!b_mn && p.N % 256 == 0, "grouped SwiGLU: K-major weights, 2I % 256 == 0");
      p.D2 = out2;
      p.ldd2 = ldo2;
      p.vec_ok = aligned16(out, ldo, 2) && aligned16(out2, ldo2, 2);
      if (gemm_tma_swiglu() && aligned16(out, ldo, 2) && (!out2 || aligned16(out2, ldo2, 2))) {
        const CUtensorMap th = make_tmap_out(out, p.M, p.N / 2, ldo, false);
        CUtensorMap tg;
        if (out2) tg = make_tmap_out(out2, p.M, p.N, ldo2, false);
        p.tma_out = 1;
        launch_t<false, false, EPI_SWIGLU>(ta, tb, p, st, &th, out2 ? &tg : nullptr);
      } else {
        launch_t<false, false, EPI_SWIGLU>(ta, tb, p, st);
      }
      break;
    case 3:
      OXI_CHECK(b_mn && p.N % 128 == 0, "grouped SwiGLU backward: MN-major weights");
      p.R = reinterpret_cast<const __nv_bfloat16*>(aux);
      p.ldr = ldaux;
      p.vec_ok = aligned16(out, ldo, 2) && aligned16(aux, ldaux, 2);
      launch_t<false, true, EPI_SWIGLU_BWD>(ta, tb, p, st);
      break;
    default:
      OXI_CHECK(false, "unknown grouped epilogue");
  }
}

}  // namespace oxi
