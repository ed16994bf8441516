#pragma once
// Persistent warp-specialised bf16 GEMM for sm_100a (tcgen05 + TMEM + TMA).
//
//   C[M,N] = sum_k A[m,k] * B[n,k]        (f32 accumulation in TMEM)
//
// A and B are each either K-major (row-major [rows, K]) or MN-major (stored
// transposed, row-major [K, rows]); the UMMA descriptors take either layout,
// so the three GEMMs of a linear layer (fwd, dX, dW) need no transposes.
//
// CTA tile 128 x 256 x 64, 4-stage TMA ring, two TMEM accumulators (2 x 256
// columns) so the epilogue of tile i overlaps the main loop of tile i+1.
// Warp roles (192 threads): warp 0 = TMA producer, warp 1 = MMA issuer and
// TMEM owner, warps 2..5 = epilogue (warp w reads TMEM lanes 32*(w%4)..+31).
//
// Epilogues (fused so no extra pass over the output is needed):
//   EPI_BF16        C -> bf16, optionally + bias[col] and + residual R (R may alias C)
//   EPI_F32         C -> f32, optionally + beta * C_old (gradient accumulation)
//   EPI_SWIGLU      B rows interleaved in blocks of 128 [gate|up]; writes
//                   H = silu(g)*u (bf16, N/2 columns) and the pre-activation GU
//   EPI_SWIGLU_BWD  C = dH; reads GU, writes dGU (interleaved like GU)
//   EPI_CE          C = logits; per (row, N-tile) max and sum(exp), target
//                   logit capture, optional bf16 logits store
//   EPI_ROPE        C = [q | k | v] projections; rotate-half RoPE on q and k
//                   heads using per-position cos/sin tables
//
// Every TMA load here is issued by one CTA for itself and reads local memory.
// Upstream: the reference's Linear / matmul calls on cuBLAS through Candle (e.g. model.rs:238,248,367,377,
// mamba2.rs:563,611,673,732) and the fused epilogue math of model.rs:68-117 (RoPE), model.rs:430-455
// (SwiGLU) and trainer.rs:166-171 (cross-entropy).
#include <cudaTypedefs.h>
#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "host_util.h"
#include "kernels_ep.h"

#include "ptx.cuh"

namespace oxi {

// An integer tuning knob from the environment, clamped to [lo, hi].
inline int gemm_env_int(const char* name, int dflt, int lo, int hi) {
  const char* e = getenv(name);
  if (!e || !*e) return dflt;
  return std::max(lo, std::min(hi, atoi(e)));
}


constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_STAGE_BYTES = BM * BK * 2;   // 16 KB
constexpr int B_STAGE_BYTES = BN * BK * 2;   // 32 KB
constexpr int STAGE_BYTES = A_STAGE_BYTES + B_STAGE_BYTES;
constexpr int GEMM_THREADS = 192;
constexpr int TMEM_COLS = 512;
constexpr int GROUP_M = 8;  // default row-tile grouping of the raster (OXI_GEMM_GROUP_M)

enum Epi : int { EPI_BF16 = 0, EPI_F32 = 1, EPI_SWIGLU = 2, EPI_SWIGLU_BWD = 3, EPI_CE = 4, EPI_ROPE = 5 };

struct GemmParams {
  int M, N, K;
  int tiles_m, tiles_n, num_tiles;  // num_tiles counts work units (tiles x splits)
  int group_m;                       // row tiles per raster group (consecutive units share B)
  int nst;                           // CTA-pair pipeline stages in use (<= PAIR_STAGES)
  int diag_nostore;                  // diagnostics: the epilogue drains TMEM but stores nothing
  int tma_out;                       // epilogue through shared memory + TMA: 0 off, 1 bf16 store,
                                     // 2 f32 store, 3 f32 reduce-add (the tmD map covers D),
                                     // 4 f32 reduce-add into expert e's slice of a 3-D [E][M][N] map
  int splits;                        // split-K factor (F32 accumulate epilogue only)
  int kb_per_split;
  void* D;                 // main output
  int64_t ldd;
  const __nv_bfloat16* R;  // residual (BF16) / GU (SWIGLU_BWD)
  int64_t ldr;
  const __nv_bfloat16* bias;  // BF16 epilogue: per-column bias [N] (may be null)
  void* D2;                // GU output (SWIGLU)
  int64_t ldd2;
  float beta;              // F32: C = acc + beta * C_old
  float alpha;             // scale applied to the accumulator
  // CE
  const int64_t* targets;
  float* part_max;         // [M, tiles_n]
  float* part_sum;         // [M, tiles_n]
  float* tgt_logit;        // [M]
  // RoPE
  const float* rope_cos;   // [S, hd/2]
  const float* rope_sin;
  int rope_seq, rope_hd, rope_q_cols, rope_k_cols;  // q columns [0,q), k columns [q, q+k)
  int vec_ok;              // output rows are 16-byte aligned
  int* status;
  // grouped (MoE) modes: 0 none; 1 group-M (A rows split into expert segments,
  // B rows offset by expert); 2 group-K (K split into expert segments, one
  // output matrix per expert).  seg_off[0..n_groups] are row offsets of the
  // segments (128-aligned; 256-aligned for CTA-pair group-M tiles), on the device.
  int group_mode;
  int n_groups;
  const int* seg_off;
  int64_t b_group_stride;  // B tensor-map rows per expert
  int64_t d_group_stride;  // output elements per expert (group-K)
  int cg;                  // 2: CTA-pair tiles (256 x 256, cta_group::2); else one CTA per 128 x 256 tile
  // BF16 epilogue, row scatter to peers (expert-parallel combine fused into the
  // expert GEMM): output row r goes to row (i % scatter_rows) of the buffer at
  // scatter_ptrs[i / scatter_rows], i = scatter_idx[r]; rows with i < 0 are
  // dropped.  The buffers may be other GPUs' memory (plain P2P stores).
  const int* scatter_idx;
  const uint64_t* scatter_ptrs;
  int scatter_rows;
  // after its last store the last CTA to finish posts flag (post_kind, post_rank)
  // = post_seq into every peer's signal pad (expert-parallel pad layout)
  int* post_ctr;
  const uint64_t* post_pads;
  int post_kind, post_rank, post_W, post_seq;
};

// CTA-pair configuration: each CTA holds 128 rows of A and 128 of B's 256 per
// k-block (32 KB per stage); six stages fit beside the epilogue's staging buffers
// (how many are used is a launch parameter, OXI_GEMM_PAIR_STAGES).
constexpr int PAIR_STAGES = 6;
// Epilogue staging for TMA stores: per epilogue warp two 4 KB boxes of 32 rows x 128 bytes.
constexpr int EPI_SMEM = 4 * 2 * 4096;
constexpr int PAIR_B_ROWS = 128;

__device__ __forceinline__ void tile_coords(int t, const GemmParams& p, int& tm, int& tn) {
  // Group GROUP_M row-tiles together so consecutive CTAs share B tiles in L2.
  t /= p.splits;
  const int group_m = p.group_m > 0 ? p.group_m : GROUP_M;
  const int per_group = group_m * p.tiles_n;
  const int g = t / per_group;
  const int first_m = g * group_m;
  const int gm = min(p.tiles_m - first_m, group_m);
  const int r = t - g * per_group;
  tm = first_m + (r % gm);
  tn = r / gm;
}

// k-block range of work unit t
__device__ __forceinline__ void unit_krange(int t, const GemmParams& p, int num_kb, int& kb0, int& kb1) {
  const int sp = t % p.splits;
  kb0 = sp * p.kb_per_split;
  kb1 = min(num_kb, kb0 + p.kb_per_split);
}

struct Unit {
  int tm, tn, kb0, kb1, e;
  bool valid;
};

// Work unit t -> output tile, k-block range, expert; identical in every role.
__device__ __forceinline__ Unit unit_info(int t, const GemmParams& p, int num_kb) {
  Unit u;
  u.e = 0;
  if (p.group_mode == 0) {
    tile_coords(t, p, u.tm, u.tn);
    unit_krange(t, p, num_kb, u.kb0, u.kb1);
    u.valid = true;
  } else if (p.group_mode == 1) {
    u.tm = t / p.tiles_n;
    u.tn = t % p.tiles_n;
    u.kb0 = 0;
    u.kb1 = num_kb;
    const int m0 = u.tm * BM * p.cg;  // a pair tile covers 2 * BM rows of one segment
    u.valid = m0 < __ldg(p.seg_off + p.n_groups);
    if (u.valid) {
      int lo = 0, hi = p.n_groups;  // last e with seg_off[e] <= m0
      while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (__ldg(p.seg_off + mid) <= m0) lo = mid; else hi = mid;
      }
      u.e = lo;
    }
  } else {
    const int per = p.tiles_m * p.tiles_n;
    u.e = t / per;
    tile_coords(t % per, p, u.tm, u.tn);
    u.kb0 = __ldg(p.seg_off + u.e) / BK;
    u.kb1 = __ldg(p.seg_off + u.e + 1) / BK;
    u.valid = u.kb1 > u.kb0;
  }
  return u;
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.f + __expf(-x)); }

// ------------------------------------------------------------------ stores
// 32 values -> bf16 at a 32-byte aligned address with two 32-byte stores (used
// for rows that go to another GPU: full-sector NVLink writes instead of 16-byte ones)
__device__ __forceinline__ void store_bf16_row32b(__nv_bfloat16* dst, const float* v) {
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    uint32_t w[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) w[i] = pack_bf16(v[q * 16 + 2 * i], v[q * 16 + 2 * i + 1]);
    asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(dst + q * 16), "r"(w[0]), "r"(w[1]),
                 "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
                 : "memory");
  }
}

__device__ __forceinline__ void store_bf16_row(__nv_bfloat16* dst, const float* v, int ncols_valid, bool vec) {
  if (vec && ncols_valid >= 32) {
    uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 w;
      w.x = pack_bf16(v[q * 8 + 0], v[q * 8 + 1]);
      w.y = pack_bf16(v[q * 8 + 2], v[q * 8 + 3]);
      w.z = pack_bf16(v[q * 8 + 4], v[q * 8 + 5]);
      w.w = pack_bf16(v[q * 8 + 6], v[q * 8 + 7]);
      d4[q] = w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < ncols_valid) dst[j] = __float2bfloat16(v[j]);
  }
}
__device__ __forceinline__ void load_bf16_row(const __nv_bfloat16* src, float* v, int ncols_valid, bool vec) {
  if (vec && ncols_valid >= 32) {
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 w = s4[q];
      float2 a = unpack_bf16(w.x), b = unpack_bf16(w.y), c = unpack_bf16(w.z), d = unpack_bf16(w.w);
      v[q * 8 + 0] = a.x; v[q * 8 + 1] = a.y; v[q * 8 + 2] = b.x; v[q * 8 + 3] = b.y;
      v[q * 8 + 4] = c.x; v[q * 8 + 5] = c.y; v[q * 8 + 6] = d.x; v[q * 8 + 7] = d.y;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = (j < ncols_valid) ? __bfloat162float(src[j]) : 0.f;
  }
}

// CG = 1: one CTA per 128 x 256 output tile.
// CG = 2: a cluster of two CTAs per 256 x 256 tile.  The even CTA ("leader")
// issues the pair MMAs (cta_group::2); each CTA TMA-loads its own 128 rows of A
// and its half of B's rows into its own shared memory and counts the bytes on the
// leader's `full` barrier; the leader's commits arrive on both CTAs' `empty` and
// `tfull` barriers; both CTAs' epilogue threads release an accumulator on the
// leader's `tempty`.  Every load reads global memory of this GPU only.
template <bool A_MN, bool B_MN, int EPI, int CG = 1>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmD, const __grid_constant__ CUtensorMap tmD2,
                GemmParams p) {
  constexpr int NST = CG == 2 ? PAIR_STAGES : STAGES;  // shared-memory layout (maximum)
  const int nst = CG == 2 ? (p.nst >= 2 && p.nst <= NST ? p.nst : NST) : STAGES;  // ring length in use
  constexpr int BROWS = CG == 2 ? PAIR_B_ROWS : BN;   // B rows held by this CTA
  constexpr int B_BYTES = BROWS * BK * 2;
  constexpr int ST_BYTES = A_STAGE_BYTES + B_BYTES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment is required by the 128B swizzle atoms.
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + NST * A_STAGE_BYTES;
  uint8_t* sEpi = smem + NST * ST_BYTES;  // 1024-aligned: stages are multiples of 16 KB
  uint64_t* bars = reinterpret_cast<uint64_t*>(sEpi + EPI_SMEM);
  uint64_t* full = bars;
  uint64_t* empty = bars + NST;
  uint64_t* tfull = bars + 2 * NST;
  uint64_t* tempty = bars + 2 * NST + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * NST + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const uint32_t rank = CG == 2 ? cluster_ctarank() : 0u;
  const int unit0 = CG == 2 ? (int)(blockIdx.x / 2) : (int)blockIdx.x;
  const int unit_step = CG == 2 ? (int)(gridDim.x / 2) : (int)gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128 * CG);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    if constexpr (CG == 2) {
      tmem_alloc_pair(tmem_slot, TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, TMEM_COLS);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  if constexpr (CG == 2) cluster_sync();  // both CTAs' barriers exist before any remote arrive
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_kb = (p.K + BK - 1) / BK;
  // shared::cluster address of an accumulator-release barrier (the leader's)
  auto release_acc = [&](int a) {
    if constexpr (CG == 2) mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[a]), 0));
    else mbar_arrive(&tempty[a]);
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed_parity[NST];
      bool armed[NST];
#pragma unroll
      for (int s = 0; s < NST; ++s) { armed[s] = false; armed_parity[s] = 0; }
      bool ok = true;
      for (int t = unit0; t < p.num_tiles && ok; t += unit_step) {
        const Unit un = unit_info(t, p, num_kb);
        if (!un.valid) continue;
        const int kb0 = un.kb0, kb1 = un.kb1;
        const int m0 = un.tm * BM * CG + (int)rank * BM;
        const int n0 = un.tn * BN + (int)rank * (CG == 2 ? PAIR_B_ROWS : 0);
        const int boff = (int)(un.e * p.b_group_stride);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.status)) { ok = false; break; }
          if (rank == 0) {
            mbar_arrive_expect_tx(&full[stage], ST_BYTES * CG);
            armed[stage] = true;
            armed_parity[stage] = phase;
          }
          uint8_t* a_dst = sA + stage * A_STAGE_BYTES;
          uint8_t* b_dst = sB + stage * B_BYTES;
          const int k0 = kb * BK;
          if constexpr (CG == 2) {
            const uint32_t bar = mapa_shared(smem_u32(&full[stage]), 0);
            if (!A_MN) {
              tma_load_2d_pair(a_dst, &tmA, bar, k0, m0);
            } else {
              tma_load_2d_pair(a_dst, &tmA, bar, m0, k0);
              tma_load_2d_pair(a_dst + BK * 128, &tmA, bar, m0 + 64, k0);
            }
            if (!B_MN) {
              tma_load_2d_pair(b_dst, &tmB, bar, k0, n0 + boff);
            } else {
#pragma unroll
              for (int q = 0; q < BROWS / 64; ++q)
                tma_load_2d_pair(b_dst + q * BK * 128, &tmB, bar, n0 + 64 * q, k0 + boff);
            }
          } else {
            if (!A_MN) {
              tma_load_2d(a_dst, &tmA, &full[stage], k0, m0);
            } else {
              tma_load_2d(a_dst, &tmA, &full[stage], m0, k0);
              tma_load_2d(a_dst + BK * 128, &tmA, &full[stage], m0 + 64, k0);
            }
            if (!B_MN) {
              tma_load_2d(b_dst, &tmB, &full[stage], k0, n0 + boff);
            } else {
#pragma unroll
              for (int q = 0; q < BROWS / 64; ++q)
                tma_load_2d(b_dst + q * BK * 128, &tmB, &full[stage], n0 + 64 * q, k0 + boff);
            }
          }
          if (++stage == nst) { stage = 0; phase ^= 1; }
        }
      }
      if (!ok) {
        // Drain the copies issued into barriers this thread armed before leaving (bounded).
        for (int s = 0; s < NST; ++s)
          if (armed[s]) mbar_wait(&full[s], armed_parity[s], nullptr, p.status);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && rank == 0) {
      constexpr uint32_t IDESC = umma_idesc_bf16(BM * CG, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = unit0; t < p.num_tiles && ok; t += unit_step) {
        const Unit un = unit_info(t, p, num_kb);
        if (!un.valid) continue;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, abort_flag, p.status)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        const int kb0 = un.kb0, kb1 = un.kb1;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.status)) { ok = false; break; }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * A_STAGE_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            uint64_t ad, bd;
            if (!A_MN) ad = umma_desc_sw128(a_addr + k * 32, 16, 1024);
            else       ad = umma_desc_sw128(a_addr + k * 2048, BK * 128, 1024);
            if (!B_MN) bd = umma_desc_sw128(b_addr + k * 32, 16, 1024);
            else       bd = umma_desc_sw128(b_addr + k * 2048, BK * 128, 1024);
            if constexpr (CG == 2) tc_mma_f16_pair(d_tmem, ad, bd, IDESC, (kb != kb0 || k != 0) ? 1u : 0u);
            else tc_mma_f16(d_tmem, ad, bd, IDESC, (kb != kb0 || k != 0) ? 1u : 0u);
          }
          if constexpr (CG == 2) {
            tc_commit_pair(mapa_shared(smem_u32(&empty[stage]), 0));
            tc_commit_pair(mapa_shared(smem_u32(&empty[stage]), 1));
          } else {
            tc_commit(&empty[stage]);
          }
          if (++stage == nst) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        if constexpr (CG == 2) {
          tc_commit_pair(mapa_shared(smem_u32(&tfull[acc]), 0));
          tc_commit_pair(mapa_shared(smem_u32(&tfull[acc]), 1));
        } else {
          tc_commit(&tfull[acc]);
        }
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;           // TMEM lane quarter this warp may access
    const int row_in_tile = quarter * 32 + lane;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    int acc = 0;
    uint32_t acc_phase = 0;
    const bool vec = p.vec_ok != 0;
    // TMA epilogue: this warp's two 4 KB staging boxes, and how many boxes it has issued
    uint8_t* eslab = sEpi + (warp - 2) * 8192;
    int ebox = 0;
    for (int t = unit0; t < p.num_tiles; t += unit_step) {
      const Unit un = unit_info(t, p, num_kb);
      if (!un.valid) continue;
      const int tn = un.tn;
      const int m0 = un.tm * BM * CG + (int)rank * BM, n0 = un.tn * BN;
      void* Dp = p.D;
      if (p.group_mode == 2) Dp = (char*)p.D + un.e * p.d_group_stride * (EPI == EPI_F32 ? 4 : 2);
      const int row = m0 + row_in_tile;
      const bool row_ok = row < p.M;
      // SwiGLU backward reads the saved gate / up values of its row: the 16-byte
      // vectors of the next 32-column chunk are loaded one chunk ahead (the first
      // before the accumulator wait), so their latency hides behind the TMEM loads
      // and the math of the current chunk instead of stalling every chunk.
      uint4 pre_g[4], pre_u[4];
      auto swb_full = [&](int cc) { return row_ok && vec && n0 + cc * 32 + 32 <= p.N; };
      auto swb_fetch = [&](int cc) {
        const int col = n0 + cc * 32;
        const uint4* gq = reinterpret_cast<const uint4*>(p.R + (int64_t)row * p.ldr + (col / 128) * 256 + col % 128);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          pre_g[q] = gq[q];
          pre_u[q] = gq[q + 16];  // the up block sits 128 columns after the gate block
        }
      };
      if constexpr (EPI == EPI_SWIGLU_BWD) {
        if (swb_full(0)) swb_fetch(0);
      }
      if (!mbar_wait(&tfull[acc], acc_phase, abort_flag, p.status)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + lane_base + acc * BN;
      // TMA epilogue helpers: a 32-row x 128-byte box in one of this warp's two staging
      // buffers (the box issued two boxes ago from it must have been read), filled from two
      // 32-value halves as bf16, then stored by one lane
      const int y = m0 + quarter * 32;  // first row of this warp's boxes
      auto box_begin = [&]() -> uint8_t* {
        uint8_t* b = eslab + (ebox & 1) * 4096;
        if (lane == 0) bulk_wait_read<1>();
        __syncwarp();
        return b;
      };
      auto box_fill = [&](uint8_t* b, const float* lo, const float* hi) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          sw128_store16(b, lane, q, make_uint4(pack_bf16(lo[q * 8], lo[q * 8 + 1]), pack_bf16(lo[q * 8 + 2], lo[q * 8 + 3]),
                                               pack_bf16(lo[q * 8 + 4], lo[q * 8 + 5]), pack_bf16(lo[q * 8 + 6], lo[q * 8 + 7])));
          sw128_store16(b, lane, 4 + q, make_uint4(pack_bf16(hi[q * 8], hi[q * 8 + 1]), pack_bf16(hi[q * 8 + 2], hi[q * 8 + 3]),
                                                   pack_bf16(hi[q * 8 + 4], hi[q * 8 + 5]), pack_bf16(hi[q * 8 + 6], hi[q * 8 + 7])));
        }
      };
      auto box_issue = [&](uint8_t* b, const CUtensorMap* tm, int x, int xmax) {
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          if (y < p.M && x < xmax && !p.diag_nostore) tma_store_2d(tm, b, x, y);
          bulk_commit();
        }
        ++ebox;
      };

      if ((EPI == EPI_BF16 || EPI == EPI_F32) && p.tma_out) {
        // Through shared memory: each warp stages its 32 rows of a 128-byte-wide column
        // block (64 bf16 or 32 f32 columns, 128B-swizzled) and one lane issues a TMA
        // store (or, for an accumulating f32 output, a TMA reduce-add performed in L2)
        // of the 32 x 128-byte box.  Full-line writes, no read of D by the threads; the
        // map clips rows past M and columns past N.
        constexpr int CPB = EPI == EPI_BF16 ? 2 : 1;  // 32-column chunks per box
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(tbase + c * 32, r);
          tc_wait_ld();
          if (c == BN / 32 - 1) { tc_fence_before(); release_acc(acc); }
          const int col = n0 + c * 32;
          const int nvalid = min(32, p.N - col);
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * p.alpha;
          if constexpr (EPI == EPI_BF16) {
            if (row_ok && nvalid > 0) {
              if (p.bias) {
                float bb[32];
                load_bf16_row(p.bias + col, bb, nvalid, vec);
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] += bb[j];
              }
              if (p.R) {
                float rr[32];
                load_bf16_row(p.R + (int64_t)row * p.ldr + col, rr, nvalid, vec);
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] += rr[j];
              }
            }
          }
          uint8_t* buf = eslab + (ebox & 1) * 4096;
          if (c % CPB == 0) {  // a new box: the box issued two boxes ago from this buffer was read
            if (lane == 0) bulk_wait_read<1>();
            __syncwarp();
          }
          if constexpr (EPI == EPI_BF16) {
#pragma unroll
            for (int q = 0; q < 4; ++q)
              sw128_store16(buf, lane, (c & 1) * 4 + q,
                            make_uint4(pack_bf16(v[q * 8], v[q * 8 + 1]), pack_bf16(v[q * 8 + 2], v[q * 8 + 3]),
                                       pack_bf16(v[q * 8 + 4], v[q * 8 + 5]), pack_bf16(v[q * 8 + 6], v[q * 8 + 7])));
          } else {
#pragma unroll
            for (int q = 0; q < 8; ++q)
              sw128_store16(buf, lane, q,
                            make_uint4(__float_as_uint(v[q * 4]), __float_as_uint(v[q * 4 + 1]),
                                       __float_as_uint(v[q * 4 + 2]), __float_as_uint(v[q * 4 + 3])));
          }
          if (c % CPB == CPB - 1) {
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) {
              const int x = n0 + (c - (CPB - 1)) * 32;
              if (y < p.M && x < p.N && !p.diag_nostore) {
                if (p.tma_out == 4) tma_reduce_add_3d(&tmD, buf, x, y, un.e);  // per-expert [E][M][N]
                else if (p.tma_out == 3) tma_reduce_add_2d(&tmD, buf, x, y);
                else tma_store_2d(&tmD, buf, x, y);
              }
              bulk_commit();
            }
            ++ebox;
          }
        }
      } else if constexpr (EPI == EPI_BF16 || EPI == EPI_F32 || EPI == EPI_SWIGLU_BWD) {
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(tbase + c * 32, r);
          uint4 cur_g[4], cur_u[4];
          if constexpr (EPI == EPI_SWIGLU_BWD) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              cur_g[q] = pre_g[q];
              cur_u[q] = pre_u[q];
            }
            if (c + 1 < BN / 32 && swb_full(c + 1)) swb_fetch(c + 1);
          }
          tc_wait_ld();
          if (c == BN / 32 - 1) { tc_fence_before(); release_acc(acc); }
          const int col = n0 + c * 32;
          const int nvalid = min(32, p.N - col);
          if (!row_ok || nvalid <= 0 || p.diag_nostore) continue;
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * p.alpha;
          if constexpr (EPI == EPI_BF16) {
            __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(Dp) + (int64_t)row * p.ldd + col;
            if (p.scatter_idx) {
              const int si = __ldg(p.scatter_idx + row);
              if (si < 0) continue;
              dst = reinterpret_cast<__nv_bfloat16*>(p.scatter_ptrs[si / p.scatter_rows]) +
                    (int64_t)(si % p.scatter_rows) * p.ldd + col;
              if (vec && nvalid >= 32 && (reinterpret_cast<uintptr_t>(dst) & 31) == 0) {
                store_bf16_row32b(dst, v);
                continue;
              }
            }
            if (p.bias) {
              float bb[32];
              load_bf16_row(p.bias + col, bb, nvalid, (reinterpret_cast<uintptr_t>(p.bias) & 15) == 0);
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] += bb[j];
            }
            if (p.R) {
              float rr[32];
              load_bf16_row(p.R + (int64_t)row * p.ldr + col, rr, nvalid, vec);
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] += rr[j];
            }
            store_bf16_row(dst, v, nvalid, vec);
          } else if constexpr (EPI == EPI_F32) {
            float* dst = reinterpret_cast<float*>(Dp) + (int64_t)row * p.ldd + col;
            if (p.splits > 1) {
              // split-K partial sums accumulate into the output (beta == 1)
              if (vec && nvalid >= 32) {
                float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
                for (int q = 0; q < 8; ++q)
                  atomicAdd(d4 + q, make_float4(v[q * 4], v[q * 4 + 1], v[q * 4 + 2], v[q * 4 + 3]));
              } else {
                for (int j = 0; j < nvalid; ++j) atomicAdd(dst + j, v[j]);
              }
            } else if (vec && nvalid >= 32) {
              float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
              for (int q = 0; q < 8; ++q) {
                float4 o = make_float4(v[q * 4], v[q * 4 + 1], v[q * 4 + 2], v[q * 4 + 3]);
                if (p.beta != 0.f) {
                  float4 old = d4[q];
                  o.x += p.beta * old.x; o.y += p.beta * old.y; o.z += p.beta * old.z; o.w += p.beta * old.w;
                }
                d4[q] = o;
              }
            } else {
              for (int j = 0; j < nvalid; ++j) dst[j] = v[j] + (p.beta != 0.f ? p.beta * dst[j] : 0.f);
            }
          } else {  // EPI_SWIGLU_BWD: v = dH columns; GU interleaved in blocks of 128
            const int blk = col / 128, off = col % 128;
            const __nv_bfloat16* gp = p.R + (int64_t)row * p.ldr + blk * 256 + off;
            const __nv_bfloat16* up = gp + 128;
            float g[32], u[32];
            if (swb_full(c)) {
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                const uint32_t gw[4] = {cur_g[q].x, cur_g[q].y, cur_g[q].z, cur_g[q].w};
                const uint32_t uw[4] = {cur_u[q].x, cur_u[q].y, cur_u[q].z, cur_u[q].w};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                  const float2 a = unpack_bf16(gw[k]), b = unpack_bf16(uw[k]);
                  g[q * 8 + 2 * k] = a.x;
                  g[q * 8 + 2 * k + 1] = a.y;
                  u[q * 8 + 2 * k] = b.x;
                  u[q * 8 + 2 * k + 1] = b.y;
                }
              }
            } else {
              load_bf16_row(gp, g, nvalid, vec);
              load_bf16_row(up, u, nvalid, vec);
            }
            float dg[32], du[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float s = 1.f / (1.f + __expf(-g[j]));
              const float sg = g[j] * s;
              du[j] = v[j] * sg;
              dg[j] = v[j] * u[j] * s * (1.f + g[j] * (1.f - s));
            }
            __nv_bfloat16* dgp = reinterpret_cast<__nv_bfloat16*>(Dp) + (int64_t)row * p.ldd + blk * 256 + off;
            store_bf16_row(dgp, dg, nvalid, vec);
            store_bf16_row(dgp + 128, du, nvalid, vec);
          }
        }
      } else if (EPI == EPI_SWIGLU && p.tma_out) {
        // TMA form: per pair of 32-column chunks, the 64 gate and 64 up pre-activation columns
        // of gu (map tmD2) and the 64 columns of h = silu(gate) * up (map tmD) each leave as
        // one 32-row x 128-byte box
#pragma unroll 1
        for (int c = 0; c < 4; c += 2) {
          uint32_t rg0[32], ru0[32], rg1[32], ru1[32];
          tmem_ld32(tbase + c * 32, rg0);
          tmem_ld32(tbase + 128 + c * 32, ru0);
          tmem_ld32(tbase + (c + 1) * 32, rg1);
          tmem_ld32(tbase + 128 + (c + 1) * 32, ru1);
          tc_wait_ld();
          if (c == 2) { tc_fence_before(); release_acc(acc); }
          float g0[32], g1[32], u0[32], u1[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            g0[j] = __uint_as_float(rg0[j]);
            g1[j] = __uint_as_float(rg1[j]);
            u0[j] = __uint_as_float(ru0[j]);
            u1[j] = __uint_as_float(ru1[j]);
          }
          if (p.D2) {
            uint8_t* b = box_begin();
            box_fill(b, g0, g1);
            box_issue(b, &tmD2, n0 + c * 32, p.N);
            b = box_begin();
            box_fill(b, u0, u1);
            box_issue(b, &tmD2, n0 + 128 + c * 32, p.N);
          }
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            g0[j] = silu_f(g0[j]) * u0[j];
            g1[j] = silu_f(g1[j]) * u1[j];
          }
          uint8_t* b = box_begin();
          box_fill(b, g0, g1);
          box_issue(b, &tmD, n0 / 2 + c * 32, p.N / 2);
        }
      } else if constexpr (EPI == EPI_SWIGLU) {
        // tile columns [0,128) gate, [128,256) up, for output columns n0/2 + [0,128)
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t rg[32], ru[32];
          tmem_ld32(tbase + c * 32, rg);
          tmem_ld32(tbase + 128 + c * 32, ru);
          tc_wait_ld();
          if (c == 3) { tc_fence_before(); release_acc(acc); }
          const int hcol = n0 / 2 + c * 32;
          const int nvalid = min(32, p.N / 2 - hcol);
          if (!row_ok || nvalid <= 0) continue;
          float g[32], u[32], h[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            g[j] = __uint_as_float(rg[j]);
            u[j] = __uint_as_float(ru[j]);
            h[j] = silu_f(g[j]) * u[j];
          }
          store_bf16_row(reinterpret_cast<__nv_bfloat16*>(Dp) + (int64_t)row * p.ldd + hcol, h, nvalid, vec);
          if (p.D2) {
            __nv_bfloat16* gu = reinterpret_cast<__nv_bfloat16*>(p.D2) + (int64_t)row * p.ldd2 + n0 + c * 32;
            store_bf16_row(gu, g, nvalid, vec);
            store_bf16_row(gu + 128, u, nvalid, vec);
          }
        }
      } else if constexpr (EPI == EPI_CE) {
        // two 32-column chunks per TMEM round trip (both loads, then one wait)
        float run_max = -INFINITY, run_sum = 0.f;
        const int64_t tgt = row_ok ? p.targets[row] : -1;
#pragma unroll 1
        for (int c = 0; c < BN / 32; c += 2) {
          uint32_t r0[32], r1[32];
          tmem_ld32(tbase + c * 32, r0);
          tmem_ld32(tbase + (c + 1) * 32, r1);
          tc_wait_ld();
          if (c + 2 == BN / 32) { tc_fence_before(); release_acc(acc); }
          const int col = n0 + c * 32;
          const int nvalid = min(64, p.N - col);
          // the TMA logit store is warp-wide: every lane takes part even without a row
          if (!p.tma_out && (!row_ok || nvalid <= 0)) continue;
          float v[64];
          float cmax = -INFINITY;
#pragma unroll
          for (int j = 0; j < 64; ++j) {
            v[j] = __uint_as_float(j < 32 ? r0[j] : r1[j - 32]) * p.alpha;
            if (j < nvalid) cmax = fmaxf(cmax, v[j]);
          }
          if (row_ok && nvalid > 0) {
            const float nmax = fmaxf(run_max, cmax);
            float s = 0.f;
#pragma unroll
            for (int j = 0; j < 64; ++j)
              if (j < nvalid) s += __expf(v[j] - nmax);
            run_sum = run_sum * __expf(run_max - nmax) + s;
            run_max = nmax;
            if (tgt >= col && tgt < col + nvalid) {
              float tv = 0.f;
#pragma unroll
              for (int j = 0; j < 64; ++j)
                if (col + j == tgt) tv = v[j];
              p.tgt_logit[row] = tv;
            }
          }
          if (Dp) {
            if (p.tma_out) {
              uint8_t* b = box_begin();
              box_fill(b, v, v + 32);
              box_issue(b, &tmD, col, p.N);
            } else {
              __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(Dp) + (int64_t)row * p.ldd + col;
              store_bf16_row(dst, v, min(32, nvalid), vec);
              if (nvalid > 32) store_bf16_row(dst + 32, v + 32, nvalid - 32, vec);
            }
          }
        }
        if (row_ok) {
          p.part_max[(int64_t)row * p.tiles_n + tn] = run_max;
          p.part_sum[(int64_t)row * p.tiles_n + tn] = run_sum;
        }
      } else if constexpr (EPI == EPI_ROPE) {
        // Heads are rope_hd wide; each pair of 32-column chunks (c, c + half/32)
        // forms the rotate-half pair for one head.
        const int hd = p.rope_hd, half = hd / 2;
        const int pos = row % p.rope_seq;
        const int nch = BN / 32, pair_off = half / 32;
#pragma unroll 1
        for (int c = 0; c < nch; ++c) {
          const int col = n0 + c * 32;
          const int in_head = (c * 32) % hd;   // tiles start at head boundaries (BN % hd == 0)
          if (in_head >= half) continue;        // handled with its partner
          const bool rot = col < p.rope_q_cols + p.rope_k_cols;
          // cos / sin of this row's position: 16-byte loads issued before the TMEM loads so
          // their latency overlaps (table rows are 16-byte aligned, in_head % 32 == 0)
          float cj[32], sj[32];
          if (rot) {
            const float4* cs4 = reinterpret_cast<const float4*>(p.rope_cos + (int64_t)pos * half + in_head);
            const float4* sn4 = reinterpret_cast<const float4*>(p.rope_sin + (int64_t)pos * half + in_head);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const float4 cv = __ldg(cs4 + q), sv = __ldg(sn4 + q);
              cj[4 * q] = cv.x; cj[4 * q + 1] = cv.y; cj[4 * q + 2] = cv.z; cj[4 * q + 3] = cv.w;
              sj[4 * q] = sv.x; sj[4 * q + 1] = sv.y; sj[4 * q + 2] = sv.z; sj[4 * q + 3] = sv.w;
            }
          }
          uint32_t r1[32], r2[32];
          tmem_ld32(tbase + c * 32, r1);
          tmem_ld32(tbase + (c + pair_off) * 32, r2);
          tc_wait_ld();
          const bool last = (c + pair_off == nch - 1) || (c == nch - 1);
          if (last) { tc_fence_before(); release_acc(acc); }
          const int nvalid = min(32, p.N - col);
          if (!row_ok || nvalid <= 0) continue;
          float x1[32], x2[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) { x1[j] = __uint_as_float(r1[j]); x2[j] = __uint_as_float(r2[j]); }
          if (rot) {
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              const float a = x1[j], b = x2[j];
              x1[j] = a * cj[j] - b * sj[j];
              x2[j] = b * cj[j] + a * sj[j];
            }
          }
          __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(Dp) + (int64_t)row * p.ldd + col;
          store_bf16_row(dst, x1, nvalid, vec);
          const int nvalid2 = min(32, p.N - (col + half));
          if (nvalid2 > 0) store_bf16_row(dst + half, x2, nvalid2, vec);
        }
      }
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    if (p.tma_out && lane == 0) bulk_wait<0>();  // every TMA store / reduce of this warp performed
  }

  tc_fence_before();
  if (p.post_ctr) __threadfence_system();  // this thread's (peer) stores before the flag
  if constexpr (CG == 2) cluster_sync();  // no remote arrive or pair MMA is still aimed at this CTA
  else __syncthreads();
  if (p.post_ctr && threadIdx.x == 0) {
    if (atomicAdd(p.post_ctr, 1) == (int)gridDim.x - 1) {
      *p.post_ctr = 0;
      __threadfence_system();
      for (int i = 0; i < p.post_W; ++i) {
        int* f = reinterpret_cast<int*>(p.post_pads[i]) + EP_FLAGS + p.post_kind * EP_MAXW + p.post_rank;
        asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(f), "r"(p.post_seq) : "memory");
      }
    }
  }
  if (warp == 1) {
    tc_fence_after();
    if constexpr (CG == 2) tmem_dealloc_pair(tmem_base, TMEM_COLS);
    else tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ====================================================================== host
inline PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* ptr = nullptr;
    OXI_CUDA_CHECK(cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000, cudaEnableDefault, &q));
    OXI_CHECK(q == cudaDriverEntryPointSuccess && ptr, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

// cuTensorMapEncodeTiled is a driver call and needs a current context.  Autograd runs
// backward on a thread of its own; when one of these ops is the first CUDA work there,
// no runtime call has made the primary context current yet (the device guard does
// nothing when the device already matches).  cudaSetDevice makes it current (CUDA 12).
inline void ensure_current_context() {
  thread_local unsigned long long ready = 0;
  int dev = 0;
  OXI_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev < 64 && ((ready >> dev) & 1ull)) return;
  OXI_CUDA_CHECK(cudaSetDevice(dev));
  if (dev < 64) ready |= 1ull << dev;
}

// 2-D bf16 tensor map over a row-major matrix [rows, cols] with row stride
// `ld` elements, box {box_cols, box_rows}, 128-byte swizzle, zero OOB fill.
inline CUtensorMap make_tmap_bf16(const void* base, int64_t rows, int64_t cols, int64_t ld, int box_cols, int box_rows,
                                  CUtensorMapL2promotion promo = CU_TENSOR_MAP_L2_PROMOTION_L2_256B) {
  OXI_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, "TMA base must be 16-byte aligned");
  OXI_CHECK((ld * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes (ld % 8 == 0)");
  ensure_current_context();
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                               estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, promo,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  OXI_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", (int)r);
  return m;
}

// 2-D tensor map over the GEMM output D [rows, cols] (row stride ld elements) for the TMA
// epilogue: boxes of 32 rows x 128 bytes (64 bf16 or 32 f32 columns), 128-byte swizzle.
inline CUtensorMap make_tmap_out(void* base, int64_t rows, int64_t cols, int64_t ld, bool f32) {
  const int es = f32 ? 4 : 2;
  OXI_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0 && (ld * es) % 16 == 0, "TMA output alignment");
  ensure_current_context();
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * es)};
  cuuint32_t box[2] = {(cuuint32_t)(128 / es), 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode_fn()(&m, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base,
                               dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  OXI_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (GEMM output) failed: ", (int)r);
  return m;
}

// 3-D f32 map over per-expert outputs [groups][rows][cols] (row stride ld, expert stride
// group_stride elements) for the grouped weight-gradient reduce-adds.
inline CUtensorMap make_tmap_out3_f32(void* base, int64_t groups, int64_t rows, int64_t cols, int64_t ld,
                                      int64_t group_stride) {
  OXI_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0 && (ld * 4) % 16 == 0 && (group_stride * 4) % 16 == 0,
            "TMA output alignment (grouped)");
  ensure_current_context();
  CUtensorMap m;
  cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)groups};
  cuuint64_t strides[2] = {(cuuint64_t)(ld * 4), (cuuint64_t)(group_stride * 4)};
  cuuint32_t box[3] = {32, 32, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = get_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, dims, strides, box, estr,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  OXI_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (grouped GEMM output) failed: ", (int)r);
  return m;
}

// Whether the TMA epilogue is enabled (OXI_GEMM_TMA_EPI=0 keeps per-thread stores;
// OXI_GEMM_TMA_SWIGLU=0 / OXI_GEMM_TMA_CE=0 only for the SwiGLU / cross-entropy epilogue).
inline bool gemm_tma_epilogue() {
  static const int on = gemm_env_int("OXI_GEMM_TMA_EPI", 1, 0, 1);
  return on != 0;
}
inline bool gemm_tma_swiglu() {
  static const int on = gemm_env_int("OXI_GEMM_TMA_SWIGLU", 1, 0, 1);
  return on != 0 && gemm_tma_epilogue();
}
inline bool gemm_tma_ce() {  // OXI_GEMM_TMA_CE=0: the cross-entropy epilogue's logits per thread
  static const int on = gemm_env_int("OXI_GEMM_TMA_CE", 1, 0, 1);
  return on != 0 && gemm_tma_epilogue();
}

inline int num_sms() {
  static int n = 0;
  if (!n) {
    int dev;
    OXI_CUDA_CHECK(cudaGetDevice(&dev));
    OXI_CUDA_CHECK(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  }
  return n;
}

constexpr int GEMM_SMEM = STAGES * STAGE_BYTES + EPI_SMEM + 1024 /*align*/ + 256 /*barriers*/;
constexpr int GEMM_PAIR_SMEM = PAIR_STAGES * (A_STAGE_BYTES + PAIR_B_ROWS * BK * 2) + EPI_SMEM + 1024 + 256;
static_assert(GEMM_SMEM <= 232448 && GEMM_PAIR_SMEM <= 232448, "GEMM shared memory budget");

// Clusters of two (one CTA per SM) that fit on the device at once.
template <typename K>
inline int max_pair_clusters(K kern) {
  static int n = -1;
  if (n < 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * num_sms(), 1, 1);
    cfg.blockDim = dim3(GEMM_THREADS, 1, 1);
    cfg.dynamicSmemBytes = GEMM_PAIR_SMEM;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int c = 0;
    OXI_CUDA_CHECK(cudaOccupancyMaxActiveClusters(&c, kern, &cfg));
    n = c;
  }
  return n;
}

template <bool A_MN, bool B_MN, int EPI>
static void launch_t(const CUtensorMap& ta, const CUtensorMap& tb, GemmParams& p, cudaStream_t st,
                     const CUtensorMap* td = nullptr, const CUtensorMap* td2 = nullptr) {
  if (p.num_tiles <= 0) return;
  CUtensorMap tdv, tdv2;
  if (td) tdv = *td;
  else memset(&tdv, 0, sizeof(tdv));
  if (td2) tdv2 = *td2;
  else memset(&tdv2, 0, sizeof(tdv2));
  if (!td) p.tma_out = 0;
  if (p.cg == 2) {
    auto kern = gemm_kernel<A_MN, B_MN, EPI, 2>;
    static bool attr = false;
    if (!attr) {
      OXI_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, GEMM_PAIR_SMEM));
      attr = true;
    }
    const int clusters = std::min(p.num_tiles, std::max(1, max_pair_clusters(kern)));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * clusters, 1, 1);
    cfg.blockDim = dim3(GEMM_THREADS, 1, 1);
    cfg.dynamicSmemBytes = GEMM_PAIR_SMEM;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 2;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    OXI_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, ta, tb, tdv, tdv2, p));
    return;
  }
  auto kern = gemm_kernel<A_MN, B_MN, EPI, 1>;
  static bool attr = false;
  if (!attr) {
    OXI_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, GEMM_SMEM));
    attr = true;
  }
  int grid = std::min(p.num_tiles, num_sms());
  kern<<<grid, GEMM_THREADS, GEMM_SMEM, st>>>(ta, tb, tdv, tdv2, p);
  OXI_CUDA_CHECK(cudaGetLastError());
}

template <int EPI>
static void launch_epi(bool a_mn, bool b_mn, const CUtensorMap& ta, const CUtensorMap& tb, GemmParams& p,
                       cudaStream_t st, const CUtensorMap* td = nullptr) {
  if (!a_mn && !b_mn) launch_t<false, false, EPI>(ta, tb, p, st, td);
  else if (!a_mn && b_mn) launch_t<false, true, EPI>(ta, tb, p, st, td);
  else if (a_mn && !b_mn) launch_t<true, false, EPI>(ta, tb, p, st, td);
  else launch_t<true, true, EPI>(ta, tb, p, st, td);
}

// Launch tuning shared by every GEMM entry point (read once per process).
inline void gemm_tuning(GemmParams& p) {
  static const int gm = gemm_env_int("OXI_GEMM_GROUP_M", GROUP_M, 1, 64);
  static const int ns = gemm_env_int("OXI_GEMM_PAIR_STAGES", PAIR_STAGES, 2, PAIR_STAGES);
  static const int ns0 = gemm_env_int("OXI_GEMM_DIAG_NOSTORE", 0, 0, 1);
  p.group_m = gm;
  p.nst = ns;
  p.diag_nostore = ns0;
}

// Operand description (row-major storage, unit inner stride):
//  K-major operand with R rows: stored [R, K]  (mn=false)
//  MN-major operand with R rows: stored [K, R] (mn=true)
struct Operand {
  const void* ptr;
  int64_t rows, k, ld;
  bool mn;
};

inline CUtensorMap operand_tmap(const Operand& o, int tile_rows) {
  // L2 sector promotion of the operand loads (OXI_GEMM_L2PROMO: 0 none, 1 64 B, 2 128 B, 3 256 B)
  static const int pr = gemm_env_int("OXI_GEMM_L2PROMO", 3, 0, 3);
  const CUtensorMapL2promotion promo = pr == 0 ? CU_TENSOR_MAP_L2_PROMOTION_NONE
                                       : pr == 1 ? CU_TENSOR_MAP_L2_PROMOTION_L2_64B
                                       : pr == 2 ? CU_TENSOR_MAP_L2_PROMOTION_L2_128B
                                                 : CU_TENSOR_MAP_L2_PROMOTION_L2_256B;
  if (!o.mn) return make_tmap_bf16(o.ptr, o.rows, o.k, o.ld, BK, tile_rows, promo);
  // stored [K, rows]; box = 64 row-elements (inner) x BK k-rows
  return make_tmap_bf16(o.ptr, o.k, o.rows, o.ld, 64, BK, promo);
}

inline void fill_common(GemmParams& p, const Operand& a, const Operand& b) {
  OXI_CHECK(a.k == b.k, "GEMM K mismatch: ", a.k, " vs ", b.k);
  p.M = (int)a.rows;
  p.N = (int)b.rows;
  p.K = (int)a.k;
  p.tiles_m = (p.M + BM - 1) / BM;
  p.tiles_n = (p.N + BN - 1) / BN;
  p.splits = 1;
  p.kb_per_split = (p.K + BK - 1) / BK;
  p.num_tiles = p.tiles_m * p.tiles_n;
  p.alpha = 1.f;
  p.cg = 1;
  gemm_tuning(p);
}

// Switch a plain (ungrouped) GEMM to CTA-pair 256 x 256 tiles when it has more
// than one 128-row tile of output (OXI_GEMM_CG=1 keeps single-CTA tiles).  Call
// before choose_splits and before building B's tensor map (b_tile_rows).
inline void use_pairs(GemmParams& p) {
  static int mode = -1;
  if (mode < 0) {
    const char* e = getenv("OXI_GEMM_CG");
    mode = (e && e[0] == '1') ? 1 : 2;
  }
  if (mode != 2 || p.group_mode != 0 || p.M <= BM) return;
  p.cg = 2;
  p.tiles_m = (p.M + 2 * BM - 1) / (2 * BM);
  p.num_tiles = p.tiles_m * p.tiles_n;
}

// The same for the grouped (MoE) GEMMs: group-M tiles need expert segments
// aligned to the pair's 2 * BM rows (seg_align); group-K pairs tile the weight
// rows of each expert's output and take any segment alignment.
inline void use_pairs_grouped(GemmParams& p, int seg_align) {
  static int mode = -1;
  if (mode < 0) {
    const char* e = getenv("OXI_GEMM_CG");
    mode = (e && e[0] == '1') ? 1 : 2;
  }
  if (mode != 2 || p.M <= BM) return;
  if (p.group_mode == 1 && seg_align % (2 * BM) != 0) return;
  p.cg = 2;
  p.tiles_m = (p.M + 2 * BM - 1) / (2 * BM);
  p.num_tiles = (p.group_mode == 2 ? p.n_groups : 1) * p.tiles_m * p.tiles_n;
}

// Rows of B per CTA tile (the box height of B's tensor map when K-major).
inline int b_tile_rows(const GemmParams& p) { return p.cg == 2 ? PAIR_B_ROWS : BN; }

// Split K across CTAs when there are too few output tiles to fill the GPU
// (weight-gradient GEMMs: small M x N, K = tokens).  Only valid for an
// accumulating f32 output, whose epilogue adds atomically (TMA reduce-add in L2,
// or per-thread f32 atomics without the TMA epilogue).  The split count
// is chosen for wave fill over the units that run at once (CTAs, or clusters
// for CTA pairs): the smallest count within 2 % of the best fill, at least 16
// k-blocks per split, at most four waves of units (more splits cost more in f32
// atomics than the better fill gains; measured on the dW shapes).
inline void choose_splits(GemmParams& p) {
  const int tiles = p.tiles_m * p.tiles_n;
  const int num_kb = (p.K + BK - 1) / BK;
  const int slots = p.cg == 2 ? num_sms() / 2 : num_sms();
  if (tiles >= 2 * slots || num_kb < 32) return;
  const int smax = std::max(1, std::min(num_kb / 16, (4 * slots + tiles - 1) / tiles));
  auto fill = [&](int s) {
    const int64_t u = (int64_t)tiles * s;
    const int64_t waves = (u + slots - 1) / slots;
    return (double)u / (double)(waves * slots);
  };
  double best = 0.0;
  for (int s = 1; s <= smax; ++s) best = std::max(best, fill(s));
  int s = 1;
  while (s < smax && fill(s) < best - 0.02) ++s;
  if (s <= 1) return;
  p.kb_per_split = (num_kb + s - 1) / s;
  p.splits = (num_kb + p.kb_per_split - 1) / p.kb_per_split;
  p.num_tiles = tiles * p.splits;
}

inline bool aligned16(const void* ptr, int64_t ld, int esize) {
  return ((reinterpret_cast<uintptr_t>(ptr) & 15) == 0) && ((ld * esize) % 16 == 0);
}

}  // namespace oxi
