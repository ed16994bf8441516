// Causal flash attention for sm_100a (tcgen05 + TMEM + TMA), forward.
//
// One CTA per (128-query tile, query head, batch).  Q (128 x D) stays in
// shared memory; K/V tiles of 128 keys stream through a 2-stage TMA ring.
//   S_j = Q K_j^T        tcgen05.mma, f32 accumulator in TMEM (2 buffers)
//   P_j = exp2(S_j*c - m) softmax warps: one thread per query row; P (bf16) is
//                        written back into the TMEM columns of S_j
//   O  += P_j V_j        tcgen05.mma with A = P from TMEM, f32 accumulator in
//                        TMEM (V as MN-major B from shared memory)
// The running max is only moved (and O rescaled) when the row max grows by
// more than 2^8, so the TMEM read-modify-write of O is rare after the first
// tiles.  S is double-buffered and P lives in its S buffer, so the softmax of
// tile j+1 never waits for PV_j (only an O rescale does); the MMA warp issues
// S_{j+1} before waiting for P_j.  MMAs issued by one thread run in order, so
// S_{j+2} overwrites P_j only after PV_j has read it.
//
// Layout: q/k are row-major [B*S, H*DQ] views and v [B*S, Hk*DV] (row strides
// ld*), head h at columns [h*DQ, (h+1)*DQ) resp. [h*DV, ...); GQA maps query
// head h to kv head h / (Hq/Hk).  DQ may exceed DV (multi-head latent attention
// concatenates a RoPE part to q and k): a DQ that is not a multiple of 64 is
// staged in whole 64-column blocks and the QK^T MMA stops at DQ.
// Outputs: o [B*S, Hq*DV] bf16, lse [B, Hq, S] f32 (natural log).
// Warps: 0 TMA, 1 MMA + TMEM owner, 2..9 softmax/correction/epilogue (two per
// 32-row TMEM lane quarter, splitting the keys of each tile).
// Every TMA load here reads local memory for one CTA; every wait is bounded.
// Upstream: GQA attention model.rs:333-386 (repeat_kv model.rs:388-399, causal mask
// model.rs:402-425); multi-head latent attention model.rs:196-256.
#include <algorithm>
#include <cudaTypedefs.h>

#include "gemm_kernel.cuh"
#include "kernels_attn.h"

namespace oxi {
namespace {

constexpr int FA_BM = 128, FA_BN = 128;
// Forward key tile: 64 keys, so that a CTA needs 256 TMEM columns (two S tiles +
// O) and about 100 KB of shared memory, and two CTAs share an SM: one CTA's
// softmax overlaps the other's MMAs and its prologue/epilogue the other's loop.
constexpr int FA_BNF = 64;
constexpr int FA_THREADS = 320;      // TMA warp, MMA warp, 8 softmax/epilogue warps
constexpr int FA_BWD_THREADS = 320;  // TMA warp, MMA warp, 8 softmax/epilogue warps

struct FaParams {
  int B, S, Hq, Hk;
  float scale_log2;  // softmax scale * log2(e)
  int causal;
  __nv_bfloat16* o;
  int64_t ldo;
  float* lse;
  int* status;
};

template <int DQ, int DV>
struct FaSmem {
  static constexpr int KBQ = (DQ + 63) / 64;  // 64-column blocks of a q/k row
  static constexpr int KBV = DV / 64;         // 64-column blocks of a v row
  static constexpr int Q_BYTES = FA_BM * KBQ * 128;
  static constexpr int K_BYTES = FA_BNF * KBQ * 128;
  static constexpr int V_BYTES = FA_BNF * KBV * 128;
  static constexpr int KST = 2;  // K stages: K_j is freed as soon as S_j is done
  static constexpr int VST = 2;  // V stages: V_j is freed after PV_j
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + Q_BYTES;
  static constexpr int OFF_V = OFF_K + KST * K_BYTES;
  static constexpr int OFF_RED = OFF_V + VST * V_BYTES;  // row-max exchange [2][2][128] + row sums [2][128]
  static constexpr int OFF_BAR = OFF_RED + 768 * 4;
  static constexpr int TOTAL = OFF_BAR + 256 + 1024;
  static_assert(2 * (TOTAL + 1024) <= 233472, "two CTAs per SM");
};

// UMMA descriptor of the kk-th K=16 slice of a K-major SW128 tile whose K
// extent is split into 64-element (128-byte) blocks of `block_bytes` each.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t base, int kk, uint32_t block_bytes) {
  return umma_desc_sw128(base + (kk >> 2) * block_bytes + (kk & 3) * 32, 16, 1024);
}

template <int DQ, int DV>
__global__ void __launch_bounds__(FA_THREADS, 2)
    fa_fwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV, FaParams p) {
  using L = FaSmem<DQ, DV>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + L::OFF_Q;
  uint8_t* sK = smem + L::OFF_K;
  uint8_t* sV = smem + L::OFF_V;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;    // [3]
  uint64_t* k_empty = bars + 4;   // [3]
  uint64_t* v_full = bars + 7;    // [3]
  uint64_t* v_empty = bars + 10;  // [3]
  uint64_t* s_full = bars + 13;   // [2]
  uint64_t* p_full = bars + 17;
  uint64_t* pv_done = bars + 18;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 19);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int n_qt = (p.S + FA_BM - 1) / FA_BM;
  // the query tile is the slowest grid index and runs backwards, so every head's
  // longest (causal) tiles are issued before any shorter one: longest-first
  // scheduling across the whole grid, not just within one head
  const int qt = n_qt - 1 - blockIdx.z;
  const int h = blockIdx.x, b = blockIdx.y;
  const int hk = h / (p.Hq / p.Hk);
  const int q0 = qt * FA_BM;
  const int row0 = b * p.S;
  const int n_kt_all = (p.S + FA_BNF - 1) / FA_BNF;
  const int nk = p.causal ? min(n_kt_all, (q0 + FA_BM - 1) / FA_BNF + 1) : n_kt_all;
  constexpr int KBQ = L::KBQ, KBV = L::KBV;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 3; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) mbar_init(&s_full[i], 1);
    mbar_init(p_full, 8);
    mbar_init(pv_done, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t TM_S0 = tmem, TM_O = tmem + 2 * FA_BNF;

  if (warp == 0) {
    if (lane == 0) {
      bool ok = true;
      mbar_arrive_expect_tx(q_full, L::Q_BYTES);
#pragma unroll
      for (int kb = 0; kb < KBQ; ++kb) tma_load_2d(sQ + kb * FA_BM * 128, &tmQ, q_full, h * DQ + kb * 64, row0 + q0);
      // K_j runs ahead of V_j: K stages free up when S_j completes, V stages
      // when PV_j completes, so K loads are issued as early as possible.
      int jv = 0;
      for (int j = 0; j < nk && ok; ++j) {
        const int ks = j % L::KST, ku = j / L::KST;
        if (!mbar_wait(&k_empty[ks], (ku & 1) ^ 1, abort_flag, p.status)) { ok = false; break; }
        mbar_arrive_expect_tx(&k_full[ks], L::K_BYTES);
#pragma unroll
        for (int kb = 0; kb < KBQ; ++kb)
          tma_load_2d(sK + ks * L::K_BYTES + kb * FA_BNF * 128, &tmK, &k_full[ks], hk * DQ + kb * 64,
                      row0 + j * FA_BNF);
        // issue every V load whose stage is already free (never more than one behind K)
        while (jv <= j) {
          const int vs = jv % L::VST, vu = jv / L::VST;
          if (jv < j && !mbar_try_wait(smem_u32(&v_empty[vs]), (vu & 1) ^ 1)) break;
          if (jv == j && !mbar_wait(&v_empty[vs], (vu & 1) ^ 1, abort_flag, p.status)) { ok = false; break; }
          mbar_arrive_expect_tx(&v_full[vs], L::V_BYTES);
#pragma unroll
          for (int kb = 0; kb < KBV; ++kb)
            tma_load_2d(sV + vs * L::V_BYTES + kb * FA_BNF * 128, &tmV, &v_full[vs], hk * DV + kb * 64,
                        row0 + jv * FA_BNF);
          ++jv;
        }
      }
      // drain: wait for every copy issued to land before leaving
      if (!ok) {
        mbar_wait(q_full, 0, nullptr, p.status);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t IDESC_S = umma_idesc_bf16(FA_BM, FA_BNF, false, false);
      constexpr uint32_t IDESC_O = umma_idesc_bf16(FA_BM, DV, false, true);
      bool ok = mbar_wait(q_full, 0, abort_flag, p.status);
      const uint32_t aQ = smem_u32(sQ);
      // S_j's buffer last held P_{j-2}, read by PV_{j-2}, issued earlier by this thread
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;
        const int ks = j % L::KST, ku = j / L::KST;
        if (!mbar_wait(&k_full[ks], ku & 1, abort_flag, p.status)) return false;
        tc_fence_after();
        const uint32_t aK = smem_u32(sK + ks * L::K_BYTES);
#pragma unroll
        for (int kk = 0; kk < DQ / 16; ++kk)
          tc_mma_f16(TM_S0 + st * FA_BNF, kmajor_desc(aQ, kk, FA_BM * 128), kmajor_desc(aK, kk, FA_BNF * 128),
                     IDESC_S, kk != 0);
        tc_commit(&s_full[st]);
        tc_commit(&k_empty[ks]);
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; j < nk && ok; ++j) {
        if (j + 1 < nk && !issue_s(j + 1)) { ok = false; break; }
        if (!mbar_wait(p_full, j & 1, abort_flag, p.status)) { ok = false; break; }
        const int vs = j % L::VST, vu = j / L::VST;
        if (!mbar_wait(&v_full[vs], vu & 1, abort_flag, p.status)) { ok = false; break; }
        tc_fence_after();
        const uint32_t tP = TM_S0 + (j & 1) * FA_BNF;  // P_j: bf16 pairs in S_j's first half
        const uint32_t aV = smem_u32(sV + vs * L::V_BYTES);
#pragma unroll
        for (int kk = 0; kk < FA_BNF / 16; ++kk)
          tc_mma_f16_ts(TM_O, tP + kk * 8, umma_desc_sw128(aV + kk * 2048, FA_BNF * 128, 1024), IDESC_O,
                        (j | kk) != 0);
        tc_commit(pv_done);
        tc_commit(&v_empty[vs]);
      }
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------- softmax warps
    // Eight warps: warps w and w + 4 own TMEM lane quarter (w & 3), i.e. the same
    // 32 query rows, and split the keys of a tile (and O's columns) in halves.
    // The two halves agree on the row max through shared memory once per tile.
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = quarter * 32 + lane;       // query row within the tile (== TMEM lane)
    const int qpos = q0 + r;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    float* s_xmax = reinterpret_cast<float*>(smem + L::OFF_RED);  // [tile parity][half][128]
    float* s_lsum = s_xmax + 512;                                 // [half][128]
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    // After a failed wait the loop keeps running without work so that every
    // softmax warp still meets the other half at each named barrier.
    for (int j = 0; j < nk; ++j) {
      const int st = j & 1, u = j >> 1;
      if (ok && !mbar_wait(&s_full[st], u & 1, abort_flag, p.status)) ok = false;
      if (!ok) {
        asm volatile("bar.sync 1, 256;" ::: "memory");
        continue;
      }
      tc_fence_after();
      // Masking is branch-free: keys past `lim` (causal diagonal or sequence end) become -inf.
      constexpr int KPT = FA_BNF / 2;   // keys per thread (the two halves split a tile)
      constexpr int NCH = KPT / 32;     // 32-key TMEM chunks per thread
      const int k0 = j * FA_BNF + half * KPT;
      const bool need_mask = (p.causal && k0 + KPT - 1 > q0) || (k0 + KPT > p.S);
      const int lim = p.causal ? min(qpos, p.S - 1) : p.S - 1;
      const uint32_t s_base = TM_S0 + st * FA_BNF + lane_base;
      uint32_t rr[NCH][32];
#pragma unroll
      for (int c = 0; c < NCH; ++c) tmem_ld32(s_base + half * KPT + c * 32, rr[c]);
      tc_wait_ld();
      float mx[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) mx[q] = -INFINITY;
      // the max is taken over the raw scores and scaled once (the scale is positive); the
      // scale is applied inside the exponent's FFMA below
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        const int kc = k0 + c * 32;
#pragma unroll
        for (int t = 0; t < 32; ++t) {
          float v = __uint_as_float(rr[c][t]);
          if (need_mask) {
            v = (kc + t > lim) ? -INFINITY : v;
            rr[c][t] = __float_as_uint(v);
          }
          mx[t & 7] = fmaxf(mx[t & 7], v);
        }
      }
      const float mloc = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                               fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7]))) * p.scale_log2;
      float* xm = s_xmax + (j & 1) * 256;
      xm[half * 128 + r] = mloc;
      // every S column of this tile has been read into registers before either
      // half writes P over the S buffer
      tc_fence_before();
      asm volatile("bar.sync 1, 256;" ::: "memory");
      tc_fence_after();
      const float mt = fmaxf(mloc, xm[(half ^ 1) * 128 + r]);
      // move the reference max only when it grows by more than 2^8
      const bool move = (mt > m + 8.f);
      const float m_new = move ? mt : m;
      const float alpha = move ? ex2_approx(m - m_new) : 1.f;  // exp2(-inf) = 0 on the first tile
      const float mref = (m_new == -INFINITY) ? 0.f : m_new;
      const bool rescale_warp = __any_sync(0xffffffffu, move && j > 0);
      m = m_new;
      if (j > 0 && rescale_warp) {
        // O is owned by the previous PV MMA until it completes (PV_j cannot have
        // completed yet, so the parity wait cannot skip a phase)
        if (!mbar_wait(pv_done, (j - 1) & 1, abort_flag, p.status)) {
          ok = false;
          continue;
        }
        tc_fence_after();
#pragma unroll 1
        for (int c = half * (DV / 64); c < (half + 1) * (DV / 64); ++c) {
          uint32_t o0[32];
          tmem_ld32(TM_O + lane_base + c * 32, o0);
          tc_wait_ld();
#pragma unroll
          for (int t = 0; t < 32; ++t) o0[t] = __float_as_uint(__uint_as_float(o0[t]) * alpha);
          tmem_st32(TM_O + lane_base + c * 32, o0);
        }
        tc_wait_st();
      }
      float rsa[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) rsa[q] = 0.f;
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        uint32_t pk[16];
#pragma unroll
        for (int t = 0; t < 32; t += 2) {
          const float a = ex2_approx(fmaf(__uint_as_float(rr[c][t]), p.scale_log2, -mref));
          const float bb = ex2_approx(fmaf(__uint_as_float(rr[c][t + 1]), p.scale_log2, -mref));
          rsa[(t >> 1) & 7] += a + bb;
          pk[t / 2] = pack_bf16(a, bb);
        }
        // keys KPT half + 32c .. +31 -> P columns KPT/2 half + 16c .. +15
        tmem_st16(s_base + half * (KPT / 2) + c * 16, pk);
      }
      const float rs = ((rsa[0] + rsa[1]) + (rsa[2] + rsa[3])) + ((rsa[4] + rsa[5]) + (rsa[6] + rsa[7]));
      l = l * alpha + rs;
      tc_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    if (ok && !mbar_wait(pv_done, (nk - 1) & 1, abort_flag, p.status)) ok = false;
    s_lsum[half * 128 + r] = l;
    asm volatile("bar.sync 1, 256;" ::: "memory");  // reached by every softmax warp
    if (ok) {
      tc_fence_after();
      const float lt = l + s_lsum[(half ^ 1) * 128 + r];
      const float inv_l = (lt > 0.f) ? 1.f / lt : 0.f;
      const bool valid = qpos < p.S;
      __nv_bfloat16* orow = p.o + (int64_t)(row0 + qpos) * p.ldo + h * DV;
#pragma unroll 1
      for (int c = half * (DV / 64); c < (half + 1) * (DV / 64); ++c) {
        uint32_t o[32];
        tmem_ld32(TM_O + lane_base + c * 32, o);
        tc_wait_ld();
        if (valid) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 w;
            w.x = pack_bf16(__uint_as_float(o[q * 8 + 0]) * inv_l, __uint_as_float(o[q * 8 + 1]) * inv_l);
            w.y = pack_bf16(__uint_as_float(o[q * 8 + 2]) * inv_l, __uint_as_float(o[q * 8 + 3]) * inv_l);
            w.z = pack_bf16(__uint_as_float(o[q * 8 + 4]) * inv_l, __uint_as_float(o[q * 8 + 5]) * inv_l);
            w.w = pack_bf16(__uint_as_float(o[q * 8 + 6]) * inv_l, __uint_as_float(o[q * 8 + 7]) * inv_l);
            dst[q] = w;
          }
        }
      }
      if (valid && half == 0) p.lse[((int64_t)b * p.Hq + h) * p.S + qpos] = (m + __log2f(lt)) * 0.69314718055994530942f;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

template <int DQ, int DV>
void launch_fa_fwd_t(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv, void* o,
                     int64_t ldo, float* lse, int B, int S, int Hq, int Hk, float scale, bool causal, int* status,
                     cudaStream_t st) {
  using L = FaSmem<DQ, DV>;
  const int64_t T = (int64_t)B * S;
  CUtensorMap tq = make_tmap_bf16(q, T, (int64_t)Hq * DQ, ldq, 64, FA_BM);
  CUtensorMap tk = make_tmap_bf16(k, T, (int64_t)Hk * DQ, ldk, 64, FA_BNF);
  CUtensorMap tv = make_tmap_bf16(v, T, (int64_t)Hk * DV, ldv, 64, FA_BNF);
  FaParams p;
  p.B = B; p.S = S; p.Hq = Hq; p.Hk = Hk;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.causal = causal ? 1 : 0;
  p.o = reinterpret_cast<__nv_bfloat16*>(o);
  p.ldo = ldo;
  p.lse = lse;
  p.status = status;
  auto kern = fa_fwd_kernel<DQ, DV>;
  static bool attr = false;
  if (!attr) {
    OXI_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL));
    attr = true;
  }
  dim3 grid(Hq, B, (S + FA_BM - 1) / FA_BM);
  kern<<<grid, FA_THREADS, L::TOTAL, st>>>(tq, tk, tv, p);
  OXI_CUDA_CHECK(cudaGetLastError());
}


// ===================================================================== backward
// One CTA per (128-key tile j, kv head hk, batch b); loops over the query heads
// of the GQA group and over the query tiles i >= j (causal).  Per (h, i):
//   S^T  = K Q_i^T, dP^T = V dO_i^T            (TMEM)
//   P^T  = exp2(S^T c - lse_i), dS^T = P^T (dP^T - delta_i) * scale
//                                              (softmax warps -> swizzled smem)
//   dV += P^T dO_i, dK += dS^T Q_i             (TMEM accumulators)
//   dQ_i = dS K -> TMA reduce-add into dq_acc  (TMEM, aliases dP^T)
// dS^T in shared memory serves as the K-major A of dK and, read as MN-major,
// as the A of dQ; Q, dO and K are read as K-major or MN-major B operands from
// the same tiles.
struct FaBwdParams {
  int B, S, Hq, Hk;
  float scale, scale_log2;
  int causal;
  const float* lse;    // [B, Hq, S]
  const float* delta;  // [B, Hq, S]
  float* dq_acc;       // [B*S, Hq*DQ] f32, zero-initialised
  int64_t ld_dq;
  __nv_bfloat16* dk;
  __nv_bfloat16* dv;
  int64_t ld_dk, ld_dv;
  const float* rope_cos;  // [S, DQ/2] or null: dk is the gradient of the unrotated k
  const float* rope_sin;
  int* status;
};

template <int DQ, int DV>
struct FaBwdSmem {
  static constexpr int KBQ = (DQ + 63) / 64;
  static constexpr int KBV = DV / 64;
  static constexpr int NQ = KBQ * 64;             // DQ rounded up to whole 64-column blocks
  static constexpr int TQ_BYTES = 128 * NQ * 2;   // K, Q tiles
  static constexpr int TV_BYTES = 128 * DV * 2;   // V, dO tiles
  static constexpr int P_BYTES = 128 * 128 * 2;   // dS^T
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = OFF_K + TQ_BYTES;
  static constexpr int OFF_Q = OFF_V + TV_BYTES;       // [2] (double-buffered)
  static constexpr int OFF_DO = OFF_Q + 2 * TQ_BYTES;  // [2]
  static constexpr int OFF_DST = OFF_DO + 2 * TV_BYTES;
  static constexpr int OFF_VEC = OFF_DST + P_BYTES;   // lse (log2), delta of the current pair: 2 x 128 f32
  static constexpr int OFF_BAR = OFF_VEC + 2 * 128 * 4;
  static constexpr int TOTAL = OFF_BAR + 256 + 1024;
  static_assert(TOTAL <= 232448, "shared memory budget");
  static_assert(DV + NQ + 256 <= 512, "TMEM budget: dV, dK, S^T and dP^T accumulators");
};

__device__ __forceinline__ void named_bar_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// One CTA per (128-key tile, kv head, batch); loops over the query heads of
// the GQA group and the query tiles i >= j.  Per (h, i):
//   S^T = K Q_i^T, dP^T = V dO_i^T               (TMEM)
//   P^T = exp2(S^T c - lse), dS^T = P^T (dP^T - delta) scale
//        P^T is written back into TMEM as bf16 (the A operand of dV), dS^T to
//        128B-swizzled shared memory (A of dK, and read MN-major, A of dQ)
//   dV += P^T dO_i, dK += dS^T Q_i                (TMEM accumulators)
//   dQ_i = dS K -> TMA reduce-add into dq_acc     (TMEM, in the dP^T columns)
// Q_i / dO_i are double-buffered so the next pair's loads overlap this one; the
// next pair's S^T MMA is issued before this pair's dQ has been drained (only its
// dP^T MMA waits for that), and lse / delta are loaded one pair ahead.
template <int DQ, int DV>
__global__ void __launch_bounds__(FA_BWD_THREADS, 1)
    fa_bwd_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                  const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmDO,
                  const __grid_constant__ CUtensorMap tmDQ, FaBwdParams p) {
  using L = FaBwdSmem<DQ, DV>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem + L::OFF_K;
  uint8_t* sV = smem + L::OFF_V;
  uint8_t* sQ = smem + L::OFF_Q;
  uint8_t* sDO = smem + L::OFF_DO;
  uint8_t* sDSt = smem + L::OFF_DST;
  float* s_lse = reinterpret_cast<float*>(smem + L::OFF_VEC);
  float* s_delta = s_lse + 128;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::OFF_BAR);
  uint64_t* kv_full = bars + 0;
  uint64_t* qdo_full = bars + 1;   // [2]
  uint64_t* qdo_empty = bars + 3;  // [2]
  uint64_t* sdp_full = bars + 5;
  uint64_t* p_ready = bars + 6;
  uint64_t* it_done = bars + 7;
  uint64_t* dq_read = bars + 8;
  uint64_t* dq_full = bars + 9;    // dK and dQ MMAs of the pair done (dS^T free, dQ readable)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 10);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  // the key tile is the slowest grid index: under causal masking key tile 0 has the
  // most query tiles, so every head's longest tiles are issued first
  const int jt = blockIdx.z, hk = blockIdx.x, b = blockIdx.y;
  const int group = p.Hq / p.Hk;
  const int n_qt = (p.S + 127) / 128;
  const int i_start = p.causal ? jt : 0;
  const int n_i = n_qt - i_start;
  const int n_it = group * n_i;
  const int row0 = b * p.S;
  const int k0 = jt * 128;
  constexpr int KBQ = L::KBQ, KBV = L::KBV, NQ = L::NQ;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&qdo_full[i], 1);
      mbar_init(&qdo_empty[i], 1);
    }
    mbar_init(sdp_full, 1);
    mbar_init(p_ready, 8);   // one arrival per softmax warp
    mbar_init(it_done, 1);
    mbar_init(dq_read, 8);
    mbar_init(dq_full, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    tma_prefetch_desc(&tmDO);
    tma_prefetch_desc(&tmDQ);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t TM_DV = tmem, TM_DK = tmem + DV, TM_S = tmem + DV + NQ, TM_DP = tmem + DV + NQ + 128;
  const uint32_t TM_DQ = TM_DP;  // dQ reuses the dP^T columns once the softmax warps consumed them

  if (warp == 0) {
    if (lane == 0) {
      mbar_arrive_expect_tx(kv_full, L::TQ_BYTES + L::TV_BYTES);
#pragma unroll
      for (int kb = 0; kb < KBQ; ++kb) tma_load_2d(sK + kb * 128 * 128, &tmK, kv_full, hk * DQ + kb * 64, row0 + k0);
#pragma unroll
      for (int kb = 0; kb < KBV; ++kb) tma_load_2d(sV + kb * 128 * 128, &tmV, kv_full, hk * DV + kb * 64, row0 + k0);
      int issued = 0;
      for (int it = 0; it < n_it; ++it) {
        const int h = hk * group + it / n_i;
        const int i = i_start + it % n_i;
        const int st = it & 1, u = it >> 1;
        if (!mbar_wait(&qdo_empty[st], (u & 1) ^ 1, abort_flag, p.status)) break;
        mbar_arrive_expect_tx(&qdo_full[st], L::TQ_BYTES + L::TV_BYTES);
        uint8_t* q = sQ + st * L::TQ_BYTES;
        uint8_t* o = sDO + st * L::TV_BYTES;
#pragma unroll
        for (int kb = 0; kb < KBQ; ++kb) tma_load_2d(q + kb * 128 * 128, &tmQ, &qdo_full[st], h * DQ + kb * 64, row0 + i * 128);
#pragma unroll
        for (int kb = 0; kb < KBV; ++kb)
          tma_load_2d(o + kb * 128 * 128, &tmDO, &qdo_full[st], h * DV + kb * 64, row0 + i * 128);
        ++issued;
      }
      // leave no copy in flight into shared memory
      for (int it = (issued > 2 ? issued - 2 : 0); it < issued; ++it)
        mbar_wait(&qdo_full[it & 1], (it >> 1) & 1, nullptr, p.status);
      mbar_wait(kv_full, 0, nullptr, p.status);
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t ID_SS = umma_idesc_bf16(128, 128, false, false);  // S^T, dP^T
      constexpr uint32_t ID_V = umma_idesc_bf16(128, DV, false, true);     // dV (A from TMEM)
      constexpr uint32_t ID_K = umma_idesc_bf16(128, NQ, false, true);     // dK
      constexpr uint32_t ID_Q = umma_idesc_bf16(128, NQ, true, true);      // dQ
      const uint32_t aK = smem_u32(sK), aV = smem_u32(sV), aDSt = smem_u32(sDSt);
      bool ok = mbar_wait(kv_full, 0, abort_flag, p.status);
      for (int it = 0; it < n_it && ok; ++it) {
        const int st = it & 1;
        const uint32_t aQ = smem_u32(sQ + st * L::TQ_BYTES), aDO = smem_u32(sDO + st * L::TV_BYTES);
        if (!mbar_wait(&qdo_full[st], (it >> 1) & 1, abort_flag, p.status)) { ok = false; break; }
        tc_fence_after();
        // S^T columns hold P^T of the previous pair until its dV MMA has read them; that
        // MMA was issued earlier by this thread, so S^T can be issued now and runs while
        // the softmax warps drain the previous dQ
#pragma unroll
        for (int kk = 0; kk < DQ / 16; ++kk)
          tc_mma_f16(TM_S, kmajor_desc(aK, kk, 128 * 128), kmajor_desc(aQ, kk, 128 * 128), ID_SS, kk != 0);
        // the dP^T columns hold the previous dQ until the softmax warps have read it
        if (it > 0 && !mbar_wait(dq_read, (it - 1) & 1, abort_flag, p.status)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < DV / 16; ++kk)
          tc_mma_f16(TM_DP, kmajor_desc(aV, kk, 128 * 128), kmajor_desc(aDO, kk, 128 * 128), ID_SS, kk != 0);
        tc_commit(sdp_full);
        if (!mbar_wait(p_ready, it & 1, abort_flag, p.status)) { ok = false; break; }
        tc_fence_after();
        // dK and dQ (the two readers of dS^T) first: the softmax warps drain dQ while dV runs
#pragma unroll
        for (int kk = 0; kk < 128 / 16; ++kk) {
          const uint32_t acc = (it > 0 || kk > 0) ? 1u : 0u;
          tc_mma_f16(TM_DK, kmajor_desc(aDSt, kk, 128 * 128), umma_desc_sw128(aQ + kk * 2048, 128 * 128, 1024),
                     ID_K, acc);
          tc_mma_f16(TM_DQ, umma_desc_sw128(aDSt + kk * 2048, 128 * 128, 1024),
                     umma_desc_sw128(aK + kk * 2048, 128 * 128, 1024), ID_Q, kk > 0 ? 1u : 0u);
        }
        tc_commit(dq_full);
#pragma unroll
        for (int kk = 0; kk < 128 / 16; ++kk) {
          const uint32_t acc = (it > 0 || kk > 0) ? 1u : 0u;
          // P^T (bf16 in TMEM): queries 0..63 in columns 0..31, 64..127 in columns 64..95
          const uint32_t aP = TM_S + (kk < 4 ? kk * 8 : 64 + (kk - 4) * 8);
          tc_mma_f16_ts(TM_DV, aP, umma_desc_sw128(aDO + kk * 2048, 128 * 128, 1024), ID_V, acc);
        }
        tc_commit(it_done);
        tc_commit(&qdo_empty[st]);
      }
    }
    __syncwarp();
  } else {
    // warps 2..9: warp w reads TMEM lanes 32*(w%4).. (its row quarter) and
    // handles column half `half` of every 128-wide tile it processes.
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = quarter * 32 + lane;  // key row for P/dS; query row for the dQ epilogue
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const int kpos = k0 + r;
    bool ok = true;
    // lse / delta of a pair's 128 queries: the first 128 softmax threads load one
    // element each, one pair ahead (registers), so no global load latency sits
    // between the pairs
    const int vtid = threadIdx.x - 64;
    float nx_lse = 0.f, nx_delta = 0.f;
    auto load_vec = [&](int it2) {
      const int h2 = hk * group + it2 / n_i;
      const int qp = (i_start + it2 % n_i) * 128 + vtid;
      const int64_t vi = ((int64_t)b * p.Hq + h2) * p.S + qp;
      nx_lse = qp < p.S ? __ldg(p.lse + vi) * 1.4426950408889634f : 0.f;
      nx_delta = qp < p.S ? __ldg(p.delta + vi) : 0.f;
    };
    if (vtid < 128 && n_it > 0) load_vec(0);
    // After a failed wait the loop keeps running without work so that every
    // softmax warp still reaches each named barrier.
    for (int it = 0; it < n_it; ++it) {
      const int h = hk * group + it / n_i;
      const int i = i_start + it % n_i;
      const int q0 = i * 128;
      named_bar_sync(1, 256);  // every softmax warp is done with the previous pair's vectors
      if (vtid < 128) {
        s_lse[vtid] = nx_lse;
        s_delta[vtid] = nx_delta;
        if (it + 1 < n_it) load_vec(it + 1);
      }
      named_bar_sync(1, 256);
      if (!ok) continue;
      if (!mbar_wait(sdp_full, it & 1, abort_flag, p.status)) { ok = false; continue; }
      // dS^T smem is free once the previous pair's MMAs completed (waited in the previous dQ step)
      tc_fence_after();
      const bool diag = p.causal && (q0 < k0 + 128);
#pragma unroll 1
      for (int cc = 0; cc < 2; ++cc) {
        const int c = half * 2 + cc;  // 32-query chunk 0..3
        uint32_t sr[32], dr[32];
        tmem_ld32(TM_S + lane_base + c * 32, sr);
        tmem_ld32(TM_DP + lane_base + c * 32, dr);
        tc_wait_ld();
        uint32_t pk[16], dk[16];
#pragma unroll
        for (int t = 0; t < 32; t += 2) {
          float pv[2], dsv[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int qc = c * 32 + t + e;
            const int qp = q0 + qc;
            const bool valid = (qp < p.S) && (kpos < p.S) && (!diag || qp >= kpos);
            const float pp = valid ? ex2_approx(__uint_as_float(sr[t + e]) * p.scale_log2 - s_lse[qc]) : 0.f;
            pv[e] = pp;
            dsv[e] = pp * (__uint_as_float(dr[t + e]) - s_delta[qc]) * p.scale;
          }
          pk[t / 2] = pack_bf16(pv[0], pv[1]);
          dk[t / 2] = pack_bf16(dsv[0], dsv[1]);
        }
        // P^T (bf16 pairs) back into this half's own, already read, S^T columns
        tmem_st16(TM_S + lane_base + (half * 64 + cc * 16), pk);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int ch = c * 4 + q;  // 8-query chunk index 0..15
          sw128_store16(sDSt + (ch >> 3) * (128 * 128), r, ch & 7,
                        make_uint4(dk[q * 4], dk[q * 4 + 1], dk[q * 4 + 2], dk[q * 4 + 3]));
        }
      }
      tc_wait_st();
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_ready);
      // dQ of this (h, i): thread r owns query row r; the two halves take alternate 32-column
      // chunks.  Each warp stages its 32 rows x 32 columns (f32, 128B-swizzled) in its own
      // 4 KB slab of the dS^T buffer -- the slab it writes dS^T into, free once this pair's
      // dK and dQ MMAs have completed -- and adds it to dq_acc with one TMA reduce-add (rows
      // past the sequence end are clipped by the tensor map).  The dV MMA runs meanwhile.
      if (!mbar_wait(dq_full, it & 1, abort_flag, p.status)) { ok = false; continue; }
      tc_fence_after();
      uint8_t* slab = sDSt + half * (128 * 128) + quarter * (32 * 128);
#pragma unroll 1
      for (int c = half; c < DQ / 32; c += 2) {
        uint32_t o[32];
        tmem_ld32(TM_DQ + lane_base + c * 32, o);
        tc_wait_ld();
        if (c != half) {  // the previous chunk's reduce has finished reading the slab
          if (lane == 0) bulk_wait_read<0>();
          __syncwarp();
        }
#pragma unroll
        for (int u = 0; u < 8; ++u)
          sw128_store16(slab, lane, u, make_uint4(o[u * 4], o[u * 4 + 1], o[u * 4 + 2], o[u * 4 + 3]));
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && q0 + quarter * 32 < p.S) {  // a box wholly past the sequence end adds nothing
          tma_reduce_add_3d(&tmDQ, slab, h * DQ + c * 32, q0 + quarter * 32, b);
          bulk_commit();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(dq_read);
        bulk_wait_read<0>();  // the slab is written again by the next pair's softmax
      }
      __syncwarp();
    }
    if (lane == 0) bulk_wait<0>();  // every dQ reduce issued by this warp has been performed
    // the last pair's dV MMA (issued after its dQ) completes the accumulators
    if (ok && n_it > 0 && !mbar_wait(it_done, (n_it - 1) & 1, abort_flag, p.status)) ok = false;
    // dK, dV of this key tile (thread r owns key row r; halves take alternate chunks)
    if (ok && n_it > 0) {
      tc_fence_after();
      const bool valid = kpos < p.S;
      // with RoPE, dK leaves through the inverse rotation: column j and j + DQ/2 form a pair,
      // so half h takes the 32-column chunks h and h + DQ/64 together
      const int n_which = (DQ == DV && p.rope_cos != nullptr) ? 1 : 2;
      if (n_which == 1) {
        constexpr int HC = DQ / 64;  // 32-column chunks in half a head
        __nv_bfloat16* dst = p.dk + (int64_t)(row0 + kpos) * p.ld_dk + hk * DQ;
        const float* cs = p.rope_cos + (int64_t)kpos * (DQ / 2);
        const float* sn = p.rope_sin + (int64_t)kpos * (DQ / 2);
#pragma unroll 1
        for (int c = half; c < HC; c += 2) {
          uint32_t o1[32], o2[32];
          tmem_ld32(TM_DK + lane_base + c * 32, o1);
          tmem_ld32(TM_DK + lane_base + (c + HC) * 32, o2);
          tc_wait_ld();
          if (valid) {
            uint4* d1 = reinterpret_cast<uint4*>(dst + c * 32);
            uint4* d2 = reinterpret_cast<uint4*>(dst + (c + HC) * 32);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              float a[8], bb[8];
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                const int j = c * 32 + q * 8 + e;
                const float cj = __ldg(cs + j), sj = __ldg(sn + j);
                const float x1 = __uint_as_float(o1[q * 8 + e]), x2 = __uint_as_float(o2[q * 8 + e]);
                a[e] = x1 * cj + x2 * sj;
                bb[e] = x2 * cj - x1 * sj;
              }
              d1[q] = make_uint4(pack_bf16(a[0], a[1]), pack_bf16(a[2], a[3]), pack_bf16(a[4], a[5]),
                                 pack_bf16(a[6], a[7]));
              d2[q] = make_uint4(pack_bf16(bb[0], bb[1]), pack_bf16(bb[2], bb[3]), pack_bf16(bb[4], bb[5]),
                                 pack_bf16(bb[6], bb[7]));
            }
          }
        }
      }
#pragma unroll 1
      for (int which = 0; which < n_which; ++which) {
        __nv_bfloat16* dst = which == 0 ? p.dv + (int64_t)(row0 + kpos) * p.ld_dv + hk * DV
                                        : p.dk + (int64_t)(row0 + kpos) * p.ld_dk + hk * DQ;
        const uint32_t src = (which == 0 ? TM_DV : TM_DK) + lane_base;
        const int ncol = which == 0 ? DV : DQ;
#pragma unroll 1
        for (int c = half; c < ncol / 32; c += 2) {
          uint32_t o[32];
          tmem_ld32(src + c * 32, o);
          tc_wait_ld();
          if (valid) {
            uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
            for (int q = 0; q < 4; ++q)
              d4[q] = make_uint4(pack_bf16(__uint_as_float(o[q * 8]), __uint_as_float(o[q * 8 + 1])),
                                 pack_bf16(__uint_as_float(o[q * 8 + 2]), __uint_as_float(o[q * 8 + 3])),
                                 pack_bf16(__uint_as_float(o[q * 8 + 4]), __uint_as_float(o[q * 8 + 5])),
                                 pack_bf16(__uint_as_float(o[q * 8 + 6]), __uint_as_float(o[q * 8 + 7])));
          }
        }
      }
    } else if (n_it == 0 && kpos < p.S && half == 0) {
      // no query attends to this key tile: zero gradients
      __nv_bfloat16* dv = p.dv + (int64_t)(row0 + kpos) * p.ld_dv + hk * DV;
      __nv_bfloat16* dk = p.dk + (int64_t)(row0 + kpos) * p.ld_dk + hk * DQ;
      for (int c = 0; c < DV; ++c) dv[c] = __float2bfloat16(0.f);
      for (int c = 0; c < DQ; ++c) dk[c] = __float2bfloat16(0.f);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// delta[b, h, s] = sum_d dO * O  (one warp per (token, head) row)
// delta[b, h, s] = <dO_row, O_row>: D / 8 threads per row, 16-byte loads,
// shuffle reduction within the row's lane group (D in {64, 96, 128, ...}, D / 8
// a power of two up to 32 -> groups never straddle a warp).
__global__ void fa_bwd_prep_kernel(const __nv_bfloat16* __restrict__ o, int64_t ldo,
                                   const __nv_bfloat16* __restrict__ dout, int64_t lddo, float* __restrict__ delta,
                                   int B, int S, int Hq, int D) {
  const int per = D / 8;  // threads per row
  const int64_t gt = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t w = gt / per;
  const int sub = (int)(gt % per);
  const int64_t rows = (int64_t)B * S * Hq;
  const bool live = w < rows;
  float s = 0.f;
  int64_t t = 0;
  int h = 0;
  if (live) {
    t = w / Hq;
    h = (int)(w % Hq);
    const uint4 ua = *reinterpret_cast<const uint4*>(o + t * ldo + (int64_t)h * D + sub * 8);
    const uint4 ug = *reinterpret_cast<const uint4*>(dout + t * lddo + (int64_t)h * D + sub * 8);
    const __nv_bfloat162* a = reinterpret_cast<const __nv_bfloat162*>(&ua);
    const __nv_bfloat162* g = reinterpret_cast<const __nv_bfloat162*>(&ug);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 x = __bfloat1622float2(a[i]), y = __bfloat1622float2(g[i]);
      s += x.x * y.x + x.y * y.y;
    }
  }
  for (int off = per / 2; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (live && sub == 0) {
    const int b = (int)(t / S), sp = (int)(t % S);
    delta[((int64_t)b * Hq + h) * S + sp] = s;
  }
}

// dq (bf16, row stride lddq) = the inverse rotate-half RoPE of dq_acc (f32): one
// thread per 8 rotation pairs (columns j..j+7 and j+hd/2..j+hd/2+7 of a head),
// position = row % S.
__global__ void fa_dq_convert_rope_kernel(const float* __restrict__ acc, int64_t ldacc,
                                          __nv_bfloat16* __restrict__ dq, int64_t lddq, int64_t rows, int cols,
                                          int hd, int S, const float* __restrict__ cs, const float* __restrict__ sn) {
  const int half = hd / 2;
  const int per_row = cols / 16;  // (heads) x (half / 8) items
  const int64_t nv = rows * per_row;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / per_row;
    const int it = (int)(i % per_row);
    const int head = it / (half / 8), j = (it % (half / 8)) * 8;
    const int pos = (int)(r % S);
    const float* a = acc + r * ldacc + head * hd + j;
    const float4 a0 = *reinterpret_cast<const float4*>(a), a1 = *reinterpret_cast<const float4*>(a + 4);
    const float4 b0 = *reinterpret_cast<const float4*>(a + half), b1 = *reinterpret_cast<const float4*>(a + half + 4);
    const float4 c0 = *reinterpret_cast<const float4*>(cs + (int64_t)pos * half + j);
    const float4 c1 = *reinterpret_cast<const float4*>(cs + (int64_t)pos * half + j + 4);
    const float4 s0 = *reinterpret_cast<const float4*>(sn + (int64_t)pos * half + j);
    const float4 s1 = *reinterpret_cast<const float4*>(sn + (int64_t)pos * half + j + 4);
    const float x1[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    const float x2[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
    const float cc[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
    const float ss[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    float y1[8], y2[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      y1[e] = x1[e] * cc[e] + x2[e] * ss[e];
      y2[e] = x2[e] * cc[e] - x1[e] * ss[e];
    }
    __nv_bfloat16* d = dq + r * lddq + head * hd + j;
    *reinterpret_cast<uint4*>(d) =
        make_uint4(pack_bf16(y1[0], y1[1]), pack_bf16(y1[2], y1[3]), pack_bf16(y1[4], y1[5]), pack_bf16(y1[6], y1[7]));
    *reinterpret_cast<uint4*>(d + half) =
        make_uint4(pack_bf16(y2[0], y2[1]), pack_bf16(y2[2], y2[3]), pack_bf16(y2[4], y2[5]), pack_bf16(y2[6], y2[7]));
  }
}

// dq (bf16, row stride lddq) = dq_acc (f32)
__global__ void fa_dq_convert_kernel(const float* __restrict__ acc, int64_t ldacc, __nv_bfloat16* __restrict__ dq,
                                     int64_t lddq, int64_t rows, int cols) {
  const int64_t nv = rows * (cols / 8);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / (cols / 8);
    const int c = (int)(i % (cols / 8)) * 8;
    const float4 a = *reinterpret_cast<const float4*>(acc + r * ldacc + c);
    const float4 b = *reinterpret_cast<const float4*>(acc + r * ldacc + c + 4);
    *reinterpret_cast<uint4*>(dq + r * lddq + c) =
        make_uint4(pack_bf16(a.x, a.y), pack_bf16(a.z, a.w), pack_bf16(b.x, b.y), pack_bf16(b.z, b.w));
  }
}

// 3-D f32 tensor map over dq_acc viewed as [B][S][cols] (row stride ld), box of 32
// columns x 32 rows x 1 batch, 128-byte swizzle: the target of the dQ reduce-adds.
// Rows past S are outside the map, so a box that reaches past a sequence's end is
// clipped there instead of spilling into the next sequence.
inline CUtensorMap make_tmap_dq(float* base, int B, int S, int64_t cols, int64_t ld) {
  OXI_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0 && (ld * 4) % 16 == 0 && cols % 32 == 0,
            "dq accumulator: 16-byte aligned rows, a multiple of 32 columns");
  ensure_current_context();
  CUtensorMap m;
  cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)S, (cuuint64_t)B};
  cuuint64_t strides[2] = {(cuuint64_t)(ld * 4), (cuuint64_t)(ld * 4 * S)};
  cuuint32_t box[3] = {32, 32, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = get_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, base, dims, strides, box, estr,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  OXI_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (dq accumulator) failed: ", (int)r);
  return m;
}

template <int DQ, int DV>
void launch_fa_bwd_t(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
                     const void* dout, int64_t lddo, const float* lse, const float* delta, float* dq_acc,
                     int64_t ld_dq, void* dk, int64_t ld_dk, void* dv, int64_t ld_dv, int B, int S, int Hq, int Hk,
                     float scale, bool causal, int* status, cudaStream_t st, const float* rope_cos,
                     const float* rope_sin) {
  using L = FaBwdSmem<DQ, DV>;
  const int64_t T = (int64_t)B * S;
  CUtensorMap tq = make_tmap_bf16(q, T, (int64_t)Hq * DQ, ldq, 64, 128);
  CUtensorMap tk = make_tmap_bf16(k, T, (int64_t)Hk * DQ, ldk, 64, 128);
  CUtensorMap tv = make_tmap_bf16(v, T, (int64_t)Hk * DV, ldv, 64, 128);
  CUtensorMap tdo = make_tmap_bf16(dout, T, (int64_t)Hq * DV, lddo, 64, 128);
  CUtensorMap tdq = make_tmap_dq(dq_acc, B, S, (int64_t)Hq * DQ, ld_dq);
  FaBwdParams p;
  p.B = B; p.S = S; p.Hq = Hq; p.Hk = Hk;
  p.scale = scale;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.causal = causal ? 1 : 0;
  p.lse = lse;
  p.delta = delta;
  p.dq_acc = dq_acc;
  p.ld_dq = ld_dq;
  p.dk = reinterpret_cast<__nv_bfloat16*>(dk);
  p.dv = reinterpret_cast<__nv_bfloat16*>(dv);
  p.ld_dk = ld_dk;
  p.ld_dv = ld_dv;
  p.rope_cos = rope_cos;
  p.rope_sin = rope_sin;
  p.status = status;
  auto kern = fa_bwd_kernel<DQ, DV>;
  static bool attr = false;
  if (!attr) {
    OXI_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::TOTAL));
    attr = true;
  }
  dim3 grid(Hk, B, (S + 127) / 128);
  kern<<<grid, FA_BWD_THREADS, L::TOTAL, st>>>(tq, tk, tv, tdo, tdq, p);
  OXI_CUDA_CHECK(cudaGetLastError());
}

}  // namespace

bool fa_supported(int Dqk, int Dv) {
  return (Dqk == 64 && Dv == 64) || (Dqk == 128 && Dv == 128) || (Dqk == 96 && Dv == 64) ||
         (Dqk == 128 && Dv == 64);
}

bool fa_bwd_supported(int Dqk, int Dv) {
  return (Dqk == 64 && Dv == 64) || (Dqk == 128 && Dv == 128) || (Dqk == 96 && Dv == 64) ||
         (Dqk == 128 && Dv == 64);
}

void launch_fa_fwd(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv, void* o,
                   int64_t ldo, float* lse, int B, int S, int Hq, int Hk, int Dqk, int Dv, float scale, bool causal,
                   int* status, cudaStream_t st) {
  OXI_CHECK(Hq % Hk == 0, "query heads must be a multiple of kv heads");
  OXI_CHECK(ldo % 8 == 0 && (reinterpret_cast<uintptr_t>(o) & 15) == 0, "output rows must be 16-byte aligned");
  OXI_CHECK(fa_supported(Dqk, Dv), "flash attention forward has no kernel for head dims (qk ", Dqk, ", v ", Dv, ")");
  if (B == 0 || S == 0) return;
#define OXI_FA_FWD(DQ_, DV_)                                                                                    \
  if (Dqk == DQ_ && Dv == DV_)                                                                                 \
    return launch_fa_fwd_t<DQ_, DV_>(q, ldq, k, ldk, v, ldv, o, ldo, lse, B, S, Hq, Hk, scale, causal, status, st);
  OXI_FA_FWD(64, 64)
  OXI_FA_FWD(128, 128)
  OXI_FA_FWD(96, 64)
  OXI_FA_FWD(128, 64)
#undef OXI_FA_FWD
}

void launch_fa_bwd(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
                   const void* o, int64_t ldo, const void* dout, int64_t lddo, const float* lse, float* delta,
                   float* dq_acc, void* dq, int64_t lddq, void* dk, int64_t ld_dk, void* dv, int64_t ld_dv, int B,
                   int S, int Hq, int Hk, int Dqk, int Dv, float scale, bool causal, int* status, cudaStream_t st,
                   const float* rope_cos, const float* rope_sin) {
  OXI_CHECK(Hq % Hk == 0, "query heads must be a multiple of kv heads");
  const bool rope = rope_cos != nullptr;
  OXI_CHECK(!rope || (rope_sin != nullptr && Dqk == Dv && (Dqk == 64 || Dqk == 128) &&
                      (reinterpret_cast<uintptr_t>(rope_cos) & 15) == 0 &&
                      (reinterpret_cast<uintptr_t>(rope_sin) & 15) == 0),
            "flash backward with RoPE: head dims 64 / 128 (qk == v), 16-byte aligned cos / sin tables");
  OXI_CHECK(ld_dk % 8 == 0 && ld_dv % 8 == 0 && lddq % 8 == 0, "gradient rows must be 16-byte aligned");
  OXI_CHECK(fa_bwd_supported(Dqk, Dv), "flash attention backward has no kernel for head dims (qk ", Dqk, ", v ", Dv,
            ")");
  if (B == 0 || S == 0) return;
  const int64_t T = (int64_t)B * S;
  const int64_t rows = T * Hq;
  OXI_CHECK(Dv % 8 == 0 && (Dv / 8) <= 32 && ((Dv / 8) & (Dv / 8 - 1)) == 0 && ldo % 8 == 0 && lddo % 8 == 0,
            "flash backward prep: v head dim / 8 must be a power of two <= 32");
  fa_bwd_prep_kernel<<<(unsigned)((rows * (Dv / 8) + 255) / 256), 256, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(o), ldo, reinterpret_cast<const __nv_bfloat16*>(dout), lddo, delta, B,
      S, Hq, Dv);
  OXI_CUDA_CHECK(cudaGetLastError());
  OXI_CUDA_CHECK(cudaMemsetAsync(dq_acc, 0, (size_t)T * Hq * Dqk * sizeof(float), st));
#define OXI_FA_BWD(DQ_, DV_)                                                                                       \
  if (Dqk == DQ_ && Dv == DV_)                                                                                    \
    launch_fa_bwd_t<DQ_, DV_>(q, ldq, k, ldk, v, ldv, dout, lddo, lse, delta, dq_acc, (int64_t)Hq * Dqk, dk, ld_dk, \
                              dv, ld_dv, B, S, Hq, Hk, scale, causal, status, st, rope_cos, rope_sin);
  OXI_FA_BWD(64, 64)
  OXI_FA_BWD(128, 128)
  OXI_FA_BWD(96, 64)
  OXI_FA_BWD(128, 64)
#undef OXI_FA_BWD
  if (rope) {
    const int64_t nr = T * (Hq * Dqk / 16);
    fa_dq_convert_rope_kernel<<<(unsigned)std::min<int64_t>((nr + 255) / 256, 148 * 16), 256, 0, st>>>(
        dq_acc, (int64_t)Hq * Dqk, reinterpret_cast<__nv_bfloat16*>(dq), lddq, T, Hq * Dqk, Dqk, S, rope_cos,
        rope_sin);
    OXI_CUDA_CHECK(cudaGetLastError());
    return;
  }
  const int64_t nv = T * (Hq * Dqk / 8);
  fa_dq_convert_kernel<<<(unsigned)std::min<int64_t>((nv + 255) / 256, 148 * 16), 256, 0, st>>>(
      dq_acc, (int64_t)Hq * Dqk, reinterpret_cast<__nv_bfloat16*>(dq), lddq, T, Hq * Dqk);
  OXI_CUDA_CHECK(cudaGetLastError());
}

}  // namespace oxi
