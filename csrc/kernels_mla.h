// Multi-head latent attention operand packing (mla.cu).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace oxi {
// q, k [T, nh, hd + dr] and v [T, nh, hd] from q_c [T, nh*hd] (row stride ldqc), kv [T, 2*nh*hd]
// (k | v, row stride ldkv) and rp [T, dr + nh*dr] (k_rope | q_rope, row stride ldrp); rotate-half
// RoPE from the f32 [S, dr/2] tables at position t % S; k_rope shared by every head.
void launch_mla_pack_fwd(const void* qc, int64_t ldqc, const void* kv, int64_t ldkv, const void* rp, int64_t ldrp,
                         const float* cos_t, const float* sin_t, int64_t T, int S, int nh, int hd, int dr, void* q,
                         void* k, void* v, cudaStream_t st);
// dq_c [T, nh*hd], dkv [T, 2*nh*hd], drp [T, dr + nh*dr] (all contiguous) from dq, dk [T, nh, hd + dr], dv [T, nh, hd].
void launch_mla_pack_bwd(const void* dq, const void* dk, const void* dv, const float* cos_t, const float* sin_t,
                         int64_t T, int S, int nh, int hd, int dr, void* dqc, void* dkv, void* drp, cudaStream_t st);
}  // namespace oxi
