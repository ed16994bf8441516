// Launchers of the attention kernels (flash_attn.cu).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace oxi {
// Head-dim pairs (qk, v) with a compiled kernel.
bool fa_supported(int Dqk, int Dv);
bool fa_bwd_supported(int Dqk, int Dv);

// q/k: row-major [B*S, H*Dqk] views, v [B*S, Hk*Dv], with row strides ld*;
// o [B*S, Hq*Dv]; lse [B, Hq, S] f32.
void launch_fa_fwd(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv, void* o,
                   int64_t ldo, float* lse, int B, int S, int Hq, int Hk, int Dqk, int Dv, float scale, bool causal,
                   int* status, cudaStream_t st);

// Backward: writes dq (bf16, via an f32 accumulator dq_acc [B*S, Hq*Dqk]), dk
// [B*S, Hk*Dqk] and dv [B*S, Hk*Dv] (bf16, row strides ld_dk / ld_dv); delta
// [B, Hq, S] f32 is scratch.  With rope_cos / rope_sin ([S, Dqk/2] f32 tables, or
// null) q and k are taken to be rotate-half RoPE outputs, and dq / dk are written
// as the gradients of the unrotated projections (the inverse rotation is applied
// in the dK epilogue and in the dQ conversion; needs Dqk == Dv in {64, 128}).
void launch_fa_bwd(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
                   const void* o, int64_t ldo, const void* dout, int64_t lddo, const float* lse, float* delta,
                   float* dq_acc, void* dq, int64_t lddq, void* dk, int64_t ld_dk, void* dv, int64_t ld_dv, int B,
                   int S, int Hq, int Hk, int Dqk, int Dv, float scale, bool causal, int* status, cudaStream_t st,
                   const float* rope_cos = nullptr, const float* rope_sin = nullptr);
}  // namespace oxi
