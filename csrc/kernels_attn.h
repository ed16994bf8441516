// Launchers of the attention kernels (flash_attn.cu).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace oxi {
// q/k/v: row-major [B*S, H*D] views with row strides ld*; o [B*S, Hq*D]; lse [B, Hq, S] f32.
void launch_fa_fwd(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv, void* o,
                   int64_t ldo, float* lse, int B, int S, int Hq, int Hk, int D, float scale, bool causal,
                   int* status, cudaStream_t st);
}  // namespace oxi

namespace oxi {
// Backward: writes dq (bf16, via an f32 accumulator dq_acc [B*S, Hq*D]), dk, dv
// (bf16, row stride ld_dkv); delta [B, Hq, S] f32 is scratch.
void launch_fa_bwd(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
                   const void* o, int64_t ldo, const void* dout, int64_t lddo, const float* lse, float* delta,
                   float* dq_acc, void* dq, int64_t lddq, void* dk, void* dv, int64_t ld_dkv, int B, int S, int Hq,
                   int Hk, int D, float scale, bool causal, int* status, cudaStream_t st);
}  // namespace oxi
