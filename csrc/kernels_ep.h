// Expert-parallel NVLink dispatch / combine (ep.cu).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace oxi {

constexpr int EP_MAXW = 8;    // ranks of one expert-parallel group (one node)
constexpr int EP_MAXE = 256;  // experts per layer
// flag kinds (one int32 per kind and source rank in every pad)
constexpr int EP_K_COUNTS = 0, EP_K_DISPATCHED = 1, EP_K_YREADY = 2, EP_K_DYPUSHED = 3, EP_K_DXREADY = 4;
constexpr int EP_NKIND = 5;
constexpr int EP_FLAGS = 0;                                 // [EP_NKIND][EP_MAXW]
constexpr int EP_COUNTS = EP_FLAGS + EP_NKIND * EP_MAXW;    // [EP_MAXW][EP_MAXE]
constexpr int EP_PAD_WORDS = EP_COUNTS + EP_MAXW * EP_MAXE;

// All-gather of per-expert counts [E] -> all_counts [W][E]; seg_off [El + 2]
// (128-aligned segment starts of this rank's receive buffer, then the skip
// marker), recv_counts [El].  When any owner would need more than `cap` rows
// the layer is skipped on every rank: empty segments, seg_off[El + 1] = 1,
// *overflow = 1 and *need_max >= the rows it would have needed.
void launch_ep_counts(const int* local_counts, const uint64_t* peer_pads, int* my_pad, int rank, int W, int E, int seq,
                      int* all_counts, int* seg_off, int* recv_counts, int cap, int* overflow, int* need_max,
                      int* status, int64_t wait_ns, cudaStream_t st);
// x [T, H] rows -> owners' xrecv; routing weights -> owners' metaw; source index
// (rank * T*k + pair) -> owners' srcidx; pos_out [T*k] = row in the owner's buffers.
void launch_ep_dispatch(const void* x, int64_t ldx, const int64_t* topi, const float* topw, int64_t T, int k, int H,
                        const int* all_counts, int rank, int W, int E, int* cursor, const uint64_t* peers_xrecv,
                        const uint64_t* peers_metaw, const uint64_t* peers_srcidx, int* pos_out, int* done_ctr,
                        const uint64_t* peer_pads, int seq, const int* seg_off, const int* status, cudaStream_t st);
// srcidx = -1 on the padding rows of this rank's expert segments
void launch_ep_mark_pad(const int* seg_off, const int* recv_counts, int El, int* srcidx, cudaStream_t st);
void launch_ep_wait(const int* my_pad, int kind, int W, int seq, int* status, int64_t wait_ns, cudaStream_t st);
void launch_ep_signal(const uint64_t* peer_pads, int kind, int rank, int W, int seq, cudaStream_t st);
// wait for flag `wait_kind` from every owner, then out [T, H] = (resid) + sum_j (w[t,j]) * rows[t*k + j]
void launch_ep_sum_pairs(const void* rows, const float* w, int64_t T, int k, int H, const void* resid, void* out,
                         const int* my_pad, int wait_kind, int W, int seq, int* status, int64_t wait_ns,
                         cudaStream_t st);
// dy rows -> owners' dyrecv; dw [T*k] = <dy_t, yret[t*k + j]>
void launch_ep_push_dy(const void* dy, const int64_t* topi, const int* pos, int64_t T, int k, int H, int El,
                       const uint64_t* peers_dyrecv, const void* yret, float* dw, int* done_ctr,
                       const uint64_t* peer_pads, int rank, int W, int seq, const int* seg_off, const int* status,
                       cudaStream_t st);
void launch_ep_scale_rows(void* dyrecv, const float* metaw, const int* seg_off, const int* recv_counts, int El, int H,
                          int64_t cap_rows, cudaStream_t st);
}  // namespace oxi
