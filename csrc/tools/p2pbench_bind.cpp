// Python bindings of the NVLink microbenchmark kernels (tools extension).
#include <torch/extension.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include "p2pbench.h"

namespace {
cudaStream_t stream() { return c10::cuda::getCurrentCUDAStream().stream(); }

void p2p_read(int64_t src, int64_t bytes, torch::Tensor sink, int64_t ctas, int64_t threads, int64_t unr) {
  c10::cuda::CUDAGuard g(sink.device());
  oxi::launch_p2p_read(reinterpret_cast<const void*>(src), bytes, sink.data_ptr(), (int)ctas, (int)threads, (int)unr,
                       stream());
}

void p2p_write(int64_t dst, int64_t bytes, torch::Tensor on_device, int64_t ctas, int64_t threads, int64_t unr) {
  c10::cuda::CUDAGuard g(on_device.device());
  oxi::launch_p2p_write(reinterpret_cast<void*>(dst), bytes, (int)ctas, (int)threads, (int)unr, stream());
}

void p2p_bulk(bool write, int64_t peer, int64_t bytes, int64_t ctas, int64_t chunk, int64_t stages,
              torch::Tensor status) {
  c10::cuda::CUDAGuard g(status.device());
  TORCH_CHECK(status.scalar_type() == torch::kInt32 && status.is_cuda(), "status: int32 CUDA tensor");
  oxi::launch_p2p_bulk(write, reinterpret_cast<void*>(peer), bytes, (int)ctas, (int)chunk, (int)stages,
                       status.data_ptr<int>(), stream());
}
}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("p2p_read", &p2p_read, "microbenchmark: SM loads from (peer) memory");
  m.def("p2p_write", &p2p_write, "microbenchmark: SM stores to (peer) memory");
  m.def("p2p_bulk", &p2p_bulk, "microbenchmark: bulk (TMA engine) copies from/to (peer) memory");
}
