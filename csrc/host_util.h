// Host-side error helpers shared by the torch-free launchers.
#pragma once
#include <cuda_runtime.h>
#include <sstream>
#include <stdexcept>
#include <string>

namespace oxi {
template <typename... Args>
[[noreturn]] inline void fail(const char* file, int line, Args&&... args) {
  std::ostringstream os;
  (os << ... << args);
  os << " (" << file << ":" << line << ")";
  throw std::runtime_error(os.str());
}
}  // namespace oxi

#define OXI_CHECK(cond, ...) \
  do { if (!(cond)) ::oxi::fail(__FILE__, __LINE__, "check failed: " #cond " ", ##__VA_ARGS__); } while (0)
#define OXI_CUDA_CHECK(expr)                                                                        \
  do {                                                                                              \
    cudaError_t _e = (expr);                                                                        \
    if (_e != cudaSuccess) ::oxi::fail(__FILE__, __LINE__, "CUDA error: ", cudaGetErrorString(_e)); \
  } while (0)
