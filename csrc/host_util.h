// Host-side error helpers shared by the torch-free launchers.
#pragma once
#include <cuda_runtime.h>
#include <cstdio>
#include <type_traits>
#include <stdexcept>
#include <string>

namespace oxi {
// Messages are assembled with std::string and snprintf: std::ostringstream
// crashed (SIGSEGV in its locale setup) inside the extension when loaded into
// this PyTorch build, which turned every failed check into a crash.
inline void append_arg(std::string& s, const char* v) { s += v ? v : "(null)"; }
inline void append_arg(std::string& s, const std::string& v) { s += v; }
inline void append_arg(std::string& s, char v) { s += v; }
inline void append_arg(std::string& s, bool v) { s += v ? "true" : "false"; }
inline void append_arg(std::string& s, double v) {
  char b[64];
  snprintf(b, sizeof b, "%g", v);
  s += b;
}
inline void append_arg(std::string& s, float v) { append_arg(s, (double)v); }
template <typename T, typename std::enable_if<std::is_integral<T>::value, int>::type = 0>
inline void append_arg(std::string& s, T v) {
  char b[32];
  if (std::is_signed<T>::value) snprintf(b, sizeof b, "%lld", (long long)v);
  else snprintf(b, sizeof b, "%llu", (unsigned long long)v);
  s += b;
}
template <typename T, typename std::enable_if<std::is_enum<T>::value, int>::type = 0>
inline void append_arg(std::string& s, T v) { append_arg(s, (long long)v); }
inline void append_arg(std::string& s, const void* p) {
  char b[32];
  snprintf(b, sizeof b, "%p", p);
  s += b;
}

template <typename... Args>
[[noreturn]] inline void fail(const char* file, int line, Args&&... args) {
  std::string msg;
  (append_arg(msg, args), ...);
  msg += " (";
  msg += file;
  msg += ":";
  append_arg(msg, line);
  msg += ")";
  throw std::runtime_error(msg);
}
}  // namespace oxi

#define OXI_CHECK(cond, ...) \
  do { if (!(cond)) ::oxi::fail(__FILE__, __LINE__, "check failed: " #cond " ", ##__VA_ARGS__); } while (0)
#define OXI_CUDA_CHECK(expr)                                                                        \
  do {                                                                                              \
    cudaError_t _e = (expr);                                                                        \
    if (_e != cudaSuccess) ::oxi::fail(__FILE__, __LINE__, "CUDA error: ", cudaGetErrorString(_e)); \
  } while (0)
