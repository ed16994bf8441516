// Native token loader for raw u32 token files (upstream format: a flat array
// of native-endian u32 token ids, data.rs:103-152).
//
// Batching follows upstream LitDataLoader::next_batch (data.rs:211-233):
// each batch is the contiguous slice [cursor, cursor + B*(S+1)) of the shard,
// viewed as [B, S+1]; inputs = [:, :S], targets = [:, 1:]; the cursor then
// advances by B*S (so consecutive batches share B tokens) and wraps to the
// shard start when the next slice would cross the shard end.
//
// Differences from upstream, by design:
//  * sharding is real: rank r of W reads [r*n/W, (r+1)*n/W) (the last rank
//    takes the remainder), the split of with_sharding (data.rs:172-188);
//  * a prefetch thread fills a ring of caller-owned (pinned) host buffers
//    ahead of the consumer, so the copy to the GPU starts from pinned memory.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <atomic>
#include <condition_variable>
#include <cstdint>
#include <cstring>
#include <deque>
#include <fcntl.h>
#include <mutex>
#include <stdexcept>
#include <string>
#include <sys/mman.h>
#include <sys/stat.h>
#include <thread>
#include <unistd.h>
#include <vector>

namespace py = pybind11;

class TokenLoader {
 public:
  // Memory-mapped file source.
  TokenLoader(const std::string& path, int64_t batch, int64_t seq, int64_t rank, int64_t world)
      : batch_(batch), seq_(seq) {
    fd_ = ::open(path.c_str(), O_RDONLY);
    if (fd_ < 0) throw std::runtime_error("Failed to open data file: " + path);
    struct stat st;
    if (fstat(fd_, &st) != 0) throw std::runtime_error("Failed to stat data file: " + path);
    if (st.st_size % 4 != 0) throw std::runtime_error("File size is not a multiple of u32 size");
    n_ = st.st_size / 4;
    if (n_ > 0) {
      map_ = ::mmap(nullptr, st.st_size, PROT_READ, MAP_SHARED, fd_, 0);
      if (map_ == MAP_FAILED) throw std::runtime_error("Failed to mmap file: " + path);
      ::madvise(map_, st.st_size, MADV_SEQUENTIAL);
      map_bytes_ = st.st_size;
      tokens_ = static_cast<const uint32_t*>(map_);
    }
    init_shard(rank, world);
  }

  // In-memory source (used for the synthetic-token path).
  TokenLoader(py::array_t<uint32_t, py::array::c_style | py::array::forcecast> arr, int64_t batch, int64_t seq,
              int64_t rank, int64_t world)
      : batch_(batch), seq_(seq) {
    owned_.assign(arr.data(), arr.data() + arr.size());
    n_ = (int64_t)owned_.size();
    tokens_ = owned_.data();
    init_shard(rank, world);
  }

  ~TokenLoader() {
    stop_prefetch();
    if (map_ && map_ != MAP_FAILED) ::munmap(map_, map_bytes_);
    if (fd_ >= 0) ::close(fd_);
  }

  int64_t dataset_size() const { return n_; }
  int64_t shard_start() const { return shard_start_; }
  int64_t shard_end() const { return shard_end_; }
  int64_t cursor() const { return cursor_; }
  void set_cursor(int64_t c) {
    if (prefetching_) throw std::runtime_error("set_cursor while prefetching");
    cursor_ = c;
  }
  int64_t tokens_per_batch() const { return batch_ * (seq_ + 1); }

  // Fill dst (int32 [B, S+1]) with the next batch; returns the start offset used.
  int64_t fill(uintptr_t dst) {
    if (prefetching_) throw std::runtime_error("fill() while prefetching; use acquire()");
    return fill_locked(reinterpret_cast<int32_t*>(dst));
  }

  // Start the prefetch thread over caller-owned slots (each int32 [B, S+1]).
  void start_prefetch(std::vector<uintptr_t> slots) {
    if (prefetching_) throw std::runtime_error("prefetch already running");
    if (slots.empty()) throw std::runtime_error("need at least one slot");
    slots_ = slots;
    free_.clear();
    ready_.clear();
    for (size_t i = 0; i < slots_.size(); ++i) free_.push_back((int)i);
    stop_ = false;
    prefetching_ = true;
    worker_ = std::thread([this] { run(); });
  }

  // Block until the next slot is filled; returns {slot, offset}.
  std::pair<int, int64_t> acquire() {
    if (!prefetching_) throw std::runtime_error("prefetch not running");
    py::gil_scoped_release nogil;
    std::unique_lock<std::mutex> lk(mu_);
    cv_.wait(lk, [this] { return !ready_.empty() || stop_ || !error_.empty(); });
    if (!error_.empty()) throw std::runtime_error(error_);
    if (ready_.empty()) throw std::runtime_error("prefetch stopped");
    auto r = ready_.front();
    ready_.pop_front();
    return r;
  }

  // Give a slot back to the worker (after its copy to the device finished).
  void release(int slot) {
    {
      std::lock_guard<std::mutex> lk(mu_);
      free_.push_back(slot);
    }
    cv_.notify_all();
  }

  void stop_prefetch() {
    if (!prefetching_) return;
    {
      std::lock_guard<std::mutex> lk(mu_);
      stop_ = true;
    }
    cv_.notify_all();
    if (worker_.joinable()) worker_.join();
    prefetching_ = false;
  }

 private:
  void init_shard(int64_t rank, int64_t world) {
    if (world < 1 || rank < 0 || rank >= world) throw std::runtime_error("bad rank/world");
    const int64_t shard = n_ / world;
    shard_start_ = rank * shard;
    shard_end_ = (rank == world - 1) ? n_ : (rank + 1) * shard;
    cursor_ = shard_start_;
    if (shard_end_ - shard_start_ < batch_ * (seq_ + 1))
      throw std::runtime_error("data shard smaller than one batch (" + std::to_string(shard_end_ - shard_start_) +
                               " < " + std::to_string(batch_ * (seq_ + 1)) + " tokens)");
  }

  int64_t fill_locked(int32_t* dst) {
    const int64_t need = batch_ * (seq_ + 1);
    if (cursor_ + need > shard_end_) cursor_ = shard_start_;
    const int64_t start = cursor_;
    cursor_ += batch_ * seq_;
    std::memcpy(dst, tokens_ + start, need * sizeof(uint32_t));
    return start;
  }

  void run() {
    try {
      while (true) {
        int slot;
        {
          std::unique_lock<std::mutex> lk(mu_);
          cv_.wait(lk, [this] { return !free_.empty() || stop_; });
          if (stop_) return;
          slot = free_.front();
          free_.pop_front();
        }
        const int64_t off = fill_locked(reinterpret_cast<int32_t*>(slots_[slot]));
        {
          std::lock_guard<std::mutex> lk(mu_);
          ready_.push_back({slot, off});
        }
        cv_.notify_all();
      }
    } catch (const std::exception& e) {
      std::lock_guard<std::mutex> lk(mu_);
      error_ = e.what();
      cv_.notify_all();
    }
  }

  int64_t batch_, seq_;
  int fd_ = -1;
  void* map_ = nullptr;
  size_t map_bytes_ = 0;
  const uint32_t* tokens_ = nullptr;
  std::vector<uint32_t> owned_;
  int64_t n_ = 0, shard_start_ = 0, shard_end_ = 0, cursor_ = 0;

  std::vector<uintptr_t> slots_;
  std::deque<int> free_;
  std::deque<std::pair<int, int64_t>> ready_;
  std::mutex mu_;
  std::condition_variable cv_;
  std::thread worker_;
  bool stop_ = false;
  std::atomic<bool> prefetching_{false};
  std::string error_;
};

// Write a flat u32 token file (upstream write_tokens_to_file, data.rs:274-291).
void write_tokens(const std::string& path, py::array_t<uint32_t, py::array::c_style | py::array::forcecast> arr) {
  FILE* f = std::fopen(path.c_str(), "wb");
  if (!f) throw std::runtime_error("cannot open " + path);
  const size_t n = arr.size();
  if (n && std::fwrite(arr.data(), sizeof(uint32_t), n, f) != n) {
    std::fclose(f);
    throw std::runtime_error("short write to " + path);
  }
  std::fclose(f);
}

PYBIND11_MODULE(oxidizr_b200_data, m) {
  m.doc() = "mmap u32 token loader with rank sharding and a prefetch thread";
  py::class_<TokenLoader>(m, "TokenLoader")
      .def(py::init<const std::string&, int64_t, int64_t, int64_t, int64_t>(), py::arg("path"), py::arg("batch"),
           py::arg("seq"), py::arg("rank") = 0, py::arg("world") = 1)
      .def(py::init<py::array_t<uint32_t, py::array::c_style | py::array::forcecast>, int64_t, int64_t, int64_t,
                    int64_t>(),
           py::arg("tokens"), py::arg("batch"), py::arg("seq"), py::arg("rank") = 0, py::arg("world") = 1)
      .def("dataset_size", &TokenLoader::dataset_size)
      .def("shard_start", &TokenLoader::shard_start)
      .def("shard_end", &TokenLoader::shard_end)
      .def("cursor", &TokenLoader::cursor)
      .def("set_cursor", &TokenLoader::set_cursor)
      .def("tokens_per_batch", &TokenLoader::tokens_per_batch)
      .def("fill", &TokenLoader::fill, py::call_guard<py::gil_scoped_release>())
      .def("start_prefetch", &TokenLoader::start_prefetch)
      .def("acquire", &TokenLoader::acquire)
      .def("release", &TokenLoader::release)
      .def("stop_prefetch", &TokenLoader::stop_prefetch, py::call_guard<py::gil_scoped_release>());
  m.def("write_tokens", &write_tokens);
}
