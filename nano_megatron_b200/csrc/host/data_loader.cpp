// Host-side data path: fixed-length token windows gathered from a memory-mapped
// (or in-memory) token stream into caller-provided (typically pinned) int64
// batch buffers, optionally on a background thread so the next batch is ready
// while the GPU runs the current step.
//
// Functional counterpart of the reference's torch DataLoader + Dataset
// __getitem__ path (src/nano_megatron/data/datasets.py:109-236,
// src/nano_megatron/data/loader.py:239-315): sample i is the window
// tokens[i*S : i*S + S + 1]; which samples form a batch (shuffle order,
// replica sharding, resume offset) is decided by the Python sampler.
#include <torch/extension.h>

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <condition_variable>
#include <cstdint>
#include <cstring>
#include <deque>
#include <map>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

namespace {

class TokenSource {
 public:
  // Memory-map `path`, a little-endian array of `count` unsigned integers of
  // `elem_bytes` bytes (2 or 4) or int64 (8).
  TokenSource(const std::string& path, int64_t elem_bytes, int64_t count)
      : elem_bytes_(elem_bytes), count_(count) {
    if (elem_bytes != 2 && elem_bytes != 4 && elem_bytes != 8)
      throw std::invalid_argument("token element size must be 2, 4 or 8 bytes");
    if (count < 1) throw std::invalid_argument("token count must be positive");
    fd_ = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
    if (fd_ < 0) throw std::runtime_error("cannot open token file: " + path);
    struct stat st;
    if (::fstat(fd_, &st) != 0) {
      ::close(fd_);
      throw std::runtime_error("cannot stat token file: " + path);
    }
    bytes_ = static_cast<size_t>(count) * static_cast<size_t>(elem_bytes);
    if (static_cast<size_t>(st.st_size) != bytes_) {
      ::close(fd_);
      throw std::runtime_error("token file size does not match count * element size: " + path);
    }
    void* p = ::mmap(nullptr, bytes_, PROT_READ, MAP_SHARED, fd_, 0);
    if (p == MAP_FAILED) {
      ::close(fd_);
      throw std::runtime_error("mmap failed for token file: " + path);
    }
    base_ = static_cast<const uint8_t*>(p);
    mapped_ = true;
  }

  // Borrow an in-memory int64 CPU tensor (kept alive by this object).
  explicit TokenSource(torch::Tensor tokens) : elem_bytes_(8) {
    TORCH_CHECK(tokens.device().is_cpu() && tokens.dim() == 1, "tokens must be a 1-D CPU tensor");
    TORCH_CHECK(tokens.scalar_type() == torch::kInt64, "tokens must be int64");
    owner_ = tokens.contiguous();
    count_ = owner_.numel();
    TORCH_CHECK(count_ >= 1, "token tensor is empty");
    base_ = reinterpret_cast<const uint8_t*>(owner_.data_ptr<int64_t>());
    bytes_ = static_cast<size_t>(count_) * 8;
  }

  ~TokenSource() {
    if (mapped_) ::munmap(const_cast<uint8_t*>(base_), bytes_);
    if (fd_ >= 0) ::close(fd_);
  }

  int64_t size() const { return count_; }
  int64_t element_bytes() const { return elem_bytes_; }

  // out[r, :] = tokens[starts[r] : starts[r] + window] widened to int64.
  void gather_rows(const int64_t* starts, int64_t rows, int64_t window, int64_t* out,
                   int threads) const {
    for (int64_t r = 0; r < rows; ++r) {
      if (starts[r] < 0 || starts[r] + window > count_)
        throw std::out_of_range("token window [" + std::to_string(starts[r]) + ", " +
                                std::to_string(starts[r] + window) + ") outside token count " +
                                std::to_string(count_));
    }
    auto work = [&](int64_t r0, int64_t r1) {
      for (int64_t r = r0; r < r1; ++r) copy_window(starts[r], window, out + r * window);
    };
    const int64_t total = rows * window;
    int nt = std::max(1, std::min<int>(threads, static_cast<int>(rows)));
    if (nt == 1 || total < (1 << 16)) {
      work(0, rows);
      return;
    }
    std::vector<std::thread> pool;
    const int64_t per = (rows + nt - 1) / nt;
    for (int t = 0; t < nt; ++t) {
      const int64_t r0 = t * per, r1 = std::min(rows, r0 + per);
      if (r0 >= r1) break;
      pool.emplace_back(work, r0, r1);
    }
    for (auto& th : pool) th.join();
  }

 private:
  void copy_window(int64_t start, int64_t n, int64_t* dst) const {
    const uint8_t* src = base_ + static_cast<size_t>(start) * elem_bytes_;
    switch (elem_bytes_) {
      case 2: {
        const uint16_t* s = reinterpret_cast<const uint16_t*>(src);
        for (int64_t i = 0; i < n; ++i) dst[i] = s[i];
        break;
      }
      case 4: {
        const uint32_t* s = reinterpret_cast<const uint32_t*>(src);
        for (int64_t i = 0; i < n; ++i) dst[i] = s[i];
        break;
      }
      default:
        std::memcpy(dst, src, static_cast<size_t>(n) * 8);
    }
  }

  int64_t elem_bytes_ = 8;
  int64_t count_ = 0;
  int fd_ = -1;
  bool mapped_ = false;
  size_t bytes_ = 0;
  const uint8_t* base_ = nullptr;
  torch::Tensor owner_;
};

void check_job(const torch::Tensor& starts, const torch::Tensor& out, int64_t window) {
  TORCH_CHECK(starts.device().is_cpu() && starts.scalar_type() == torch::kInt64 &&
                  starts.dim() == 1 && starts.is_contiguous(),
              "starts must be a contiguous 1-D int64 CPU tensor");
  TORCH_CHECK(out.device().is_cpu() && out.scalar_type() == torch::kInt64 && out.dim() == 2 &&
                  out.is_contiguous(),
              "out must be a contiguous 2-D int64 CPU tensor");
  TORCH_CHECK(out.size(0) == starts.numel() && out.size(1) == window,
              "out must have shape [len(starts), window]");
}

// One background worker that fills submitted (starts, out) jobs in order.
class BatchPrefetcher {
 public:
  BatchPrefetcher(std::shared_ptr<TokenSource> src, int64_t window, int threads)
      : src_(std::move(src)), window_(window), threads_(threads) {
    TORCH_CHECK(window >= 1, "window must be positive");
    worker_ = std::thread([this] { run(); });
  }
  ~BatchPrefetcher() {
    if (Py_IsInitialized() && !_Py_IsFinalizing()) {
      shutdown();  // normal destruction from Python (GIL held)
      return;
    }
    // Interpreter teardown: no GIL operations; stop the worker and let the
    // process reclaim the remaining references.
    {
      std::lock_guard<std::mutex> lk(mu_);
      stop_ = true;
      cv_.notify_all();
    }
    if (worker_.joinable()) worker_.detach();
    for (auto& j : queue_) {
      (void)j.starts.unsafeReleaseTensorImpl();
      (void)j.out.unsafeReleaseTensorImpl();
    }
  }

  int64_t submit(torch::Tensor starts, torch::Tensor out) {
    check_job(starts, out, window_);
    // The mutex is never taken with the GIL held: the worker may need the GIL
    // (to drop the last reference to a Python-owned tensor) while it holds the mutex.
    py::gil_scoped_release nogil;
    std::lock_guard<std::mutex> lk(mu_);
    if (stop_) throw std::runtime_error("prefetcher is shut down");
    const int64_t id = next_id_++;
    queue_.push_back(Job{id, std::move(starts), std::move(out)});
    cv_.notify_all();
    return id;
  }

  // Block until job `id` is filled; rethrow its error, if any.
  void wait(int64_t id) {
    std::string err;
    {
      py::gil_scoped_release nogil;
      std::unique_lock<std::mutex> lk(mu_);
      cv_.wait(lk, [&] { return done_through_ >= id || stop_; });
      auto it = errors_.find(id);
      if (it != errors_.end()) {
        err = it->second;
        errors_.erase(it);
      } else if (done_through_ < id) {
        err = "prefetcher stopped before the job completed";
      }
    }
    if (!err.empty()) throw std::runtime_error(err);
  }

  int64_t pending() {
    py::gil_scoped_release nogil;
    std::lock_guard<std::mutex> lk(mu_);
    return static_cast<int64_t>(queue_.size()) + (busy_ ? 1 : 0);
  }

  void shutdown() {
    py::gil_scoped_release nogil;
    {
      std::lock_guard<std::mutex> lk(mu_);
      stop_ = true;
      cv_.notify_all();
    }
    if (worker_.joinable()) worker_.join();
    // Jobs that never ran hold tensor references; drop them with the GIL held.
    std::deque<Job> left;
    {
      std::lock_guard<std::mutex> lk(mu_);
      left.swap(queue_);
    }
    py::gil_scoped_acquire gil;
    left.clear();
  }

 private:
  struct Job {
    int64_t id;
    torch::Tensor starts, out;
  };

  void run() {
    for (;;) {
      Job job;
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return stop_ || !queue_.empty(); });
        if (stop_) return;
        job = std::move(queue_.front());
        queue_.pop_front();
        busy_ = true;
      }
      std::string err;
      try {
        src_->gather_rows(job.starts.data_ptr<int64_t>(), job.starts.numel(), window_,
                          job.out.data_ptr<int64_t>(), threads_);
      } catch (const std::exception& e) {
        err = e.what();
      }
      // Drop the job's tensor references before publishing completion and outside
      // the mutex: releasing the last reference to a tensor that Python created can
      // take the GIL.
      const int64_t id = job.id;
      job.starts = torch::Tensor();
      job.out = torch::Tensor();
      {
        std::lock_guard<std::mutex> lk(mu_);
        if (!err.empty()) errors_[id] = err;
        done_through_ = id;
        busy_ = false;
        cv_.notify_all();
      }
    }
  }

  std::shared_ptr<TokenSource> src_;
  int64_t window_;
  int threads_;
  std::mutex mu_;
  std::condition_variable cv_;
  std::deque<Job> queue_;
  std::map<int64_t, std::string> errors_;
  int64_t next_id_ = 0;
  int64_t done_through_ = -1;
  bool busy_ = false;
  bool stop_ = false;
  std::thread worker_;
};

}  // namespace

void register_data_loader(py::module& m) {
  py::class_<TokenSource, std::shared_ptr<TokenSource>>(m, "TokenSource")
      .def(py::init<const std::string&, int64_t, int64_t>(), py::arg("path"),
           py::arg("element_bytes"), py::arg("count"))
      .def(py::init<torch::Tensor>(), py::arg("tokens"))
      .def("size", &TokenSource::size)
      .def("element_bytes", &TokenSource::element_bytes)
      .def(
          "gather",
          [](const TokenSource& s, torch::Tensor starts, int64_t window, torch::Tensor out,
             int threads) {
            check_job(starts, out, window);
            py::gil_scoped_release nogil;
            s.gather_rows(starts.data_ptr<int64_t>(), starts.numel(), window,
                          out.data_ptr<int64_t>(), threads);
          },
          py::arg("starts"), py::arg("window"), py::arg("out"), py::arg("threads") = 4);
  py::class_<BatchPrefetcher>(m, "BatchPrefetcher")
      .def(py::init<std::shared_ptr<TokenSource>, int64_t, int>(), py::arg("source"),
           py::arg("window"), py::arg("threads") = 4)
      .def("submit", &BatchPrefetcher::submit)
      .def("wait", &BatchPrefetcher::wait)
      .def("pending", &BatchPrefetcher::pending)
      .def("shutdown", &BatchPrefetcher::shutdown);
}
