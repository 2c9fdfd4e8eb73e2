// Host-side row gathers from a pinned arena (reference
// csrc/kernels/gather_rows.cu:6-21): the staged variant copies the selected
// rows into pinned staging with a small persistent thread pool (one memcpy
// stream per core instead of the reference's single thread), then issues one
// cudaMemcpyAsync of the whole block; the naive variant issues one
// cudaMemcpyAsync per row.  Indices are bounds-checked before any copy.
#include <condition_variable>
#include <cstring>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

#include <cuda_runtime.h>

#include "../../include/soinfer_b200.h"
#include "capi_util.h"

namespace {

class CopyPool {
 public:
  static CopyPool& get() {
    static CopyPool pool;
    return pool;
  }

  // Runs fn(part) for part in [0, parts) across the pool and the caller.
  void run(int parts, const std::function<void(int)>& fn) {
    if (parts <= 1 || workers_.empty()) {
      for (int p = 0; p < parts; ++p) fn(p);
      return;
    }
    std::unique_lock<std::mutex> call_lock(call_mu_);  // one gather at a time through the pool
    {
      std::lock_guard<std::mutex> lk(mu_);
      fn_ = &fn;
      parts_ = parts;
      next_ = 0;
      pending_ = parts;
      ++generation_;
    }
    cv_.notify_all();
    work();
    std::unique_lock<std::mutex> lk(mu_);
    done_cv_.wait(lk, [&] { return pending_ == 0; });
    fn_ = nullptr;
  }

  int size() const { return (int)workers_.size() + 1; }

 private:
  CopyPool() {
    unsigned n = std::thread::hardware_concurrency();
    if (n == 0) n = 1;
    if (n > 16) n = 16;
    for (unsigned i = 1; i < n; ++i) workers_.emplace_back([this] { loop(); });
  }
  ~CopyPool() {
    {
      std::lock_guard<std::mutex> lk(mu_);
      stop_ = true;
    }
    cv_.notify_all();
    for (auto& t : workers_) t.join();
  }

  void work() {
    for (;;) {
      int p;
      const std::function<void(int)>* fn;
      {
        std::lock_guard<std::mutex> lk(mu_);
        if (!fn_ || next_ >= parts_) return;
        p = next_++;
        fn = fn_;
      }
      (*fn)(p);
      std::lock_guard<std::mutex> lk(mu_);
      if (--pending_ == 0) done_cv_.notify_all();
    }
  }

  void loop() {
    uint64_t seen = 0;
    for (;;) {
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return stop_ || generation_ != seen; });
        if (stop_) return;
        seen = generation_;
      }
      work();
    }
  }

  std::vector<std::thread> workers_;
  std::mutex call_mu_, mu_;
  std::condition_variable cv_, done_cv_;
  const std::function<void(int)>* fn_ = nullptr;
  int parts_ = 0, next_ = 0, pending_ = 0;
  uint64_t generation_ = 0;
  bool stop_ = false;
};

int check_indices(const char* name, const int64_t* indices, int64_t k, int64_t num_rows) {
  for (int64_t i = 0; i < k; ++i) {
    if (indices[i] < 0 || indices[i] >= num_rows)
      return soinfer::set_error(SOINFER_ERR_INVALID_ARGUMENT, "%s: index %lld at position %lld out of range [0, %lld)",
                                name, (long long)indices[i], (long long)i, (long long)num_rows);
  }
  return SOINFER_OK;
}

}  // namespace

extern "C" {

int soinfer_gather_rows_staged(const uint8_t* matrix, int64_t num_rows, int64_t row_nbytes, const int64_t* indices,
                               int64_t k, uint8_t* staging, int64_t staging_bytes, uint8_t* gpu_dst,
                               int64_t dst_bytes, void* stream) {
  const char* name = "gather_rows_staged";
  if (num_rows < 0 || row_nbytes < 0 || k < 0)
    return soinfer::set_error(SOINFER_ERR_INVALID_ARGUMENT, "%s: sizes must be >= 0", name);
  const int64_t bytes = k * row_nbytes;
  if (staging_bytes < bytes)
    return soinfer::set_error(SOINFER_ERR_INVALID_ARGUMENT, "%s(staging): too small for k * row_nbytes bytes", name);
  if (dst_bytes < bytes)
    return soinfer::set_error(SOINFER_ERR_INVALID_ARGUMENT, "%s(gpu_dst): too small for k * row_nbytes bytes", name);
  if (bytes == 0) return SOINFER_OK;
  if (!matrix || !indices || !staging || !gpu_dst)
    return soinfer::set_error(SOINFER_ERR_INVALID_ARGUMENT, "%s: null pointer", name);
  if (int st = check_indices(name, indices, k, num_rows)) return st;

  CopyPool& pool = CopyPool::get();
  // ~256 KB per part keeps every core busy without tiny tasks
  int64_t parts = bytes / (256 * 1024);
  if (parts > pool.size() * 4) parts = pool.size() * 4;
  if (parts > k) parts = k;
  if (parts < 1) parts = 1;
  const int64_t per = (k + parts - 1) / parts;
  pool.run((int)parts, [&](int p) {
    const int64_t i0 = p * per;
    const int64_t i1 = (i0 + per < k) ? i0 + per : k;
    for (int64_t i = i0; i < i1; ++i)
      std::memcpy(staging + i * row_nbytes, matrix + indices[i] * row_nbytes, (size_t)row_nbytes);
  });
  return soinfer::cuda_result(cudaMemcpyAsync(gpu_dst, staging, (size_t)bytes, cudaMemcpyHostToDevice,
                                              reinterpret_cast<cudaStream_t>(stream)),
                              name);
}

int soinfer_gather_rows_naive(const uint8_t* matrix, int64_t num_rows, int64_t row_nbytes, const int64_t* indices,
                              int64_t k, uint8_t* gpu_dst, int64_t dst_bytes, void* stream) {
  const char* name = "gather_rows_naive";
  if (num_rows < 0 || row_nbytes < 0 || k < 0)
    return soinfer::set_error(SOINFER_ERR_INVALID_ARGUMENT, "%s: sizes must be >= 0", name);
  if (dst_bytes < k * row_nbytes)
    return soinfer::set_error(SOINFER_ERR_INVALID_ARGUMENT, "%s(gpu_dst): too small for k * row_nbytes bytes", name);
  if (k == 0 || row_nbytes == 0) return SOINFER_OK;
  if (!matrix || !indices || !gpu_dst)
    return soinfer::set_error(SOINFER_ERR_INVALID_ARGUMENT, "%s: null pointer", name);
  if (int st = check_indices(name, indices, k, num_rows)) return st;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  for (int64_t i = 0; i < k; ++i) {
    cudaError_t e = cudaMemcpyAsync(gpu_dst + i * row_nbytes, matrix + indices[i] * row_nbytes, (size_t)row_nbytes,
                                    cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) return soinfer::cuda_result(e, name);
  }
  return SOINFER_OK;
}

}  // extern "C"
