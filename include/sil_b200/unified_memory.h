// Storage for silarray on the B200 backend (replaces the reference's
// include/unified_memory.h:17-79).  Same `storage` fields; buffers are CUDA
// managed memory, so array.h keeps reading `data` on the host after a flush,
// and `mtl_buf` carries the same pointer to mark a GPU-visible buffer.  The
// pool recycles buffers by exact byte size and never frees, like the original.
#pragma once

#include <cuda_runtime_api.h>

#include <cstddef>
#include <memory>
#include <mutex>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

namespace sil {

struct storage {
  std::shared_ptr<void> buf;
  void *data = nullptr;
  void *mtl_buf = nullptr;  // device-visible pointer (== data, managed memory)
  size_t off = 0;
  size_t len = 0;

  static storage make(size_t bytes);
};

class buffer_pool {
 public:
  static buffer_pool &instance() {
    static auto *pool = new buffer_pool();
    return *pool;
  }

  void *acquire(size_t bytes) {
    {
      std::lock_guard<std::mutex> lk(mu_);
      auto it = free_.find(bytes);
      if (it != free_.end() && !it->second.empty()) {
        void *p = it->second.back();
        it->second.pop_back();
        return p;
      }
    }
    void *p = nullptr;
    cudaError_t e = cudaMallocManaged(&p, bytes ? bytes : 16, cudaMemAttachGlobal);
    if (e != cudaSuccess)
      throw std::runtime_error(std::string("storage: cudaMallocManaged: ") + cudaGetErrorString(e));
    return p;
  }

  void release(void *p, size_t bytes) {
    std::lock_guard<std::mutex> lk(mu_);
    free_[bytes].push_back(p);
  }

 private:
  std::mutex mu_;
  std::unordered_map<size_t, std::vector<void *>> free_;
};

inline storage storage::make(size_t bytes) {
  void *p = buffer_pool::instance().acquire(bytes);
  storage s;
  s.buf = std::shared_ptr<void>(p, [bytes](void *q) { buffer_pool::instance().release(q, bytes); });
  s.data = p;
  s.mtl_buf = p;
  return s;
}

};  // namespace sil
