// Test infrastructure only: host-memory stand-in for silarray's Metal-backed
// storage (include/unified_memory.h).  Same fields, plain aligned_alloc, and a
// pool keyed by exact byte size like the original (include/unified_memory.h:29-62).
#pragma once

#include <cstddef>
#include <cstdlib>
#include <memory>
#include <stdexcept>
#include <unordered_map>
#include <vector>

namespace sil {

struct storage {
  std::shared_ptr<void> buf;
  void *data = nullptr;
  void *mtl_buf = nullptr;  // always null: there is no GPU in the oracle build
  size_t off = 0;
  size_t len = 0;

  static storage make(size_t bytes);
};

inline storage storage::make(size_t bytes) {
  size_t rounded = ((bytes + 63) / 64) * 64;
  if (rounded == 0) rounded = 64;
  void *p = std::aligned_alloc(64, rounded);
  if (!p) throw std::runtime_error("oracle: out of host memory");
  storage s;
  s.buf = std::shared_ptr<void>(p, [](void *q) { std::free(q); });
  s.data = p;
  return s;
}

};  // namespace sil
