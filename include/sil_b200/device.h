// Device selection for silarray with the B200 backend (replaces the
// reference's include/device.h:5-16).  CUDA takes the slot of the reference's
// GPU device, so array.h's `case Device::MPS:` branches run on the B200 and
// sil::use_cuda() joins use_cpu().  gpu_pending_ keeps its meaning: work is
// queued on the GPU and a host read must flush first.
#pragma once

#include <unified_memory.h>

namespace sil {

enum class Device {
  MPS,
  CPU,
  CUDA = MPS,
};

inline Device device_ = Device::CUDA;
inline bool gpu_pending_ = false;

inline void use_cpu() { device_ = Device::CPU; }
inline void use_cuda() { device_ = Device::CUDA; }
inline void use_mps() { use_cuda(); }  // source compatibility: the GPU device is CUDA here

};  // namespace sil
