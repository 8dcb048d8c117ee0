// Linux stand-in for the one Mach call silarray's benchmark harness makes
// (bench/bench_common.h: task_info(MACH_TASK_BASIC_INFO) for the resident
// set size).  resident_size is the peak resident set of the process, from
// getrusage; the other fields of the Mach structure are not provided.
#pragma once
#include <sys/resource.h>

#include <cstdint>

typedef int kern_return_t;
typedef unsigned int mach_msg_type_number_t;
typedef unsigned int mach_port_t;
typedef int task_flavor_t;
typedef int *task_info_t;

struct mach_task_basic_info {
  uint64_t virtual_size;
  uint64_t resident_size;
  uint64_t resident_size_max;
};
typedef mach_task_basic_info mach_task_basic_info_data_t;

#define KERN_SUCCESS 0
#define MACH_TASK_BASIC_INFO 20
#define MACH_TASK_BASIC_INFO_COUNT \
  (sizeof(mach_task_basic_info_data_t) / sizeof(int))

inline mach_port_t mach_task_self() { return 0; }

inline kern_return_t task_info(mach_port_t, task_flavor_t, task_info_t out, mach_msg_type_number_t *count) {
  rusage ru{};
  getrusage(RUSAGE_SELF, &ru);
  auto *info = reinterpret_cast<mach_task_basic_info_data_t *>(out);
  info->virtual_size = 0;
  info->resident_size = uint64_t(ru.ru_maxrss) * 1024;  // Linux reports KiB
  info->resident_size_max = info->resident_size;
  if (count) *count = MACH_TASK_BASIC_INFO_COUNT;
  return KERN_SUCCESS;
}
