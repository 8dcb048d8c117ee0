// Umbrella header for silarray on the B200 backend: put include/sil_b200 (and,
// on Linux, include/sil_b200/compat) ahead of silarray's include/ directory;
// device.h, unified_memory.h and gpu.h then resolve to this backend, while
// types.h, cpu.h and array.h remain silarray's own.
#pragma once
#include <device.h>
#include <cpu.h>
#include <gpu.h>
#include <array.h>
