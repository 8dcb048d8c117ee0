// Test infrastructure only: umbrella header for the CPU-only oracle build.
// Resolves to the reference's own device.h / cpu.h / array.h (array.h after
// the mechanical g++-13 rewrite) and to the host-memory stand-ins in this
// folder for unified_memory.h and gpu.h.
#pragma once
#include <device.h>
#include <cpu.h>
#include <gpu.h>
#include <array.h>
