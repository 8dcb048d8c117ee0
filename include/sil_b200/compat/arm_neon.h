// Linux stand-in (scalar) for the four NEON intrinsics the
// silarray CPU backend uses (include/cpu.h affine).  vfmaq_f32 is a fused
// multiply-add on ARM, so it maps to fmaf lane by lane.
#pragma once
#include <cmath>

struct float32x4_t { float v[4]; };

inline float32x4_t vdupq_n_f32(float s) { return {{s, s, s, s}}; }
inline float32x4_t vld1q_f32(const float *p) { return {{p[0], p[1], p[2], p[3]}}; }
inline void vst1q_f32(float *p, float32x4_t a) {
  for (int i = 0; i < 4; i++) p[i] = a.v[i];
}
// vfmaq_f32(a, b, c) = a + b * c, fused
inline float32x4_t vfmaq_f32(float32x4_t a, float32x4_t b, float32x4_t c) {
  float32x4_t r;
  for (int i = 0; i < 4; i++) r.v[i] = fmaf(b.v[i], c.v[i], a.v[i]);
  return r;
}
