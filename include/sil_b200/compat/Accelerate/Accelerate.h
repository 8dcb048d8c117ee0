// Linux stand-in for the subset of Apple Accelerate
// (vDSP, vForce, CBLAS) that the silarray CPU backend calls, so that the
// reference's own include/cpu.h and include/array.h compile with g++ on Linux.
//
// Semantics follow Apple's published vDSP/vForce documentation:
//   vDSP_vsub(B, .., A, .., C)  -> C = A - B     (operand order is reversed)
//   vDSP_vdiv(B, .., A, .., C)  -> C = A / B
//   vDSP_svdiv(&a, B, .., C)    -> C = a / B
//   vDSP_vsdiv(A, .., &b, C)    -> C = A / b
//   vDSP_vsmsa(A, .., &b, &c, D)-> D = A * b + c
//   vDSP_vthres(A, .., &t, C)   -> C = A >= t ? A : 0
//   vvpowf(z, y, x, &n)         -> z = x ^ y
// Reductions (sve, meanv, dotpr) accumulate sequentially in fp32; Apple's
// vectorised order is not published, so this is the documented stand-in.
// cblas_sgemm is resolved at link time from the host's OpenBLAS.
#pragma once

#include <cmath>
#include <cstddef>
#include <cstring>  // Apple's umbrella header pulls in <string.h>

typedef unsigned long vDSP_Length;
typedef long vDSP_Stride;

extern "C" {
enum CBLAS_ORDER { CblasRowMajor = 101, CblasColMajor = 102 };
enum CBLAS_TRANSPOSE { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 };
void cblas_sgemm(enum CBLAS_ORDER order, enum CBLAS_TRANSPOSE ta,
                 enum CBLAS_TRANSPOSE tb, int M, int N, int K, float alpha,
                 const float *A, int lda, const float *B, int ldb, float beta,
                 float *C, int ldc);
}

inline void vDSP_vadd(const float *A, vDSP_Stride sa, const float *B,
                      vDSP_Stride sb, float *C, vDSP_Stride sc, vDSP_Length n) {
  for (vDSP_Length i = 0; i < n; i++) C[i * sc] = A[i * sa] + B[i * sb];
}
inline void vDSP_vsub(const float *B, vDSP_Stride sb, const float *A,
                      vDSP_Stride sa, float *C, vDSP_Stride sc, vDSP_Length n) {
  for (vDSP_Length i = 0; i < n; i++) C[i * sc] = A[i * sa] - B[i * sb];
}
inline void vDSP_vmul(const float *A, vDSP_Stride sa, const float *B,
                      vDSP_Stride sb, float *C, vDSP_Stride sc, vDSP_Length n) {
  for (vDSP_Length i = 0; i < n; i++) C[i * sc] = A[i * sa] * B[i * sb];
}
inline void vDSP_vdiv(const float *B, vDSP_Stride sb, const float *A,
                      vDSP_Stride sa, float *C, vDSP_Stride sc, vDSP_Length n) {
  for (vDSP_Length i = 0; i < n; i++) C[i * sc] = A[i * sa] / B[i * sb];
}
inline void vDSP_vsadd(const float *A, vDSP_Stride sa, const float *b,
                       float *C, vDSP_Stride sc, vDSP_Length n) {
  const float s = *b;
  for (vDSP_Length i = 0; i < n; i++) C[i * sc] = A[i * sa] + s;
}
inline void vDSP_vsmul(const float *A, vDSP_Stride sa, const float *b,
                       float *C, vDSP_Stride sc, vDSP_Length n) {
  const float s = *b;
  for (vDSP_Length i = 0; i < n; i++) C[i * sc] = A[i * sa] * s;
}
inline void vDSP_vsdiv(const float *A, vDSP_Stride sa, const float *b,
                       float *C, vDSP_Stride sc, vDSP_Length n) {
  const float s = *b;
  for (vDSP_Length i = 0; i < n; i++) C[i * sc] = A[i * sa] / s;
}
inline void vDSP_svdiv(const float *a, const float *B, vDSP_Stride sb,
                       float *C, vDSP_Stride sc, vDSP_Length n) {
  const float s = *a;
  for (vDSP_Length i = 0; i < n; i++) C[i * sc] = s / B[i * sb];
}
inline void vDSP_vsmsa(const float *A, vDSP_Stride sa, const float *b,
                       const float *c, float *D, vDSP_Stride sd, vDSP_Length n) {
  const float s = *b, o = *c;
  for (vDSP_Length i = 0; i < n; i++) {
    volatile float p = A[i * sa] * s;  // unfused multiply, then add
    D[i * sd] = p + o;
  }
}
inline void vDSP_vneg(const float *A, vDSP_Stride sa, float *C,
                      vDSP_Stride sc, vDSP_Length n) {
  for (vDSP_Length i = 0; i < n; i++) C[i * sc] = -A[i * sa];
}
inline void vDSP_vthres(const float *A, vDSP_Stride sa, const float *t,
                        float *C, vDSP_Stride sc, vDSP_Length n) {
  const float th = *t;
  for (vDSP_Length i = 0; i < n; i++) {
    const float v = A[i * sa];
    C[i * sc] = v >= th ? v : 0.0f;
  }
}
inline void vDSP_sve(const float *A, vDSP_Stride sa, float *c, vDSP_Length n) {
  float s = 0.0f;
  for (vDSP_Length i = 0; i < n; i++) s += A[i * sa];
  *c = s;
}
inline void vDSP_meanv(const float *A, vDSP_Stride sa, float *c,
                       vDSP_Length n) {
  float s = 0.0f;
  for (vDSP_Length i = 0; i < n; i++) s += A[i * sa];
  *c = n ? s / static_cast<float>(n) : 0.0f;
}
inline void vDSP_dotpr(const float *A, vDSP_Stride sa, const float *B,
                       vDSP_Stride sb, float *c, vDSP_Length n) {
  float s = 0.0f;
  for (vDSP_Length i = 0; i < n; i++) {
    volatile float p = A[i * sa] * B[i * sb];
    s += p;
  }
  *c = s;
}
inline void vDSP_minvi(const float *A, vDSP_Stride sa, float *c,
                       vDSP_Length *idx, vDSP_Length n) {
  float m = INFINITY;
  vDSP_Length k = 0;
  for (vDSP_Length i = 0; i < n; i++)
    if (A[i * sa] < m) { m = A[i * sa]; k = i * sa; }
  *c = m;
  *idx = k;
}
inline void vDSP_maxvi(const float *A, vDSP_Stride sa, float *c,
                       vDSP_Length *idx, vDSP_Length n) {
  float m = -INFINITY;
  vDSP_Length k = 0;
  for (vDSP_Length i = 0; i < n; i++)
    if (A[i * sa] > m) { m = A[i * sa]; k = i * sa; }
  *c = m;
  *idx = k;
}
inline void vvexpf(float *y, const float *x, const int *n) {
  for (int i = 0; i < *n; i++) y[i] = expf(x[i]);
}
inline void vvrecf(float *y, const float *x, const int *n) {
  for (int i = 0; i < *n; i++) y[i] = 1.0f / x[i];
}
inline void vvpowf(float *z, const float *y, const float *x, const int *n) {
  for (int i = 0; i < *n; i++) z[i] = powf(x[i], y[i]);
}
