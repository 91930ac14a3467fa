/*
 * Stand-in for Apple's Accelerate framework, used ONLY to compile the
 * reference's CPU sources on Linux as a test oracle (oracle/_ref).  Each
 * routine is a plain scalar loop with the semantics Apple documents for it;
 * where Accelerate's internal order or exp implementation is unknowable,
 * the pinned definitions of oracle/oracle.h are used (vDSP_svesq: 32-lane
 * order over 4-float chunks; vDSP_sve: 1024-thread order; vvexpf: or_expf).
 * Test infrastructure; never part of the product.
 */
#pragma once
#include <stddef.h>
#include <math.h>
#include "../../oracle.h"

typedef unsigned long vDSP_Length;
typedef long vDSP_Stride;

static inline void vDSP_vneg(const float* a, vDSP_Stride ia, float* c, vDSP_Stride ic, vDSP_Length n) {
    for (vDSP_Length i = 0; i < n; i++) c[i * ic] = -a[i * ia];
}
static inline void vDSP_vsadd(const float* a, vDSP_Stride ia, const float* b, float* c, vDSP_Stride ic, vDSP_Length n) {
    float s = *b;
    for (vDSP_Length i = 0; i < n; i++) c[i * ic] = a[i * ia] + s;
}
/* C = A / B with the (B, A, C) argument order of vDSP_vdiv */
static inline void vDSP_vdiv(const float* b, vDSP_Stride ib, const float* a, vDSP_Stride ia, float* c, vDSP_Stride ic, vDSP_Length n) {
    for (vDSP_Length i = 0; i < n; i++) c[i * ic] = a[i * ia] / b[i * ib];
}
static inline void vDSP_vadd(const float* a, vDSP_Stride ia, const float* b, vDSP_Stride ib, float* c, vDSP_Stride ic, vDSP_Length n) {
    for (vDSP_Length i = 0; i < n; i++) c[i * ic] = a[i * ia] + b[i * ib];
}
/* C = B - A */
static inline void vDSP_vsub(const float* a, vDSP_Stride ia, const float* b, vDSP_Stride ib, float* c, vDSP_Stride ic, vDSP_Length n) {
    for (vDSP_Length i = 0; i < n; i++) c[i * ic] = b[i * ib] - a[i * ia];
}
static inline void vDSP_vmul(const float* a, vDSP_Stride ia, const float* b, vDSP_Stride ib, float* c, vDSP_Stride ic, vDSP_Length n) {
    for (vDSP_Length i = 0; i < n; i++) c[i * ic] = a[i * ia] * b[i * ib];
}
static inline void vDSP_vsmul(const float* a, vDSP_Stride ia, const float* b, float* c, vDSP_Stride ic, vDSP_Length n) {
    float s = *b;
    for (vDSP_Length i = 0; i < n; i++) c[i * ic] = a[i * ia] * s;
}
/* E = A*B - C*D, each product rounded */
static inline void vDSP_vmmsb(const float* a, vDSP_Stride ia, const float* b, vDSP_Stride ib,
                              const float* c, vDSP_Stride ic, const float* d, vDSP_Stride id,
                              float* e, vDSP_Stride ie, vDSP_Length n) {
    for (vDSP_Length i = 0; i < n; i++) {
        float p = a[i * ia] * b[i * ib];
        float q = c[i * ic] * d[i * id];
        e[i * ie] = p - q;
    }
}
/* E = A*B + C*D, each product rounded */
static inline void vDSP_vmma(const float* a, vDSP_Stride ia, const float* b, vDSP_Stride ib,
                             const float* c, vDSP_Stride ic, const float* d, vDSP_Stride id,
                             float* e, vDSP_Stride ie, vDSP_Length n) {
    for (vDSP_Length i = 0; i < n; i++) {
        float p = a[i * ia] * b[i * ib];
        float q = c[i * ic] * d[i * id];
        e[i * ie] = p + q;
    }
}
static inline void vDSP_svesq(const float* a, vDSP_Stride ia, float* c, vDSP_Length n) {
    if (ia == 1) { *c = or_sumsq(a, (int)n, 4); return; }
    float s = 0.0f;
    for (vDSP_Length i = 0; i < n; i++) s = fmaf(a[i * ia], a[i * ia], s);
    *c = s;
}
static inline void vDSP_sve(const float* a, vDSP_Stride ia, float* c, vDSP_Length n) {
    if (ia == 1) { *c = or_softmax_sum(a, (int)n); return; }
    float s = 0.0f;
    for (vDSP_Length i = 0; i < n; i++) s += a[i * ia];
    *c = s;
}
static inline void vDSP_maxv(const float* a, vDSP_Stride ia, float* c, vDSP_Length n) {
    float m = -INFINITY;
    for (vDSP_Length i = 0; i < n; i++) if (a[i * ia] > m) m = a[i * ia];
    *c = m;
}
static inline void vDSP_dotpr(const float* a, vDSP_Stride ia, const float* b, vDSP_Stride ib, float* c, vDSP_Length n) {
    float s = 0.0f;
    for (vDSP_Length i = 0; i < n; i++) s += a[i * ia] * b[i * ib];
    *c = s;
}
static inline void vvexpf(float* y, const float* x, const int* n) {
    for (int i = 0; i < *n; i++) y[i] = or_expf(x[i]);
}

enum CBLAS_ORDER { CblasRowMajor = 101, CblasColMajor = 102 };
enum CBLAS_TRANSPOSE { CblasNoTrans = 111, CblasTrans = 112 };

static inline void cblas_sgemv(enum CBLAS_ORDER order, enum CBLAS_TRANSPOSE tr, int m, int n, float alpha,
                               const float* A, int lda, const float* x, int incx, float beta, float* y, int incy) {
    (void)order;
    if (tr == CblasNoTrans) {
        for (int i = 0; i < m; i++) {
            float s = 0.0f;
            for (int j = 0; j < n; j++) s += A[(size_t)i * lda + j] * x[j * incx];
            y[i * incy] = alpha * s + (beta == 0.0f ? 0.0f : beta * y[i * incy]);
        }
    } else {
        for (int j = 0; j < n; j++) {
            float s = 0.0f;
            for (int i = 0; i < m; i++) s += A[(size_t)i * lda + j] * x[i * incx];
            y[j * incy] = alpha * s + (beta == 0.0f ? 0.0f : beta * y[j * incy]);
        }
    }
}
static inline void cblas_sscal(int n, float a, float* x, int incx) {
    for (int i = 0; i < n; i++) x[i * incx] *= a;
}
static inline void cblas_sger(enum CBLAS_ORDER order, int m, int n, float alpha, const float* x, int incx,
                              const float* y, int incy, float* A, int lda) {
    (void)order;
    for (int i = 0; i < m; i++)
        for (int j = 0; j < n; j++) A[(size_t)i * lda + j] += alpha * x[i * incx] * y[j * incy];
}
static inline void cblas_saxpy(int n, float a, const float* x, int incx, float* y, int incy) {
    for (int i = 0; i < n; i++) y[i * incy] += a * x[i * incx];
}
