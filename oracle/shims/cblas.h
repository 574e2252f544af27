/* TEST INFRASTRUCTURE (oracle) -- not part of the product.
 * Minimal CBLAS header, written for this repository, that forwards
 * cblas_sgemm to the OpenBLAS 0.3.x bundled with scipy (exported there as
 * scipy_cblas_sgemm).  The enum values are the standard CBLAS ones. */
#pragma once

#ifdef __cplusplus
extern "C" {
#endif

enum CBLAS_ORDER { CblasRowMajor = 101, CblasColMajor = 102 };
enum CBLAS_TRANSPOSE { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 };
typedef enum CBLAS_ORDER CBLAS_LAYOUT;

void scipy_cblas_sgemm(enum CBLAS_ORDER order, enum CBLAS_TRANSPOSE ta, enum CBLAS_TRANSPOSE tb,
                       int m, int n, int k, float alpha, const float* a, int lda,
                       const float* b, int ldb, float beta, float* c, int ldc);
void scipy_openblas_set_num_threads(int n);

static inline void cblas_sgemm(enum CBLAS_ORDER order, enum CBLAS_TRANSPOSE ta, enum CBLAS_TRANSPOSE tb,
                               int m, int n, int k, float alpha, const float* a, int lda,
                               const float* b, int ldb, float beta, float* c, int ldc) {
    scipy_cblas_sgemm(order, ta, tb, m, n, k, alpha, a, lda, b, ldb, beta, c, ldc);
}

#ifdef __cplusplus
}
#endif
