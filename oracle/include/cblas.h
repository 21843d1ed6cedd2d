/* Minimal CBLAS prototype for building the reference's v0 ground truth against the
 * OpenBLAS shipped inside this image's Python wheels (no system cblas.h here).
 * TEST INFRASTRUCTURE ONLY: used by oracle/Makefile, never by the product library.
 * Enum values follow the published CBLAS standard (RowMajor=101, NoTrans=111). */
#pragma once
#ifdef __cplusplus
extern "C" {
#endif
enum CBLAS_ORDER { CblasRowMajor = 101, CblasColMajor = 102 };
enum CBLAS_TRANSPOSE { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 };
void cblas_sgemm(enum CBLAS_ORDER order, enum CBLAS_TRANSPOSE ta, enum CBLAS_TRANSPOSE tb,
                 int m, int n, int k, float alpha, const float* A, int lda,
                 const float* B, int ldb, float beta, float* C, int ldc);
#ifdef __cplusplus
}
#endif
