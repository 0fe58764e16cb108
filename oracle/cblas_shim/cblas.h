/*
 * Prototype-only CBLAS header used when compiling the reference's CPU path
 * (this image has the OpenBLAS shared library but no development headers).
 * Only the single routine the reference calls is declared; the enum values
 * are the standard CBLAS ABI constants.  Test infrastructure only.
 */
#ifndef VO_CBLAS_SHIM_H
#define VO_CBLAS_SHIM_H

#ifdef __cplusplus
extern "C" {
#endif

enum CBLAS_ORDER { CblasRowMajor = 101, CblasColMajor = 102 };
enum CBLAS_TRANSPOSE { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 };

void cblas_sgemm(enum CBLAS_ORDER order, enum CBLAS_TRANSPOSE ta,
                 enum CBLAS_TRANSPOSE tb, int M, int N, int K, float alpha,
                 const float *A, int lda, const float *B, int ldb, float beta,
                 float *C, int ldc);

#ifdef __cplusplus
}
#endif
#endif
