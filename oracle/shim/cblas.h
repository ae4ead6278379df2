/* Minimal CBLAS declarations for building the reference CPU path as the oracle.
 *
 * Oracle infrastructure only: nothing in the nova_b200 package includes this.
 * The reference includes <cblas.h> at fusion/src/Fusion/cpu/blas/backend/BlasCblas.hpp:86
 * and calls only cblas_sgemm (BlasCblas.hpp:94). This image ships no CBLAS header, so
 * this file declares the standard netlib CBLAS enum values and the sgemm prototype; the
 * symbol itself comes from the OpenBLAS shared object bundled in the Python venv. */
#ifndef FUSION_ORACLE_CBLAS_SHIM_H
#define FUSION_ORACLE_CBLAS_SHIM_H
#ifdef __cplusplus
extern "C" {
#endif

enum CBLAS_ORDER { CblasRowMajor = 101, CblasColMajor = 102 };
enum CBLAS_TRANSPOSE { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 };

void cblas_sgemm(enum CBLAS_ORDER order, enum CBLAS_TRANSPOSE transa,
                 enum CBLAS_TRANSPOSE transb, int m, int n, int k, float alpha,
                 const float *a, int lda, const float *b, int ldb, float beta,
                 float *c, int ldc);

#ifdef __cplusplus
}
#endif
#endif
