// mkl.h stand-in used ONLY to compile the reference's own CPU sources in place
// (oracle/Makefile -> oracle/_ref/). The reference is built with icpx + oneMKL
// (baseline/scripts/build.sh:6-8), neither of which exists in this image. This
// header supplies the handful of oneMKL declarations the reference uses:
//  - MKL_BF16, CBLAS enums, MKLVersion;
//  - cblas_gemm_bf16bf16f32 and the Fortran sgemm_ are the real oneMKL entry
//    points exported by PyTorch's libtorch_cpu.so (linked at build time);
//  - cblas_sgemm maps row-major C = A*B onto the column-major sgemm_;
//  - mkl_set_* are no-ops: the oneMKL inside libtorch_cpu.so threads through the
//    process-wide OpenMP runtime, which the reference already configures with
//    omp_set_num_threads (baseline/bench/main.cpp:33);
//  - _mm512_exp_ps (an SVML function, absent from GCC) is a per-lane std::exp.
//    This is a disclosed deviation: std::exp is slower than SVML and rounds
//    differently in the last ulp.
#pragma once
#include <cmath>
#include <cstdint>
#include <immintrin.h>

typedef uint16_t MKL_BF16;
typedef int MKL_INT;
enum CBLAS_LAYOUT { CblasRowMajor = 101, CblasColMajor = 102 };
enum CBLAS_TRANSPOSE { CblasNoTrans = 111, CblasTrans = 112, CblasConjTrans = 113 };

extern "C" {
void sgemm_(const char* transa, const char* transb, const int* m, const int* n, const int* k,
            const float* alpha, const float* a, const int* lda, const float* b, const int* ldb,
            const float* beta, float* c, const int* ldc);
void cblas_gemm_bf16bf16f32(CBLAS_LAYOUT layout, CBLAS_TRANSPOSE transa, CBLAS_TRANSPOSE transb,
                            MKL_INT m, MKL_INT n, MKL_INT k, float alpha, const MKL_BF16* a,
                            MKL_INT lda, const MKL_BF16* b, MKL_INT ldb, float beta, float* c,
                            MKL_INT ldc);
}

inline void cblas_sgemm(CBLAS_LAYOUT layout, CBLAS_TRANSPOSE ta, CBLAS_TRANSPOSE tb, int m, int n,
                        int k, float alpha, const float* a, int lda, const float* b, int ldb,
                        float beta, float* c, int ldc) {
    // Only the row-major, no-transpose form is used by the reference.
    (void)layout;
    (void)ta;
    (void)tb;
    // Row-major C[m][n] = A[m][k] B[k][n]  <=>  column-major C^T = B^T A^T.
    const char nt = 'N';
    sgemm_(&nt, &nt, &n, &m, &k, &alpha, b, &ldb, a, &lda, &beta, c, &ldc);
}

struct MKLVersion {
    int MajorVersion, MinorVersion, UpdateVersion;
    const char* ProductStatus;
    const char* Build;
    const char* Processor;
    const char* Platform;
};
inline void mkl_get_version(MKLVersion* v) {
    v->MajorVersion = 2024;
    v->MinorVersion = 2;
    v->UpdateVersion = 0;
    v->ProductStatus = "libtorch_cpu";
    v->Build = "shim";
    v->Processor = "oneMKL-in-libtorch_cpu";
    v->Platform = "x86_64";
}
inline void mkl_set_num_threads(int) {}
inline void mkl_set_dynamic(int) {}

inline __m512 _mm512_exp_ps(__m512 x) {
    alignas(64) float t[16];
    _mm512_store_ps(t, x);
    for (float& v : t) v = std::exp(v);
    return _mm512_load_ps(t);
}
