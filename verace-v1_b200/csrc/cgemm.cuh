// Batched planar-complex fp32 GEMM used by the Newton-Schulz retraction and by the
// readout polynomial of the CHAM scan:
//     C = alpha * opA(A) opB(B) + beta * X
// opA(A)(m,k) = A[m][k]  or (trans) A[k][m], optionally conjugated; likewise opB.
// Matrices are row-major with leading dimension ld*, batch stride s* (elements),
// real and imaginary parts in separate arrays.  Ai/Bi may be NULL (real operand);
// X may be NULL (beta ignored).  C must not alias A or B.
#pragma once
#include "common.cuh"

namespace verace {

struct CMat {
  const float* re;
  const float* im;
  int ld;
  long long stride;
};

int cgemm(int M, int N, int K, int batch, float alpha,
          CMat A, bool transA, bool conjA,
          CMat B, bool transB, bool conjB,
          float beta, CMat X,
          float* Cr, float* Ci, int ldc, long long sC, cudaStream_t st);

}  // namespace verace
