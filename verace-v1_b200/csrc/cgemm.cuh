// Batched planar-complex fp32 GEMM used by the Newton-Schulz retraction and by the
// readout polynomial of the CHAM scan (cgemm_tc below):
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

// On the tcgen05 tensor cores (cgemm_tc.cu; fp32 operands as three bf16 parts, six
// products per real product): the operands are packed into caller scratch of at least
// cgemm_tc_scratch(M, N, K, batch) bytes (one batch item's worth at least; up to four
// items' worth are used per launch group).
size_t cgemm_tc_scratch(int M, int N, int K, int batch);
int cgemm_tc(int M, int N, int K, int batch, float alpha,
             CMat A, bool transA, bool conjA,
             CMat B, bool transB, bool conjB,
             float beta, CMat X,
             float* Cr, float* Ci, int ldc, long long sC, void* scratch, size_t scratch_bytes,
             cudaStream_t st);
int cgemm_tc_read_status(int* status);

}  // namespace verace
