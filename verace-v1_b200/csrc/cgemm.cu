// SIMT planar-complex GEMM (64x64 output tiles, K-steps of 16, 4x4 complex
// micro-tiles per thread).  See cgemm.cuh for the contract.
#include "cgemm.cuh"

namespace verace {
namespace {

constexpr int BM = 64, BN = 64, BK = 16, PAD = 4;

template <bool TA, bool CA, bool TB, bool CB>
__global__ void __launch_bounds__(256)
cgemm_kernel(int M, int N, int K, float alpha,
             const float* __restrict__ Ar, const float* __restrict__ Ai, int lda, long long sA,
             const float* __restrict__ Br, const float* __restrict__ Bi, int ldb, long long sB,
             float beta, const float* __restrict__ Xr, const float* __restrict__ Xi, int ldx, long long sX,
             float* __restrict__ Cr, float* __restrict__ Ci, int ldc, long long sC) {
  __shared__ __align__(16) float sAr[BK][BM + PAD];
  __shared__ __align__(16) float sAi[BK][BM + PAD];
  __shared__ __align__(16) float sBr[BK][BN + PAD];
  __shared__ __align__(16) float sBi[BK][BN + PAD];
  const int z = blockIdx.z;
  Ar += z * sA; if (Ai) Ai += z * sA;
  Br += z * sB; if (Bi) Bi += z * sB;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  const int tid = threadIdx.x, tx = tid % 16, ty = tid / 16;
  float accr[4][4], acci[4][4];
#pragma unroll
  for (int a = 0; a < 4; ++a)
#pragma unroll
    for (int b = 0; b < 4; ++b) accr[a][b] = acci[a][b] = 0.f;

  for (int k0 = 0; k0 < K; k0 += BK) {
    for (int e = tid; e < BM * BK; e += 256) {
      int mm, kk;
      if (!TA) { mm = e / BK; kk = e % BK; } else { kk = e / BM; mm = e % BM; }
      const int m = m0 + mm, kx = k0 + kk;
      float re = 0.f, im = 0.f;
      if (m < M && kx < K) {
        const size_t off = TA ? (size_t)kx * lda + m : (size_t)m * lda + kx;
        re = Ar[off];
        im = Ai ? Ai[off] : 0.f;
      }
      sAr[kk][mm] = re;
      sAi[kk][mm] = CA ? -im : im;
    }
    for (int e = tid; e < BN * BK; e += 256) {
      int nn, kk;
      if (!TB) { kk = e / BN; nn = e % BN; } else { nn = e / BK; kk = e % BK; }
      const int n = n0 + nn, kx = k0 + kk;
      float re = 0.f, im = 0.f;
      if (n < N && kx < K) {
        const size_t off = TB ? (size_t)n * ldb + kx : (size_t)kx * ldb + n;
        re = Br[off];
        im = Bi ? Bi[off] : 0.f;
      }
      sBr[kk][nn] = re;
      sBi[kk][nn] = CB ? -im : im;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      const float4 ar = *reinterpret_cast<const float4*>(&sAr[kk][ty * 4]);
      const float4 ai = *reinterpret_cast<const float4*>(&sAi[kk][ty * 4]);
      const float4 br = *reinterpret_cast<const float4*>(&sBr[kk][tx * 4]);
      const float4 bi = *reinterpret_cast<const float4*>(&sBi[kk][tx * 4]);
      const float avr[4] = {ar.x, ar.y, ar.z, ar.w}, avi[4] = {ai.x, ai.y, ai.z, ai.w};
      const float bvr[4] = {br.x, br.y, br.z, br.w}, bvi[4] = {bi.x, bi.y, bi.z, bi.w};
#pragma unroll
      for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          accr[a][b] = fmaf(avr[a], bvr[b], accr[a][b]);
          accr[a][b] = fmaf(-avi[a], bvi[b], accr[a][b]);
          acci[a][b] = fmaf(avr[a], bvi[b], acci[a][b]);
          acci[a][b] = fmaf(avi[a], bvr[b], acci[a][b]);
        }
    }
    __syncthreads();
  }
  Cr += z * sC; Ci += z * sC;
  if (Xr) { Xr += z * sX; if (Xi) Xi += z * sX; }
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const int m = m0 + ty * 4 + a;
    if (m >= M) continue;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const int n = n0 + tx * 4 + b;
      if (n >= N) continue;
      float re = alpha * accr[a][b], im = alpha * acci[a][b];
      if (Xr) {
        re += beta * Xr[(size_t)m * ldx + n];
        if (Xi) im += beta * Xi[(size_t)m * ldx + n];
      }
      Cr[(size_t)m * ldc + n] = re;
      Ci[(size_t)m * ldc + n] = im;
    }
  }
}

template <bool TA, bool CA, bool TB, bool CB>
void launch(dim3 g, int M, int N, int K, float alpha, const CMat& A, const CMat& B, float beta,
            const CMat& X, float* Cr, float* Ci, int ldc, long long sC, cudaStream_t st) {
  cgemm_kernel<TA, CA, TB, CB><<<g, 256, 0, st>>>(M, N, K, alpha, A.re, A.im, A.ld, A.stride,
                                                  B.re, B.im, B.ld, B.stride, beta, X.re, X.im,
                                                  X.ld, X.stride, Cr, Ci, ldc, sC);
}

}  // namespace

int cgemm(int M, int N, int K, int batch, float alpha, CMat A, bool transA, bool conjA,
          CMat B, bool transB, bool conjB, float beta, CMat X, float* Cr, float* Ci, int ldc,
          long long sC, cudaStream_t st) {
  if (M <= 0 || N <= 0 || batch <= 0) return VERACE_OK;
  dim3 g((N + BN - 1) / BN, (M + BM - 1) / BM, batch);
  const int code = (transA ? 8 : 0) | (conjA ? 4 : 0) | (transB ? 2 : 0) | (conjB ? 1 : 0);
  switch (code) {
#define VERACE_CG_CASE(c, ta, ca, tb, cb) \
  case c: launch<ta, ca, tb, cb>(g, M, N, K, alpha, A, B, beta, X, Cr, Ci, ldc, sC, st); break;
    VERACE_CG_CASE(0, false, false, false, false)
    VERACE_CG_CASE(1, false, false, false, true)
    VERACE_CG_CASE(2, false, false, true, false)
    VERACE_CG_CASE(3, false, false, true, true)
    VERACE_CG_CASE(4, false, true, false, false)
    VERACE_CG_CASE(5, false, true, false, true)
    VERACE_CG_CASE(6, false, true, true, false)
    VERACE_CG_CASE(7, false, true, true, true)
    VERACE_CG_CASE(8, true, false, false, false)
    VERACE_CG_CASE(9, true, false, false, true)
    VERACE_CG_CASE(10, true, false, true, false)
    VERACE_CG_CASE(11, true, false, true, true)
    VERACE_CG_CASE(12, true, true, false, false)
    VERACE_CG_CASE(13, true, true, false, true)
    VERACE_CG_CASE(14, true, true, true, false)
    VERACE_CG_CASE(15, true, true, true, true)
#undef VERACE_CG_CASE
  }
  return check_launch("cgemm_kernel");
}

}  // namespace verace
