// Shared helpers for the Verace V1 B200 kernels: element loads/stores for the
// supported input dtypes, the status / last-error plumbing of the C ABI, and a
// small shared-memory SIMT GEMM used by the fp32 chunk kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stddef.h>

#include <type_traits>

#include "../../include/verace_b200.h"

namespace verace {

// ------------------------------------------------------------------ status
void set_error(const char* fmt, ...);
int check_launch(const char* what);

#define VERACE_REQUIRE(cond, code, ...)            \
  do {                                             \
    if (!(cond)) {                                 \
      ::verace::set_error(__VA_ARGS__);            \
      return (code);                               \
    }                                              \
  } while (0)

#define VERACE_CUDA(call)                                                         \
  do {                                                                            \
    cudaError_t _e = (call);                                                      \
    if (_e != cudaSuccess) {                                                      \
      ::verace::set_error("%s failed: %s", #call, cudaGetErrorString(_e));        \
      return VERACE_ERR_CUDA;                                                     \
    }                                                                             \
  } while (0)

static inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// ------------------------------------------------------------------ element IO
__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }

// Two 16-bit values in a 32-bit word <-> floats, by value (no address taken, so arrays of
// words stay in registers).  T is __nv_bfloat16 or __half.
template <typename T>
__device__ __forceinline__ float2 unpack2(uint32_t w) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
  } else {
    return __half22float2(__halves2half2(__ushort_as_half((unsigned short)(w & 0xffffu)),
                                         __ushort_as_half((unsigned short)(w >> 16))));
  }
}
template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(a)) |
           ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(b)) << 16);
  } else {
    return (uint32_t)__half_as_ushort(__float2half_rn(a)) | ((uint32_t)__half_as_ushort(__float2half_rn(b)) << 16);
  }
}
// The 8 values of a 16-byte word of 16-bit elements, and back.
template <typename T>
__device__ __forceinline__ void unpack8(const uint4& u, float* x) {
  float2 f = unpack2<T>(u.x); x[0] = f.x; x[1] = f.y;
  f = unpack2<T>(u.y); x[2] = f.x; x[3] = f.y;
  f = unpack2<T>(u.z); x[4] = f.x; x[5] = f.y;
  f = unpack2<T>(u.w); x[6] = f.x; x[7] = f.y;
}
template <typename T>
__device__ __forceinline__ uint4 pack8(const float* x) {
  return make_uint4(pack2<T>(x[0], x[1]), pack2<T>(x[2], x[3]), pack2<T>(x[4], x[5]), pack2<T>(x[6], x[7]));
}

// ------------------------------------------------------------------ SMEM GEMM
// C(m,n) (=|+=) alpha * sum_k A(m,k) B(k,n) over an M x N output with K terms, where
// A(m,k) = A[m*sam + k*sak], B(k,n) = B[k*sbk + n*sbn], C(m,n) = C[m*scm + n*scn].
// Each participating thread owns TM x TN micro-tiles; consecutive threads step
// along n so that B loads of a warp are contiguous when sbn == 1.
template <int TM, int TN, bool ACC>
__device__ __forceinline__ void smem_gemm(int M, int N, int K,
                                          const float* __restrict__ A, int sam, int sak,
                                          const float* __restrict__ B, int sbk, int sbn,
                                          float* __restrict__ C, int scm, int scn,
                                          int tid, int nthr, float alpha = 1.f) {
  const int tn_count = (N + TN - 1) / TN;
  const int tiles = ((M + TM - 1) / TM) * tn_count;
  for (int tile = tid; tile < tiles; tile += nthr) {
    const int m0 = (tile / tn_count) * TM;
    const int n0 = (tile % tn_count) * TN;
    float acc[TM][TN];
#pragma unroll
    for (int a = 0; a < TM; ++a)
#pragma unroll
      for (int b = 0; b < TN; ++b) acc[a][b] = 0.f;
    for (int k = 0; k < K; ++k) {
      float av[TM], bv[TN];
#pragma unroll
      for (int a = 0; a < TM; ++a) av[a] = (m0 + a < M) ? A[(m0 + a) * sam + k * sak] : 0.f;
#pragma unroll
      for (int b = 0; b < TN; ++b) bv[b] = (n0 + b < N) ? B[k * sbk + (n0 + b) * sbn] : 0.f;
#pragma unroll
      for (int a = 0; a < TM; ++a)
#pragma unroll
        for (int b = 0; b < TN; ++b) acc[a][b] = fmaf(av[a], bv[b], acc[a][b]);
    }
#pragma unroll
    for (int a = 0; a < TM; ++a)
#pragma unroll
      for (int b = 0; b < TN; ++b)
        if (m0 + a < M && n0 + b < N) {
          float* c = &C[(m0 + a) * scm + (n0 + b) * scn];
          if (ACC) *c += alpha * acc[a][b]; else *c = alpha * acc[a][b];
        }
  }
}

}  // namespace verace
