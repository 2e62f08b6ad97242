// Projection epilogue shared by the two mixers: from one concatenated projection
//     y = x [W_q; W_k; W_v; W_gate]ᵀ           (row r: q | k | v | gate, each h·d wide, gate g)
// produce q, k, v L2-normalised per head (F.normalize(·, p=2, dim=-1), eps 1e-12), with
// CHAM's v passed through SiLU first, and the gates 0.1·sigmoid(·)·mask in fp32.
//   SSSDAttention.project:               sssd_attention.py:116-126 (h heads of d, g = h)
//   ContinuousHolographicMemory.project: cham_memory.py:129-153   (one "head" of D, g = 1, SiLU on v)
// The reference runs these as separate projections and a dozen elementwise and reduction
// kernels; here they are one GEMM (outside this file) and one pass over its output.
//
// Work split: one warp per (row, vector, head) normalises d values with 16-byte loads
// (norms in fp32); the gates are a grid-stride tail of the same launch.
#include "common.cuh"

namespace verace {
namespace {

constexpr int PT = 256;   // threads per CTA

__device__ __forceinline__ float warp_sum32(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

template <typename T>
__device__ __forceinline__ void load8v(const T* p, float* x);
template <>
__device__ __forceinline__ void load8v<__nv_bfloat16>(const __nv_bfloat16* p, float* x) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __bfloat1622float2(h[i]);
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
}
template <>
__device__ __forceinline__ void load8v<__half>(const __half* p, float* x) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    x[2 * i] = f.x;
    x[2 * i + 1] = f.y;
  }
}
template <>
__device__ __forceinline__ void load8v<float>(const float* p, float* x) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  const float4 b = *reinterpret_cast<const float4*>(p + 4);
  x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}

template <typename T>
__device__ __forceinline__ void store8v(T* p, const float* x) {
  if constexpr (sizeof(T) == 4) {
    *reinterpret_cast<float4*>(p) = make_float4(x[0], x[1], x[2], x[3]);
    *reinterpret_cast<float4*>(p + 4) = make_float4(x[4], x[5], x[6], x[7]);
  } else {
    uint4 u;
    T* h = reinterpret_cast<T*>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) h[i] = from_f32<T>(x[i]);
    *reinterpret_cast<uint4*>(p) = u;
  }
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.f + expf(-x)); }
__device__ __forceinline__ float sigmoid_f(float x) { return 1.f / (1.f + expf(-x)); }

// Up to MAXV values per lane are held between the norm and the scaling.
constexpr int MAXV = 8;   // chunks of 8 per lane: d <= 32 * 8 * 8 = 2048

template <typename T>
__global__ void __launch_bounds__(PT)
mixer_prologue_kernel(const T* __restrict__ y, long long ld, T* __restrict__ q, T* __restrict__ k,
                      T* __restrict__ v, float* __restrict__ gate, const unsigned char* __restrict__ mask,
                      long long n, int h, int d, int g, int silu_v, long long nvec_blocks) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int hd = h * d;
  if ((long long)blockIdx.x < nvec_blocks) {
    const long long unit = (long long)blockIdx.x * (PT / 32) + w;   // (row, part, head)
    if (unit >= n * 3 * h) return;
    const long long r = unit / (3 * h);
    const int rem = (int)(unit % (3 * h)), part = rem / h, head = rem % h;
    const T* src = y + r * ld + (long long)part * hd + (long long)head * d;
    T* dst = (part == 0 ? q : part == 1 ? k : v) + r * hd + (long long)head * d;
    const bool act = part == 2 && silu_v;
    const int nc = d / 8;
    float x[MAXV][8];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int cc = lane + 32 * i;
      if (cc < nc) {
        load8v<T>(src + 8 * cc, x[i]);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (act) x[i][j] = silu_f(x[i][j]);
          ss += x[i][j] * x[i][j];
        }
      }
    }
    ss = warp_sum32(ss);
    const float inv = 1.f / fmaxf(sqrtf(ss), 1e-12f);
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int cc = lane + 32 * i;
      if (cc < nc) {
#pragma unroll
        for (int j = 0; j < 8; ++j) x[i][j] *= inv;
        store8v<T>(dst + 8 * cc, x[i]);
      }
    }
    return;
  }
  // gates: 0.1 sigmoid(y_gate) * mask
  const long long e = ((long long)blockIdx.x - nvec_blocks) * PT + threadIdx.x;
  if (e >= n * g) return;
  const long long r = e / g;
  const int j = (int)(e % g);
  float val = 0.1f * sigmoid_f(to_f32(y[r * ld + 3LL * hd + j]));
  if (mask && !mask[r]) val = 0.f;
  gate[e] = val;
}

}  // namespace
}  // namespace verace

using namespace verace;

extern "C" int verace_mixer_prologue(const void* y, long long ld, void* q, void* k, void* v, float* gate,
                                     const unsigned char* mask, long long n, int heads, int head_dim,
                                     int gate_cols, int silu_v, int dtype, void* stream) {
  VERACE_REQUIRE(n >= 0 && heads >= 1 && head_dim >= 1 && gate_cols >= 0, VERACE_ERR_INVALID,
                 "verace_mixer_prologue: invalid sizes n=%lld heads=%d head_dim=%d gate_cols=%d", n, heads,
                 head_dim, gate_cols);
  VERACE_REQUIRE(dtype == VERACE_F32 || dtype == VERACE_BF16 || dtype == VERACE_F16, VERACE_ERR_INVALID,
                 "verace_mixer_prologue: unknown dtype %d", dtype);
  VERACE_REQUIRE(head_dim % 8 == 0 && head_dim <= 32 * 8 * MAXV, VERACE_ERR_UNSUPPORTED,
                 "verace_mixer_prologue: head_dim %d unsupported (a multiple of 8, at most %d)", head_dim,
                 32 * 8 * MAXV);
  const long long hd = (long long)heads * head_dim;
  VERACE_REQUIRE(ld >= 3 * hd + gate_cols && ld % 8 == 0, VERACE_ERR_INVALID,
                 "verace_mixer_prologue: row stride %lld must be >= %lld and a multiple of 8", ld, 3 * hd + gate_cols);
  if (n == 0) return VERACE_OK;
  VERACE_REQUIRE(y && q && k && v && (gate || gate_cols == 0), VERACE_ERR_INVALID,
                 "verace_mixer_prologue: NULL pointer");
  const long long nvec_blocks = (n * 3 * heads + PT / 32 - 1) / (PT / 32);
  const long long ngate_blocks = (n * gate_cols + PT - 1) / PT;
  const long long grid = nvec_blocks + ngate_blocks;
  VERACE_REQUIRE(grid < (1LL << 31), VERACE_ERR_UNSUPPORTED, "verace_mixer_prologue: too many rows");
  cudaStream_t st = (cudaStream_t)stream;
  switch (dtype) {
    case VERACE_F32:
      mixer_prologue_kernel<float><<<(unsigned)grid, PT, 0, st>>>(
          (const float*)y, ld, (float*)q, (float*)k, (float*)v, gate, mask, n, heads, head_dim, gate_cols, silu_v,
          nvec_blocks);
      break;
    case VERACE_BF16:
      mixer_prologue_kernel<__nv_bfloat16><<<(unsigned)grid, PT, 0, st>>>(
          (const __nv_bfloat16*)y, ld, (__nv_bfloat16*)q, (__nv_bfloat16*)k, (__nv_bfloat16*)v, gate, mask, n, heads,
          head_dim, gate_cols, silu_v, nvec_blocks);
      break;
    default:
      mixer_prologue_kernel<__half><<<(unsigned)grid, PT, 0, st>>>(
          (const __half*)y, ld, (__half*)q, (__half*)k, (__half*)v, gate, mask, n, heads, head_dim, gate_cols, silu_v,
          nvec_blocks);
  }
  return check_launch("mixer_prologue_kernel");
}
