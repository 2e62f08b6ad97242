// Projection epilogue shared by the two mixers: from one concatenated projection
//     y = x [W_q; W_k; W_v; W_gate]ᵀ           (row r: q | k | v | gate, each h·d wide, gate g)
// produce q, k, v L2-normalised per head (F.normalize(·, p=2, dim=-1), eps 1e-12), with
// CHAM's v passed through SiLU first, and the gates 0.1·sigmoid(·)·mask in fp32.
//   SSSDAttention.project:               sssd_attention.py:116-126 (h heads of d, g = h)
//   ContinuousHolographicMemory.project: cham_memory.py:129-153   (one "head" of D, g = 1, SiLU on v)
// The reference runs these as separate projections and a dozen elementwise and reduction
// kernels; here they are one GEMM (outside this file) and one pass over its output.
//
// Work split: each head vector is normalised by a group of lanes of one warp (16-byte
// loads, fp32 norms, segmented shuffle reductions): several short vectors share a warp,
// long ones take a whole warp.  A lane group takes UPT consecutive vectors (adjacent
// heads of a row) and issues all of their loads before the first reduction, so short
// vectors still keep several 16-byte loads per thread in flight.  The gates are a
// grid-stride tail of the same launch.
#include "common.cuh"

namespace verace {
namespace {

constexpr int PT = 256;   // threads per CTA

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

// A "unit" is one head vector of d values (d/8 chunks of 8).  Units of at most 16 chunks
// share a warp (32 / L lanes per unit, one chunk per lane); longer units take the whole
// warp with CPL chunks per lane.
constexpr int MAXV = 8;   // chunks of 8 per lane: d <= 32 * 8 * 8 = 2048

template <typename T, int CPL, int UPT>
__global__ void __launch_bounds__(PT, 2)
mixer_prologue_kernel(const T* __restrict__ y, long long ld, T* __restrict__ q, T* __restrict__ k,
                      T* __restrict__ v, float* __restrict__ gate, const unsigned char* __restrict__ mask,
                      long long n, int h, int d, int g, int silu_v, int L, long long nvec_blocks) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int hd = h * d;
  if ((long long)blockIdx.x < nvec_blocks) {
    const int upw = 32 / L;                                    // lane groups per warp
    const long long unit0 = (((long long)blockIdx.x * (PT / 32) + w) * upw + lane / L) * UPT;   // (row, part, head)
    const int sl = lane % L;                                   // lane within the group
    const int nc = d / 8;
    const long long nunits = n * 3 * h;
    // unit = (row * 3 + part) * h + head: one 64-bit division per lane group, then steps
    long long row0;
    int rem0;
    if (nunits < (1LL << 31)) {   // 32-bit division when it fits
      row0 = (int)unit0 / (3 * h);
      rem0 = (int)unit0 - (int)row0 * (3 * h);
    } else {
      row0 = unit0 / (3 * h);
      rem0 = (int)(unit0 - row0 * (3 * h));
    }
    float x[UPT][CPL][8];
#pragma unroll
    for (int u = 0; u < UPT; ++u) {
      const bool active = unit0 + u < nunits;
      const int wrap = (rem0 + u) / (3 * h), rem = rem0 + u - wrap * (3 * h);
      const int part = rem / h, head = rem - part * h;
      const T* src = y + (row0 + wrap) * ld + (long long)part * hd + (long long)head * d;
#pragma unroll
      for (int i = 0; i < CPL; ++i) {
        const int cc = sl + L * i;
        if (active && cc < nc) load8v<T>(src + 8 * cc, x[u][i]);
      }
    }
#pragma unroll
    for (int u = 0; u < UPT; ++u) {
      const bool active = unit0 + u < nunits;
      const int wrap = (rem0 + u) / (3 * h), rem = rem0 + u - wrap * (3 * h);
      const int part = rem / h, head = rem - part * h;
      T* dst = (part == 0 ? q : part == 1 ? k : v) + (row0 + wrap) * hd + (long long)head * d;
      const bool act = part == 2 && silu_v;
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < CPL; ++i) {
        const int cc = sl + L * i;
        if (active && cc < nc) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            if (act) x[u][i][j] = silu_f(x[u][i][j]);
            ss += x[u][i][j] * x[u][i][j];
          }
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
        if (o < L) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float inv = 1.f / fmaxf(sqrtf(ss), 1e-12f);
#pragma unroll
      for (int i = 0; i < CPL; ++i) {
        const int cc = sl + L * i;
        if (active && cc < nc) {
#pragma unroll
          for (int j = 0; j < 8; ++j) x[u][i][j] *= inv;
          store8v<T>(dst + 8 * cc, x[u][i]);
        }
      }
    }
    return;
  }
  // gates: 0.1 sigmoid(y_gate) * mask
  const long long e = ((long long)blockIdx.x - nvec_blocks) * PT + threadIdx.x;
  if (e >= n * g) return;
  long long r;
  int j;
  if (n * g < (1LL << 31)) {   // 32-bit division when it fits
    r = (int)e / g;
    j = (int)e - (int)r * g;
  } else {
    r = e / g;
    j = (int)(e - r * g);
  }
  float val = 0.1f * sigmoid_f(to_f32(y[r * ld + 3LL * hd + j]));
  if (mask && !mask[r]) val = 0.f;
  gate[e] = val;
}

template <typename T>
int launch_prologue(const void* y, long long ld, void* q, void* k, void* v, float* gate, const unsigned char* mask,
                    long long n, int h, int d, int g, int silu_v, cudaStream_t st) {
  const int nc = d / 8;
  int L, cpl;
  if (nc <= 16 && (16 % nc) == 0) { L = nc; cpl = 1; }
  else { L = 32; cpl = (nc + 31) / 32; }
  const int upt = 1;                  // vectors per lane group
  const long long units = n * 3 * h;
  const long long per_block = (long long)(PT / 32) * (32 / L) * upt;
  const long long nvec_blocks = (units + per_block - 1) / per_block;
  const long long ngate_blocks = (n * g + PT - 1) / PT;
  const long long grid = nvec_blocks + ngate_blocks;
  VERACE_REQUIRE(grid < (1LL << 31), VERACE_ERR_UNSUPPORTED, "verace_mixer_prologue: too many rows");
  const T* yy = (const T*)y;
  T *qq = (T*)q, *kk = (T*)k, *vv = (T*)v;
  if (cpl == 1)
    mixer_prologue_kernel<T, 1, 1><<<(unsigned)grid, PT, 0, st>>>(yy, ld, qq, kk, vv, gate, mask, n, h, d, g, silu_v,
                                                                   L, nvec_blocks);
  else if (cpl <= 4)
    mixer_prologue_kernel<T, 4, 1><<<(unsigned)grid, PT, 0, st>>>(yy, ld, qq, kk, vv, gate, mask, n, h, d, g, silu_v,
                                                                   L, nvec_blocks);
  else
    mixer_prologue_kernel<T, MAXV, 1><<<(unsigned)grid, PT, 0, st>>>(yy, ld, qq, kk, vv, gate, mask, n, h, d, g,
                                                                      silu_v, L, nvec_blocks);
  return check_launch("mixer_prologue_kernel");
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
  cudaStream_t st = (cudaStream_t)stream;
  switch (dtype) {
    case VERACE_F32:
      return launch_prologue<float>(y, ld, q, k, v, gate, mask, n, heads, head_dim, gate_cols, silu_v, st);
    case VERACE_BF16:
      return launch_prologue<__nv_bfloat16>(y, ld, q, k, v, gate, mask, n, heads, head_dim, gate_cols, silu_v, st);
    default:
      return launch_prologue<__half>(y, ld, q, k, v, gate, mask, n, heads, head_dim, gate_cols, silu_v, st);
  }
}

