// Projection epilogue shared by the two mixers: from one concatenated projection
//     y = x [W_q; W_k; W_v; W_gate]ᵀ           (row r: q | k | v | gate, each h·d wide, gate g)
// produce q, k, v L2-normalised per head (F.normalize(·, p=2, dim=-1), eps 1e-12), with
// CHAM's v passed through SiLU first, and the gates 0.1·sigmoid(·)·mask in fp32.
//   SSSDAttention.project:               sssd_attention.py:116-126 (h heads of d, g = h)
//   ContinuousHolographicMemory.project: cham_memory.py:129-153   (one "head" of D, g = 1, SiLU on v)
// The reference runs these as separate projections and a dozen elementwise and reduction
// kernels; here they are one GEMM (outside this file) and one pass over its output.
//
// Work split, from 4096 rows of 16-bit activations with h·d a multiple of 256 and head
// vectors that divide or span whole 32-lane rounds of 16-byte chunks (the configs' 8 x 128
// and 1 x 1024): one row per warp, every lane issuing its 12 loads of a 1024-wide row
// before the first reduction (mixer_prologue_rows; 53 us against 72 us for the general
// split at 16384 rows of 8 x 128 heads).  Otherwise each head vector is normalised by a
// group of lanes of one warp (16-byte loads, fp32 norms, segmented shuffle reductions):
// several short vectors share a warp, long ones take a whole warp, and the gates are a
// grid-stride tail of the same launch.
#include "common.cuh"

#include <algorithm>
#include <type_traits>

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
  // a kernel launched after this one as a programmatic dependent (the deferred decode
  // step's lazy_pre_kernel) may start; it waits for this grid's completion before reading
  asm volatile("griddepcontrol.launch_dependents;");
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
            if (act) x[u][i][j] = to_f32(from_f32<T>(silu_f(x[u][i][j])));   // in the input type, as the
                                                                            // reference's SiLU output is
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

// Row-per-warp variant for 16-bit activations when h d is a multiple of 256 and each head
// vector either divides a 32-lane round of 16-byte chunks (RV = 0: d / 8 a divisor of 32)
// or is RV whole rounds (d / 8 = 32 RV, RV dividing NR): a lane issues NR of a row's
// 16-byte loads (6 KB a warp at h d = 1024) before the first reduction, so the loads in
// flight are not limited by the vectors a lane group holds.  Chunk c = lane + 32 i of the
// row's q | k | v part lies in part c / (h d / 8), head (c mod (h d / 8)) / (d / 8).
template <typename T>
__device__ __forceinline__ uint32_t silu2(uint32_t w) {
  const float2 f = unpack2<T>(w);
  return pack2<T>(silu_f(f.x), silu_f(f.y));
}
template <typename T>
__device__ __forceinline__ float ss2(uint32_t w) {
  const float2 f = unpack2<T>(w);
  return f.x * f.x + f.y * f.y;
}

// Normalise one row segment held as NR rounds of 16-byte words (round i = chunks
// lane + 32 (r0 + i) of the row's q | k | v part) and store it; the gates are separate.
template <typename T, int NR, int RV>
__device__ __forceinline__ void rows_finish(uint4 (&raw)[NR], int r0, int rounds, int lane, int nc, int pc, int silu_v,
                                            long long row, int hd, T* __restrict__ q, T* __restrict__ k,
                                            T* __restrict__ v) {
  float sc[NR];   // per round: this lane's sum of squares, then the vector's 1 / norm
#pragma unroll
  for (int i = 0; i < NR; ++i) {
    if (silu_v && (lane + 32 * (r0 + i)) / pc == 2) {   // v through SiLU, kept in the input type (as
      raw[i].x = silu2<T>(raw[i].x);                     // the reference's SiLU output is)
      raw[i].y = silu2<T>(raw[i].y);
      raw[i].z = silu2<T>(raw[i].z);
      raw[i].w = silu2<T>(raw[i].w);
    }
    sc[i] = ss2<T>(raw[i].x) + ss2<T>(raw[i].y) + ss2<T>(raw[i].z) + ss2<T>(raw[i].w);
  }
  if constexpr (RV == 0) {   // 32 / nc vectors per round: segmented reduction over nc lanes
#pragma unroll
    for (int i = 0; i < NR; ++i) {
      float ss = sc[i];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1)
        if (o < nc) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      sc[i] = 1.f / fmaxf(sqrtf(ss), 1e-12f);
    }
  } else {                   // one vector per RV consecutive rounds
#pragma unroll
    for (int i0 = 0; i0 < NR; i0 += RV) {
      float ss = 0.f;
#pragma unroll
      for (int i = i0; i < i0 + RV; ++i) ss += sc[i];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float r = 1.f / fmaxf(sqrtf(ss), 1e-12f);
#pragma unroll
      for (int i = i0; i < i0 + RV; ++i) sc[i] = r;
    }
  }
#pragma unroll
  for (int i = 0; i < NR; ++i) {
    if (r0 + i < rounds) {
      const int c = lane + 32 * (r0 + i), part = c / pc, cc = c - part * pc;
      const float r = sc[i];
      const float2 a = unpack2<T>(raw[i].x), b = unpack2<T>(raw[i].y), c2 = unpack2<T>(raw[i].z),
                   d2 = unpack2<T>(raw[i].w);
      const uint4 o = make_uint4(pack2<T>(a.x * r, a.y * r), pack2<T>(b.x * r, b.y * r), pack2<T>(c2.x * r, c2.y * r),
                                 pack2<T>(d2.x * r, d2.y * r));
      *reinterpret_cast<uint4*>((part == 0 ? q : part == 1 ? k : v) + row * hd + 8LL * cc) = o;
    }
  }
}

// One row per warp, NR rounds of loads in flight per lane (a segment loop for rows of more
// than NR rounds).
template <typename T, int NR, int RV>
__global__ void __launch_bounds__(PT, 3) mixer_prologue_rows(const T* __restrict__ y, long long ld, T* __restrict__ q,
                                                            T* __restrict__ k, T* __restrict__ v,
                                                            float* __restrict__ gate,
                                                            const unsigned char* __restrict__ mask, long long n, int h,
                                                            int d, int g, int silu_v) {
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * (PT / 32) + (threadIdx.x >> 5);
  if (row >= n) return;
  const int hd = h * d, nc = d / 8, pc = hd / 8;
  const int rounds = 3 * pc / 32;
  const T* src = y + row * ld;
  const bool keep = mask == nullptr || mask[row];
  for (int j = lane; j < g; j += 32) gate[row * g + j] = keep ? 0.1f * sigmoid_f(to_f32(src[3LL * hd + j])) : 0.f;
  for (int r0 = 0; r0 < rounds; r0 += NR) {
    uint4 raw[NR];
#pragma unroll
    for (int i = 0; i < NR; ++i)
      if (r0 + i < rounds) raw[i] = *reinterpret_cast<const uint4*>(src + 8 * (lane + 32 * (r0 + i)));
    rows_finish<T, NR, RV>(raw, r0, rounds, lane, nc, pc, silu_v, row, hd, q, k, v);
  }
}

template <typename T>
int launch_prologue(const void* y, long long ld, void* q, void* k, void* v, float* gate, const unsigned char* mask,
                    long long n, int h, int d, int g, int silu_v, cudaStream_t st) {
  const int nc = d / 8;
  int L, cpl;
  if (nc <= 16 && (16 % nc) == 0) { L = nc; cpl = 1; }
  else { L = 32; cpl = (nc + 31) / 32; }
  constexpr int UPT = 1;   // vectors per lane group (2 and 4 measured slower)
  const int upt = UPT;
  const long long units = n * 3 * h;
  const int hd = h * d;
  const long long per_block = (long long)(PT / 32) * (32 / L) * upt;
  const long long nvec_blocks = (units + per_block - 1) / per_block;
  const long long ngate_blocks = (n * g + PT - 1) / PT;
  const long long grid = nvec_blocks + ngate_blocks;
  VERACE_REQUIRE(grid < (1LL << 31), VERACE_ERR_UNSUPPORTED, "verace_mixer_prologue: too many rows");
  const T* yy = (const T*)y;
  T *qq = (T*)q, *kk = (T*)k, *vv = (T*)v;
  if constexpr (sizeof(T) == 2) {
    // (for a few rows, e.g. a decode step's batch, one warp per row leaves most SMs idle and
    // the general split's many small lane groups are faster)
    const bool fits = n >= 4096 && hd % 256 == 0 && (nc <= 32 ? 32 % nc == 0 : (nc == 64 || nc == 128));
    const int rv = nc <= 32 ? 0 : nc / 32;
    if (fits) {   // one row per warp, 12 rounds per segment
      const unsigned gr = (unsigned)((n + PT / 32 - 1) / (PT / 32));
      if (rv == 0)
        mixer_prologue_rows<T, 12, 0><<<gr, PT, 0, st>>>(yy, ld, qq, kk, vv, gate, mask, n, h, d, g, silu_v);
      else if (rv == 2)
        mixer_prologue_rows<T, 12, 2><<<gr, PT, 0, st>>>(yy, ld, qq, kk, vv, gate, mask, n, h, d, g, silu_v);
      else
        mixer_prologue_rows<T, 12, 4><<<gr, PT, 0, st>>>(yy, ld, qq, kk, vv, gate, mask, n, h, d, g, silu_v);
      return check_launch("mixer_prologue_rows");
    }
  }
  if (cpl == 1)
    mixer_prologue_kernel<T, 1, UPT><<<(unsigned)grid, PT, 0, st>>>(yy, ld, qq, kk, vv, gate, mask, n, h, d, g, silu_v,
                                                                   L, nvec_blocks);
  else if (cpl <= 4)
    mixer_prologue_kernel<T, 4, UPT><<<(unsigned)grid, PT, 0, st>>>(yy, ld, qq, kk, vv, gate, mask, n, h, d, g, silu_v,
                                                                   L, nvec_blocks);
  else
    mixer_prologue_kernel<T, MAXV, UPT><<<(unsigned)grid, PT, 0, st>>>(yy, ld, qq, kk, vv, gate, mask, n, h, d, g,
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
  VERACE_REQUIRE((((uintptr_t)y | (uintptr_t)q | (uintptr_t)k | (uintptr_t)v) & 15) == 0, VERACE_ERR_INVALID,
                 "verace_mixer_prologue: y, q, k and v must be 16-byte aligned");
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

