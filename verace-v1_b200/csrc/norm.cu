// Residual and RMS-normalisation glue around the two mixers of a block
// (verace_v1/modules/backbone.py: h <- h + SSSD(RMSNorm(h)); h <- h + CHAM(RMSNorm(h)),
// with SSSDAttention's per-head RMSNorm before w_out (sssd_attention.py:177-182) and
// ContinuousHolographicMemory's RMSNorm after w_out (cham_memory.py:241)).
//
// RMSNorm follows torch.nn.RMSNorm: r = x * rsqrt(mean(x^2) + eps) in fp32, rounded to the
// input dtype, then multiplied by the weight (rounded again).  A residual add rounds its
// fp32 sum once.  The fused entry point does a block's residual step in one pass:
//     h <- h + (y_weight ? RMSNorm(y) : y);   n <- RMSNorm(h)   (when n is given)
// Work split: one row per group of L lanes (L = 16 for rows of 128, else 32), 16-byte
// vector loads, fp32 sums by segmented shuffles.  For rows of up to 1024 the weights are
// loaded together with the rows, so a small launch (a decode step's 64 rows) waits for
// one round trip to memory before its reductions instead of one per weight vector.
#include "common.cuh"

namespace verace {
namespace {

constexpr int NT = 256;    // threads per CTA
constexpr int MAXV = 8;    // 8-element chunks per lane: rows <= 32 * 8 * 8 = 2048

template <typename T>
__device__ __forceinline__ void ld8(const T* p, float* x) {
  if constexpr (sizeof(T) == 4) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    const float4 b = *reinterpret_cast<const float4*>(p + 4);
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
  } else {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) x[i] = to_f32(e[i]);
  }
}

template <typename T>
__device__ __forceinline__ void st8(T* p, const float* x) {
  if constexpr (sizeof(T) == 4) {
    *reinterpret_cast<float4*>(p) = make_float4(x[0], x[1], x[2], x[3]);
    *reinterpret_cast<float4*>(p + 4) = make_float4(x[4], x[5], x[6], x[7]);
  } else {
    uint4 u;
    T* e = reinterpret_cast<T*>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) e[i] = from_f32<T>(x[i]);
    *reinterpret_cast<uint4*>(p) = u;
  }
}

// round to the storage dtype and back
template <typename T>
__device__ __forceinline__ float rnd(float x) {
  if constexpr (sizeof(T) == 4) return x;
  else return to_f32(from_f32<T>(x));
}

template <int L>
__device__ __forceinline__ float group_sum(float s) {
#pragma unroll
  for (int o = L / 2; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  return s;
}

// 8 consecutive elements as loaded (16 bytes for 2-byte types, 32 for fp32)
template <typename T>
struct Raw8 {
  uint4 u[sizeof(T) / 2];
};

template <typename T>
__device__ __forceinline__ void ldraw(const T* p, Raw8<T>& r) {
#pragma unroll
  for (int k = 0; k < (int)(sizeof(T) / 2); ++k) r.u[k] = __ldg(reinterpret_cast<const uint4*>(p) + k);
}

template <typename T>
__device__ __forceinline__ void unraw(const Raw8<T>& r, float* x) {
  if constexpr (sizeof(T) == 4) {
    x[0] = __uint_as_float(r.u[0].x); x[1] = __uint_as_float(r.u[0].y);
    x[2] = __uint_as_float(r.u[0].z); x[3] = __uint_as_float(r.u[0].w);
    x[4] = __uint_as_float(r.u[1].x); x[5] = __uint_as_float(r.u[1].y);
    x[6] = __uint_as_float(r.u[1].z); x[7] = __uint_as_float(r.u[1].w);
  } else {
    const uint4 u = r.u[0];
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) x[i] = to_f32(e[i]);
  }
}

// weights loaded up front for rows of at most 4 chunks per lane
template <int V>
constexpr bool prefetch_w() { return V <= 4; }

// the lane's weight chunks (when prefetch_w<V>() and w is given)
template <typename T, int L, int V>
__device__ __forceinline__ void load_w(const T* __restrict__ w, int sl, int nc, Raw8<T> (&wr)[V]) {
  if constexpr (prefetch_w<V>()) {
    if (w) {
#pragma unroll
      for (int i = 0; i < V; ++i)
        if (sl + L * i < nc) ldraw<T>(w + 8 * (sl + L * i), wr[i]);
    }
  }
}

// x[V][8] <- RMSNorm(x) (with weight w when given; its chunks in wr when prefetched),
// rounded as torch does
template <typename T, int L, int V>
__device__ __forceinline__ void rms_apply(float (&x)[V][8], const T* __restrict__ w, const Raw8<T> (&wr)[V], int sl,
                                          int nc, int cols, float eps) {
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i)
    if (sl + L * i < nc)
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = fmaf(x[i][j], x[i][j], ss);
  ss = group_sum<L>(ss);
  const float rs = rsqrtf(ss / (float)cols + eps);
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int cc = sl + L * i;
    if (cc < nc) {
      float wv[8];
      if (w) {
        if constexpr (prefetch_w<V>()) unraw<T>(wr[i], wv);
        else ld8<T>(w + 8 * cc, wv);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float r = rnd<T>(x[i][j] * rs);
        x[i][j] = w ? rnd<T>(r * wv[j]) : r;
      }
    }
  }
}

template <typename T, int L, int V>
__global__ void __launch_bounds__(NT)
rmsnorm_kernel(const T* __restrict__ x, const T* __restrict__ w, T* __restrict__ y, long long rows, int cols,
               float eps) {
  const int lane = threadIdx.x & 31;
  const long long row = ((long long)blockIdx.x * NT + threadIdx.x) / L;
  const int sl = lane % L, nc = cols / 8;
  const bool act = row < rows;
  const T* xr = x + (act ? row : 0) * cols;
  Raw8<T> wr[V];
  load_w<T, L, V>(w, sl, nc, wr);
  // launched as a programmatic dependent of the kernel before it (the SSSD decode step ahead
  // of its per-head norm triggers early): the weights above need nothing from it, x does
  asm volatile("griddepcontrol.wait;" ::: "memory");
  float v[V][8];
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int cc = sl + L * i;
    if (cc < nc) ld8<T>(xr + 8 * cc, v[i]);
    else
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = 0.f;
  }
  rms_apply<T, L, V>(v, w, wr, sl, nc, cols, eps);
  if (!act) return;
  T* yr = y + row * cols;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int cc = sl + L * i;
    if (cc < nc) st8<T>(yr + 8 * cc, v[i]);
  }
}

template <typename T, int L, int V>
__global__ void __launch_bounds__(NT)
add_rmsnorm_kernel(T* __restrict__ h, const T* __restrict__ y, const T* __restrict__ wy, float eps_y,
                   const T* __restrict__ wn, float eps_n, T* __restrict__ n, long long rows, int cols, int norm_y) {
  const int lane = threadIdx.x & 31;
  const long long row = ((long long)blockIdx.x * NT + threadIdx.x) / L;
  const int sl = lane % L, nc = cols / 8;
  const bool act = row < rows;
  const long long off = (act ? row : 0) * cols;
  Raw8<T> wyr[V], wnr[V];
  load_w<T, L, V>(norm_y ? wy : nullptr, sl, nc, wyr);
  load_w<T, L, V>(n ? wn : nullptr, sl, nc, wnr);
  float a[V][8], b[V][8];
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int cc = sl + L * i;
    if (cc < nc) {
      ld8<T>(h + off + 8 * cc, a[i]);
      ld8<T>(y + off + 8 * cc, b[i]);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) a[i][j] = b[i][j] = 0.f;
    }
  }
  if (norm_y) rms_apply<T, L, V>(b, wy, wyr, sl, nc, cols, eps_y);
#pragma unroll
  for (int i = 0; i < V; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) a[i][j] = rnd<T>(a[i][j] + b[i][j]);
  if (act) {
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int cc = sl + L * i;
      if (cc < nc) st8<T>(h + off + 8 * cc, a[i]);
    }
  }
  if (!n) return;
  rms_apply<T, L, V>(a, wn, wnr, sl, nc, cols, eps_n);
  if (!act) return;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int cc = sl + L * i;
    if (cc < nc) st8<T>(n + off + 8 * cc, a[i]);
  }
}

// add_rmsnorm for 16-bit activations and rows of at most 4 chunks per lane: the same
// arithmetic in the same order, with the row's h and y chunks held as the loaded 16-byte
// words (unpacked where used) instead of floats, so that a thread holds a quarter of the
// registers and more rows' loads are in flight per SM.
template <typename T, int L, int V>
__global__ void __launch_bounds__(NT, 3)
add_rmsnorm16_kernel(T* __restrict__ h, const T* __restrict__ y, const T* __restrict__ wy, float eps_y,
                     const T* __restrict__ wn, float eps_n, T* __restrict__ n, long long rows, int cols, int norm_y) {
  static_assert(sizeof(T) == 2 && prefetch_w<V>(), "16-bit rows of at most 4 chunks per lane");
  const int lane = threadIdx.x & 31;
  const long long row = ((long long)blockIdx.x * NT + threadIdx.x) / L;
  const int sl = lane % L, nc = cols / 8;
  const bool act = row < rows;
  const long long off = (act ? row : 0) * cols;
  Raw8<T> wyr[V], wnr[V];
  load_w<T, L, V>(norm_y ? wy : nullptr, sl, nc, wyr);
  load_w<T, L, V>(n ? wn : nullptr, sl, nc, wnr);
  uint4 ar[V], br[V];
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int cc = sl + L * i;
    if (cc < nc) {
      ar[i] = *reinterpret_cast<const uint4*>(h + off + 8 * cc);
      br[i] = *reinterpret_cast<const uint4*>(y + off + 8 * cc);
    } else {
      ar[i] = br[i] = make_uint4(0, 0, 0, 0);
    }
  }
  // sum of squares of a row held as words, in rms_apply's order; then 1 / rms
  auto inv_rms = [&](const uint4 (&r)[V], float eps) {
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < V; ++i)
      if (sl + L * i < nc) {
        float x[8];
        unpack8<T>(r[i], x);
#pragma unroll
        for (int j = 0; j < 8; ++j) ss = fmaf(x[j], x[j], ss);
      }
    ss = group_sum<L>(ss);
    return rsqrtf(ss / (float)cols + eps);
  };
  const float rs_y = norm_y ? inv_rms(br, eps_y) : 0.f;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    float xa[8], xb[8];
    unpack8<T>(ar[i], xa);
    unpack8<T>(br[i], xb);
    if (norm_y && sl + L * i < nc) {
      float wv[8];
      if (wy) unraw<T>(wyr[i], wv);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float r = rnd<T>(xb[j] * rs_y);
        xb[j] = wy ? rnd<T>(r * wv[j]) : r;
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) xa[j] = rnd<T>(xa[j] + xb[j]);
    ar[i] = pack8<T>(xa);   // (exact: every value is already rounded to T)
  }
  if (act) {
#pragma unroll
    for (int i = 0; i < V; ++i) {
      const int cc = sl + L * i;
      if (cc < nc) *reinterpret_cast<uint4*>(h + off + 8 * cc) = ar[i];
    }
  }
  if (!n) return;
  const float rs_n = inv_rms(ar, eps_n);
  if (!act) return;
#pragma unroll
  for (int i = 0; i < V; ++i) {
    const int cc = sl + L * i;
    if (cc < nc) {
      float x[8], wv[8];
      unpack8<T>(ar[i], x);
      if (wn) unraw<T>(wnr[i], wv);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float r = rnd<T>(x[j] * rs_n);
        x[j] = wn ? rnd<T>(r * wv[j]) : r;
      }
      *reinterpret_cast<uint4*>(n + off + 8 * cc) = pack8<T>(x);
    }
  }
}

// lanes per row and chunks per lane for a row of `cols`
struct Shape {
  int L, V;
};
Shape shape_for(int cols) {
  const int nc = cols / 8;
  if (nc <= 16) return {16, 1};
  const int v = (nc + 31) / 32;
  return {32, v <= 1 ? 1 : v <= 4 ? 4 : MAXV};
}

template <typename T>
int launch_rmsnorm(const void* x, const void* w, void* y, long long rows, int cols, float eps, cudaStream_t st) {
  const Shape sh = shape_for(cols);
  const long long grid = (rows * sh.L + NT - 1) / NT;
  VERACE_REQUIRE(grid < (1LL << 31), VERACE_ERR_UNSUPPORTED, "verace_rmsnorm: too many rows");
  const T* xx = (const T*)x;
  const T* ww = (const T*)w;
  T* yy = (T*)y;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(NT);
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (sh.L == 16) VERACE_CUDA(cudaLaunchKernelEx(&cfg, rmsnorm_kernel<T, 16, 1>, xx, ww, yy, rows, cols, eps));
  else if (sh.V == 1) VERACE_CUDA(cudaLaunchKernelEx(&cfg, rmsnorm_kernel<T, 32, 1>, xx, ww, yy, rows, cols, eps));
  else if (sh.V == 4) VERACE_CUDA(cudaLaunchKernelEx(&cfg, rmsnorm_kernel<T, 32, 4>, xx, ww, yy, rows, cols, eps));
  else VERACE_CUDA(cudaLaunchKernelEx(&cfg, rmsnorm_kernel<T, 32, MAXV>, xx, ww, yy, rows, cols, eps));
  return check_launch("rmsnorm_kernel");
}

template <typename T>
int launch_add_rmsnorm(void* h, const void* y, const void* wy, float eps_y, int norm_y, const void* wn, float eps_n,
                       void* n, long long rows, int cols, cudaStream_t st) {
  const Shape sh = shape_for(cols);
  const long long grid = (rows * sh.L + NT - 1) / NT;
  VERACE_REQUIRE(grid < (1LL << 31), VERACE_ERR_UNSUPPORTED, "verace_add_rmsnorm: too many rows");
  T* hh = (T*)h;
  const T* yy = (const T*)y;
  const T* a = (const T*)wy;
  const T* bw = (const T*)wn;
  T* nn = (T*)n;
  if constexpr (sizeof(T) == 2) {
    if (sh.L == 16) {
      add_rmsnorm16_kernel<T, 16, 1><<<(unsigned)grid, NT, 0, st>>>(hh, yy, a, eps_y, bw, eps_n, nn, rows, cols, norm_y);
      return check_launch("add_rmsnorm16_kernel");
    }
    if (sh.V <= 4) {
      if (sh.V == 1)
        add_rmsnorm16_kernel<T, 32, 1><<<(unsigned)grid, NT, 0, st>>>(hh, yy, a, eps_y, bw, eps_n, nn, rows, cols,
                                                                      norm_y);
      else
        add_rmsnorm16_kernel<T, 32, 4><<<(unsigned)grid, NT, 0, st>>>(hh, yy, a, eps_y, bw, eps_n, nn, rows, cols,
                                                                      norm_y);
      return check_launch("add_rmsnorm16_kernel");
    }
  }
  if (sh.L == 16)
    add_rmsnorm_kernel<T, 16, 1><<<(unsigned)grid, NT, 0, st>>>(hh, yy, a, eps_y, bw, eps_n, nn, rows, cols, norm_y);
  else if (sh.V == 1)
    add_rmsnorm_kernel<T, 32, 1><<<(unsigned)grid, NT, 0, st>>>(hh, yy, a, eps_y, bw, eps_n, nn, rows, cols, norm_y);
  else if (sh.V == 4)
    add_rmsnorm_kernel<T, 32, 4><<<(unsigned)grid, NT, 0, st>>>(hh, yy, a, eps_y, bw, eps_n, nn, rows, cols, norm_y);
  else
    add_rmsnorm_kernel<T, 32, MAXV><<<(unsigned)grid, NT, 0, st>>>(hh, yy, a, eps_y, bw, eps_n, nn, rows, cols,
                                                                    norm_y);
  return check_launch("add_rmsnorm_kernel");
}

int check_shape(const char* what, long long rows, int cols, int dtype) {
  VERACE_REQUIRE(rows >= 0 && cols >= 1, VERACE_ERR_INVALID, "%s: invalid sizes rows=%lld cols=%d", what, rows, cols);
  VERACE_REQUIRE(dtype == VERACE_F32 || dtype == VERACE_BF16 || dtype == VERACE_F16, VERACE_ERR_INVALID,
                 "%s: unknown dtype %d", what, dtype);
  VERACE_REQUIRE(cols % 8 == 0 && cols <= 32 * 8 * MAXV, VERACE_ERR_UNSUPPORTED,
                 "%s: cols %d unsupported (a multiple of 8, at most %d)", what, cols, 32 * 8 * MAXV);
  return VERACE_OK;
}

}  // namespace
}  // namespace verace

using namespace verace;

extern "C" int verace_rmsnorm(const void* x, const void* weight, void* y, long long rows, int cols, float eps,
                              int dtype, void* stream) {
  if (int rc = check_shape("verace_rmsnorm", rows, cols, dtype)) return rc;
  if (rows == 0) return VERACE_OK;
  VERACE_REQUIRE(x && y, VERACE_ERR_INVALID, "verace_rmsnorm: NULL pointer");
  cudaStream_t st = (cudaStream_t)stream;
  switch (dtype) {
    case VERACE_F32: return launch_rmsnorm<float>(x, weight, y, rows, cols, eps, st);
    case VERACE_BF16: return launch_rmsnorm<__nv_bfloat16>(x, weight, y, rows, cols, eps, st);
    default: return launch_rmsnorm<__half>(x, weight, y, rows, cols, eps, st);
  }
}

extern "C" int verace_add_rmsnorm(void* h, const void* y, int norm_y, const void* y_weight, float y_eps,
                                  const void* n_weight, float n_eps, void* n, long long rows, int cols, int dtype,
                                  void* stream) {
  if (int rc = check_shape("verace_add_rmsnorm", rows, cols, dtype)) return rc;
  if (rows == 0) return VERACE_OK;
  VERACE_REQUIRE(h && y, VERACE_ERR_INVALID, "verace_add_rmsnorm: NULL pointer");
  cudaStream_t st = (cudaStream_t)stream;
  switch (dtype) {
    case VERACE_F32:
      return launch_add_rmsnorm<float>(h, y, y_weight, y_eps, norm_y, n_weight, n_eps, n, rows, cols, st);
    case VERACE_BF16:
      return launch_add_rmsnorm<__nv_bfloat16>(h, y, y_weight, y_eps, norm_y, n_weight, n_eps, n, rows, cols, st);
    default:
      return launch_add_rmsnorm<__half>(h, y, y_weight, y_eps, norm_y, n_weight, n_eps, n, rows, cols, st);
  }
}
