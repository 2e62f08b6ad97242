// M-CMoE (Manifold Continuous Mixture-of-Experts) routing, manifold projection and
// SiTU-GLU activation on sm_100a.
//
// Reference: ManifoldContinuousMoE.forward (verace_v1/modules/mcmoe.py:58-120), its GPU
// kernel launch_mcmoe_triton_projection / mcmoe_manifold_gpu_kernel
// (verace_v1/serving/triton_kernels.py:688-723, :313-353) and SiTUGLU.forward
// (verace_v1/modules/activations.py):
//   top-K of the router logits (mcmoe.py:92), softmax over the K kept logits (:93-96),
//   manifold[t] = sum_k w[t,k] U_c (sigma[t,c,:] * (V_c x_t)),  c = idx[t,k]   (:98-120)
//   SiTU-GLU(g, u) = [b1 tanh(g / b1) sigmoid(g)] * [b2 tanh(u / b2)]
//
// The projection on the tensor cores (bf16, d % 128 == 0, C*r % 128 == 0).  A token
// selects K of the C components, but on B200 a dense pass over all components costs less
// than scattering K fp32 d-vectors per token into the output (K*d*4 bytes of L2
// reductions per token against 4*C*r*d flops per token at tensor-core rate), so the
// projection runs as two GEMMs with the routing folded into the first one's epilogue:
//     Yhat[t, c*r + j] = (x_t . V[c, j, :]) * sigma[t, c, j] * wsel[t, c]     (bf16)
//     out[t, f]        = sum_{c, j} Yhat[t, c*r + j] * U[c, f, j]
// with wsel[t, c] the routing weight of component c for token t and 0 when it is not
// selected, so every unselected term is an exact zero (r % 8 == 0: each 8-column group of
// Yhat belongs to one component).  Each GEMM: 128 x 128 output tiles,
// K blocks of 64 loaded by TMA with 128-byte swizzle, tcgen05 MMAs (M = N = 128, K = 16)
// into a 128-column TMEM accumulator, three stages, two CTAs per SM; eight epilogue warps
// (a TMEM lane quarter and half of the columns each) stage the tile in shared memory and
// it leaves by TMA store.  U is first re-laid out as
// [d][C*r] so that the second GEMM's B operand is K-major like the first one's.
// Other dtypes and shapes: one CTA per token evaluates the reference's formula in fp32.
#include "common.cuh"
#include "tc.cuh"
#include "tmap.cuh"

namespace verace {

__device__ int g_mcmoe_status = 0;   // non-zero after a bounded wait gave up

namespace {

constexpr int MAX_TOPK = 16;
constexpr int MAX_C = 256;
constexpr uint32_t GPOLLS = 1u << 22;

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

template <typename T>
__device__ __forceinline__ float rnd(float x) {
  if constexpr (sizeof(T) == 4) return x;
  else return to_f32(from_f32<T>(x));
}

__device__ __forceinline__ float sigmoid_f(float x) { return 1.f / (1.f + expf(-x)); }
// The GEMM epilogue's sigmoid, whose result is rounded to bf16 at once: the fast exponent
// and reciprocal intrinsics are well inside that rounding.
__device__ __forceinline__ float sigmoid_fast(float x) { return __frcp_rn(1.f + __expf(-x)); }

// ------------------------------------------------------------------------- routing
// One warp per token: K rounds of a warp arg-max over the C logits (NaN ranks above every
// number, ties go to the lower index), then the softmax over the K kept logits, which is
// torch.softmax of the masked row (the others are -inf) computed in fp32 and rounded once.
template <typename T>
__global__ void __launch_bounds__(256) mcmoe_route_kernel(const T* __restrict__ logits, long long n, int C, int K,
                                                          long long* __restrict__ idx, T* __restrict__ wout) {
  constexpr int PER = MAX_C / 32;
  const int lane = threadIdx.x & 31;
  const long long t = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t >= n) return;
  const T* row = logits + t * C;
  float v[PER];
  bool taken[PER];
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    const int c = lane + 32 * i;
    v[i] = c < C ? to_f32(row[c]) : 0.f;
    taken[i] = c >= C;
  }
  auto better = [](float a, int ia, float b, int ib) {   // does (a, ia) rank before (b, ib)?
    const bool na = a != a, nb = b != b;
    if (na != nb) return na;
    if (!na && a != b) return a > b;
    return ia < ib;
  };
  float sel_v[MAX_TOPK];
  int sel_i[MAX_TOPK];
#pragma unroll 1
  for (int k = 0; k < K; ++k) {
    float bv = 0.f;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < PER; ++i) {
      const int c = lane + 32 * i;
      if (!taken[i] && (bi == 0x7fffffff || better(v[i], c, bv, bi))) { bv = v[i]; bi = c; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (oi != 0x7fffffff && (bi == 0x7fffffff || better(ov, oi, bv, bi))) { bv = ov; bi = oi; }
    }
#pragma unroll
    for (int i = 0; i < PER; ++i)
      if (lane + 32 * i == bi) taken[i] = true;
    sel_v[k < MAX_TOPK ? k : 0] = bv;
    sel_i[k < MAX_TOPK ? k : 0] = bi;
  }
  if (lane == 0) {
    const float m = sel_v[0];
    float e[MAX_TOPK], s = 0.f;
#pragma unroll 1
    for (int k = 0; k < K; ++k) {
      e[k] = expf(sel_v[k] - m);
      s += e[k];
    }
#pragma unroll 1
    for (int k = 0; k < K; ++k) {
      idx[t * K + k] = sel_i[k];
      wout[t * K + k] = from_f32<T>(e[k] / s);
    }
  }
}

// ------------------------------------------------------------------------- U re-layout
// Ut[f][c*r + j] = U[c][f][j]  (bf16)
__global__ void mcmoe_u_relayout_kernel(const __nv_bfloat16* __restrict__ U, __nv_bfloat16* __restrict__ Ut, int d,
                                        int C, int r) {
  const long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long ncr = (long long)C * r;
  if (e >= (long long)d * ncr) return;
  const int f = (int)(e / ncr), col = (int)(e % ncr), c = col / r, j = col % r;
  Ut[e] = U[((size_t)c * d + f) * r + j];
}

// ------------------------------------------------------------------------- tensor-core GEMM
// C[M][N] = A[M][K] B[N][K]^T (bf16 in, fp32 accumulate), both operands K-major.
constexpr int GBM = 128, GBN = 128, GBK = 64, GST = 3;
constexpr int G_STAGE = (GBM + GBN) * GBK * 2;   // 32 KB
constexpr int G_BAR = GST * G_STAGE;             // 96 KB
constexpr int G_SMEM = G_BAR + 128;
constexpr int G_THREADS = 320;                   // warp 0 TMA, warp 1 MMA (+ TMEM), warps 2-9 epilogue
enum { EPI_STORE = 0, EPI_MASK = 1 };

struct MaskArgs {
  const __nv_bfloat16* sigma;   // [M][N]
  const long long* idx;         // [M][K]
  const __nv_bfloat16* w;       // [M][K]
  int r, K, sigma_is_logits;
};

template <int EPI>
__global__ void __launch_bounds__(G_THREADS, 2)
mcmoe_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                  const __grid_constant__ CUtensorMap tmC, int M, int N, int K, MaskArgs ma) {
  extern __shared__ __align__(1024) unsigned char gsm[];
  uint64_t* full = reinterpret_cast<uint64_t*>(gsm + G_BAR);
  uint64_t* empty = full + GST;
  uint64_t* accf = empty + GST;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(accf + 1);
  volatile int* fail = reinterpret_cast<volatile int*>(tslot + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int m0 = blockIdx.y * GBM, n0 = blockIdx.x * GBN;
  const int nk = K / GBK;
  if (warp == 1) tc::tmem_alloc(tslot, GBN);
  if (tid == 0) {
    for (int s = 0; s < GST; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    tc::mbar_init(accf, 1);
    *fail = 0;
    tc::fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tacc = *tslot;
  auto sA = [&](int s) { return gsm + s * G_STAGE; };
  auto sB = [&](int s) { return gsm + s * G_STAGE + GBM * GBK * 2; };

  if (warp == 0) {
    if (lane == 0) {   // ---- TMA producer
      int kb = 0;
      for (; kb < nk; ++kb) {
        const int s = kb % GST;
        if (kb >= GST && (*fail || !tc::mbar_wait(&empty[s], ((kb / GST) - 1) & 1, GPOLLS))) {
          *fail = 1;
          atomicExch(&g_mcmoe_status, 1);
          break;
        }
        tc::mbar_expect_tx(&full[s], G_STAGE);
        tc::tma_load_2d(sA(s), &tmA, kb * GBK, m0, &full[s]);
        tc::tma_load_2d(sB(s), &tmB, kb * GBK, n0, &full[s]);
      }
      // copies still in flight land before the CTA may exit
      for (int j = kb - GST < 0 ? 0 : kb - GST; j < kb; ++j) tc::mbar_wait(&full[j % GST], (j / GST) & 1, GPOLLS);
    }
  } else if (warp == 1) {
    if (lane == 0) {   // ---- MMA issuer
      constexpr uint32_t ID = tc::idesc_bf16(GBM, GBN, false, false);
      bool ok = true;
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % GST;
        if (*fail || !tc::mbar_wait(&full[s], (kb / GST) & 1, GPOLLS)) {
          ok = false;
          *fail = 1;
          atomicExch(&g_mcmoe_status, 1);
          break;
        }
        tc::fence_after_sync();
        const uint32_t a = tc::smem_addr(sA(s)), b = tc::smem_addr(sB(s));
#pragma unroll
        for (int ks = 0; ks < GBK / 16; ++ks)
          tc::mma_bf16(tacc, tc::sdesc_sw128(a + ks * 32, 16, 1024), tc::sdesc_sw128(b + ks * 32, 16, 1024), ID,
                       (kb > 0 || ks > 0) ? 1u : 0u);
        tc::commit(&empty[s]);   // the stage is free once these MMAs have read it
      }
      tc::commit(accf);          // (also after a failure: every issued MMA completes)
      if (!ok) tc::mbar_wait(accf, 0, GPOLLS);
    }
  } else {
    // ---- epilogue: warps 2-9; TMEM lane quarter warp % 4, columns [64 hf, 64 hf + 64) with
    // hf = (warp - 2) / 4; thread = one output row
    const int q = warp & 3, hf = (warp - 2) >> 2, rl = 32 * q + lane, row = m0 + rl;
    float wg[8];    // routing weight of each 8-column group of the thread's 64 columns (r % 8 == 0)
    uint4 sgn[2];   // the next chunk's sigma (bf16), loaded while the current one is processed
    auto load_sigma = [&](int u) {
      if (row < M) {
        const uint4* sp = reinterpret_cast<const uint4*>(ma.sigma + (size_t)row * N + n0 + 64 * hf + 16 * u);
        sgn[0] = __ldg(sp);
        sgn[1] = __ldg(sp + 1);
      } else {
        sgn[0] = sgn[1] = make_uint4(0, 0, 0, 0);
      }
    };
    if constexpr (EPI == EPI_MASK) {   // (while the MMAs run)
#pragma unroll
      for (int gi = 0; gi < 8; ++gi) wg[gi] = 0.f;
      if (row < M) {
        int cg[8];   // component of each group
#pragma unroll
        for (int gi = 0; gi < 8; ++gi) cg[gi] = (n0 + 64 * hf + 8 * gi) / ma.r;
#pragma unroll 1
        for (int k = 0; k < ma.K; ++k) {
          const int c = (int)ma.idx[(size_t)row * ma.K + k];
          const float wk = to_f32(ma.w[(size_t)row * ma.K + k]);
#pragma unroll
          for (int gi = 0; gi < 8; ++gi)
            if (c == cg[gi]) wg[gi] += wk;
        }
      }
      load_sigma(0);
    }
    // one thread waits for the accumulator; the others sleep at the named barrier
    __shared__ int acc_ok;
    if (tid == 64) acc_ok = tc::mbar_wait(accf, 0, GPOLLS) && !*fail;
    tc::named_sync(1, G_THREADS - 64);
    const bool got = acc_ok != 0;
    if (!got) {
      atomicExch(&g_mcmoe_status, 1);
    } else {
      tc::fence_after_sync();
      const uint32_t lb = (uint32_t)(32 * q) << 16;
#pragma unroll 1
      for (int u = 0; u < 4; ++u) {
        const int cl = 64 * hf + 16 * u;   // tile column of the chunk
        float v[16];
        tc::tmem_ld16(tacc + lb + cl, v);
        if constexpr (EPI == EPI_MASK) {
          float sg[16];
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&sgn[h]);
#pragma unroll
            for (int j = 0; j < 8; ++j) sg[8 * h + j] = __bfloat162float(e[j]);
          }
          if (u + 1 < 4) load_sigma(u + 1);
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float sv = sg[j];
            if (ma.sigma_is_logits) sv = rnd<__nv_bfloat16>(sigmoid_fast(sv));
            v[j] = v[j] * sv * wg[2 * u + (j >> 3)];
          }
        }
        // bf16 into the staged tile: two 64-column boxes, 128-byte rows, 128-byte swizzle
        const int box = cl >> 6, cb = cl & 63;
        unsigned char* base = gsm + box * (GBM * 128) + rl * 128;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint4 pk;
          __nv_bfloat16* pe = reinterpret_cast<__nv_bfloat16*>(&pk);
#pragma unroll
          for (int j = 0; j < 8; ++j) pe[j] = __float2bfloat16_rn(v[8 * h + j]);
          const int chunk = (cb >> 3) + h;
          *reinterpret_cast<uint4*>(base + ((chunk ^ (rl & 7)) << 4)) = pk;
        }
      }
      tc::fence_proxy_async();
    }
    tc::named_sync(1, G_THREADS - 64);
    if (got && tid == 64) {
      tc::tma_store_2d(&tmC, n0, m0, gsm);
      tc::tma_store_2d(&tmC, n0 + 64, m0, gsm + GBM * 128);
      tc::bulk_commit();
      tc::bulk_wait<0>();
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) tc::tmem_dealloc(tacc, GBN);
}

// ------------------------------------------------------------------------- direct path
// One CTA per token, the reference kernel's formula in fp32:
//   acc[f] = sum_k w_k sum_j (x . V[c_k, j, :]) sigma[t, c_k, j] U[c_k, f, j]
template <typename T>
__global__ void __launch_bounds__(256)
mcmoe_direct_kernel(const T* __restrict__ x, const T* __restrict__ U, const T* __restrict__ Vb,
                    const long long* __restrict__ idx, const T* __restrict__ w, const T* __restrict__ sigma,
                    int sigma_is_logits, T* __restrict__ out, int d, int C, int r, int K) {
  extern __shared__ float dsm[];
  float* xs = dsm;                 // [d]
  float* ys = dsm + d;             // [K][r]: (x . V) * sigma
  const int tid = threadIdx.x, lane = tid & 31, wp = tid >> 5;
  const size_t t = blockIdx.x;
  for (int f = tid; f < d; f += 256) xs[f] = to_f32(x[t * d + f]);
  __syncthreads();
  for (int kj = wp; kj < K * r; kj += 8) {
    const int k = kj / r, j = kj % r;
    const long long c = idx[t * K + k];
    float dp = 0.f;
    if (c >= 0 && c < C) {
      const T* vr = Vb + ((size_t)c * r + j) * d;
      for (int f = lane; f < d; f += 32) dp += xs[f] * to_f32(vr[f]);
    }
    dp = warp_sum(dp);
    if (lane == 0) {
      float s = (c >= 0 && c < C) ? to_f32(sigma[(t * C + c) * r + j]) : 0.f;
      if (sigma_is_logits) s = rnd<T>(sigmoid_f(s));
      ys[kj] = dp * s;
    }
  }
  __syncthreads();
  for (int f = tid; f < d; f += 256) {
    float acc = 0.f;
    for (int k = 0; k < K; ++k) {
      const long long c = idx[t * K + k];
      if (c < 0 || c >= C) continue;
      const T* ur = U + ((size_t)c * d + f) * r;
      float up = 0.f;
      for (int j = 0; j < r; ++j) up += ys[k * r + j] * to_f32(ur[j]);
      acc += to_f32(w[t * K + k]) * up;
    }
    out[t * d + f] = from_f32<T>(acc);
  }
}

// ------------------------------------------------------------------------- SiTU-GLU
// out = [b1 tanh(g / b1) sigmoid(g)] * [b2 tanh(u / b2)], rounded to T after each
// elementwise op as the reference's sequence of torch ops is.
template <typename T>
__global__ void __launch_bounds__(256) situ_glu_kernel(const T* __restrict__ g, const T* __restrict__ u, long long ld,
                                                       T* __restrict__ out, long long n, int cols, float b1,
                                                       float b2) {
  const long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= n * cols) return;
  const long long r = e / cols;
  const int c = (int)(e - r * cols);
  const float gv = to_f32(g[r * ld + c]), uv = to_f32(u[r * ld + c]);
  const float gc = rnd<T>(b1 * rnd<T>(tanhf(rnd<T>(gv / b1))));
  const float ga = rnd<T>(gc * rnd<T>(sigmoid_f(gv)));
  const float uc = rnd<T>(b2 * rnd<T>(tanhf(rnd<T>(uv / b2))));
  out[e] = from_f32<T>(ga * uc);
}

// ------------------------------------------------------------------------- host side
int make_map_2d(CUtensorMap* m, const void* base, long long rows, int cols, int box_cols, int box_rows) {
  auto enc = tmap_encoder();
  VERACE_REQUIRE(enc != nullptr, VERACE_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  const cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
  const cuuint32_t es[2] = {1, 1};
  CUresult rc = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  VERACE_REQUIRE(rc == CUDA_SUCCESS, VERACE_ERR_CUDA, "cuTensorMapEncodeTiled (M-CMoE operand) failed: %d", (int)rc);
  return VERACE_OK;
}

template <int EPI>
int launch_gemm(const void* A, const void* B, void* Cout, long long M, int N, int K, const MaskArgs& ma,
                cudaStream_t st) {
  CUtensorMap ta, tb, tcm;
  int rc;
  if ((rc = make_map_2d(&ta, A, M, K, GBK, GBM)) || (rc = make_map_2d(&tb, B, N, K, GBK, GBN)) ||
      (rc = make_map_2d(&tcm, Cout, M, N, 64, GBM)))
    return rc;
  VERACE_CUDA(cudaFuncSetAttribute(mcmoe_gemm_kernel<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize, G_SMEM));
  const dim3 grid((unsigned)(N / GBN), (unsigned)((M + GBM - 1) / GBM));
  mcmoe_gemm_kernel<EPI><<<grid, G_THREADS, G_SMEM, st>>>(ta, tb, tcm, (int)M, N, K, ma);
  return check_launch("mcmoe_gemm_kernel");
}

struct McWs {
  size_t ut, yhat, total;
};
McWs mc_ws(long long n, int d, int C, int r) {
  McWs L{};
  size_t off = 0;
  L.ut = off;   off = align_up(off + (size_t)d * C * r * 2, 1024);
  L.yhat = off; off = align_up(off + (size_t)n * C * r * 2, 1024);
  L.total = off + 1024;
  return L;
}

bool tc_path(int dtype, int d, int C, int r, int K) {
  return dtype == VERACE_BF16 && d % GBN == 0 && d % GBK == 0 && ((long long)C * r) % GBN == 0 &&
         ((long long)C * r) % GBK == 0 && r % 8 == 0 && K <= MAX_TOPK;
}

}  // namespace

int mcmoe_read_status(int* status) {
  int h = 0;
  VERACE_CUDA(cudaMemcpyFromSymbol(&h, g_mcmoe_status, sizeof(int)));
  if (h) {
    const int zero = 0;
    VERACE_CUDA(cudaMemcpyToSymbol(g_mcmoe_status, &zero, sizeof(int)));
  }
  *status = h;
  return VERACE_OK;
}

}  // namespace verace

using namespace verace;

extern "C" size_t verace_mcmoe_workspace(long long n, int d, int C, int r, int dtype) {
  if (n <= 0 || d <= 0 || C <= 0 || r <= 0 || !tc_path(dtype, d, C, r, 1)) return 256;
  return mc_ws(n, d, C, r).total;
}

extern "C" int verace_mcmoe_route(const void* logits, long long n, int C, int K, long long* idx, void* weights,
                                  int dtype, void* stream) {
  VERACE_REQUIRE(n >= 0 && C >= 1 && K >= 1, VERACE_ERR_INVALID, "verace_mcmoe_route: invalid sizes n=%lld C=%d K=%d",
                 n, C, K);
  VERACE_REQUIRE(dtype == VERACE_F32 || dtype == VERACE_BF16 || dtype == VERACE_F16, VERACE_ERR_INVALID,
                 "verace_mcmoe_route: unknown dtype %d", dtype);
  VERACE_REQUIRE(C <= MAX_C && K <= C && K <= MAX_TOPK, VERACE_ERR_UNSUPPORTED,
                 "verace_mcmoe_route: C=%d K=%d unsupported (C <= %d, K <= min(C, %d))", C, K, MAX_C, MAX_TOPK);
  if (n == 0) return VERACE_OK;
  VERACE_REQUIRE(logits && idx && weights, VERACE_ERR_INVALID, "verace_mcmoe_route: NULL pointer");
  cudaStream_t st = (cudaStream_t)stream;
  const unsigned grid = (unsigned)((n + 7) / 8);
  switch (dtype) {
    case VERACE_F32:
      mcmoe_route_kernel<float><<<grid, 256, 0, st>>>((const float*)logits, n, C, K, idx, (float*)weights);
      break;
    case VERACE_BF16:
      mcmoe_route_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((const __nv_bfloat16*)logits, n, C, K, idx,
                                                              (__nv_bfloat16*)weights);
      break;
    default:
      mcmoe_route_kernel<__half><<<grid, 256, 0, st>>>((const __half*)logits, n, C, K, idx, (__half*)weights);
      break;
  }
  return check_launch("mcmoe_route_kernel");
}

extern "C" int verace_mcmoe_projection(const void* x, const void* u_basis, const void* v_basis, const long long* idx,
                                       const void* weights, const void* sigma, int sigma_is_logits, void* out,
                                       long long n, int d, int C, int r, int K, int dtype, void* workspace,
                                       size_t workspace_bytes, void* stream) {
  VERACE_REQUIRE(n >= 0 && d >= 1 && C >= 1 && r >= 1 && K >= 1, VERACE_ERR_INVALID,
                 "verace_mcmoe_projection: invalid sizes n=%lld d=%d C=%d r=%d K=%d", n, d, C, r, K);
  VERACE_REQUIRE(dtype == VERACE_F32 || dtype == VERACE_BF16 || dtype == VERACE_F16, VERACE_ERR_INVALID,
                 "verace_mcmoe_projection: unknown dtype %d", dtype);
  if (n == 0) return VERACE_OK;
  VERACE_REQUIRE(x && u_basis && v_basis && idx && weights && sigma && out, VERACE_ERR_INVALID,
                 "verace_mcmoe_projection: NULL pointer");
  cudaStream_t st = (cudaStream_t)stream;
  if (tc_path(dtype, d, C, r, K)) {
    const McWs L = mc_ws(n, d, C, r);
    VERACE_REQUIRE(workspace != nullptr && workspace_bytes >= L.total, VERACE_ERR_WORKSPACE,
                   "verace_mcmoe_projection: workspace of %zu bytes required, %zu given", L.total,
                   workspace ? workspace_bytes : (size_t)0);
    VERACE_REQUIRE((((uintptr_t)x | (uintptr_t)v_basis | (uintptr_t)out | (uintptr_t)sigma) & 15) == 0,
                   VERACE_ERR_INVALID, "verace_mcmoe_projection: x, v_basis, sigma and out must be 16-byte aligned");
    char* base = (char*)align_up((size_t)workspace, 1024);
    __nv_bfloat16* Ut = (__nv_bfloat16*)(base + L.ut);
    __nv_bfloat16* Yh = (__nv_bfloat16*)(base + L.yhat);
    const long long ncr = (long long)C * r;
    const long long nu = (long long)d * ncr;
    mcmoe_u_relayout_kernel<<<(unsigned)((nu + 255) / 256), 256, 0, st>>>((const __nv_bfloat16*)u_basis, Ut, d, C, r);
    int rc = check_launch("mcmoe_u_relayout_kernel");
    if (rc) return rc;
    MaskArgs ma{(const __nv_bfloat16*)sigma, idx, (const __nv_bfloat16*)weights, r, K, sigma_is_logits};
    // Yhat = (x V^T) * sigma * wsel, then out = Yhat Ut^T
    if ((rc = launch_gemm<EPI_MASK>(x, v_basis, Yh, n, (int)ncr, d, ma, st))) return rc;
    MaskArgs none{nullptr, nullptr, nullptr, 1, 0, 0};
    return launch_gemm<EPI_STORE>(Yh, Ut, out, n, d, (int)ncr, none, st);
  }
  VERACE_REQUIRE(K <= MAX_TOPK * 64 && (size_t)(d + K * r) * 4 <= 200 * 1024, VERACE_ERR_UNSUPPORTED,
                 "verace_mcmoe_projection: d=%d, K*r=%d too large for the direct path", d, K * r);
  const size_t smem = (size_t)(d + K * r) * 4;
  switch (dtype) {
    case VERACE_F32:
      VERACE_CUDA(cudaFuncSetAttribute(mcmoe_direct_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem));
      mcmoe_direct_kernel<float><<<(unsigned)n, 256, smem, st>>>(
          (const float*)x, (const float*)u_basis, (const float*)v_basis, idx, (const float*)weights,
          (const float*)sigma, sigma_is_logits, (float*)out, d, C, r, K);
      break;
    case VERACE_BF16:
      VERACE_CUDA(cudaFuncSetAttribute(mcmoe_direct_kernel<__nv_bfloat16>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      mcmoe_direct_kernel<__nv_bfloat16><<<(unsigned)n, 256, smem, st>>>(
          (const __nv_bfloat16*)x, (const __nv_bfloat16*)u_basis, (const __nv_bfloat16*)v_basis, idx,
          (const __nv_bfloat16*)weights, (const __nv_bfloat16*)sigma, sigma_is_logits, (__nv_bfloat16*)out, d, C, r,
          K);
      break;
    default:
      VERACE_CUDA(cudaFuncSetAttribute(mcmoe_direct_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem));
      mcmoe_direct_kernel<__half><<<(unsigned)n, 256, smem, st>>>(
          (const __half*)x, (const __half*)u_basis, (const __half*)v_basis, idx, (const __half*)weights,
          (const __half*)sigma, sigma_is_logits, (__half*)out, d, C, r, K);
      break;
  }
  return check_launch("mcmoe_direct_kernel");
}

extern "C" int verace_situ_glu(const void* gate, const void* up, long long ld, void* out, long long n, int cols,
                               float beta1, float beta2, int dtype, void* stream) {
  VERACE_REQUIRE(n >= 0 && cols >= 1 && ld >= cols, VERACE_ERR_INVALID,
                 "verace_situ_glu: invalid sizes n=%lld cols=%d ld=%lld", n, cols, ld);
  VERACE_REQUIRE(dtype == VERACE_F32 || dtype == VERACE_BF16 || dtype == VERACE_F16, VERACE_ERR_INVALID,
                 "verace_situ_glu: unknown dtype %d", dtype);
  if (n == 0) return VERACE_OK;
  VERACE_REQUIRE(gate && up && out, VERACE_ERR_INVALID, "verace_situ_glu: NULL pointer");
  cudaStream_t st = (cudaStream_t)stream;
  const long long tot = n * cols;
  const unsigned grid = (unsigned)((tot + 255) / 256);
  switch (dtype) {
    case VERACE_F32:
      situ_glu_kernel<float><<<grid, 256, 0, st>>>((const float*)gate, (const float*)up, ld, (float*)out, n, cols,
                                                   beta1, beta2);
      break;
    case VERACE_BF16:
      situ_glu_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>((const __nv_bfloat16*)gate, (const __nv_bfloat16*)up, ld,
                                                           (__nv_bfloat16*)out, n, cols, beta1, beta2);
      break;
    default:
      situ_glu_kernel<__half><<<grid, 256, 0, st>>>((const __half*)gate, (const __half*)up, ld, (__half*)out, n,
                                                    cols, beta1, beta2);
      break;
  }
  return check_launch("situ_glu_kernel");
}
