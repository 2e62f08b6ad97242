// Planar-complex fp32 GEMM on the tcgen05 tensor cores (sm_100a), the contract of
// cgemm.cuh: C = alpha * opA(A) opB(B) + beta * X.  Used by the dense Newton-Schulz
// retraction (cham_memory.py:21-51) and by the readout polynomial of the CHAM scan from a
// hologram far from unitary (cham_memory.py:229-239), both D^3 contractions.
//
// fp32 operands enter the bf16 tensor cores as three bf16 parts, x = h + m + l (h =
// bf16(x), m = bf16(x - h), l = bf16(x - h - m): 24 significant bits), and each real
// product takes the six terms down to the 2^-24 level, hh + hm + mh + hl + lh + mm:
// fp32 accuracy (two parts, three terms, leave ~1e-5 relative, short of the 1e-5 the
// retraction's tests hold it to).  A complex product is folded into ONE real GEMM over a
// twelve-fold K (each segment Kp long), the hh terms first:
//   A' row m      = [ar h, -ai h | ar: h m h l m, -ai: h m h l m]
//   B' row n      = [br h,  bi h | br: m h l h m,  bi: m h l h m]   -> Re C = ar br - ai bi
//   B' row Np + n = [bi h, -br h | bi: m h l h m, -br: m h l h m]   -> Im C = ar bi + ai br
// so C' = A' B'^T (M x 2N) holds Re C in its first Np columns and Im C in the rest.  The
// hh segments and the small terms accumulate into two separate tensor-memory
// accumulators, summed in fp32 by the epilogue, so that the small terms are not added
// one k-step at a time into an accumulator of the full result's magnitude.  Two pack
// kernels build A' and B' (K-major, bf16) in caller scratch; the GEMM streams 128 x 64
// K-major tiles of both by TMA (128-byte swizzle) through three stages into one 128 x 128
// fp32 accumulator in tensor memory (one elected thread issues the MMAs), and the
// epilogue applies alpha, beta and X and writes the planar result.
#include "cgemm.cuh"

#include <algorithm>

#include "tc.cuh"
#include "tmap.cuh"

namespace verace {
namespace {

constexpr int TBM = 128, TBN = 128, TBK = 64, TST = 3;
constexpr int T_STAGE = (TBM + TBN) * TBK * 2;   // 32 KB
constexpr int T_BAR = TST * T_STAGE;             // 96 KB
constexpr int T_SMEM = T_BAR + 128;
constexpr int T_THREADS = 192;                   // warp 0 TMA, warp 1 MMA (+ TMEM), warps 2-5 epilogue
constexpr uint32_t CPOLLS = 1u << 22;

__device__ int g_cgemm_status = 0;

int round_up(int x, int m) { return (x + m - 1) / m * m; }

constexpr int SEG = 12;   // K segments of the packed operands

// 8 fp32 values -> three bf16 parts each, packed as three 16-byte chunks
__device__ __forceinline__ void split3_8(const float* x, uint4& h, uint4& m, uint4& l) {
  __nv_bfloat16* ph = reinterpret_cast<__nv_bfloat16*>(&h);
  __nv_bfloat16* pm = reinterpret_cast<__nv_bfloat16*>(&m);
  __nv_bfloat16* pl = reinterpret_cast<__nv_bfloat16*>(&l);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const __nv_bfloat16 a = __float2bfloat16_rn(x[j]);
    const float r = x[j] - __bfloat162float(a);
    const __nv_bfloat16 b = __float2bfloat16_rn(r);
    ph[j] = a;
    pm[j] = b;
    pl[j] = __float2bfloat16_rn(r - __bfloat162float(b));
  }
}

// A'[z][m][seg * Kp + k] (m < Mp, k < Kp; zero outside M x K).  Thread: one m, 8 k.
__global__ void cgemm_pack_a(const float* __restrict__ Ar, const float* __restrict__ Ai, int lda, long long sA,
                             int trans, int conj, int M, int K, int Mp, int Kp, int z0,
                             __nv_bfloat16* __restrict__ out) {
  const long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int z = blockIdx.y;
  if (e >= (long long)Mp * (Kp / 8)) return;
  const int m = (int)(e % Mp), k0 = (int)(e / Mp) * 8;
  const float* ar = Ar + (z0 + z) * sA;
  const float* ai = Ai ? Ai + (z0 + z) * sA : nullptr;
  float re[8], im[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int k = k0 + j;
    float a = 0.f, b = 0.f;
    if (m < M && k < K) {
      const size_t off = trans ? (size_t)k * lda + m : (size_t)m * lda + k;
      a = ar[off];
      b = ai ? ai[off] : 0.f;
    }
    re[j] = a;
    im[j] = conj ? b : -b;   // the A' row holds -Im(opA)
  }
  uint4 p[2][3];   // [re, -im][h, m, l]
  split3_8(re, p[0][0], p[0][1], p[0][2]);
  split3_8(im, p[1][0], p[1][1], p[1][2]);
  unsigned char* row = reinterpret_cast<unsigned char*>(out + ((size_t)z * Mp + m) * (SEG * (size_t)Kp));
  const size_t seg = (size_t)Kp * 2;   // bytes per segment
  const size_t kb = (size_t)k0 * 2;
  // segment t: part APC[t] (0 re, 1 -im), piece APP[t] (0 h, 1 m, 2 l)
  constexpr int APC[SEG] = {0, 1, 0, 0, 0, 0, 0, 1, 1, 1, 1, 1};
  constexpr int APP[SEG] = {0, 0, 0, 1, 0, 2, 1, 0, 1, 0, 2, 1};
#pragma unroll
  for (int t = 0; t < SEG; ++t) *reinterpret_cast<uint4*>(row + t * seg + kb) = p[APC[t]][APP[t]];
}

// B'[z][n][.] (real output column n) and B'[z][Np + n][.] (imaginary output column n).
__global__ void cgemm_pack_b(const float* __restrict__ Br, const float* __restrict__ Bi, int ldb, long long sB,
                             int trans, int conj, int N, int K, int Np, int Kp, int z0,
                             __nv_bfloat16* __restrict__ out) {
  const long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const int z = blockIdx.y;
  if (e >= (long long)Np * (Kp / 8)) return;
  const int n = (int)(e % Np), k0 = (int)(e / Np) * 8;
  const float* br = Br + (z0 + z) * sB;
  const float* bi = Bi ? Bi + (z0 + z) * sB : nullptr;
  float re[8], im[8], nre[8];   // Re(opB), Im(opB), -Re(opB)
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int k = k0 + j;
    float a = 0.f, b = 0.f;
    if (n < N && k < K) {
      const size_t off = trans ? (size_t)n * ldb + k : (size_t)k * ldb + n;
      a = br[off];
      b = bi ? bi[off] : 0.f;
    }
    re[j] = a;
    im[j] = conj ? -b : b;
    nre[j] = -a;
  }
  uint4 p[3][3];   // [re, im, -re][h, m, l]
  split3_8(re, p[0][0], p[0][1], p[0][2]);
  split3_8(im, p[1][0], p[1][1], p[1][2]);
  split3_8(nre, p[2][0], p[2][1], p[2][2]);
  const size_t seg = (size_t)Kp * 2, kb = (size_t)k0 * 2, rowb = SEG * (size_t)Kp;
  unsigned char* rr = reinterpret_cast<unsigned char*>(out + ((size_t)z * 2 * Np + n) * rowb);
  unsigned char* ri = reinterpret_cast<unsigned char*>(out + ((size_t)z * 2 * Np + Np + n) * rowb);
  // segment t: Re column part BRC[t] (0 re, 1 im), Im column part BIC[t] (1 im, 2 -re),
  // piece BPP[t] (0 h, 1 m, 2 l)
  constexpr int BRC[SEG] = {0, 1, 0, 0, 0, 0, 0, 1, 1, 1, 1, 1};
  constexpr int BIC[SEG] = {1, 2, 1, 1, 1, 1, 1, 2, 2, 2, 2, 2};
  constexpr int BPP[SEG] = {0, 0, 1, 0, 2, 0, 1, 1, 0, 2, 0, 1};
#pragma unroll
  for (int t = 0; t < SEG; ++t) {
    *reinterpret_cast<uint4*>(rr + t * seg + kb) = p[BRC[t]][BPP[t]];
    *reinterpret_cast<uint4*>(ri + t * seg + kb) = p[BIC[t]][BPP[t]];
  }
}

struct EpiArgs {
  int M, N, Mp, Np;
  float alpha, beta;
  const float* Xr; const float* Xi; int ldx; long long sX;
  float* Cr; float* Ci; int ldc; long long sC;
  int z0;
};

__global__ void __launch_bounds__(T_THREADS, 2)
cgemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int nk,
                EpiArgs E) {
  extern __shared__ __align__(1024) unsigned char gsm[];
  uint64_t* full = reinterpret_cast<uint64_t*>(gsm + T_BAR);
  uint64_t* empty = full + TST;
  uint64_t* accf = empty + TST;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(accf + 1);
  volatile int* fail = reinterpret_cast<volatile int*>(tslot + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int z = blockIdx.z;
  const int m0 = blockIdx.y * TBM, n0 = blockIdx.x * TBN;   // n0 in [0, 2 Np)
  if (warp == 1) tc::tmem_alloc(tslot, 2 * TBN);   // [0, 128) hh terms, [128, 256) the small terms
  if (tid == 0) {
    for (int s = 0; s < TST; ++s) {
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
  auto sA = [&](int s) { return gsm + s * T_STAGE; };
  auto sB = [&](int s) { return gsm + s * T_STAGE + TBM * TBK * 2; };

  if (warp == 0) {
    if (lane == 0) {   // ---- TMA producer
      int kb = 0;
      for (; kb < nk; ++kb) {
        const int s = kb % TST;
        if (kb >= TST && (*fail || !tc::mbar_wait(&empty[s], ((kb / TST) - 1) & 1, CPOLLS))) {
          *fail = 1;
          atomicExch(&g_cgemm_status, 1);
          break;
        }
        tc::mbar_expect_tx(&full[s], T_STAGE);
        tc::tma_load_2d(sA(s), &tmA, kb * TBK, z * E.Mp + m0, &full[s]);
        tc::tma_load_2d(sB(s), &tmB, kb * TBK, z * 2 * E.Np + n0, &full[s]);
      }
      // copies still in flight land before the CTA may exit
      for (int j = kb - TST < 0 ? 0 : kb - TST; j < kb; ++j) tc::mbar_wait(&full[j % TST], (j / TST) & 1, CPOLLS);
    }
  } else if (warp == 1) {
    if (lane == 0) {   // ---- MMA issuer
      constexpr uint32_t ID = tc::idesc_bf16(TBM, TBN, false, false);
      const int ksplit = nk / 6;   // k-blocks of the two hh segments (nk = 12 Kp / TBK)
      bool ok = true;
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % TST;
        if (*fail || !tc::mbar_wait(&full[s], (kb / TST) & 1, CPOLLS)) {
          ok = false;
          *fail = 1;
          atomicExch(&g_cgemm_status, 1);
          break;
        }
        tc::fence_after_sync();
        const uint32_t a = tc::smem_addr(sA(s)), b = tc::smem_addr(sB(s));
        const uint32_t acc = kb < ksplit ? tacc : tacc + TBN;
        const bool first = kb == 0 || kb == ksplit;
#pragma unroll
        for (int ks = 0; ks < TBK / 16; ++ks)
          tc::mma_bf16(acc, tc::sdesc_sw128(a + ks * 32, 16, 1024), tc::sdesc_sw128(b + ks * 32, 16, 1024), ID,
                       (!first || ks > 0) ? 1u : 0u);
        tc::commit(&empty[s]);   // the stage is free once these MMAs have read it
      }
      tc::commit(accf);          // (also after a failure: every issued MMA completes)
      if (!ok) tc::mbar_wait(accf, 0, CPOLLS);
    }
  } else {
    // ---- epilogue: warps 2-5, TMEM lane quarter warp % 4; thread = one output row, 128 columns
    __shared__ int acc_ok;
    if (tid == 64) acc_ok = tc::mbar_wait(accf, 0, CPOLLS) && !*fail;
    tc::named_sync(1, T_THREADS - 64);
    if (acc_ok == 0) {
      if (tid == 64) atomicExch(&g_cgemm_status, 1);
    } else {
      tc::fence_after_sync();
      const int q = warp & 3, rl = 32 * q + lane, m = m0 + rl;
      const uint32_t lb = (uint32_t)(32 * q) << 16;
      const bool imag = n0 >= E.Np;
      const int c0 = imag ? n0 - E.Np : n0;   // output column of the tile's first column
      float* C = (imag ? E.Ci : E.Cr) + (E.z0 + z) * E.sC + (size_t)m * E.ldc;
      const float* X = E.beta != 0.f && E.Xr != nullptr
                           ? (imag ? E.Xi : E.Xr) + (E.z0 + z) * E.sX + (size_t)m * E.ldx : nullptr;
      const bool xzero = imag && E.Xi == nullptr;   // a real X has no imaginary part
#pragma unroll 1
      for (int u = 0; u < TBN / 16; ++u) {
        float v[16], w[16];
        tc::tmem_ld16(tacc + lb + 16 * u, v);
        tc::tmem_ld16(tacc + lb + TBN + 16 * u, w);
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] += w[j];
        if (m < E.M) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int c = c0 + 16 * u + j;
            if (c < E.N) {
              float r = E.alpha * v[j];
              if (X != nullptr && !xzero) r += E.beta * X[c];
              C[c] = r;
            }
          }
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) tc::tmem_dealloc(tacc, 2 * TBN);
}

int make_op_map(CUtensorMap* m, const void* base, long long rows, long long cols) {
  auto enc = tmap_encoder();
  VERACE_REQUIRE(enc != nullptr, VERACE_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  const cuuint32_t box[2] = {(cuuint32_t)TBK, (cuuint32_t)TBM};
  const cuuint32_t es[2] = {1, 1};
  CUresult rc = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  VERACE_REQUIRE(rc == CUDA_SUCCESS, VERACE_ERR_CUDA, "cuTensorMapEncodeTiled (complex GEMM operand) failed: %d",
                 (int)rc);
  return VERACE_OK;
}

size_t per_item_bytes(int M, int N, int K) {
  const size_t Mp = round_up(M, TBM), Np = round_up(N, TBN), Kp = round_up(K, TBK);
  return (Mp + 2 * Np) * SEG * Kp * 2;
}

}  // namespace

size_t cgemm_tc_scratch(int M, int N, int K, int batch) {
  if (M <= 0 || N <= 0 || K <= 0 || batch <= 0) return 0;
  return per_item_bytes(M, N, K) * (size_t)(batch < 4 ? batch : 4) + 1024;
}

int cgemm_tc(int M, int N, int K, int batch, float alpha, CMat A, bool transA, bool conjA, CMat B, bool transB,
             bool conjB, float beta, CMat X, float* Cr, float* Ci, int ldc, long long sC, void* scratch,
             size_t scratch_bytes, cudaStream_t st) {
  if (M <= 0 || N <= 0 || batch <= 0) return VERACE_OK;
  const int Mp = round_up(M, TBM), Np = round_up(N, TBN), Kp = round_up(K, TBK);
  const size_t per = per_item_bytes(M, N, K);
  char* base = (char*)(((uintptr_t)scratch + 1023) & ~(uintptr_t)1023);
  const size_t usable = scratch_bytes > (size_t)(base - (char*)scratch) ? scratch_bytes - (base - (char*)scratch) : 0;
  const int group = (int)std::min<size_t>((size_t)batch, usable / per);
  VERACE_REQUIRE(group >= 1, VERACE_ERR_WORKSPACE, "complex GEMM: %zu bytes of scratch needed, %zu given", per,
                 usable);
  VERACE_CUDA(cudaFuncSetAttribute(cgemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, T_SMEM));
  for (int z0 = 0; z0 < batch; z0 += group) {
    const int g = std::min(group, batch - z0);
    __nv_bfloat16* Ap = (__nv_bfloat16*)base;
    __nv_bfloat16* Bp = Ap + (size_t)g * Mp * SEG * Kp;
    const long long na = (long long)Mp * (Kp / 8), nb = (long long)Np * (Kp / 8);
    cgemm_pack_a<<<dim3((unsigned)((na + 255) / 256), g), 256, 0, st>>>(A.re, A.im, A.ld, A.stride, transA, conjA, M,
                                                                       K, Mp, Kp, z0, Ap);
    int rc = check_launch("cgemm_pack_a");
    if (rc) return rc;
    cgemm_pack_b<<<dim3((unsigned)((nb + 255) / 256), g), 256, 0, st>>>(B.re, B.im, B.ld, B.stride, transB, conjB, N,
                                                                       K, Np, Kp, z0, Bp);
    if ((rc = check_launch("cgemm_pack_b"))) return rc;
    CUtensorMap ta, tb;
    if ((rc = make_op_map(&ta, Ap, (long long)g * Mp, (long long)SEG * Kp)) ||
        (rc = make_op_map(&tb, Bp, (long long)g * 2 * Np, (long long)SEG * Kp)))
      return rc;
    EpiArgs E{M, N, Mp, Np, alpha, beta, X.re, X.im, X.ld, X.stride, Cr, Ci, ldc, sC, z0};
    cgemm_tc_kernel<<<dim3(2 * Np / TBN, Mp / TBM, g), T_THREADS, T_SMEM, st>>>(ta, tb, SEG * Kp / TBK, E);
    if ((rc = check_launch("cgemm_tc_kernel"))) return rc;
  }
  return VERACE_OK;
}

int cgemm_tc_read_status(int* status) {
  int h = 0;
  VERACE_CUDA(cudaMemcpyFromSymbol(&h, g_cgemm_status, sizeof(int)));
  if (h) {
    const int zero = 0;
    VERACE_CUDA(cudaMemcpyToSymbol(g_cgemm_status, &zero, sizeof(int)));
  }
  *status = h;
  return VERACE_OK;
}

}  // namespace verace
