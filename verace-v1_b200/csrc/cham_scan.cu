// CHAM holographic-memory scan (fp32 complex state, chunked compact-WY form) and the
// dense Newton-Schulz retraction.
//
// Reference semantics (verace_v1/modules/cham_memory.py:177-243): per token
//     U_t = (I - iG_t/2)^-1 (I + iG_t/2),  G_t = g_t (k vᵀ + v kᵀ)
//     H_t = U_t H_{t-1}     (raw, exported, never retracted)
//     rec_t = Re(NS3(H_t)) q_t,   NS(H) = H (3I - HᴴH)/2
// With U_t = [k_t, v_t]:  U_t = I + U_t N_t U_tᵀ,  c = g/2,
//     N_t = (2c/det) [[-c vv, i + c kv], [i + c kv, -c kk]],
//     det = 1 + c² (kk vv - kv²) - 2i c kv
// (exact; N_t -> 0 continuously as g -> 0).  A chunk of C tokens composes to
// I + W T Wᵀ with real W = [U_1 .. U_C] (D x 2C) and complex block lower-triangular
// T = (I - Nblk L)^-1 Nblk, L the strictly block-lower part of the real Gram WᵀW.
//
// Readout.  Every U_t is unitary, so for H_t = P_t H_0 (P_t a product of U's):
//     Hᴴ_t H_t = H_0ᴴ H_0 =: A   and   NS3(H_t) = H_t p(A),
//     p(A) = g(A) g(A1) g(A2),  g(X) = (3I - X)/2,  A1 = A g(A)², A2 = A1 g(A1)²
// (NS3(H) = H g(A) g(A1) g(A2) because each NS step right-multiplies by a polynomial
// of HᴴH).  Hence rec_t = Re(H_t y_t) with y_t = p(A) q_t, which is computed once per
// call from H_0 with 13 applications of A (26 complex matrix products on the D x s
// block of query vectors).  For H_0 = I, p(I) = I and y_t = q_t exactly.
//
// Per chunk (state S = H at the chunk start, Y = [y_t] of the chunk):
//     Z = Wᵀ S,  Cm = T Z,  S_next = S + W Cm
//     rec_t = Re(S y_t) + sum_{tau<=t} U_tau Re(Cm_tau y_t)
// Kernels: cham_prep (T for all chunks in parallel), then per chunk
//   cham_colpass  -- one CTA per (item, block of NB columns): Z, Cm, the chunk's
//                    Re(Cm Y) partial (atomically reduced over column blocks) and the
//                    column block of S_next;
//   cham_readout  -- one CTA per (item, block of RB rows): Re(S Y) + W mask(Re(Cm Y)).
#include "common.cuh"
#include "cgemm.cuh"

#include <stdlib.h>

namespace verace {

// tcgen05 path (cham_tc.cu)
bool cham_tc_supported(int D, int dtype, bool has_h0);
bool cham_tc_supported_unitary(int D, int dtype);
size_t cham_tc_workspace(int b, int s, int D);
int cham_tc_scan(const void* q, const void* k, const void* v, const float* gamma, const float* h0r,
                 const float* h0i, void* out, float* hr, float* hi, int b, int s, int D, int dtype, void* workspace,
                 cudaStream_t st);
int tc_read_status(cudaStream_t st, int* status);
int sssd_tc_read_status(int* status);
int decode_read_status(unsigned int* status);
int mcmoe_read_status(int* status);

namespace {

// VERACE_CHAM_SIMT=1 forces the fp32 SIMT kernels (used to compare the two paths).
bool force_simt() {
  const char* e = getenv("VERACE_CHAM_SIMT");
  return e && e[0] && e[0] != '0';
}

constexpr int CC = 32;       // tokens per chunk
constexpr int CR = 2 * CC;   // rank of a chunk transform
constexpr int NB = 32;       // columns per colpass CTA
constexpr int RT = 32;       // row tile of the colpass streams
constexpr int RB = 32;       // rows per readout CTA
constexpr int JT = 64;       // K tile of the readout
constexpr int DT = 64;       // row tile of the prep Gram matrix
constexpr int THREADS = 256;

struct ChamWs {
  float* T;                  // [b][nch][2][CR][CR]   (re plane, im plane)
  float* E;                  // [b][nch][CR][CC]      Re(Cm Y), reduced over column blocks
  unsigned long long* bad;   // [b][nch]
  float* Hre;                // [b][D][D]  ping-pong partner of the output state
  float* Him;
  float* Y;                  // [6][2][b][s][D]  readout polynomial vectors (has_h0 only)
  void* pack;                // the tensor-core complex GEMM's operand scratch (has_h0 only)
  size_t pack_bytes;
};

size_t ws_layout(int b, int s, int D, int has_h0, ChamWs* w, char* base) {
  const size_t nch = ((size_t)s + CC - 1) / CC;
  size_t off = 0;
  auto take = [&](size_t bytes) { size_t o = off; off += align_up(bytes, 256); return base ? (void*)(base + o) : nullptr; };
  ChamWs t;
  t.T = (float*)take((size_t)b * nch * 2 * CR * CR * sizeof(float));
  t.E = (float*)take((size_t)b * nch * CR * CC * sizeof(float));
  t.bad = (unsigned long long*)take((size_t)b * nch * sizeof(unsigned long long));
  const bool need_ping = nch >= 2;
  t.Hre = (float*)take(need_ping ? (size_t)b * D * D * sizeof(float) : 0);
  t.Him = (float*)take(need_ping ? (size_t)b * D * D * sizeof(float) : 0);
  t.Y = (float*)take(has_h0 ? (size_t)12 * b * s * D * sizeof(float) : 0);
  t.pack_bytes = has_h0 ? cgemm_tc_scratch(s, D, D, b) : 0;
  t.pack = take(t.pack_bytes);
  if (w) *w = t;
  return off + 256;
}

// ---------------------------------------------------------------------------------
// prep: G = WᵀW over D in row tiles, N_t, complex T by forward substitution, zero E.
// smem: Wt [DT][CR+1], Gs [CR][CR+1], Tr/Ti [CR][CR+1], Ns [CC][6]
template <typename T>
__global__ void __launch_bounds__(THREADS)
cham_prep_kernel(const T* __restrict__ k, const T* __restrict__ v, const float* __restrict__ gamma,
                 float* __restrict__ Tws, float* __restrict__ Ews, unsigned long long* __restrict__ badws,
                 int S, int D, int nch) {
  extern __shared__ float sm[];
  float* Wt = sm;
  float* Gs = Wt + DT * (CR + 1);
  float* Tr = Gs + CR * (CR + 1);
  float* Ti = Tr + CR * (CR + 1);
  float* Ns = Ti + CR * (CR + 1);
  __shared__ unsigned long long bad_bits;
  const int c = blockIdx.x, item = blockIdx.y, tid = threadIdx.x;
  const int t0 = c * CC, nt = min(CC, S - t0);
  if (tid == 0) bad_bits = 0ull;
  for (int e = tid; e < CR * (CR + 1); e += blockDim.x) Gs[e] = 0.f;
  for (int i0 = 0; i0 < D; i0 += DT) {
    __syncthreads();
    for (int e = tid; e < DT * CR; e += blockDim.x) {
      const int i = e / CR, r = e % CR, tau = r >> 1;
      float val = 0.f;
      if (tau < nt && i0 + i < D) {
        const size_t off = ((size_t)item * S + t0 + tau) * D + i0 + i;
        val = to_f32((r & 1) ? v[off] : k[off]);
      }
      Wt[i * (CR + 1) + r] = val;
      // a non-finite k or v element marks its token for identity substitution
      if (!isfinite(val)) atomicOr(&bad_bits, 1ull << tau);
    }
    __syncthreads();
    if (bad_bits) {  // zero flagged columns before they reach the Gram matrix
      for (int e = tid; e < DT * CR; e += blockDim.x)
        if ((bad_bits >> ((e % CR) >> 1)) & 1ull) Wt[(e / CR) * (CR + 1) + e % CR] = 0.f;
      __syncthreads();
    }
    smem_gemm<4, 4, true>(CR, CR, DT, Wt, 1, CR + 1, Wt, CR + 1, 1, Gs, CR + 1, 1, tid, blockDim.x);
  }
  __syncthreads();
  if (tid < CC && tid < nt && !isfinite(gamma[(size_t)item * S + t0 + tid])) atomicOr(&bad_bits, 1ull << tid);
  __syncthreads();
  if (tid < CC) {
    const int tau = tid;
    float n00r = 0.f, n00i = 0.f, n01r = 0.f, n01i = 0.f, n11r = 0.f, n11i = 0.f;
    const bool flagged = (bad_bits >> tau) & 1ull;
    if (tau < nt || flagged) {  // flagged tokens: clear their Gram rows/columns below
      for (int r = 0; r < CR && flagged; ++r) {
        Gs[(2 * tau) * (CR + 1) + r] = 0.f; Gs[(2 * tau + 1) * (CR + 1) + r] = 0.f;
        Gs[r * (CR + 1) + 2 * tau] = 0.f; Gs[r * (CR + 1) + 2 * tau + 1] = 0.f;
      }
    }
    if (tau < nt && !flagged) {
      const float kk = Gs[(2 * tau) * (CR + 1) + 2 * tau];
      const float vv = Gs[(2 * tau + 1) * (CR + 1) + 2 * tau + 1];
      const float kv = Gs[(2 * tau) * (CR + 1) + 2 * tau + 1];
      const float g = gamma[(size_t)item * S + t0 + tau];
      const float cc = 0.5f * g;
      const float dr = 1.f + cc * cc * (kk * vv - kv * kv);
      const float di = -2.f * cc * kv;
      const float m2 = dr * dr + di * di;
      const float fr = 2.f * cc * dr / m2;     // 2c / det
      const float fi = -2.f * cc * di / m2;
      // N00 = f (-c vv), N01 = N10 = f (c kv + i), N11 = f (-c kk)
      n00r = fr * (-cc * vv); n00i = fi * (-cc * vv);
      n11r = fr * (-cc * kk); n11i = fi * (-cc * kk);
      n01r = fr * (cc * kv) - fi; n01i = fr + fi * (cc * kv);
      const bool ok = isfinite(kk) && isfinite(vv) && isfinite(kv) && isfinite(g) &&
                      isfinite(n00r) && isfinite(n00i) && isfinite(n01r) && isfinite(n01i) &&
                      isfinite(n11r) && isfinite(n11i);
      if (!ok) {  // identity substitution, as the reference's _solve_cham_cayley does
        n00r = n00i = n01r = n01i = n11r = n11i = 0.f;
        atomicOr(&bad_bits, 1ull << tau);
        for (int r = 0; r < CR; ++r) {
          Gs[(2 * tau) * (CR + 1) + r] = 0.f; Gs[(2 * tau + 1) * (CR + 1) + r] = 0.f;
          Gs[r * (CR + 1) + 2 * tau] = 0.f; Gs[r * (CR + 1) + 2 * tau + 1] = 0.f;
        }
      }
    }
    float* n = Ns + tau * 6;
    n[0] = n00r; n[1] = n00i; n[2] = n01r; n[3] = n01i; n[4] = n11r; n[5] = n11i;
  }
  __syncthreads();
  if (tid < CR) {
    const int sg = tid, blk = sg >> 1;
    for (int r = 0; r < 2 * blk; ++r) { Tr[r * (CR + 1) + sg] = 0.f; Ti[r * (CR + 1) + sg] = 0.f; }
    for (int t = blk; t < CC; ++t) {
      float x0r = (sg == 2 * t) ? 1.f : 0.f, x0i = 0.f;
      float x1r = (sg == 2 * t + 1) ? 1.f : 0.f, x1i = 0.f;
      for (int tp = blk; tp < t; ++tp) {
        const float a0r = Tr[(2 * tp) * (CR + 1) + sg], a0i = Ti[(2 * tp) * (CR + 1) + sg];
        const float a1r = Tr[(2 * tp + 1) * (CR + 1) + sg], a1i = Ti[(2 * tp + 1) * (CR + 1) + sg];
        const float g00 = Gs[(2 * t) * (CR + 1) + 2 * tp], g01 = Gs[(2 * t) * (CR + 1) + 2 * tp + 1];
        const float g10 = Gs[(2 * t + 1) * (CR + 1) + 2 * tp], g11 = Gs[(2 * t + 1) * (CR + 1) + 2 * tp + 1];
        x0r += g00 * a0r + g01 * a1r; x0i += g00 * a0i + g01 * a1i;
        x1r += g10 * a0r + g11 * a1r; x1i += g10 * a0i + g11 * a1i;
      }
      const float* n = Ns + t * 6;
      // [T0; T1] = N_t [x0; x1], N_t = [[n00, n01], [n01, n11]]
      Tr[(2 * t) * (CR + 1) + sg] = n[0] * x0r - n[1] * x0i + n[2] * x1r - n[3] * x1i;
      Ti[(2 * t) * (CR + 1) + sg] = n[0] * x0i + n[1] * x0r + n[2] * x1i + n[3] * x1r;
      Tr[(2 * t + 1) * (CR + 1) + sg] = n[2] * x0r - n[3] * x0i + n[4] * x1r - n[5] * x1i;
      Ti[(2 * t + 1) * (CR + 1) + sg] = n[2] * x0i + n[3] * x0r + n[4] * x1i + n[5] * x1r;
    }
  }
  __syncthreads();
  const size_t chunk = (size_t)item * nch + c;
  float* To = Tws + chunk * 2 * CR * CR;
  for (int e = tid; e < CR * CR; e += blockDim.x) {
    To[e] = Tr[(e / CR) * (CR + 1) + e % CR];
    To[CR * CR + e] = Ti[(e / CR) * (CR + 1) + e % CR];
  }
  float* Eo = Ews + chunk * CR * CC;
  for (int e = tid; e < CR * CC; e += blockDim.x) Eo[e] = 0.f;
  if (tid == 0) badws[chunk] = bad_bits;
}

// Load the chunk's W rows [i0, i0+rows) into Wt[i][r] (pitch CR+1).
template <typename T>
__device__ __forceinline__ void load_w_rows(float* Wt, const T* __restrict__ k, const T* __restrict__ v,
                                            int item, int S, int D, int t0, int nt,
                                            unsigned long long bad, int i0, int rows, int tid, int nthr) {
  for (int e = tid; e < rows * CR; e += nthr) {
    const int i = e / CR, r = e % CR, tau = r >> 1;
    float val = 0.f;
    if (tau < nt && i0 + i < D && !((bad >> tau) & 1ull)) {
      const size_t off = ((size_t)item * S + t0 + tau) * D + i0 + i;
      val = to_f32((r & 1) ? v[off] : k[off]);
    }
    Wt[i * (CR + 1) + r] = val;
  }
}

// Load a rows x cols tile of a [D][D] state (or of the identity when re == nullptr).
__device__ __forceinline__ void load_state_tile(float* tr, float* ti, int pitch,
                                                const float* __restrict__ re, const float* __restrict__ im,
                                                int D, int i0, int j0, int rows, int cols, int tid, int nthr) {
  for (int e = tid; e < rows * cols; e += nthr) {
    const int i = e / cols, j = e % cols;
    const int gi = i0 + i, gj = j0 + j;
    float a = 0.f, b = 0.f;
    if (gi < D && gj < D) {
      if (re) { a = re[(size_t)gi * D + gj]; b = im[(size_t)gi * D + gj]; }
      else a = (gi == gj) ? 1.f : 0.f;
    }
    tr[i * pitch + j] = a;
    ti[i * pitch + j] = b;
  }
}

// ---------------------------------------------------------------------------------
// colpass.  smem: Wt [RT][CR+1], Htr/Hti [RT][NB+1], Zr/Zi [CR][NB+1], Cr/Ci [CR][NB+1],
//                 Tsr/Tsi [CR][CR+1], Yr/Yi [NB][CC+1], Ep [CR][CC+1]
template <typename T, bool YC>
__global__ void __launch_bounds__(THREADS)
cham_colpass_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                    const float* __restrict__ ybuf_r, const float* __restrict__ ybuf_i,
                    const float* __restrict__ Tws, float* __restrict__ Ews,
                    const unsigned long long* __restrict__ badws,
                    const float* __restrict__ src_r, const float* __restrict__ src_i,
                    float* __restrict__ dst_r, float* __restrict__ dst_i,
                    int S, int D, int nch, int c) {
  extern __shared__ float sm[];
  float* Wt = sm;
  float* Htr = Wt + RT * (CR + 1);
  float* Hti = Htr + RT * (NB + 1);
  float* Zr = Hti + RT * (NB + 1);
  float* Zi = Zr + CR * (NB + 1);
  float* Cr = Zi + CR * (NB + 1);
  float* Ci = Cr + CR * (NB + 1);
  float* Tsr = Ci + CR * (NB + 1);
  float* Tsi = Tsr + CR * (CR + 1);
  float* Yr = Tsi + CR * (CR + 1);
  float* Yi = Yr + NB * (CC + 1);
  float* Ep = Yi + NB * (CC + 1);

  const int item = blockIdx.y, j0 = blockIdx.x * NB, tid = threadIdx.x, nthr = blockDim.x;
  const int t0 = c * CC, nt = min(CC, S - t0);
  const size_t chunk = (size_t)item * nch + c;
  const unsigned long long bad = badws[chunk];
  const size_t soff = (size_t)item * D * D;
  const float* sr = src_r ? src_r + soff : nullptr;
  const float* si = src_i ? src_i + soff : nullptr;

  for (int e = tid; e < CR * (NB + 1); e += nthr) { Zr[e] = 0.f; Zi[e] = 0.f; }
  const float* Tin = Tws + chunk * 2 * CR * CR;
  for (int e = tid; e < CR * CR; e += nthr) {
    Tsr[(e / CR) * (CR + 1) + e % CR] = Tin[e];
    Tsi[(e / CR) * (CR + 1) + e % CR] = Tin[CR * CR + e];
  }
  for (int e = tid; e < NB * CC; e += nthr) {
    const int t = e / NB, j = e % NB;
    float a = 0.f, b = 0.f;
    if (t < nt && j0 + j < D) {
      const size_t off = ((size_t)item * S + t0 + t) * D + j0 + j;
      if (YC) { a = ybuf_r[off]; b = ybuf_i[off]; } else a = to_f32(q[off]);
    }
    Yr[j * (CC + 1) + t] = a;
    Yi[j * (CC + 1) + t] = b;
  }
  // Z = Wᵀ S[:, block]
  for (int i0 = 0; i0 < D; i0 += RT) {
    __syncthreads();
    load_w_rows(Wt, k, v, item, S, D, t0, nt, bad, i0, RT, tid, nthr);
    load_state_tile(Htr, Hti, NB + 1, sr, si, D, i0, j0, RT, NB, tid, nthr);
    __syncthreads();
    smem_gemm<4, 2, true>(CR, NB, RT, Wt, 1, CR + 1, Htr, NB + 1, 1, Zr, NB + 1, 1, tid, nthr);
    smem_gemm<4, 2, true>(CR, NB, RT, Wt, 1, CR + 1, Hti, NB + 1, 1, Zi, NB + 1, 1, tid, nthr);
  }
  __syncthreads();
  // Cm = T Z (complex)
  smem_gemm<4, 2, false>(CR, NB, CR, Tsr, CR + 1, 1, Zr, NB + 1, 1, Cr, NB + 1, 1, tid, nthr);
  smem_gemm<4, 2, false>(CR, NB, CR, Tsr, CR + 1, 1, Zi, NB + 1, 1, Ci, NB + 1, 1, tid, nthr);
  __syncthreads();
  smem_gemm<4, 2, true>(CR, NB, CR, Tsi, CR + 1, 1, Zi, NB + 1, 1, Cr, NB + 1, 1, tid, nthr, -1.f);
  smem_gemm<4, 2, true>(CR, NB, CR, Tsi, CR + 1, 1, Zr, NB + 1, 1, Ci, NB + 1, 1, tid, nthr);
  __syncthreads();
  // Re(Cm Y) over this column block -> atomically reduced into E
  smem_gemm<4, 4, false>(CR, CC, NB, Cr, NB + 1, 1, Yr, CC + 1, 1, Ep, CC + 1, 1, tid, nthr);
  if (YC) {
    __syncthreads();
    smem_gemm<4, 4, true>(CR, CC, NB, Ci, NB + 1, 1, Yi, CC + 1, 1, Ep, CC + 1, 1, tid, nthr, -1.f);
  }
  __syncthreads();
  float* Eo = Ews + chunk * CR * CC;
  for (int e = tid; e < CR * CC; e += nthr) atomicAdd(&Eo[e], Ep[(e / CC) * (CC + 1) + e % CC]);
  // S_next[:, block] = S[:, block] + W Cm
  for (int i0 = 0; i0 < D; i0 += RT) {
    __syncthreads();
    load_w_rows(Wt, k, v, item, S, D, t0, nt, bad, i0, RT, tid, nthr);
    load_state_tile(Htr, Hti, NB + 1, sr, si, D, i0, j0, RT, NB, tid, nthr);
    __syncthreads();
    smem_gemm<4, 2, true>(RT, NB, CR, Wt, CR + 1, 1, Cr, NB + 1, 1, Htr, NB + 1, 1, tid, nthr);
    smem_gemm<4, 2, true>(RT, NB, CR, Wt, CR + 1, 1, Ci, NB + 1, 1, Hti, NB + 1, 1, tid, nthr);
    __syncthreads();
    for (int e = tid; e < RT * NB; e += nthr) {
      const int i = e / NB, j = e % NB;
      if (i0 + i < D && j0 + j < D) {
        const size_t o = soff + (size_t)(i0 + i) * D + j0 + j;
        dst_r[o] = Htr[i * (NB + 1) + j];
        dst_i[o] = Hti[i * (NB + 1) + j];
      }
    }
  }
}

// ---------------------------------------------------------------------------------
// readout.  smem: Os [RB][CC+1], Htr/Hti [RB][JT+1], Ytr/Yti [JT][CC+1], Wt [RB][CR+1], Es [CR][CC+1]
template <typename T, bool YC>
__global__ void __launch_bounds__(THREADS)
cham_readout_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                    const float* __restrict__ ybuf_r, const float* __restrict__ ybuf_i,
                    const float* __restrict__ Ews, const unsigned long long* __restrict__ badws,
                    const float* __restrict__ src_r, const float* __restrict__ src_i,
                    T* __restrict__ out, int S, int D, int nch, int c) {
  extern __shared__ float sm[];
  float* Os = sm;
  float* Htr = Os + RB * (CC + 1);
  float* Hti = Htr + RB * (JT + 1);
  float* Ytr = Hti + RB * (JT + 1);
  float* Yti = Ytr + JT * (CC + 1);
  float* Wt = Yti + JT * (CC + 1);
  float* Es = Wt + RB * (CR + 1);
  const int item = blockIdx.y, i0 = blockIdx.x * RB, tid = threadIdx.x, nthr = blockDim.x;
  const int t0 = c * CC, nt = min(CC, S - t0);
  const size_t chunk = (size_t)item * nch + c;
  const size_t soff = (size_t)item * D * D;
  const float* sr = src_r ? src_r + soff : nullptr;
  const float* si = src_i ? src_i + soff : nullptr;

  for (int e = tid; e < RB * (CC + 1); e += nthr) Os[e] = 0.f;
  for (int j0 = 0; j0 < D; j0 += JT) {
    __syncthreads();
    load_state_tile(Htr, Hti, JT + 1, sr, si, D, i0, j0, RB, JT, tid, nthr);
    for (int e = tid; e < JT * CC; e += nthr) {
      const int t = e / JT, j = e % JT;
      float a = 0.f, b = 0.f;
      if (t < nt && j0 + j < D) {
        const size_t off = ((size_t)item * S + t0 + t) * D + j0 + j;
        if (YC) { a = ybuf_r[off]; b = ybuf_i[off]; } else a = to_f32(q[off]);
      }
      Ytr[j * (CC + 1) + t] = a;
      Yti[j * (CC + 1) + t] = b;
    }
    __syncthreads();
    smem_gemm<2, 4, true>(RB, CC, JT, Htr, JT + 1, 1, Ytr, CC + 1, 1, Os, CC + 1, 1, tid, nthr);
    if (YC) smem_gemm<2, 4, true>(RB, CC, JT, Hti, JT + 1, 1, Yti, CC + 1, 1, Os, CC + 1, 1, tid, nthr, -1.f);
  }
  __syncthreads();
  load_w_rows(Wt, k, v, item, S, D, t0, nt, badws[chunk], i0, RB, tid, nthr);
  const float* Ein = Ews + chunk * CR * CC;
  for (int e = tid; e < CR * CC; e += nthr) {
    const int r = e / CC, t = e % CC;
    Es[r * (CC + 1) + t] = ((r >> 1) <= t) ? Ein[e] : 0.f;
  }
  __syncthreads();
  smem_gemm<2, 4, true>(RB, CC, CR, Wt, CR + 1, 1, Es, CC + 1, 1, Os, CC + 1, 1, tid, nthr);
  __syncthreads();
  for (int e = tid; e < nt * RB; e += nthr) {
    const int t = e / RB, i = e % RB;
    if (i0 + i < D) out[((size_t)item * S + t0 + t) * D + i0 + i] = from_f32<T>(Os[i * (CC + 1) + t]);
  }
}

template <typename T>
__global__ void to_complex_kernel(const T* __restrict__ x, float* __restrict__ re, float* __restrict__ im, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    re[i] = to_f32(x[i]);
    im[i] = 0.f;
  }
}

__global__ void identity_fill_kernel(float* __restrict__ re, float* __restrict__ im, int D, size_t n) {
  for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < n; e += (size_t)gridDim.x * blockDim.x) {
    const size_t r = e % ((size_t)D * D);
    re[e] = (r / D == r % D) ? 1.f : 0.f;
    im[e] = 0.f;
  }
}

size_t prep_smem() { return sizeof(float) * (DT * (CR + 1) + 3 * CR * (CR + 1) + CC * 6); }
size_t colpass_smem() {
  return sizeof(float) * (RT * (CR + 1) + 2 * RT * (NB + 1) + 4 * CR * (NB + 1) + 2 * CR * (CR + 1) +
                          2 * NB * (CC + 1) + CR * (CC + 1));
}
size_t readout_smem() {
  return sizeof(float) * (RB * (CC + 1) + 2 * RB * (JT + 1) + 2 * JT * (CC + 1) + RB * (CR + 1) + CR * (CC + 1));
}

// y = p(A) q with A = H0ᴴ H0 (see the file comment).  All vector sets are [b][s][D]
// planar complex in the workspace; returns the index of the set holding y.
int readout_polynomial(const float* h0r, const float* h0i, int b, int s, int D, float* Y,
                       void* pack, size_t pack_bytes, int* y_index, cudaStream_t st) {
  const size_t set = (size_t)2 * b * s * D;
  auto re = [&](int i) { return Y + i * set; };
  auto im = [&](int i) { return Y + i * set + set / 2; };
  const long long vs = (long long)s * D, hs = (long long)D * D;
  const int TMP = 5;
  // out = alpha * A in + beta * comb   (A in = H0ᴴ (H0 in))
  auto applyA = [&](int in, int outi, float alpha, float beta, int comb) -> int {
    int rc = cgemm_tc(s, D, D, b, 1.f, CMat{re(in), im(in), D, vs}, false, false,
                      CMat{h0r, h0i, D, hs}, true, false, 0.f, CMat{nullptr, nullptr, 0, 0},
                      re(TMP), im(TMP), D, vs, pack, pack_bytes, st);
    if (rc) return rc;
    return cgemm_tc(s, D, D, b, alpha, CMat{re(TMP), im(TMP), D, vs}, false, false,
                    CMat{h0r, h0i, D, hs}, false, true, beta, CMat{re(comb), im(comb), D, vs},
                    re(outi), im(outi), D, vs, pack, pack_bytes, st);
  };
  auto g0 = [&](int in, int outi) { return applyA(in, outi, -0.5f, 1.5f, in); };
  int rc = 0;
  // g1(B0) -> B1
  if ((rc = g0(0, 2)) || (rc = g0(2, 3)) || (rc = applyA(3, 1, -0.5f, 1.5f, 0))) return rc;
  // g1(B1) -> B2
  if ((rc = g0(1, 3)) || (rc = g0(3, 4)) || (rc = applyA(4, 2, -0.5f, 1.5f, 1))) return rc;
  // g2(B0) = 1.5 B0 - 0.5 A1(B2) -> B1
  if ((rc = g0(2, 3)) || (rc = g0(3, 4)) || (rc = applyA(4, 1, -0.5f, 1.5f, 0))) return rc;
  // g1(B1) -> B2
  if ((rc = g0(1, 3)) || (rc = g0(3, 4)) || (rc = applyA(4, 2, -0.5f, 1.5f, 1))) return rc;
  // g0(B2) -> B3
  if ((rc = g0(2, 3))) return rc;
  *y_index = 3;
  return VERACE_OK;
}

template <typename T>
int launch_cham(const void* q, const void* k, const void* v, const float* gamma,
                const float* h0r, const float* h0i, void* out, float* hr, float* hi,
                int b, int s, int D, const ChamWs& w, cudaStream_t st, bool exact_readout = true) {
  const int nch = (s + CC - 1) / CC;
  int rc;
  const size_t ps = prep_smem(), cs = colpass_smem(), rs = readout_smem();
  VERACE_CUDA(cudaFuncSetAttribute(cham_prep_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ps));
  cham_prep_kernel<T><<<dim3(nch, b), THREADS, ps, st>>>((const T*)k, (const T*)v, gamma, w.T, w.E, w.bad, s, D, nch);
  if ((rc = check_launch("cham_prep_kernel"))) return rc;

  const bool yc = h0r != nullptr && exact_readout;   // readout vectors p(H0ᴴH0) q
  const float* yr = nullptr;
  const float* yi = nullptr;
  if (yc) {
    const size_t set = (size_t)2 * b * s * D;
    to_complex_kernel<T><<<1024, 256, 0, st>>>((const T*)q, w.Y, w.Y + set / 2, set / 2);
    if ((rc = check_launch("to_complex_kernel"))) return rc;
    int yidx = 0;
    if ((rc = readout_polynomial(h0r, h0i, b, s, D, w.Y, w.pack, w.pack_bytes, &yidx, st))) return rc;
    yr = w.Y + yidx * set;
    yi = yr + set / 2;
  }
  auto colpass = yc ? cham_colpass_kernel<T, true> : cham_colpass_kernel<T, false>;
  auto readout = yc ? cham_readout_kernel<T, true> : cham_readout_kernel<T, false>;
  VERACE_CUDA(cudaFuncSetAttribute(colpass, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)cs));
  VERACE_CUDA(cudaFuncSetAttribute(readout, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)rs));
  const dim3 gc((D + NB - 1) / NB, b), gr((D + RB - 1) / RB, b);
  const float* cur_r = h0r;
  const float* cur_i = h0i;
  for (int c = 0; c < nch; ++c) {
    const bool to_out = ((nch - 1 - c) % 2) == 0;
    float* dr = to_out ? hr : w.Hre;
    float* di = to_out ? hi : w.Him;
    colpass<<<gc, THREADS, cs, st>>>((const T*)q, (const T*)k, (const T*)v, yr, yi, w.T, w.E, w.bad,
                                     cur_r, cur_i, dr, di, s, D, nch, c);
    if ((rc = check_launch("cham_colpass_kernel"))) return rc;
    readout<<<gr, THREADS, rs, st>>>((const T*)q, (const T*)k, (const T*)v, yr, yi, w.E, w.bad,
                                     cur_r, cur_i, (T*)out, s, D, nch, c);
    if ((rc = check_launch("cham_readout_kernel"))) return rc;
    cur_r = dr;
    cur_i = di;
  }
  return VERACE_OK;
}

}  // namespace
}  // namespace verace

using namespace verace;

extern "C" size_t verace_cham_scan_workspace(int b, int s, int D, int has_h0) {
  if (b <= 0 || s <= 0 || D <= 0) return 256;
  size_t n = ws_layout(b, s, D, has_h0 ? 1 : 0, nullptr, nullptr);
  if (D % 128 == 0) {   // (with has_h0: the tensor-core continuation of verace_cham_scan_unitary)
    const size_t t = cham_tc_workspace(b, s, D);
    if (t > n) n = t;
  }
  return n;
}

extern "C" int verace_cham_scan(const void* q, const void* k, const void* v, const float* gamma,
                                const float* h0_re, const float* h0_im, void* out, float* h_re,
                                float* h_im, int b, int s, int D, int dtype, void* workspace,
                                size_t workspace_bytes, void* stream) {
  VERACE_REQUIRE(b >= 0 && s >= 0 && D >= 1, VERACE_ERR_INVALID,
                 "verace_cham_scan: invalid sizes b=%d s=%d D=%d", b, s, D);
  VERACE_REQUIRE(dtype == VERACE_F32 || dtype == VERACE_BF16 || dtype == VERACE_F16,
                 VERACE_ERR_INVALID, "verace_cham_scan: unknown dtype %d", dtype);
  VERACE_REQUIRE((h0_re == nullptr) == (h0_im == nullptr), VERACE_ERR_INVALID,
                 "verace_cham_scan: h0_re and h0_im must both be given or both be NULL");
  if (b == 0) return VERACE_OK;
  VERACE_REQUIRE(h_re && h_im, VERACE_ERR_INVALID, "verace_cham_scan: NULL state output");
  cudaStream_t st = (cudaStream_t)stream;
  const size_t state_elems = (size_t)b * D * D;
  if (s == 0) {
    if (h0_re) {
      VERACE_CUDA(cudaMemcpyAsync(h_re, h0_re, state_elems * sizeof(float), cudaMemcpyDeviceToDevice, st));
      VERACE_CUDA(cudaMemcpyAsync(h_im, h0_im, state_elems * sizeof(float), cudaMemcpyDeviceToDevice, st));
    } else {
      identity_fill_kernel<<<1024, 256, 0, st>>>(h_re, h_im, D, state_elems);
      return check_launch("identity_fill_kernel");
    }
    return VERACE_OK;
  }
  VERACE_REQUIRE(q && k && v && gamma && out, VERACE_ERR_INVALID, "verace_cham_scan: NULL input/output pointer");
  const int has_h0 = h0_re ? 1 : 0;
  const size_t need = verace_cham_scan_workspace(b, s, D, has_h0);
  VERACE_REQUIRE(workspace != nullptr && workspace_bytes >= need, VERACE_ERR_WORKSPACE,
                 "verace_cham_scan: workspace of %zu bytes required, %zu given", need,
                 workspace ? workspace_bytes : (size_t)0);
  if (cham_tc_supported(D, dtype, has_h0 != 0) && !force_simt())
    return cham_tc_scan(q, k, v, gamma, nullptr, nullptr, out, h_re, h_im, b, s, D, dtype, workspace, st);
  ChamWs w;
  char* base = (char*)align_up((size_t)workspace, 256);
  ws_layout(b, s, D, has_h0, &w, base);
  switch (dtype) {
    case VERACE_F32: return launch_cham<float>(q, k, v, gamma, h0_re, h0_im, out, h_re, h_im, b, s, D, w, st);
    case VERACE_BF16: return launch_cham<__nv_bfloat16>(q, k, v, gamma, h0_re, h0_im, out, h_re, h_im, b, s, D, w, st);
    default: return launch_cham<__half>(q, k, v, gamma, h0_re, h0_im, out, h_re, h_im, b, s, D, w, st);
  }
}

// ---------------------------------------------------------------------------------
// Continuation from a unitary hologram.  The Newton-Schulz readout of the scan is
// Re(NS3(H_t) q_t) = Re(H_t p(A) q_t) with A = H0ᴴ H0 (every U_t is unitary), and
// p(I + E) = I - E/2 + O(E^2): for a unitary H0, p(A) = I and the readout is Re(H_t q_t),
// which the tensor-core scan computes.  verace_cham_unitarity measures how far H0 is from
// unitary, so that a caller can choose between that scan and the exact one.
namespace verace {
namespace {
constexpr int PROBES = 4;

__device__ __forceinline__ double probe_sign(int j, int c) {
  const unsigned int h = ((unsigned int)c * 2654435761u) ^ ((unsigned int)(j + 1) * 0x9E3779B9u);
  return ((h >> 15) & 1u) ? 1.0 : -1.0;
}

// u_j = H r_j for PROBES fixed +-1 vectors r_j: one warp per row, fp64 sums; u [b][J][D] (re, im)
__global__ void unitarity_rows_kernel(const float* __restrict__ hr, const float* __restrict__ hi,
                                      double2* __restrict__ u, int b, int D) {
  const long long row = (long long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= (long long)b * D) return;
  const float* pr = hr + row * D;
  const float* pi = hi + row * D;
  double ar[PROBES], ai[PROBES];
#pragma unroll
  for (int j = 0; j < PROBES; ++j) ar[j] = ai[j] = 0.0;
  for (int c = lane; c < D; c += 32) {
    const double xr = pr[c], xi = pi[c];
#pragma unroll
    for (int j = 0; j < PROBES; ++j) {
      const double sg = probe_sign(j, c);
      ar[j] += sg * xr;
      ai[j] += sg * xi;
    }
  }
#pragma unroll
  for (int j = 0; j < PROBES; ++j) {
    for (int o = 16; o > 0; o >>= 1) {
      ar[j] += __shfl_xor_sync(0xffffffffu, ar[j], o);
      ai[j] += __shfl_xor_sync(0xffffffffu, ai[j], o);
    }
  }
  if (lane == 0) {
    const long long item = row / D, r = row % D;
#pragma unroll
    for (int j = 0; j < PROBES; ++j) u[(item * PROBES + j) * D + r] = make_double2(ar[j], ai[j]);
  }
}

// w_j = Hᴴ u_j for a stripe of 32 columns (8 warps over the rows), then the stripe's
// sum of |w_j - r_j|^2, added into err [b][J]
__global__ void unitarity_cols_kernel(const float* __restrict__ hr, const float* __restrict__ hi,
                                      const double2* __restrict__ u, double* __restrict__ err, int D) {
  __shared__ double sr[8][PROBES][32], si[8][PROBES][32];
  const int item = blockIdx.y, c = blockIdx.x * 32 + (threadIdx.x & 31), wv = threadIdx.x / 32;
  double ar[PROBES], ai[PROBES];
#pragma unroll
  for (int j = 0; j < PROBES; ++j) ar[j] = ai[j] = 0.0;
  const float* pr = hr + (size_t)item * D * D;
  const float* pi = hi + (size_t)item * D * D;
  const double2* uu = u + (size_t)item * PROBES * D;
  if (c < D) {
    for (int r = wv; r < D; r += 8) {
      const double xr = pr[(size_t)r * D + c], xi = pi[(size_t)r * D + c];
#pragma unroll
      for (int j = 0; j < PROBES; ++j) {
        const double2 q = uu[j * D + r];   // conj(H[r][c]) u[r]
        ar[j] += xr * q.x + xi * q.y;
        ai[j] += xr * q.y - xi * q.x;
      }
    }
  }
#pragma unroll
  for (int j = 0; j < PROBES; ++j) { sr[wv][j][threadIdx.x & 31] = ar[j]; si[wv][j][threadIdx.x & 31] = ai[j]; }
  __syncthreads();
  if (wv < PROBES) {
    const int j = wv, l = threadIdx.x & 31;
    double wr = 0.0, wi = 0.0;
    for (int k = 0; k < 8; ++k) { wr += sr[k][j][l]; wi += si[k][j][l]; }
    double e = 0.0;
    if (blockIdx.x * 32 + l < D) {
      const double d = wr - probe_sign(j, blockIdx.x * 32 + l);
      e = d * d + wi * wi;
    }
    for (int o = 16; o > 0; o >>= 1) e += __shfl_xor_sync(0xffffffffu, e, o);
    if (l == 0) atomicAdd(&err[item * PROBES + j], e);
  }
}

__global__ void unitarity_final_kernel(const double* __restrict__ err, float* __restrict__ eps, int b, int D) {
  const int item = blockIdx.x * blockDim.x + threadIdx.x;
  if (item >= b) return;
  double m = 0.0;
  for (int j = 0; j < PROBES; ++j) m = fmax(m, err[item * PROBES + j]);
  eps[item] = (float)sqrt(m / (double)D);   // |E r| / |r|, |r|^2 = D
}
}  // namespace
}  // namespace verace

extern "C" size_t verace_cham_unitarity_workspace(int b, int D) {
  if (b <= 0 || D <= 0) return 256;
  return align_up((size_t)b * PROBES * D * sizeof(double2), 256) + align_up((size_t)b * PROBES * sizeof(double), 256) +
         256;
}

extern "C" int verace_cham_unitarity(const float* h_re, const float* h_im, int b, int D, float* eps,
                                     void* workspace, size_t workspace_bytes, void* stream) {
  VERACE_REQUIRE(b >= 0 && D >= 1, VERACE_ERR_INVALID, "verace_cham_unitarity: invalid sizes b=%d D=%d", b, D);
  if (b == 0) return VERACE_OK;
  VERACE_REQUIRE(h_re && h_im && eps, VERACE_ERR_INVALID, "verace_cham_unitarity: NULL pointer");
  const size_t need = verace_cham_unitarity_workspace(b, D);
  VERACE_REQUIRE(workspace != nullptr && workspace_bytes >= need, VERACE_ERR_WORKSPACE,
                 "verace_cham_unitarity: workspace of %zu bytes required, %zu given", need,
                 workspace ? workspace_bytes : (size_t)0);
  cudaStream_t st = (cudaStream_t)stream;
  char* base = (char*)align_up((size_t)workspace, 256);
  double2* u = (double2*)base;
  double* err = (double*)(base + align_up((size_t)b * PROBES * D * sizeof(double2), 256));
  VERACE_CUDA(cudaMemsetAsync(err, 0, (size_t)b * PROBES * sizeof(double), st));
  const long long rows = (long long)b * D;
  unitarity_rows_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(h_re, h_im, u, b, D);
  int rc = check_launch("unitarity_rows_kernel");
  if (rc) return rc;
  unitarity_cols_kernel<<<dim3((D + 31) / 32, b), 256, 0, st>>>(h_re, h_im, u, err, D);
  if ((rc = check_launch("unitarity_cols_kernel"))) return rc;
  unitarity_final_kernel<<<(b + 127) / 128, 128, 0, st>>>(err, eps, b, D);
  return check_launch("unitarity_final_kernel");
}

extern "C" int verace_cham_scan_unitary(const void* q, const void* k, const void* v, const float* gamma,
                                        const float* h0_re, const float* h0_im, void* out, float* h_re,
                                        float* h_im, int b, int s, int D, int dtype, void* workspace,
                                        size_t workspace_bytes, void* stream) {
  VERACE_REQUIRE(b >= 0 && s >= 0 && D >= 1, VERACE_ERR_INVALID,
                 "verace_cham_scan_unitary: invalid sizes b=%d s=%d D=%d", b, s, D);
  VERACE_REQUIRE(dtype == VERACE_F32 || dtype == VERACE_BF16 || dtype == VERACE_F16,
                 VERACE_ERR_INVALID, "verace_cham_scan_unitary: unknown dtype %d", dtype);
  VERACE_REQUIRE((h0_re == nullptr) == (h0_im == nullptr), VERACE_ERR_INVALID,
                 "verace_cham_scan_unitary: h0_re and h0_im must both be given or both be NULL");
  if (h0_re == nullptr || b == 0 || s == 0)   // nothing to assume: the exact scan
    return verace_cham_scan(q, k, v, gamma, h0_re, h0_im, out, h_re, h_im, b, s, D, dtype, workspace,
                            workspace_bytes, stream);
  VERACE_REQUIRE(h_re && h_im, VERACE_ERR_INVALID, "verace_cham_scan_unitary: NULL state output");
  VERACE_REQUIRE(q && k && v && gamma && out, VERACE_ERR_INVALID,
                 "verace_cham_scan_unitary: NULL input/output pointer");
  const size_t need = verace_cham_scan_workspace(b, s, D, 1);
  VERACE_REQUIRE(workspace != nullptr && workspace_bytes >= need, VERACE_ERR_WORKSPACE,
                 "verace_cham_scan_unitary: workspace of %zu bytes required, %zu given", need,
                 workspace ? workspace_bytes : (size_t)0);
  cudaStream_t st = (cudaStream_t)stream;
  if (cham_tc_supported_unitary(D, dtype) && !force_simt())
    return cham_tc_scan(q, k, v, gamma, h0_re, h0_im, out, h_re, h_im, b, s, D, dtype, workspace, st);
  ChamWs w;
  char* base = (char*)align_up((size_t)workspace, 256);
  ws_layout(b, s, D, 0, &w, base);
  switch (dtype) {
    case VERACE_F32:
      return launch_cham<float>(q, k, v, gamma, h0_re, h0_im, out, h_re, h_im, b, s, D, w, st, false);
    case VERACE_BF16:
      return launch_cham<__nv_bfloat16>(q, k, v, gamma, h0_re, h0_im, out, h_re, h_im, b, s, D, w, st, false);
    default:
      return launch_cham<__half>(q, k, v, gamma, h0_re, h0_im, out, h_re, h_im, b, s, D, w, st, false);
  }
}

extern "C" size_t verace_cham_retract_workspace(int b, int D) {
  if (b <= 0 || D <= 0) return 256;
  return align_up((size_t)4 * b * D * D * sizeof(float), 256) + cgemm_tc_scratch(D, D, D, b) + 256;
}

extern "C" int verace_cham_retract(const float* h_re, const float* h_im, float* out_re, float* out_im,
                                   int b, int D, int steps, void* workspace, size_t workspace_bytes,
                                   void* stream) {
  VERACE_REQUIRE(b >= 0 && D >= 1 && steps >= 0, VERACE_ERR_INVALID,
                 "verace_cham_retract: invalid sizes b=%d D=%d steps=%d", b, D, steps);
  if (b == 0) return VERACE_OK;
  VERACE_REQUIRE(h_re && h_im && out_re && out_im, VERACE_ERR_INVALID, "verace_cham_retract: NULL pointer");
  cudaStream_t st = (cudaStream_t)stream;
  const size_t n = (size_t)b * D * D;
  if (steps == 0) {
    VERACE_CUDA(cudaMemcpyAsync(out_re, h_re, n * sizeof(float), cudaMemcpyDeviceToDevice, st));
    VERACE_CUDA(cudaMemcpyAsync(out_im, h_im, n * sizeof(float), cudaMemcpyDeviceToDevice, st));
    return VERACE_OK;
  }
  const size_t need = verace_cham_retract_workspace(b, D);
  VERACE_REQUIRE(workspace != nullptr && workspace_bytes >= need, VERACE_ERR_WORKSPACE,
                 "verace_cham_retract: workspace of %zu bytes required, %zu given", need,
                 workspace ? workspace_bytes : (size_t)0);
  float* base = (float*)align_up((size_t)workspace, 256);
  float* HHr = base;
  float* HHi = base + n;
  float* Pr = base + 2 * n;
  float* Pi = base + 3 * n;
  void* pack = base + 4 * n;
  const size_t pack_bytes = need - 256 - align_up((size_t)4 * n * sizeof(float), 256);
  const long long hs = (long long)D * D;
  const float* cr = h_re;
  const float* ci = h_im;
  for (int i = 0; i < steps; ++i) {
    const bool to_out = ((steps - 1 - i) % 2) == 0;
    float* nr = to_out ? out_re : Pr;
    float* ni = to_out ? out_im : Pi;
    // HH = curᴴ cur
    int rc = cgemm_tc(D, D, D, b, 1.f, CMat{cr, ci, D, hs}, true, true, CMat{cr, ci, D, hs}, false, false,
                      0.f, CMat{nullptr, nullptr, 0, 0}, HHr, HHi, D, hs, pack, pack_bytes, st);
    if (rc) return rc;
    // next = 1.5 cur - 0.5 cur HH
    rc = cgemm_tc(D, D, D, b, -0.5f, CMat{cr, ci, D, hs}, false, false, CMat{HHr, HHi, D, hs}, false, false,
                  1.5f, CMat{cr, ci, D, hs}, nr, ni, D, hs, pack, pack_bytes, st);
    if (rc) return rc;
    cr = nr;
    ci = ni;
  }
  return VERACE_OK;
}

extern "C" int verace_device_status(void* stream) {
  int status = 0, status2 = 0;
  int rc = tc_read_status((cudaStream_t)stream, &status);
  if (rc) return rc;
  rc = sssd_tc_read_status(&status2);
  if (rc) return rc;
  status |= status2;
  rc = mcmoe_read_status(&status2);
  if (rc) return rc;
  status |= status2;
  rc = cgemm_tc_read_status(&status2);
  if (rc) return rc;
  status |= status2;
  unsigned int dstat = 0;   // bit 0: a hologram far from unitary; bit 1: a decode wait gave up
  rc = decode_read_status(&dstat);
  if (rc) return rc;
  if (dstat & 2u) status = 1;
  dstat &= 1u;
  VERACE_REQUIRE(status == 0, VERACE_ERR_TIMEOUT,
                 "a bounded device-side wait gave up (tensor-core completion never arrived)");
  VERACE_REQUIRE(dstat == 0, VERACE_ERR_STATE,
                 "a decode step met a hologram too far from unitary (|(H^H H - I) q| > 1e-2 |q|)");
  return VERACE_OK;
}
