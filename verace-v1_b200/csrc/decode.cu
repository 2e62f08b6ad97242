// Fused single-token decode step for a batch: the SSSD head-state rotations and the CHAM
// hologram updates of one layer, with both readouts, in one launch.
//
// One incremental-decode step of the reference runs, per layer and per batch item,
// SSSDAttention.forward with s = 1 and initial_state (sssd_attention.py:103-182) and
// ContinuousHolographicMemory.forward with s = 1 and initial_hologram
// (cham_memory.py:117-243), reached through layer_states (backbone.py:53-101,
// hyper_generate.py:58-77) and, on the GPU, the launchers of triton_kernels.py:603-685
// (D > 128: _cham_tiled_step, triton_kernels.py:477-549).  This file does the same step
// for all items at once.
//
// SSSD, per item and head (state Ψ, d x d, fp32):
//     Ψ' = Ψ + [k v] M [kᵀΨ; vᵀΨ],      o = Ψ' q
// with M the 2x2 Woodbury factor of the Cayley transform (same formula as the scans).
//
// CHAM, per item (state H = Hr + i Hi, D x D, fp32):
//     H' = H + [k v] N [kᵀH; vᵀH],      y = Re(NS3(H') q)
// NS3 is the reference's 3-step Newton-Schulz retraction applied to the raw state at every
// readout (cham_memory.py:233-241, triton_kernels.py:532-547).  The Cayley factor is
// unitary, so NS3(H') = H' p(HᴴH) with p the Newton-Schulz polynomial, and
// p(I + E) = I - E/2 + O(E²).  Two readout modes:
//   VERACE_DECODE_UNITARY      y = Re(H' q): exact when HᴴH = I, off by |E q|/2 otherwise;
//                              every state that an identity start produces (the prefill's
//                              H0 = None, then decode steps) has E at the level of fp32
//                              rounding.  One pass over H.
//   VERACE_DECODE_FIRST_ORDER  y = Re(H' z),  z = q - E q / 2 = 1.5 q - 0.5 Hᴴ(H q):
//                              off by O(|E|²).  A pre-pass forms u = H q (one more read
//                              of H).  The step also measures |E q| and raises the
//                              decode status flag when |E q| > 1e-2 |q| (state too far
//                              from unitary for either mode).
//
// Work split: CTA i < b·h handles SSSD (item, head) i: two passes over its 128 x 128
// state (column sums, then update, readout and store; the second pass re-reads the rows
// from L2).  The CHAM hologram is cut into column stripes of 32; one CTA owns a stripe
// over all D rows and streams it twice: pass 1 forms the column reductions kᵀH, vᵀH
// (and Hᴴu), pass 2 re-reads the stripe (from L2), updates it, stores it and forms the
// readout partials of all rows over the stripe's columns, last-read rows first so that
// the re-read finds them in L2.  The last CTA of an item to
// finish sums the stripes' partials in stripe order and writes y.  No CTA waits on
// another.
#include "common.cuh"
#include "tc.cuh"
#include "tmap.cuh"

namespace verace {

__device__ unsigned int g_decode_status;

namespace {

constexpr int DT = 256;        // threads per CTA
#ifndef VERACE_DECODE_CWD
#define VERACE_DECODE_CWD 32
#endif
constexpr int CWD = VERACE_DECODE_CWD;   // CHAM stripe width (columns)
constexpr int TPR = CWD / 4;             // threads per row (4 columns each)
constexpr int RPG = 256 / TPR;           // rows per row group
constexpr int MAXD = 2048;     // largest hologram dimension
constexpr int MAXHD = 128;     // largest SSSD head dimension
constexpr int UNR = 4;         // row groups of 32 in flight per thread and pass
constexpr float DRIFT_TOL = 1e-2f;
constexpr uint32_t LPOLLS_SD = 1u << 22;   // bounded wait of the SSSD decode state copy

struct DecodeArgs {
  const void* sq; const void* sk; const void* sv; const float* delta;
  float* psi; void* sout;
  const void* cq; const void* ck; const void* cv; const float* gamma;
  float* hr; float* hi; void* cout;
  const float* u;              // FIRST_ORDER: [b][2][D] (re, im) of H q
  float* part;                 // [b][D/32][D] readout partials
  unsigned int* cnt;           // [b] stripe counters
  float* err2;                 // [b] |E q|² accumulators
  int b, h, d, D, mode, ns;
};

template <typename T>
__device__ __forceinline__ float ld1(const void* p, size_t i) {
  return to_f32(static_cast<const T*>(p)[i]);
}

// Elements i .. i + 3 as floats in one 8-byte (16-bit types) or 16-byte (fp32) load: i a
// multiple of 4 and the base aligned to four elements.
template <typename T>
__device__ __forceinline__ void ld4(const void* p, size_t i, float (&x)[4]) {
  if constexpr (sizeof(T) == 4) {
    const float4 v = *reinterpret_cast<const float4*>(static_cast<const float*>(p) + i);
    x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
  } else {
    const uint2 v = *reinterpret_cast<const uint2*>(static_cast<const T*>(p) + i);
    const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j] = to_f32(e[j]);
  }
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

__device__ __forceinline__ float& comp(float4& v, int j) {
  return j == 0 ? v.x : (j == 1 ? v.y : (j == 2 ? v.z : v.w));
}
__device__ __forceinline__ float compc(const float4& v, int j) {
  return j == 0 ? v.x : (j == 1 ? v.y : (j == 2 ? v.z : v.w));
}

// Block-wide sums of four per-thread values (all threads), and the AND of a flag.
__device__ __forceinline__ void block_sum4(float (&x)[4], bool& flag, float (*scratch)[4]) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int j = 0; j < 4; ++j) x[j] = warp_sum(x[j]);
  if (lane == 0) {
#pragma unroll
    for (int j = 0; j < 4; ++j) scratch[w][j] = x[j];
  }
  flag = __syncthreads_and(flag) != 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float t = 0.f;
#pragma unroll
    for (int ww = 0; ww < DT / 32; ++ww) t += scratch[ww][j];
    x[j] = t;
  }
}

// ------------------------------------------------------------------------- SSSD
// The 2x2 Woodbury factor M of the Cayley transform for gate delta (a = delta / 2),
//     M = -2a / (1 + a²(kk vv - kv²)) [[a vv, 1 - a kv], [-1 - a kv, a kk]],
// with every fused multiply-add written out, so that the two SSSD decode kernels round alike.
__device__ __forceinline__ void sssd_factor(float kk, float vv, float kv, float dl, float& m00, float& m01,
                                            float& m10, float& m11) {
  const float a = 0.5f * dl;
  const float det = fmaf(a * a, fmaf(kk, vv, -(kv * kv)), 1.f);
  const float f = -2.f * a / det;
  m00 = f * (a * vv); m01 = f * fmaf(-a, kv, 1.f);
  m10 = f * fmaf(-a, kv, -1.f); m11 = f * (a * kk);
}

// The warp's sums over its 32 lanes of 16 per-lane values (the readout partials of the
// warp's 16 state rows), as a reduce-scatter: 16 shuffles instead of 5 per value.  Lane l
// (and l ^ 1) ends with the total of value 8 b4 + 4 b3 + 2 b2 + b1, b_i = bit i of l.
__device__ __forceinline__ float warp_sum16_scatter(const float (&o)[16]) {
  const int lane = threadIdx.x & 31;
  float a[8], c[4], e[2];
  const bool h4 = (lane & 16) != 0, h3 = (lane & 8) != 0, h2 = (lane & 4) != 0, h1 = (lane & 2) != 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) a[i] = (h4 ? o[i + 8] : o[i]) + __shfl_xor_sync(0xffffffffu, h4 ? o[i] : o[i + 8], 16);
#pragma unroll
  for (int i = 0; i < 4; ++i) c[i] = (h3 ? a[i + 4] : a[i]) + __shfl_xor_sync(0xffffffffu, h3 ? a[i] : a[i + 4], 8);
#pragma unroll
  for (int i = 0; i < 2; ++i) e[i] = (h2 ? c[i + 2] : c[i]) + __shfl_xor_sync(0xffffffffu, h2 ? c[i] : c[i + 2], 4);
  const float f = (h1 ? e[1] : e[0]) + __shfl_xor_sync(0xffffffffu, h1 ? e[0] : e[1], 2);
  return f + __shfl_xor_sync(0xffffffffu, f, 1);
}
__device__ __forceinline__ int warp_sum16_slot(int lane) {
  return 8 * ((lane >> 4) & 1) + 4 * ((lane >> 3) & 1) + 2 * ((lane >> 2) & 1) + ((lane >> 1) & 1);
}

template <typename T>
__device__ void sssd_part(const DecodeArgs& A, int chain) {
  __shared__ float ks[MAXHD], vs[MAXHD], qs[MAXHD];
  __shared__ float red[8][MAXHD][2];
  __shared__ float dsc[8][4];
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int d = A.d;
  const size_t vec = (size_t)chain * d;
  float* P = A.psi + (size_t)chain * d * d;
  const bool colok = 4 * lane < d;
  // state rows w + 8 m, columns 4 lane .. 4 lane + 3; pass 1: column sums kᵀΨ, vᵀΨ
  float4 ps[MAXHD / 16];
#pragma unroll
  for (int m = 0; m < MAXHD / 16; ++m) {
    const int r = w + 8 * m;
    ps[m] = (colok && r < d) ? *reinterpret_cast<const float4*>(P + (size_t)r * d + 4 * lane)
                             : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  float dots[4] = {0.f, 0.f, 0.f, 0.f};
  bool fin = true;
  for (int i = tid; i < d; i += DT) {
    const float kx = ld1<T>(A.sk, vec + i), vx = ld1<T>(A.sv, vec + i);
    ks[i] = kx; vs[i] = vx; qs[i] = ld1<T>(A.sq, vec + i);
    dots[0] += kx * kx; dots[1] += vx * vx; dots[2] += kx * vx;
    fin = fin && isfinite(kx) && isfinite(vx);
  }
  block_sum4(dots, fin, dsc);      // also makes ks/vs/qs visible
  float ak[4] = {0.f, 0.f, 0.f, 0.f}, av[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    if (half == 1) {
#pragma unroll
      for (int m = 0; m < MAXHD / 16; ++m) {
        const int r = w + 8 * (m + MAXHD / 16);
        ps[m] = (colok && r < d) ? *reinterpret_cast<const float4*>(P + (size_t)r * d + 4 * lane)
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
#pragma unroll
    for (int m = 0; m < MAXHD / 16; ++m) {
      const int r = w + 8 * (m + half * MAXHD / 16);
      if (r < d) {
        const float kr = ks[r], vr = vs[r];
        ak[0] = fmaf(kr, ps[m].x, ak[0]); ak[1] = fmaf(kr, ps[m].y, ak[1]);
        ak[2] = fmaf(kr, ps[m].z, ak[2]); ak[3] = fmaf(kr, ps[m].w, ak[3]);
        av[0] = fmaf(vr, ps[m].x, av[0]); av[1] = fmaf(vr, ps[m].y, av[1]);
        av[2] = fmaf(vr, ps[m].z, av[2]); av[3] = fmaf(vr, ps[m].w, av[3]);
      }
    }
  }
  if (colok) {
#pragma unroll
    for (int j = 0; j < 4; ++j) { red[w][4 * lane + j][0] = ak[j]; red[w][4 * lane + j][1] = av[j]; }
  }
  __syncthreads();
  const float dl = A.delta[chain];
  float m00, m01, m10, m11;
  sssd_factor(dots[0], dots[1], dots[2], dl, m00, m01, m10, m11);
  // Non-finite k, v, gate or factor: identity, as the reference's _solve_cayley
  // substitution does (sssd_attention.py:52-71).
  const bool ok = fin && isfinite(dl) && isfinite(m00) && isfinite(m01) && isfinite(m10) && isfinite(m11);
  float al[4], be[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float sa = 0.f, sb = 0.f;
    if (colok) {
#pragma unroll
      for (int ww = 0; ww < 8; ++ww) { sa += red[ww][4 * lane + j][0]; sb += red[ww][4 * lane + j][1]; }
    }
    al[j] = fmaf(m00, sa, m01 * sb);   // coefficient of k_r
    be[j] = fmaf(m10, sa, m11 * sb);   // coefficient of v_r
  }
  const float4 q4 = colok ? make_float4(qs[4 * lane], qs[4 * lane + 1], qs[4 * lane + 2], qs[4 * lane + 3])
                          : make_float4(0.f, 0.f, 0.f, 0.f);
  T* out = static_cast<T*>(A.sout) + vec;
  // pass 2: update, readout, store (rows re-read from L2); the readout partials of the
  // warp's rows w + 8 m are summed over the lanes together afterwards
  static_assert(MAXHD / 8 == 16, "16 rows per warp");
  float ov[16];
#pragma unroll 4
  for (int m = 0; m < MAXHD / 8; ++m) {
    const int r = w + 8 * m;
    ov[m] = 0.f;
    if (r >= d) continue;            // warp-uniform
    float4 x = colok ? *reinterpret_cast<const float4*>(P + (size_t)r * d + 4 * lane)
                     : make_float4(0.f, 0.f, 0.f, 0.f);
    if (ok) {
      const float kr = ks[r], vr = vs[r];
      x.x += fmaf(kr, al[0], vr * be[0]); x.y += fmaf(kr, al[1], vr * be[1]);
      x.z += fmaf(kr, al[2], vr * be[2]); x.w += fmaf(kr, al[3], vr * be[3]);
    }
    ov[m] = fmaf(x.w, q4.w, fmaf(x.z, q4.z, fmaf(x.y, q4.y, x.x * q4.x)));
    if (colok) __stcs(reinterpret_cast<float4*>(P + (size_t)r * d + 4 * lane), x);
  }
  const float o = warp_sum16_scatter(ov);
  const int r = w + 8 * warp_sum16_slot(lane);
  if ((lane & 1) == 0 && r < d) out[r] = from_f32<T>(o);
}

// SSSD-only step for head_dim 128 (the step's SSSD half when the CHAM half runs deferred):
// one CTA per (item, head) holds the 128 x 128 state on chip, rows 0..39 in registers
// (thread: rows w + 8m, m < 5, columns 4 lane .. 4 lane + 3) and rows 40..127 (44 KB,
// contiguous in memory) in shared memory by one bulk copy, so the state is read once and
// written once and four CTAs share an SM (all b*h chains of a decode batch of 64 in one
// wave).  Same arithmetic and summation order as sssd_part.
constexpr int SD_NREG = 5;                                  // row groups of 8 held in registers
constexpr int SD_SROWS = 128 - 8 * SD_NREG;                 // rows in shared memory
constexpr int SD_SMEM = SD_SROWS * 128 * 4;                 // 44 KB
template <typename T>
__global__ void __launch_bounds__(DT, 4) sssd_decode128_kernel(DecodeArgs A) {
  constexpr int HD = 128, NR = HD / 8;
  extern __shared__ __align__(128) float4 srow[];           // [SD_SROWS][HD / 4]
  __shared__ float ks[HD], vs[HD], qs[HD];
  // column partials of the warps, [warp][kᵀΨ x y z w, vᵀΨ x y z w][lane], and their sums
  // over the warps (warp c forms sum c, adding the warps in order as sssd_part does)
  __shared__ float red[8][8][HD / 4];
  __shared__ float rsum[8][HD / 4];
  __shared__ float dsc[8][4];
  __shared__ __align__(8) uint64_t sbar;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int chain = blockIdx.x;
  const size_t vec = (size_t)chain * HD;
  float* P = A.psi + (size_t)chain * HD * HD;
  if (tid == 0) {
    tc::mbar_init(&sbar, 1);
    tc::fence_mbar_init();
    tc::mbar_expect_tx(&sbar, SD_SMEM);
    tc::bulk_load(srow, P + 8 * SD_NREG * HD, SD_SMEM, &sbar);
  }
  float4 ps[SD_NREG];
#pragma unroll
  for (int m = 0; m < SD_NREG; ++m) ps[m] = __ldcs(reinterpret_cast<const float4*>(P + (size_t)(w + 8 * m) * HD) + lane);
  // The state depends on no earlier kernel of this step and is requested above; launched as
  // a programmatic dependent of the projection epilogue, the kernel waits here for k, v, q
  // and the gate.  The kernel after it (the per-head norm of the readout, a programmatic
  // dependent) may launch now; it waits for this grid's completion before reading.
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  float dots[4] = {0.f, 0.f, 0.f, 0.f};
  bool fin = true;
  if (tid < HD) {
    const float kx = ld1<T>(A.sk, vec + tid), vx = ld1<T>(A.sv, vec + tid);
    ks[tid] = kx; vs[tid] = vx; qs[tid] = ld1<T>(A.sq, vec + tid);
    dots[0] = kx * kx; dots[1] = vx * vx; dots[2] = kx * vx;
    fin = isfinite(kx) && isfinite(vx);
  }
  block_sum4(dots, fin, dsc);      // also makes ks/vs/qs and the barrier init visible
  const bool got = tc::mbar_wait(&sbar, 0, LPOLLS_SD);
  if (__syncthreads_or(!got)) {
    // the copy may still land: wait for it (bounded) before the CTA releases its memory
    if (tid == 0) {
      atomicOr(&g_decode_status, 2u);
      tc::mbar_wait(&sbar, 0, LPOLLS_SD);
    }
    return;
  }
  auto row_of = [&](int m) -> float4 {   // row w + 8m, this thread's 4 columns
    return m < SD_NREG ? ps[m] : srow[(w + 8 * m - 8 * SD_NREG) * (HD / 4) + lane];
  };
  float4 ak = make_float4(0.f, 0.f, 0.f, 0.f), av = ak;
#pragma unroll
  for (int m = 0; m < NR; ++m) {
    const float4 x = row_of(m);
    const float kr = ks[w + 8 * m], vr = vs[w + 8 * m];
    ak.x = fmaf(kr, x.x, ak.x); ak.y = fmaf(kr, x.y, ak.y);
    ak.z = fmaf(kr, x.z, ak.z); ak.w = fmaf(kr, x.w, ak.w);
    av.x = fmaf(vr, x.x, av.x); av.y = fmaf(vr, x.y, av.y);
    av.z = fmaf(vr, x.z, av.z); av.w = fmaf(vr, x.w, av.w);
  }
  red[w][0][lane] = ak.x; red[w][1][lane] = ak.y; red[w][2][lane] = ak.z; red[w][3][lane] = ak.w;
  red[w][4][lane] = av.x; red[w][5][lane] = av.y; red[w][6][lane] = av.z; red[w][7][lane] = av.w;
  __syncthreads();
  {
    float t = 0.f;
#pragma unroll
    for (int ww = 0; ww < 8; ++ww) t += red[ww][w][lane];
    rsum[w][lane] = t;
  }
  __syncthreads();
  const float dl = A.delta[chain];
  float m00, m01, m10, m11;
  sssd_factor(dots[0], dots[1], dots[2], dl, m00, m01, m10, m11);
  // Non-finite k, v, gate or factor: identity, as the reference's _solve_cayley
  // substitution does (sssd_attention.py:52-71).
  const bool ok = fin && isfinite(dl) && isfinite(m00) && isfinite(m01) && isfinite(m10) && isfinite(m11);
  const float4 sa = make_float4(rsum[0][lane], rsum[1][lane], rsum[2][lane], rsum[3][lane]);
  const float4 sb = make_float4(rsum[4][lane], rsum[5][lane], rsum[6][lane], rsum[7][lane]);
  // coefficients of k_r (al) and v_r (be) in each of the thread's columns
  const float4 al = make_float4(fmaf(m00, sa.x, m01 * sb.x), fmaf(m00, sa.y, m01 * sb.y),
                                fmaf(m00, sa.z, m01 * sb.z), fmaf(m00, sa.w, m01 * sb.w));
  const float4 be = make_float4(fmaf(m10, sa.x, m11 * sb.x), fmaf(m10, sa.y, m11 * sb.y),
                                fmaf(m10, sa.z, m11 * sb.z), fmaf(m10, sa.w, m11 * sb.w));
  const float4 q4 = make_float4(qs[4 * lane], qs[4 * lane + 1], qs[4 * lane + 2], qs[4 * lane + 3]);
  T* out = static_cast<T*>(A.sout) + vec;
  static_assert(NR == 16, "16 rows per warp");
  float ov[NR];
#pragma unroll
  for (int m = 0; m < NR; ++m) {
    const int r = w + 8 * m;
    float4 x = row_of(m);
    if (ok) {
      const float kr = ks[r], vr = vs[r];
      x.x += fmaf(kr, al.x, vr * be.x); x.y += fmaf(kr, al.y, vr * be.y);
      x.z += fmaf(kr, al.z, vr * be.z); x.w += fmaf(kr, al.w, vr * be.w);
    }
    __stcs(reinterpret_cast<float4*>(P + (size_t)r * HD) + lane, x);
    ov[m] = fmaf(x.w, q4.w, fmaf(x.z, q4.z, fmaf(x.y, q4.y, x.x * q4.x)));
  }
  const float o = warp_sum16_scatter(ov);   // (the readout sums as sssd_part forms them)
  if ((lane & 1) == 0) out[w + 8 * warp_sum16_slot(lane)] = from_f32<T>(o);
}

// ------------------------------------------------------------------------- CHAM
// Per-column quantities summed over the rows: kᵀHr, kᵀHi, vᵀHr, vᵀHi, and for
// FIRST_ORDER (Hᴴu)re, (Hᴴu)im.
constexpr int NQ = 6;

// Thread layout over a stripe (D rows x CWD columns, re and im): TPR = CWD / 4 threads per
// row (columns 4 c8 .. 4 c8 + 3), RPG = 256 / TPR rows per row group.
template <typename T, bool FO>
__device__ void cham_part(const DecodeArgs& A, int unit) {
  __shared__ float ks[MAXD], vs[MAXD];
  __shared__ float qs[CWD];
  __shared__ float red[8][CWD][NQ];
  __shared__ float coef[CWD][6];         // per column: α (re, im), β (re, im), z (re, im)
  __shared__ float dsc[8][4];
  __shared__ int last_flag;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int D = A.D;
  const int nst = D / CWD;
  const int item = unit / nst, stripe = unit % nst;
  const int c8 = lane % TPR;
  const int c0 = stripe * CWD + 4 * c8;
  const int rp = threadIdx.x / TPR;     // row within a row group
  constexpr int nq = FO ? NQ : 4;

  const size_t hoff = (size_t)item * D * D;
  float* Hr = A.hr + hoff;
  float* Hi = A.hi + hoff;
  const size_t voff = (size_t)item * D;
  float dots[4] = {0.f, 0.f, 0.f, 0.f};
  bool fin = true;
  const int cs0 = stripe * CWD;
  for (int i = tid; i < D; i += DT) {
    const float kx = ld1<T>(A.ck, voff + i), vx = ld1<T>(A.cv, voff + i), qx = ld1<T>(A.cq, voff + i);
    ks[i] = kx; vs[i] = vx;
    if (i >= cs0 && i < cs0 + CWD) qs[i - cs0] = qx;
    dots[0] += kx * kx; dots[1] += vx * vx; dots[2] += kx * vx; dots[3] += qx * qx;
    fin = fin && isfinite(kx) && isfinite(vx);
  }
  block_sum4(dots, fin, dsc);      // also makes ks/vs/qs visible
  const float* ur = A.u + (size_t)item * 2 * D;
  const float* ui = ur + D;

  // ---- pass 1: column sums over all rows
  float acc[NQ][4];
#pragma unroll
  for (int qn = 0; qn < NQ; ++qn)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[qn][j] = 0.f;
  for (int g0 = 0; g0 < D; g0 += RPG * UNR) {
    float4 xr[UNR], xi[UNR];
#pragma unroll
    for (int u = 0; u < UNR; ++u) {
      const int r = g0 + RPG * u + rp;
      if (r < D) {
        xr[u] = *reinterpret_cast<const float4*>(Hr + (size_t)r * D + c0);
        xi[u] = *reinterpret_cast<const float4*>(Hi + (size_t)r * D + c0);
      } else {
        xr[u] = xi[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
#pragma unroll
    for (int u = 0; u < UNR; ++u) {
      const int r = g0 + RPG * u + rp;
      if (r >= D) continue;
      const float kr = ks[r], vr = vs[r];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float hr_ = comp(xr[u], j), hi_ = comp(xi[u], j);
        acc[0][j] += kr * hr_; acc[1][j] += kr * hi_;
        acc[2][j] += vr * hr_; acc[3][j] += vr * hi_;
      }
      if (FO) {
        const float a = __ldg(ur + r), bq = __ldg(ui + r);
#pragma unroll
        for (int j = 0; j < 4; ++j) {   // conj(H) u
          const float hr_ = comp(xr[u], j), hi_ = comp(xi[u], j);
          acc[4][j] += hr_ * a + hi_ * bq;
          acc[5][j] += hr_ * bq - hi_ * a;
        }
      }
    }
  }
  // lanes l, l^8, l^16, l^24 share columns; then the 8 warps
#pragma unroll
  for (int qn = 0; qn < nq; ++qn)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float x = acc[qn][j];
#pragma unroll
      for (int o = TPR; o < 32; o <<= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
      acc[qn][j] = x;
    }
  if (lane < TPR) {
#pragma unroll
    for (int qn = 0; qn < nq; ++qn)
#pragma unroll
      for (int j = 0; j < 4; ++j) red[w][4 * lane + j][qn] = acc[qn][j];
  }
  __syncthreads();
  const float kk = dots[0], vv = dots[1], kv = dots[2], qq = dots[3];
  const float g = A.gamma[item];
  const float cc = 0.5f * g;
  const float dr = 1.f + cc * cc * (kk * vv - kv * kv);
  const float di = -2.f * cc * kv;
  const float m2 = dr * dr + di * di;
  const float fr = 2.f * cc * dr / m2;     // 2c / det
  const float fi = -2.f * cc * di / m2;
  // N00 = f (-c vv), N01 = N10 = f (c kv + i), N11 = f (-c kk)
  const float n00r = fr * (-cc * vv), n00i = fi * (-cc * vv);
  const float n11r = fr * (-cc * kk), n11i = fi * (-cc * kk);
  const float n01r = fr * (cc * kv) - fi, n01i = fr + fi * (cc * kv);
  // Non-finite k, v, gate or factor: identity (the reference's _solve_cham_cayley
  // substitution, cham_memory.py:54-96).
  const bool ok = fin && isfinite(g) && isfinite(n00r) && isfinite(n00i) && isfinite(n01r) &&
                  isfinite(n01i) && isfinite(n11r) && isfinite(n11i);
  float e2 = 0.f;
  if (tid < CWD) {
    const int c = tid;
    float t[NQ];
#pragma unroll
    for (int qn = 0; qn < NQ; ++qn) {
      float x = 0.f;
      if (qn < nq) {
#pragma unroll
        for (int ww = 0; ww < 8; ++ww) x += red[ww][c][qn];
      }
      t[qn] = x;
    }
    // α = N00 a + N01 b (coefficient of k_r), β = N01 a + N11 b (coefficient of v_r)
    coef[c][0] = n00r * t[0] - n00i * t[1] + n01r * t[2] - n01i * t[3];
    coef[c][1] = n00r * t[1] + n00i * t[0] + n01r * t[3] + n01i * t[2];
    coef[c][2] = n01r * t[0] - n01i * t[1] + n11r * t[2] - n11i * t[3];
    coef[c][3] = n01r * t[1] + n01i * t[0] + n11r * t[3] + n11i * t[2];
    const float qc = qs[c];
    if (FO) {
      coef[c][4] = 1.5f * qc - 0.5f * t[4];
      coef[c][5] = -0.5f * t[5];
      e2 = (t[4] - qc) * (t[4] - qc) + t[5] * t[5];
    } else {
      coef[c][4] = qc;
      coef[c][5] = 0.f;
    }
  }
  __syncthreads();
  float alr[4], ali[4], ber[4], bei[4], zr[4], zi[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float* cf = coef[4 * c8 + j];
    alr[j] = cf[0]; ali[j] = cf[1]; ber[j] = cf[2]; bei[j] = cf[3]; zr[j] = cf[4]; zi[j] = cf[5];
  }

  // ---- pass 2: update, store, readout partials (rows re-read from L2, last-read first)
  float* part = A.part + ((size_t)item * nst + stripe) * D;
  for (int g0 = (D - 1) / (RPG * UNR) * (RPG * UNR); g0 >= 0; g0 -= RPG * UNR) {
    float4 xr[UNR], xi[UNR];
#pragma unroll
    for (int u = 0; u < UNR; ++u) {
      const int r = g0 + RPG * u + rp;
      if (r < D) {
        xr[u] = __ldcs(reinterpret_cast<const float4*>(Hr + (size_t)r * D + c0));
        xi[u] = __ldcs(reinterpret_cast<const float4*>(Hi + (size_t)r * D + c0));
      } else {
        xr[u] = xi[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
#pragma unroll
    for (int u = 0; u < UNR; ++u) {
      const int r = g0 + RPG * u + rp;
      float o = 0.f;
      if (r < D) {
        if (ok) {
          const float kr = ks[r], vr = vs[r];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            comp(xr[u], j) += kr * alr[j] + vr * ber[j];
            comp(xi[u], j) += kr * ali[j] + vr * bei[j];
          }
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          o += comp(xr[u], j) * zr[j];
          if (FO) o -= comp(xi[u], j) * zi[j];
        }
        __stcs(reinterpret_cast<float4*>(Hr + (size_t)r * D + c0), xr[u]);
        __stcs(reinterpret_cast<float4*>(Hi + (size_t)r * D + c0), xi[u]);
      }
#pragma unroll
      for (int sh = 1; sh < TPR; sh <<= 1) o += __shfl_xor_sync(0xffffffffu, o, sh);
      if (c8 == 0 && r < D) part[r] = o;
    }
  }
  if (FO && w == 0) {   // |E q|² of this stripe's columns
    e2 = warp_sum(e2);
    if (tid == 0) atomicAdd(&A.err2[item], e2);
  }
  // publish the partials: CTA barrier, then one release fence and the stripe count
  __syncthreads();
  if (tid == 0) {
    __threadfence();
    const unsigned int prev = atomicAdd(&A.cnt[item], 1u);
    last_flag = (prev == (unsigned int)(nst - 1));
    if (last_flag) __threadfence();
  }
  __syncthreads();
  if (last_flag) {
    const float* pb = A.part + (size_t)item * nst * D;
    T* y = static_cast<T*>(A.cout) + voff;
    for (int i = tid; i < D; i += DT) {
      float s = 0.f;
#pragma unroll 8
      for (int st = 0; st < nst; ++st) s += __ldcg(pb + (size_t)st * D + i);
      y[i] = from_f32<T>(s);
    }
    if (FO && tid == 0) {
      const float err = __ldcg(&A.err2[item]);
      if (!(err <= DRIFT_TOL * DRIFT_TOL * qq)) atomicOr(&g_decode_status, 1u);
    }
  }
}

// ------------------------------------------------------------------------- lazy CHAM
// Deferred hologram updates (unitary readout).  The stored state S lags the true state by
// the pending rank-2 factors of up to P earlier steps:
//     H = S + sum_j A_j B_j,   A_j = [k_j v_j] (D x 2, real),   B_j = N_j [k_jᵀH_j; v_jᵀH_j]
// (2 x D, complex; H_j the state before step j).  A step needs kᵀH, vᵀH and Re(H' q):
//     kᵀH = kᵀS + sum_j (kᵀk_j) B_j0 + (kᵀv_j) B_j1,      likewise vᵀH,
//     Re(H' q) = S_re q + sum_j (k_j Re(B_j0 q) + v_j Re(B_j1 q)) + k Re(B0' q) + v Re(B1' q)
// with B' = N [kᵀH; vᵀH] the step's new factor, so one read pass over S suffices.  A step
// that finds all P slots taken first folds them into S during its pass (read + write) and
// starts the list again with its own factor.  Exact up to fp32 rounding order.
// Pending storage per item: count (int) | A [P][2][D] | B [P][4][D] (row 0 re, im; row 1 re, im).
constexpr int LP_MAX = 16;

struct LazyArgs {
  const void* cq; const void* ck; const void* cv; const float* gamma;
  float* hr; float* hi; void* cout;
  int* pcount;                 // [b]
  float* pa;                   // [b][P][2][D]
  float* pb;                   // [b][P][4][D]
  float* g;                    // [b][LP_MAX][4]: kᵀk_j, kᵀv_j, vᵀk_j, vᵀv_j
  float* bq;                   // [b][LP_MAX][2]: Re(B_j0 q), Re(B_j1 q)
  float* part;                 // [b][D/32][D] readout partials
  float* cqp;                  // [b][D/32][4] per stripe: kᵀH q (re, im), vᵀH q (re, im)
  int* pcold;                  // [b] the pending counts as this step found them
  const void* y; long long yld;   // projected steps: the raw projection rows (q | k | v | gate)
  void* pq; void* pk; void* pv; float* pg;   // ... and where lazy_pre_kernel leaves q, k, v, gamma
  int b, D, P, nst;            // nst: column stripes of lazy_cham_kernel
};

// The 2x2 complex factor N of a CHAM Cayley step for gate g (c = g / 2) from the Gram
// entries kk, vv, kv:  N = 2c / det [[-c vv, c kv + i], [c kv + i, -c kk]],
// det = 1 + c² (kk vv - kv²) - 2 i c kv; `ok` is false when k, v, the gate or N is not
// finite, and such a step is the identity (cham_memory.py:54-96).  The stripe kernel and
// the readout kernel of a step both form N here, from the same Gram sums.
struct ChamN {
  float n00r, n00i, n01r, n01i, n11r, n11i;
  bool ok;
};
__device__ __forceinline__ ChamN cham_factor(float kk, float vv, float kv, float g, bool fin) {
  ChamN n;
  const float cc = 0.5f * g;
  const float dr = 1.f + cc * cc * (kk * vv - kv * kv);
  const float di = -2.f * cc * kv;
  const float m2 = dr * dr + di * di;
  const float fr = 2.f * cc * dr / m2;
  const float fi = -2.f * cc * di / m2;
  n.n00r = fr * (-cc * vv); n.n00i = fi * (-cc * vv);
  n.n11r = fr * (-cc * kk); n.n11i = fi * (-cc * kk);
  n.n01r = fr * (cc * kv) - fi; n.n01i = fr + fi * (cc * kv);
  n.ok = fin && isfinite(g) && isfinite(n.n00r) && isfinite(n.n00i) && isfinite(n.n01r) && isfinite(n.n01i) &&
         isfinite(n.n11r) && isfinite(n.n11i);
  return n;
}

// k, v (and the stripe's q columns when qs != nullptr) of one item into shared memory,
// with the Gram sums kk, vv, kv, qq (per thread; block_sum4 finishes them) and the
// finiteness of k, v.  Four elements per load when the bases allow it; every kernel that
// forms a step's N calls this with the same thread count, so their sums agree bitwise.
template <typename T>
__device__ __forceinline__ void load_kvq(const LazyArgs& A, size_t voff, int D, float* ks, float* vs, float* qs,
                                         int cs0, int W, float (&dots)[4], bool& fin) {
  const int tid = threadIdx.x;
  const bool vec4 = ((reinterpret_cast<uintptr_t>(A.ck) | reinterpret_cast<uintptr_t>(A.cv) |
                      reinterpret_cast<uintptr_t>(A.cq)) & (4 * sizeof(T) - 1)) == 0;
  if (vec4) {
    for (int i = 4 * tid; i < D; i += 4 * DT) {
      float kx[4], vx[4], qx[4];
      ld4<T>(A.ck, voff + i, kx);
      ld4<T>(A.cv, voff + i, vx);
      ld4<T>(A.cq, voff + i, qx);
      *reinterpret_cast<float4*>(ks + i) = make_float4(kx[0], kx[1], kx[2], kx[3]);
      *reinterpret_cast<float4*>(vs + i) = make_float4(vx[0], vx[1], vx[2], vx[3]);
      if (qs != nullptr && i >= cs0 && i < cs0 + W)
        *reinterpret_cast<float4*>(qs + i - cs0) = make_float4(qx[0], qx[1], qx[2], qx[3]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        dots[0] += kx[j] * kx[j]; dots[1] += vx[j] * vx[j]; dots[2] += kx[j] * vx[j]; dots[3] += qx[j] * qx[j];
        fin = fin && isfinite(kx[j]) && isfinite(vx[j]);
      }
    }
  } else {
    for (int i = tid; i < D; i += DT) {
      const float kx = ld1<T>(A.ck, voff + i), vx = ld1<T>(A.cv, voff + i), qx = ld1<T>(A.cq, voff + i);
      ks[i] = kx; vs[i] = vx;
      if (qs != nullptr && i >= cs0 && i < cs0 + W) qs[i - cs0] = qx;
      dots[0] += kx * kx; dots[1] += vx * vx; dots[2] += kx * vx; dots[3] += qx * qx;
      fin = fin && isfinite(kx) && isfinite(vx);
    }
  }
}

// The dot products between this step's k, v, q and the pending factors: one CTA per
// (item, factor slot) (slots past the item's count return at once), each thread a few
// rows of the six contiguous vectors, then a block reduction.  The slot-0 CTA of each item
// also keeps the item's pending count for lazy_out_kernel (which rewrites the count).
//
// PROJ: the step starts from the layer's raw projection row y = q | k | v | gate and this
// kernel is also its projection epilogue (the mixer prologue's CHAM row, one launch fewer):
// v through SiLU rounded to the input type (as the reference's SiLU output is), q, k, v
// L2-normalised (eps 1e-12) and rounded to the input type, gamma = 0.1 sigmoid(y_gate)
// (cham_memory.py:129-153).  Every CTA of the item that has a dot product to form
// normalises the row itself (the same threads and order, so bitwise alike) and the slot-0
// CTA stores q, k, v and gamma for the two kernels after it.
template <typename T, bool PROJ>
__global__ void __launch_bounds__(DT) lazy_pre_kernel(LazyArgs A) {
  __shared__ float red[DT / 32][6];
  __shared__ float nsc[DT / 32][4];
  constexpr int NPT = MAXD / DT;   // row elements per thread (PROJ)
  const int D = A.D, P = A.P;
  const int item = blockIdx.x / P, j = blockIdx.x % P;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  // launched as a programmatic dependent of the projection epilogue (k, v, q) or, PROJ, of
  // the projection itself; the stripe kernel that follows may start its hologram loads
  // once every CTA here has started
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int p = A.pcount[item];
  if (j == 0 && tid == 0) A.pcold[item] = p;
  const bool dots = p < P && j < p;   // (a folding step needs none of them)
  if (!dots && !(PROJ && j == 0)) return;
  const size_t voff = (size_t)item * D;
  float nq[NPT], nk[NPT], nv[NPT];
  if constexpr (PROJ) {
    const size_t yr = (size_t)item * A.yld;
    float ss[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int u = 0; u < NPT; ++u) {
      const int i = tid + DT * u;
      nq[u] = nk[u] = nv[u] = 0.f;
      if (i < D) {
        nq[u] = ld1<T>(A.y, yr + i);
        nk[u] = ld1<T>(A.y, yr + D + i);
        const float xv = ld1<T>(A.y, yr + 2 * (size_t)D + i);
        nv[u] = to_f32(from_f32<T>(xv / (1.f + expf(-xv))));
        ss[0] += nq[u] * nq[u]; ss[1] += nk[u] * nk[u]; ss[2] += nv[u] * nv[u];
      }
    }
    bool all = true;
    block_sum4(ss, all, nsc);
    const float iq = 1.f / fmaxf(sqrtf(ss[0]), 1e-12f), ik = 1.f / fmaxf(sqrtf(ss[1]), 1e-12f),
                iv = 1.f / fmaxf(sqrtf(ss[2]), 1e-12f);
#pragma unroll
    for (int u = 0; u < NPT; ++u) {
      const int i = tid + DT * u;
      if (i < D) {
        const T tq = from_f32<T>(nq[u] * iq), tk = from_f32<T>(nk[u] * ik), tv = from_f32<T>(nv[u] * iv);
        nq[u] = to_f32(tq); nk[u] = to_f32(tk); nv[u] = to_f32(tv);
        if (j == 0) {
          static_cast<T*>(A.pq)[voff + i] = tq;
          static_cast<T*>(A.pk)[voff + i] = tk;
          static_cast<T*>(A.pv)[voff + i] = tv;
        }
      }
    }
    if (j == 0 && tid == 0) A.pg[item] = 0.1f * (1.f / (1.f + expf(-ld1<T>(A.y, yr + 3 * (size_t)D))));
    if (!dots) return;
  }
  const float* a0 = A.pa + ((size_t)item * P + j) * 2 * D;
  const float* a1 = a0 + D;
  const float* b0 = A.pb + ((size_t)item * P + j) * 4 * D;   // Re(B_j0)
  const float* b1 = b0 + 2 * (size_t)D;                       // Re(B_j1)
  float x[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};   // k.k_j, k.v_j, v.k_j, v.v_j, Re(B_j0) q, Re(B_j1) q
  if constexpr (PROJ) {
#pragma unroll
    for (int u = 0; u < NPT; ++u) {
      const int i = tid + DT * u;
      if (i < D) {
        const float kx = nk[u], vx = nv[u], qx = nq[u];
        const float y0 = a0[i], y1 = a1[i];
        x[0] += kx * y0; x[1] += kx * y1; x[2] += vx * y0; x[3] += vx * y1;
        x[4] += b0[i] * qx; x[5] += b1[i] * qx;
      }
    }
  } else {
#pragma unroll 4
    for (int i = tid; i < D; i += DT) {
      const float kx = ld1<T>(A.ck, voff + i), vx = ld1<T>(A.cv, voff + i), qx = ld1<T>(A.cq, voff + i);
      const float y0 = a0[i], y1 = a1[i];
      x[0] += kx * y0; x[1] += kx * y1; x[2] += vx * y0; x[3] += vx * y1;
      x[4] += b0[i] * qx; x[5] += b1[i] * qx;
    }
  }
#pragma unroll
  for (int e = 0; e < 6; ++e) {
    x[e] = warp_sum(x[e]);
    if (lane == 0) red[w][e] = x[e];
  }
  __syncthreads();
  if (tid < 6) {
    float t = 0.f;
#pragma unroll
    for (int ww = 0; ww < DT / 32; ++ww) t += red[ww][tid];
    if (tid < 4) A.g[((size_t)item * LP_MAX + j) * 4 + tid] = t;
    else A.bq[((size_t)item * LP_MAX + j) * 2 + (tid - 4)] = t;
  }
}

// The stripe (W = 64 columns when D is a multiple of 64, else 32) streams through NSTG
// shared-memory stages of 16 KB (ROWS rows: re box | im box, W floats a row; unswizzled,
// or for the tensor-core fold two 32-column swizzled boxes per plane, see sw_off), loaded by
// TMA: thread 0 keeps every stage in flight, so the read pass is not limited by
// the loads a thread can hold in registers.  Each thread takes two rows of four columns
// per stage.  A folding step updates each stage in place and TMA-stores it back.  The
// wider stripe halves the CTAs, and with them the per-CTA set-up (k, v, q and the pending
// factors' columns) and reductions, for the same bytes streamed.
constexpr int NSTG = 5;                      // stages
template <int W, bool MF = false>
struct LazyGeom {
  static constexpr int TPR = W / 4;                 // threads per row
  static constexpr int RPG = DT / TPR;              // rows per row group
  static constexpr int ROWS = 2 * RPG;              // rows per stage
  static constexpr int STAGE = 2 * ROWS * W * 4;    // bytes per stage (16 KB)
  // dynamic smem: stages | A rows of the stage (fold steps): fp32 [LP_MAX][2][ROWS], two
  // buffers of [LP_MAX / 2][2][ROWS] when P <= LP_MAX / 2; with the tensor-core fold (MF) two
  // buffers of three bf16 pieces [ROWS][8 words] | pending B over the stripe [P][4][W] |
  // ks [D] | vs [D] | barriers
  static constexpr int AS_OFF = NSTG * STAGE;
  static constexpr int AS_BYTES = MF ? 2 * 3 * ROWS * 8 * 4 : LP_MAX * 2 * ROWS * 4;
  static constexpr int PBS_OFF = AS_OFF + AS_BYTES;
  __host__ __device__ static size_t ks_off(int P) { return PBS_OFF + (size_t)P * 4 * W * 4; }
  static size_t smem(int D, int P) { return ks_off(P) + 2 * (size_t)D * 4 + 8 * NSTG + 16; }
};
static_assert(LazyGeom<32>::STAGE == 16384 && LazyGeom<64>::STAGE == 16384, "16 KB stages");
static_assert(LazyGeom<64, true>::ROWS == 32, "the tensor-core fold tiles a stage as 2 x 16 rows");

// The tensor-core fold's stage layout: each plane of a 64-column stage is two 32-column
// boxes of 32 rows x 128 bytes, stored by TMA with the 128-byte swizzle (16-byte chunk
// index XOR row mod 8), so that the m16n8 accumulator fragments (eight rows by two chunks
// per warp) and the read pass's float4s both spread over all banks.  Float offset of
// (row r, column c) within a plane:
__device__ __forceinline__ int sw_off(int r, int c) {
  return (c >> 5) * 1024 + r * 32 + ((((c & 31) >> 2) ^ (r & 7)) << 2) + (c & 3);
}

// D += A B for one m16n8k16 tile, bf16 operands, fp32 accumulators (PTX mma.sync; the
// fragment layouts are the ISA's: A rows gid / gid + 8, k pairs 2 tig (+8); B k pairs
// 2 tig (+8), column gid; D rows gid / gid + 8, columns 2 tig, 2 tig + 1).
__device__ __forceinline__ void mma_m16n8k16_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// x = hi + mid + lo as three bf16 values (each the round-to-nearest of what the previous
// ones leave; the residuals are exact in fp32), 24 significant bits in all.
__device__ __forceinline__ void split3_bf16(float x, uint16_t& h, uint16_t& m, uint16_t& l) {
  const __nv_bfloat16 bh = __float2bfloat16_rn(x);
  const float r1 = x - __bfloat162float(bh);
  const __nv_bfloat16 bm = __float2bfloat16_rn(r1);
  const __nv_bfloat16 bl = __float2bfloat16_rn(r1 - __bfloat162float(bm));
  h = __bfloat16_as_ushort(bh); m = __bfloat16_as_ushort(bm); l = __bfloat16_as_ushort(bl);
}
constexpr uint32_t LPOLLS = 1u << 22;

//
// MF (bf16 steps, W = 64, P <= 8): the stages are in the swizzled layout of sw_off and a
// folding step runs S += sum_j A_j B_j on the tensor cores, as a 32 x 64 x 2P product per
// plane and stage (mma.sync m16n8k16; each warp one plane, 16 rows, 32 columns).  A (the
// pending factors' k, v rows) enters as bf16 pieces hi + mid + lo (a bf16 step's k, v are
// exact in the first; the others are zero and their products skipped, warp by warp), B
// (the factors' columns over the stripe, fp32) as three bf16 pieces held in registers for
// the whole pass.  The update is accumulated from zero and added to the state in fp32, so
// the tensor cores' rounding is relative to the update, not to the state.
template <typename T, int W, bool MF>
__global__ void __launch_bounds__(DT, 2)
lazy_cham_kernel(LazyArgs A, const __grid_constant__ CUtensorMap tm_r, const __grid_constant__ CUtensorMap tm_i) {
  static_assert(!MF || W == 64, "the tensor-core fold tiles 64-column stripes");
  using G = LazyGeom<W, MF>;
  constexpr int TPR = G::TPR, RPG = G::RPG, LROWS = G::ROWS, LSTAGE = G::STAGE;
  extern __shared__ __align__(1024) unsigned char lsm[];
  float* as = reinterpret_cast<float*>(lsm + G::AS_OFF);   // [j][kv][row of the stage] (MF: bf16 pieces)
  float* pbs = reinterpret_cast<float*>(lsm + G::PBS_OFF);  // pending B_j over the stripe: [j][4][W]
  float* ks = reinterpret_cast<float*>(lsm + G::ks_off(A.P));
  float* vs = ks + A.D;
  uint64_t* full = reinterpret_cast<uint64_t*>(vs + A.D);   // TMA landed (8-byte aligned: D % 32 == 0)
  __shared__ __align__(16) float qs[W];
  __shared__ float red[8][W][4];
  __shared__ float gs[LP_MAX][4];
  __shared__ float dsc[8][4];
  __shared__ float cq4[8][4];
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int D = A.D, P = A.P;
  const int nst = D / W;
  const int item = blockIdx.x / nst, stripe = blockIdx.x % nst;
  const int c8 = lane % TPR;
  const int rp = threadIdx.x / TPR;       // rows rp and rp + RPG of each stage
  const int NRB = D / LROWS;
  auto stage = [&](int s) { return reinterpret_cast<float*>(lsm + s * LSTAGE); };
  auto issue = [&](int rb) {
    const int s = rb % NSTG;
    const int y = item * D + rb * LROWS;
    tc::mbar_expect_tx(&full[s], LSTAGE);
    if constexpr (MF) {   // per plane two 32-column boxes (x stays a multiple of 32 floats)
      tc::tma_load_2d(stage(s), &tm_r, stripe * W, y, &full[s]);
      tc::tma_load_2d(stage(s) + 1024, &tm_r, stripe * W + 32, y, &full[s]);
      tc::tma_load_2d(stage(s) + 2048, &tm_i, stripe * W, y, &full[s]);
      tc::tma_load_2d(stage(s) + 3072, &tm_i, stripe * W + 32, y, &full[s]);
    } else {
      tc::tma_load_2d(stage(s), &tm_r, stripe * W, y, &full[s]);
      tc::tma_load_2d(stage(s) + LROWS * W, &tm_i, stripe * W, y, &full[s]);
    }
  };
  auto store = [&](int rb, const float* sr, const float* si) {
    const int y = item * D + rb * LROWS;
    if constexpr (MF) {
      tc::tma_store_2d(&tm_r, stripe * W, y, sr);
      tc::tma_store_2d(&tm_r, stripe * W + 32, y, sr + 1024);
      tc::tma_store_2d(&tm_i, stripe * W, y, si);
      tc::tma_store_2d(&tm_i, stripe * W + 32, y, si + 1024);
    } else {
      tc::tma_store_2d(&tm_r, stripe * W, y, sr);
      tc::tma_store_2d(&tm_i, stripe * W, y, si);
    }
  };
  // float offset of a thread's float4 (row i, columns 4 c8 ..) within a stage plane
  auto xoff = [&](int i) { return MF ? sw_off(i, 4 * c8) : i * W + 4 * c8; };
  if (MF && (tc::smem_addr(lsm) & 1023u)) {   // the swizzle needs 1024-byte aligned stages
    if (tid == 0) atomicOr(&g_decode_status, 2u);   // (reported as a pass that did not run)
    return;
  }
  // The hologram stages depend on no earlier kernel of this step: they are requested
  // before griddepcontrol.wait, which (this kernel being launched as a programmatic
  // dependent of lazy_pre_kernel) returns once lazy_pre_kernel and, through it, the
  // projection epilogue are complete and their writes visible.
  if (tid == 0) {
    for (int s = 0; s < NSTG; ++s) tc::mbar_init(&full[s], 1);
    tc::fence_mbar_init();
    for (int rb = 0; rb < NSTG && rb < NRB; ++rb) issue(rb);
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int p = A.pcount[item];
  const bool fold = p >= P;               // fold the P pending factors into S this step
  const int np = fold ? P : p;            // pending factors read by this step
  const int snew = fold ? 0 : p;          // slot of this step's factor

  const size_t voff = (size_t)item * D;
  const float* pa = A.pa + (size_t)item * P * 2 * D;
  float* pb = A.pb + (size_t)item * P * 4 * D;
  float dots[4] = {0.f, 0.f, 0.f, 0.f};
  bool fin = true;
  const int cs0 = stripe * W;
  // The small per-step inputs, all requested before any is used: the pending factors' B
  // rows over this stripe (float4s) and their dot products with this step's k, v (gs),
  // then k, v, q.
  constexpr int PBV = (LP_MAX * W + DT - 1) / DT;   // float4s of B per thread, at most
  float4 pbv[PBV];
#pragma unroll
  for (int u = 0; u < PBV; ++u) {
    const int e = tid + DT * u;   // W float4s per factor: 4 rows x W / 4
    if (e < np * W) {
      const int j = e / W, rr = (e / (W / 4)) % 4, c4 = e % (W / 4);
      pbv[u] = *reinterpret_cast<const float4*>(pb + ((size_t)j * 4 + rr) * D + cs0 + 4 * c4);
    }
  }
  const float gv = (!fold && tid < 4 * p) ? A.g[((size_t)item * LP_MAX + tid / 4) * 4 + tid % 4] : 0.f;
  load_kvq<T>(A, voff, D, ks, vs, qs, cs0, W, dots, fin);
#pragma unroll
  for (int u = 0; u < PBV; ++u) {
    const int e = tid + DT * u;
    if (e < np * W) {
      const int j = e / W, rr = (e / (W / 4)) % 4, c4 = e % (W / 4);
      *reinterpret_cast<float4*>(pbs + (j * 4 + rr) * W + 4 * c4) = pbv[u];
    }
  }
  if (!fold && tid < 4 * p) gs[tid / 4][tid % 4] = gv;
  // Fold steps with P <= LP_MAX / 2 double-buffer the A rows: stage rb + 1's rows are
  // loaded into registers during stage rb and stored to the other buffer after its
  // compute, so no stage waits for them.
  const bool adbl = fold && P <= LP_MAX / 2;
  const int an = P * 2 * LROWS;            // A values per stage
  float apre[LP_MAX / 2];
  auto a_fetch = [&](int rb) {
    if constexpr (MF) {   // (k_j, v_j) of row e % LROWS for factor j = e / LROWS, one pair a thread
      const int e = tid;
      if (e < P * LROWS) {
        const float* src = pa + (size_t)(2 * (e / LROWS)) * D + rb * LROWS + e % LROWS;
        apre[0] = __ldg(src);
        apre[1] = __ldg(src + D);
      }
    } else {
#pragma unroll
      for (int u = 0; u < LP_MAX / 2; ++u) {
        const int e = tid + DT * u;
        if (e < an) apre[u] = __ldg(pa + (size_t)(e / LROWS) * D + rb * LROWS + e % LROWS);
      }
    }
  };
  // MF: the A buffer of a stage is three arrays (hi, mid, lo) of [row][8 words], each word a
  // (k_j, v_j) bf16 pair; word c = 2 (j & 3) + (j >> 2) of a row sits at position
  // c ^ ((row >> 2) & 7), so that the writes (a warp: one factor, 32 rows) and the fragment
  // reads (8 rows x 4 factors) both reach 32 distinct banks.
  constexpr int AWORDS = LROWS * 8;      // words per piece array
  auto a_word = [](int row, int c) { return row * 8 + (c ^ ((row >> 2) & 7)); };
  auto a_put = [&](int rb) {
    if constexpr (MF) {
      uint32_t* dst = reinterpret_cast<uint32_t*>(as) + (rb & 1) * 3 * AWORDS;
      const int e = tid;
      if (e < P * LROWS) {
        const int j = e / LROWS, row = e % LROWS;
        const int wd = a_word(row, 2 * (j & 3) + (j >> 2));
        uint16_t hk, mk, lk, hv, mv, lv;
        split3_bf16(apre[0], hk, mk, lk);
        split3_bf16(apre[1], hv, mv, lv);
        dst[wd] = hk | ((uint32_t)hv << 16);
        dst[AWORDS + wd] = mk | ((uint32_t)mv << 16);
        dst[2 * AWORDS + wd] = lk | ((uint32_t)lv << 16);
      }
    } else {
      float* dst = as + (rb & 1) * (LP_MAX / 2) * 2 * LROWS;
#pragma unroll
      for (int u = 0; u < LP_MAX / 2; ++u) {
        const int e = tid + DT * u;
        if (e < an) dst[e] = apre[u];
      }
    }
  };
  if (MF && fold) {   // the words of factors j >= P (never written by a_put) are zero
    uint32_t* aw = reinterpret_cast<uint32_t*>(as);
    for (int e = tid; e < 2 * 3 * AWORDS; e += DT) {
      const int row = (e % AWORDS) >> 3;
      const int c = (e & 7) ^ ((row >> 2) & 7);
      if ((c >> 1) + 4 * (c & 1) >= P) aw[e] = 0u;
    }
  }
  if (adbl) {
    a_fetch(0);
    a_put(0);
    if (NRB > 1) a_fetch(1);
  }
  block_sum4(dots, fin, dsc);      // also makes ks/vs/qs/pbs/gs, stage 0's A rows and the barrier inits visible
  // every read of the pending count is behind us: lazy_out_kernel may start (it waits for
  // this grid's completion before it reads what the stripes write)
  asm volatile("griddepcontrol.launch_dependents;");

  // MF fold: this warp's plane, 16-row half of the stage, 32-column box; its B fragments
  // (factor j = tig, tig + 4; column gid of each 8-column tile) in three bf16 pieces
  const int gid = lane >> 2, tig = lane & 3;
  const int fpl = w >> 2, fmt = (w >> 1) & 1, fnh = w & 1;
  uint32_t bfr[3][4][2];
#pragma unroll
  for (int t = 0; t < 3; ++t)
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) bfr[t][nt][0] = bfr[t][nt][1] = 0u;
  if (MF && fold) {
#pragma unroll
    for (int nt = 0; nt < 4; ++nt)
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        const int j = tig + 4 * hf, n = fnh * 32 + nt * 8 + gid;
        float x0 = 0.f, x1 = 0.f;    // rows k = 2j (with k_j) and 2j + 1 (with v_j) of B
        if (j < P) {
          x0 = pbs[(j * 4 + fpl) * W + n];
          x1 = pbs[(j * 4 + 2 + fpl) * W + n];
        }
        uint16_t h0, m0, l0, h1, m1, l1;
        split3_bf16(x0, h0, m0, l0);
        split3_bf16(x1, h1, m1, l1);
        bfr[0][nt][hf] = h0 | ((uint32_t)h1 << 16);
        bfr[1][nt][hf] = m0 | ((uint32_t)m1 << 16);
        bfr[2][nt][hf] = l0 | ((uint32_t)l1 << 16);
      }
  }

  // ---- one pass: column sums kᵀS, vᵀS and the readout partials S_re q, folding first
  float acc[4][4];
#pragma unroll
  for (int qn = 0; qn < 4; ++qn)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[qn][j] = 0.f;
  float* part = A.part + ((size_t)item * nst + stripe) * D;
  int issued = NSTG < NRB ? NSTG : NRB;    // row blocks whose loads thread 0 has issued
  bool failed = false;
  for (int rb = 0; rb < NRB; ++rb) {
    const int s = rb % NSTG;
    // (a wait that gives up still reaches this stage's barrier, which votes on it)
    const bool got = tc::mbar_wait(&full[s], (rb / NSTG) & 1, LPOLLS);
    float* sr = stage(s);
    float* si = sr + LROWS * W;
    if (MF && fold) {   // S += sum_j A_j B_j on the tensor cores, in place in the stage
      const uint32_t* ab = reinterpret_cast<const uint32_t*>(as) + (rb & 1) * 3 * AWORDS;
      const int r0 = fmt * 16 + gid;
      uint32_t af[3][4];
#pragma unroll
      for (int t = 0; t < 3; ++t) {   // rows r0, r0 + 8; factors tig (k 2 tig, 2 tig + 1) and tig + 4
        af[t][0] = ab[t * AWORDS + a_word(r0, 2 * tig)];
        af[t][1] = ab[t * AWORDS + a_word(r0 + 8, 2 * tig)];
        af[t][2] = ab[t * AWORDS + a_word(r0, 2 * tig + 1)];
        af[t][3] = ab[t * AWORDS + a_word(r0 + 8, 2 * tig + 1)];
      }
      const bool use_m = __any_sync(0xffffffffu, (af[1][0] | af[1][1] | af[1][2] | af[1][3]) != 0u);
      const bool use_l = __any_sync(0xffffffffu, (af[2][0] | af[2][1] | af[2][2] | af[2][3]) != 0u);
      float* tile = (fpl ? si : sr) + fnh * 1024;
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
        float d[4] = {0.f, 0.f, 0.f, 0.f};   // smallest products first
        if (use_l) mma_m16n8k16_bf16(d, af[2], bfr[0][nt][0], bfr[0][nt][1]);
        if (use_m) {
          mma_m16n8k16_bf16(d, af[1], bfr[1][nt][0], bfr[1][nt][1]);
          mma_m16n8k16_bf16(d, af[1], bfr[0][nt][0], bfr[0][nt][1]);
        }
        mma_m16n8k16_bf16(d, af[0], bfr[2][nt][0], bfr[2][nt][1]);
        mma_m16n8k16_bf16(d, af[0], bfr[1][nt][0], bfr[1][nt][1]);
        mma_m16n8k16_bf16(d, af[0], bfr[0][nt][0], bfr[0][nt][1]);
        // rows r0 and r0 + 8 (same swizzle phase), columns 8 nt + 2 tig + {0, 1} of the box
        const int o = r0 * 32 + (((2 * nt + (tig >> 1)) ^ (r0 & 7)) << 2) + (tig & 1) * 2;
        float2* p0 = reinterpret_cast<float2*>(tile + o);
        float2* p1 = reinterpret_cast<float2*>(tile + o + 8 * 32);
        float2 c0 = *p0, c1 = *p1;
        c0.x += d[0]; c0.y += d[1]; c1.x += d[2]; c1.y += d[3];
        *p0 = c0;
        *p1 = c1;
      }
      __syncthreads();   // the folded stage, before the pass below reads other warps' rows
      if (rb + 1 < NRB) {   // the other A buffer was last read in stage rb - 1
        a_put(rb + 1);
        if (rb + 2 < NRB) a_fetch(rb + 2);
      }
    }
    float4 xr2[2], xi2[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int i = rp + RPG * h;
      xr2[h] = *reinterpret_cast<const float4*>(sr + xoff(i));
      xi2[h] = *reinterpret_cast<const float4*>(si + xoff(i));
    }
    if (!MF && fold) {   // S += sum_j A_j B_j; each factor's four columns of B serve both rows
      const float* asb = as;
      if (adbl) {
        asb = as + (rb & 1) * (LP_MAX / 2) * 2 * LROWS;
      } else {
        for (int e = tid; e < an; e += DT)   // the stage's rows of every A_j (coalesced)
          as[e] = __ldg(pa + (size_t)(e / LROWS) * D + rb * LROWS + e % LROWS);
        __syncthreads();
      }
#pragma unroll 2
      for (int j = 0; j < P; ++j) {
        const float4 b0r = *reinterpret_cast<const float4*>(pbs + (j * 4 + 0) * W + 4 * c8);
        const float4 b0i = *reinterpret_cast<const float4*>(pbs + (j * 4 + 1) * W + 4 * c8);
        const float4 b1r = *reinterpret_cast<const float4*>(pbs + (j * 4 + 2) * W + 4 * c8);
        const float4 b1i = *reinterpret_cast<const float4*>(pbs + (j * 4 + 3) * W + 4 * c8);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int i = rp + RPG * h;
          const float a0 = asb[(2 * j) * LROWS + i], a1 = asb[(2 * j + 1) * LROWS + i];
#pragma unroll
          for (int jj = 0; jj < 4; ++jj) {
            comp(xr2[h], jj) += a0 * compc(b0r, jj) + a1 * compc(b1r, jj);
            comp(xi2[h], jj) += a0 * compc(b0i, jj) + a1 * compc(b1i, jj);
          }
        }
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int i = rp + RPG * h;
        *reinterpret_cast<float4*>(sr + i * W + 4 * c8) = xr2[h];
        *reinterpret_cast<float4*>(si + i * W + 4 * c8) = xi2[h];
      }
      if (adbl && rb + 1 < NRB) {   // the other buffer was last read in stage rb - 1
        a_put(rb + 1);
        if (rb + 2 < NRB) a_fetch(rb + 2);
      }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int i = rp + RPG * h, r = rb * LROWS + i;
      const float4 xr = xr2[h], xi = xi2[h];
      const float kr = ks[r], vr = vs[r];
      float o = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float hr_ = compc(xr, j), hi_ = compc(xi, j);
        acc[0][j] += kr * hr_; acc[1][j] += kr * hi_;
        acc[2][j] += vr * hr_; acc[3][j] += vr * hi_;
        o += hr_ * qs[4 * c8 + j];
      }
#pragma unroll
      for (int sh = 1; sh < TPR; sh <<= 1) o += __shfl_xor_sync(0xffffffffu, o, sh);
      if (c8 == 0) part[r] = o;
    }
    if (fold) tc::fence_proxy_async();     // the in-place updates, before the store reads them
    if (__syncthreads_or(!got)) {          // stage s consumed; any wait that gave up stops all
      failed = true;
      break;
    }
    if (tid == 0) {
      if (fold) {
        // stage rb leaves by TMA store; the stage stored one step earlier, whose store has
        // had a stage's compute to read it, takes the next load
        store(rb, sr, si);
        tc::bulk_commit();
        if (rb >= 1) {
          tc::bulk_wait_read<1>();
          tc::fence_proxy_async();
          if (rb - 1 + NSTG < NRB) {
            issue(rb - 1 + NSTG);
            issued = rb + NSTG;
          }
        }
      } else {
        tc::fence_proxy_async();
        if (rb + NSTG < NRB) {
          issue(rb + NSTG);
          issued = rb + NSTG + 1;
        }
      }
    }
  }
  if (failed) {
    // let the copies in flight land before the shared memory is released; no partials
    if (tid == 0) {
      atomicOr(&g_decode_status, 2u);
      for (int rb = issued - NSTG < 0 ? 0 : issued - NSTG; rb < issued; ++rb)
        tc::mbar_wait(&full[rb % NSTG], (rb / NSTG) & 1, LPOLLS);
      tc::bulk_wait<0>();
    }
    return;
  }
  if (fold && tid == 0) tc::bulk_wait<0>();   // the folded state is written
#pragma unroll
  for (int qn = 0; qn < 4; ++qn)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float x = acc[qn][j];
#pragma unroll
      for (int o = TPR; o < 32; o <<= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
      acc[qn][j] = x;
    }
  if (lane < TPR) {
#pragma unroll
    for (int qn = 0; qn < 4; ++qn)
#pragma unroll
      for (int j = 0; j < 4; ++j) red[w][4 * lane + j][qn] = acc[qn][j];
  }
  __syncthreads();
  const ChamN N = cham_factor(dots[0], dots[1], dots[2], A.gamma[item], fin);
  float cqv[4] = {0.f, 0.f, 0.f, 0.f};
  if (tid < W) {
    const int c = tid;
    float t[4];
#pragma unroll
    for (int qn = 0; qn < 4; ++qn) {
      float x = 0.f;
#pragma unroll
      for (int ww = 0; ww < 8; ++ww) x += red[ww][c][qn];
      t[qn] = x;
    }
    // the pending factors' share of kᵀH and vᵀH (none after a fold)
    for (int j = 0; j < (fold ? 0 : p); ++j) {
      const float gkk = gs[j][0], gkv = gs[j][1], gvk = gs[j][2], gvv = gs[j][3];
      const float* pj = pbs + j * 4 * W + c;
      t[0] += gkk * pj[0] + gkv * pj[2 * W];
      t[1] += gkk * pj[W] + gkv * pj[3 * W];
      t[2] += gvk * pj[0] + gvv * pj[2 * W];
      t[3] += gvk * pj[W] + gvv * pj[3 * W];
    }
    const float qc = qs[c];
    cqv[0] = t[0] * qc; cqv[1] = t[1] * qc; cqv[2] = t[2] * qc; cqv[3] = t[3] * qc;
    float b0r = 0.f, b0i = 0.f, b1r = 0.f, b1i = 0.f;
    if (N.ok) {
      b0r = N.n00r * t[0] - N.n00i * t[1] + N.n01r * t[2] - N.n01i * t[3];
      b0i = N.n00r * t[1] + N.n00i * t[0] + N.n01r * t[3] + N.n01i * t[2];
      b1r = N.n01r * t[0] - N.n01i * t[1] + N.n11r * t[2] - N.n11i * t[3];
      b1i = N.n01r * t[1] + N.n01i * t[0] + N.n11r * t[3] + N.n11i * t[2];
    }
    float* nb = pb + (size_t)snew * 4 * D + cs0 + c;
    nb[0] = b0r; nb[D] = b0i; nb[2 * D] = b1r; nb[3 * D] = b1i;
  }
  if (w < W / 32) {   // this stripe's share of kᵀH q and vᵀH q: one partial per column warp
#pragma unroll
    for (int j = 0; j < 4; ++j) cqv[j] = warp_sum(cqv[j]);
    if (lane == 0) {
#pragma unroll
      for (int j = 0; j < 4; ++j) cq4[w][j] = cqv[j];
    }
  }
  __syncthreads();
  if (tid == 0) {
    float* dst = A.cqp + ((size_t)item * nst + stripe) * 4;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float x = 0.f;
#pragma unroll
      for (int ww = 0; ww < W / 32; ++ww) x += cq4[ww][j];
      dst[j] = x;
    }
  }
}

// The step's readout, one CTA per (item, 256 rows), launched as a programmatic dependent of
// lazy_cham_kernel: the part that does not read the stripes' results (k, v and the step's
// factor N) runs while the stripe kernel's last CTAs finish, then griddepcontrol.wait
// (the stripe kernel complete and its writes visible) and
//     y = sum over stripes of the S_re q partials (in stripe order)
//       + sum_j (k_j Re(B_j0 q) + v_j Re(B_j1 q))          (pending factors)
//       + k Re(B0' q) + v Re(B1' q)                          (this step's factor)
// with Re(B' q) = Re(N [kᵀHq; vᵀHq]) from the stripes' shares; then this step's factor's
// A part (k, v; zero for an identity step) over the CTA's rows, and the item's pending
// count.  The pending count is read from the copy lazy_pre_kernel took (pcold), because
// the count itself is rewritten here.
template <typename T>
__global__ void __launch_bounds__(DT) lazy_out_kernel(LazyArgs A) {
  extern __shared__ __align__(16) float lso[];   // ks [D] | vs [D]
  __shared__ float dsc[8][4], dsc2[8][4];
  const int item = blockIdx.y, tid = threadIdx.x, r = blockIdx.x * DT + tid;
  const int D = A.D, P = A.P, nst = A.nst;
  float* ks = lso;
  float* vs = lso + D;
  const size_t voff = (size_t)item * D;
  const int p = A.pcold[item];
  const bool fold = p >= P;
  const int npend = fold ? 0 : p, snew = fold ? 0 : p;
  float dots[4] = {0.f, 0.f, 0.f, 0.f};
  bool fin = true;
  load_kvq<T>(A, voff, D, ks, vs, nullptr, 0, 0, dots, fin);
  block_sum4(dots, fin, dsc);     // also makes ks, vs visible
  const ChamN N = cham_factor(dots[0], dots[1], dots[2], A.gamma[item], fin);
  float bq[LP_MAX][2];
#pragma unroll
  for (int j = 0; j < LP_MAX; ++j)   // (written by lazy_pre_kernel, complete before the stripe kernel began)
    if (j < npend) {
      bq[j][0] = __ldcg(A.bq + ((size_t)item * LP_MAX + j) * 2);
      bq[j][1] = __ldcg(A.bq + ((size_t)item * LP_MAX + j) * 2 + 1);
    }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  float x[4] = {0.f, 0.f, 0.f, 0.f};
  for (int st = tid; st < nst; st += DT) {
    const float* src = A.cqp + ((size_t)item * nst + st) * 4;
#pragma unroll
    for (int j = 0; j < 4; ++j) x[j] = __ldcg(src + j);
  }
  float sacc = 0.f;
  const float* pa = A.pa + (size_t)item * P * 2 * D;
  if (r < D) {   // the row's pending factor rows and stripe partials (in order), loads in flight together
    float av[LP_MAX][2];
#pragma unroll
    for (int j = 0; j < LP_MAX; ++j)
      if (j < npend) {
        av[j][0] = pa[(size_t)j * 2 * D + r];
        av[j][1] = pa[((size_t)j * 2 + 1) * D + r];
      }
    const float* pb0 = A.part + (size_t)item * nst * D + r;
    for (int s0 = 0; s0 < nst; s0 += 16) {
      float pv[16];
#pragma unroll
      for (int st = 0; st < 16; ++st)
        if (s0 + st < nst) pv[st] = __ldcg(pb0 + (size_t)(s0 + st) * D);
#pragma unroll
      for (int st = 0; st < 16; ++st)
        if (s0 + st < nst) sacc += pv[st];
    }
#pragma unroll
    for (int j = 0; j < LP_MAX; ++j)
      if (j < npend) sacc += av[j][0] * bq[j][0] + av[j][1] * bq[j][1];
  }
  bool dummy = true;
  block_sum4(x, dummy, dsc2);
  // Re of the new factor times q: B0'q = N00 (kᵀHq) + N01 (vᵀHq), B1'q = N01 (kᵀHq) + N11 (vᵀHq)
  const float u0 = N.ok ? N.n00r * x[0] - N.n00i * x[1] + N.n01r * x[2] - N.n01i * x[3] : 0.f;
  const float u1 = N.ok ? N.n01r * x[0] - N.n01i * x[1] + N.n11r * x[2] - N.n11i * x[3] : 0.f;
  if (r < D) {
    if (N.ok) sacc += ks[r] * u0 + vs[r] * u1;   // (an identity step adds nothing; k, v may be non-finite)
    static_cast<T*>(A.cout)[voff + r] = from_f32<T>(sacc);
    // this step's A part (slot snew is not among the pending rows read above)
    float* na = A.pa + ((size_t)item * P + snew) * 2 * D;
    na[r] = N.ok ? ks[r] : 0.f;
    na[D + r] = N.ok ? vs[r] : 0.f;
  }
  if (blockIdx.x == 0 && tid == 0) A.pcount[item] = snew + 1;
}

// Fold every pending factor into S and empty the list (one CTA per (item, stripe)).
__global__ void __launch_bounds__(DT) lazy_flush_kernel(float* __restrict__ hr, float* __restrict__ hi,
                                                        const int* __restrict__ pcount, const float* __restrict__ pa,
                                                        const float* __restrict__ pb, int D, int P) {
  __shared__ float pbs[LP_MAX][4][CWD];
  const int nst = D / CWD;
  const int item = blockIdx.x / nst, stripe = blockIdx.x % nst, tid = threadIdx.x, lane = tid & 31;
  const int p = pcount[item];
  if (p == 0) return;
  const int cs0 = stripe * CWD, c8 = lane % TPR, c0 = cs0 + 4 * c8, rp = tid / TPR;
  const float* a = pa + (size_t)item * P * 2 * D;
  const float* bb = pb + (size_t)item * P * 4 * D;
  for (int e = tid; e < p * 4 * CWD; e += DT) {
    const int j = e / (4 * CWD), rr = (e / CWD) % 4, c = e % CWD;
    pbs[j][rr][c] = bb[((size_t)j * 4 + rr) * D + cs0 + c];
  }
  __syncthreads();
  float* Hr = hr + (size_t)item * D * D;
  float* Hi = hi + (size_t)item * D * D;
  for (int r = rp; r < D; r += RPG) {
    float4 xr = *reinterpret_cast<const float4*>(Hr + (size_t)r * D + c0);
    float4 xi = *reinterpret_cast<const float4*>(Hi + (size_t)r * D + c0);
    for (int j = 0; j < p; ++j) {
      const float2 av = make_float2(__ldg(a + (size_t)j * 2 * D + r), __ldg(a + ((size_t)j * 2 + 1) * D + r));
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const int c = 4 * c8 + jj;
        comp(xr, jj) += av.x * pbs[j][0][c] + av.y * pbs[j][2][c];
        comp(xi, jj) += av.x * pbs[j][1][c] + av.y * pbs[j][3][c];
      }
    }
    *reinterpret_cast<float4*>(Hr + (size_t)r * D + c0) = xr;
    *reinterpret_cast<float4*>(Hi + (size_t)r * D + c0) = xi;
  }
}

template <typename T, bool CHAM, bool FO>
__global__ void __launch_bounds__(DT, 3) decode_step_kernel(DecodeArgs A) {
  const int bid = blockIdx.x;
  if (bid < A.ns) {
    sssd_part<T>(A, bid);
    return;
  }
  if constexpr (CHAM) cham_part<T, FO>(A, bid - A.ns);
}

// u = H q for FIRST_ORDER: one warp per row; u layout [b][2][D].
__global__ void __launch_bounds__(DT) decode_hq_kernel(const float* __restrict__ hr, const float* __restrict__ hi,
                                                       const void* q, int dtype, float* __restrict__ u,
                                                       int b, int D) {
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * (DT / 32) + (threadIdx.x >> 5);
  if (row >= (long long)b * D) return;
  const int item = (int)(row / D), r = (int)(row % D);
  const float* pr = hr + (size_t)row * D;
  const float* pi = hi + (size_t)row * D;
  float sr = 0.f, si = 0.f;
  for (int c = 4 * lane; c < D; c += 128) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(pr + c));
    const float4 bb = __ldg(reinterpret_cast<const float4*>(pi + c));
    float q0, q1, q2, q3;
    const size_t qo = (size_t)item * D + c;
    if (dtype == VERACE_BF16) {
      const __nv_bfloat16* qq = static_cast<const __nv_bfloat16*>(q) + qo;
      q0 = to_f32(qq[0]); q1 = to_f32(qq[1]); q2 = to_f32(qq[2]); q3 = to_f32(qq[3]);
    } else if (dtype == VERACE_F16) {
      const __half* qq = static_cast<const __half*>(q) + qo;
      q0 = to_f32(qq[0]); q1 = to_f32(qq[1]); q2 = to_f32(qq[2]); q3 = to_f32(qq[3]);
    } else {
      const float* qq = static_cast<const float*>(q) + qo;
      q0 = qq[0]; q1 = qq[1]; q2 = qq[2]; q3 = qq[3];
    }
    sr += a.x * q0 + a.y * q1 + a.z * q2 + a.w * q3;
    si += bb.x * q0 + bb.y * q1 + bb.z * q2 + bb.w * q3;
  }
  sr = warp_sum(sr);
  si = warp_sum(si);
  if (lane == 0) {
    u[(size_t)item * 2 * D + r] = sr;
    u[(size_t)item * 2 * D + D + r] = si;
  }
}

struct WsLayout {
  size_t part, cnt, err2, u, total;
};

WsLayout ws_layout(int b, int D) {
  WsLayout L{};
  size_t off = 0;
  L.part = off; off = align_up(off + (size_t)b * (D / CWD) * D * sizeof(float), 256);
  L.cnt = off;  off = align_up(off + (size_t)b * sizeof(unsigned int), 256);
  L.err2 = off; off = align_up(off + (size_t)b * sizeof(float), 256);
  L.u = off;    off = align_up(off + (size_t)b * 2 * D * sizeof(float), 256);
  L.total = off + 256;
  return L;
}

template <typename T>
int launch_typed(const DecodeArgs& A, cudaStream_t st) {
  const int ncham = (A.D > 0) ? A.b * (A.D / CWD) : 0;
  const int grid = A.ns + ncham;
  const bool fo = A.mode == VERACE_DECODE_FIRST_ORDER;
  if (A.D == 0 && A.d == 128) {
    VERACE_CUDA(cudaFuncSetAttribute(sssd_decode128_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, SD_SMEM));
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(DT);
    cfg.dynamicSmemBytes = SD_SMEM;
    cfg.stream = st;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    VERACE_CUDA(cudaLaunchKernelEx(&cfg, sssd_decode128_kernel<T>, A));
  } else if (A.D == 0)
    decode_step_kernel<T, false, false><<<grid, DT, 0, st>>>(A);
  else if (fo)
    decode_step_kernel<T, true, true><<<grid, DT, 0, st>>>(A);
  else
    decode_step_kernel<T, true, false><<<grid, DT, 0, st>>>(A);
  return check_launch("decode_step_kernel");
}

// one hologram plane as a [b*D rows][D] fp32 tensor, boxes of `cols` columns x `rows` rows,
// unswizzled or with the 128-byte swizzle (cols = 32)
int make_plane_map(CUtensorMap* m, const float* base, int b, int D, int cols, int rows, bool swizzle128) {
  auto enc = tmap_encoder();
  VERACE_REQUIRE(enc != nullptr, VERACE_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  const cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)b * D};
  const cuuint64_t strides[1] = {(cuuint64_t)D * 4};
  const cuuint32_t box[2] = {(cuuint32_t)cols, (cuuint32_t)rows};
  const cuuint32_t es[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  VERACE_REQUIRE(r == CUDA_SUCCESS, VERACE_ERR_CUDA, "cuTensorMapEncodeTiled (hologram plane) failed: %d", (int)r);
  return VERACE_OK;
}

struct LazyWs {
  size_t part, cqp, cnt, g, bq, pq, pk, pv, pg, total;
};

LazyWs lazy_ws_layout(int b, int D) {
  LazyWs L{};
  size_t off = 0;
  const int nst = D / CWD;
  L.part = off; off = align_up(off + (size_t)b * nst * D * sizeof(float), 256);
  L.cqp = off;  off = align_up(off + (size_t)b * nst * 4 * sizeof(float), 256);
  L.cnt = off;  off = align_up(off + (size_t)b * sizeof(int), 256);
  L.g = off;    off = align_up(off + (size_t)b * LP_MAX * 4 * sizeof(float), 256);
  L.bq = off;   off = align_up(off + (size_t)b * LP_MAX * 2 * sizeof(float), 256);
  // projected steps: q, k, v (at most fp32) and gamma as the pre-pass leaves them
  L.pq = off;   off = align_up(off + (size_t)b * D * sizeof(float), 256);
  L.pk = off;   off = align_up(off + (size_t)b * D * sizeof(float), 256);
  L.pv = off;   off = align_up(off + (size_t)b * D * sizeof(float), 256);
  L.pg = off;   off = align_up(off + (size_t)b * sizeof(float), 256);
  L.total = off + 256;
  return L;
}

// pending storage: counts [b] (256-byte block) | A [b][P][2][D] | B [b][P][4][D]
size_t pending_bytes(int b, int D, int P) {
  return align_up((size_t)b * sizeof(int), 256) + (size_t)b * P * 6 * D * sizeof(float);
}

void pending_ptrs(void* pending, int b, int D, int P, int** cnt, float** pa, float** pb) {
  char* base = (char*)pending;
  *cnt = (int*)base;
  *pa = (float*)(base + align_up((size_t)b * sizeof(int), 256));
  *pb = *pa + (size_t)b * P * 2 * D;
}

}  // namespace

int decode_read_status(unsigned int* status) {
  unsigned int v = 0, zero = 0;
  VERACE_CUDA(cudaMemcpyFromSymbol(&v, g_decode_status, sizeof(v)));
  if (v) VERACE_CUDA(cudaMemcpyToSymbol(g_decode_status, &zero, sizeof(zero)));
  *status = v;
  return VERACE_OK;
}

}  // namespace verace

using namespace verace;

extern "C" size_t verace_decode_workspace(int b, int D) {
  if (b <= 0 || D <= 0) return 256;
  return ws_layout(b, D).total;
}

extern "C" int verace_decode_step(const void* sssd_q, const void* sssd_k, const void* sssd_v,
                                  const float* delta, float* psi, void* sssd_out,
                                  const void* cham_q, const void* cham_k, const void* cham_v,
                                  const float* gamma, float* h_re, float* h_im, void* cham_out,
                                  int b, int h, int d, int D, int dtype, int mode,
                                  void* workspace, size_t workspace_bytes, void* stream) {
  VERACE_REQUIRE(b >= 0 && h >= 0 && d >= 0 && D >= 0, VERACE_ERR_INVALID,
                 "verace_decode_step: invalid sizes b=%d h=%d d=%d D=%d", b, h, d, D);
  VERACE_REQUIRE(dtype == VERACE_F32 || dtype == VERACE_BF16 || dtype == VERACE_F16,
                 VERACE_ERR_INVALID, "verace_decode_step: unknown dtype %d", dtype);
  VERACE_REQUIRE(mode == VERACE_DECODE_UNITARY || mode == VERACE_DECODE_FIRST_ORDER, VERACE_ERR_INVALID,
                 "verace_decode_step: unknown mode %d", mode);
  const bool do_sssd = h > 0 && d > 0;
  const bool do_cham = D > 0;
  if (b == 0 || (!do_sssd && !do_cham)) return VERACE_OK;
  if (do_sssd) {
    VERACE_REQUIRE(sssd_q && sssd_k && sssd_v && delta && psi && sssd_out, VERACE_ERR_INVALID,
                   "verace_decode_step: NULL SSSD pointer");
    VERACE_REQUIRE(d % 4 == 0 && d <= MAXHD, VERACE_ERR_UNSUPPORTED,
                   "verace_decode_step: head_dim %d unsupported (multiple of 4, at most %d)", d, MAXHD);
    VERACE_REQUIRE(((uintptr_t)psi & 15) == 0, VERACE_ERR_INVALID,
                   "verace_decode_step: SSSD state must be 16-byte aligned");
  }
  if (do_cham) {
    VERACE_REQUIRE(cham_q && cham_k && cham_v && gamma && h_re && h_im && cham_out, VERACE_ERR_INVALID,
                   "verace_decode_step: NULL CHAM pointer");
    VERACE_REQUIRE(D % CWD == 0 && D <= MAXD, VERACE_ERR_UNSUPPORTED,
                   "verace_decode_step: holographic dim %d unsupported (a multiple of %d, at most %d)", D, CWD,
                   MAXD);
    VERACE_REQUIRE((((uintptr_t)h_re | (uintptr_t)h_im) & 15) == 0, VERACE_ERR_INVALID,
                   "verace_decode_step: hologram must be 16-byte aligned");
    const size_t need = verace_decode_workspace(b, D);
    VERACE_REQUIRE(workspace != nullptr && workspace_bytes >= need, VERACE_ERR_WORKSPACE,
                   "verace_decode_step: workspace of %zu bytes required, %zu given", need,
                   workspace ? workspace_bytes : (size_t)0);
  }
  cudaStream_t st = (cudaStream_t)stream;
  DecodeArgs A{};
  A.sq = sssd_q; A.sk = sssd_k; A.sv = sssd_v; A.delta = delta; A.psi = psi; A.sout = sssd_out;
  A.cq = cham_q; A.ck = cham_k; A.cv = cham_v; A.gamma = gamma; A.hr = h_re; A.hi = h_im; A.cout = cham_out;
  A.b = b;
  A.h = do_sssd ? h : 0;
  A.d = do_sssd ? d : 0;
  A.D = do_cham ? D : 0;
  A.mode = mode;
  A.ns = A.b * A.h;
  if (do_cham) {
    const WsLayout L = ws_layout(b, D);
    char* base = (char*)align_up((size_t)workspace, 256);
    A.part = (float*)(base + L.part);
    A.cnt = (unsigned int*)(base + L.cnt);
    A.err2 = (float*)(base + L.err2);
    float* u = (float*)(base + L.u);
    A.u = u;
    VERACE_CUDA(cudaMemsetAsync(base + L.cnt, 0, L.u - L.cnt, st));   // counters and |E q|²
    if (mode == VERACE_DECODE_FIRST_ORDER) {
      const long long rows = (long long)b * D;
      decode_hq_kernel<<<(unsigned)((rows + DT / 32 - 1) / (DT / 32)), DT, 0, st>>>(h_re, h_im, cham_q, dtype,
                                                                                u, b, D);
      int rc = check_launch("decode_hq_kernel");
      if (rc) return rc;
    }
  }
  switch (dtype) {
    case VERACE_F32: return launch_typed<float>(A, st);
    case VERACE_BF16: return launch_typed<__nv_bfloat16>(A, st);
    default: return launch_typed<__half>(A, st);
  }
}

// lazy_pre_kernel, lazy_cham_kernel over (item, stripe) CTAs with the widest stripe D
// allows (MF: the tensor-core fold and its swizzled stages), then lazy_out_kernel over the
// items.
template <typename T, int W, bool MF>
int launch_lazy_w(const LazyArgs& A, const float* h_re, const float* h_im, cudaStream_t st) {
  using G = LazyGeom<W, MF>;
  CUtensorMap mr, mi;
  if (int rc = make_plane_map(&mr, h_re, A.b, A.D, MF ? 32 : W, G::ROWS, MF)) return rc;
  if (int rc = make_plane_map(&mi, h_im, A.b, A.D, MF ? 32 : W, G::ROWS, MF)) return rc;
  // all three launched as programmatic dependents of the kernel before them
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cfg.blockDim = dim3(DT);
  cfg.gridDim = dim3((unsigned)(A.b * A.P));
  cfg.dynamicSmemBytes = 0;
  if (A.y != nullptr)
    VERACE_CUDA(cudaLaunchKernelEx(&cfg, lazy_pre_kernel<T, true>, A));   // (also keeps the pending counts)
  else
    VERACE_CUDA(cudaLaunchKernelEx(&cfg, lazy_pre_kernel<T, false>, A));
  if (int rc = check_launch("lazy_pre_kernel")) return rc;
  const size_t smem = G::smem(A.D, A.P);
  VERACE_CUDA(cudaFuncSetAttribute(lazy_cham_kernel<T, W, MF>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   (int)smem));
  LazyArgs B = A;
  B.nst = A.D / W;
  cfg.gridDim = dim3((unsigned)(A.b * B.nst));
  cfg.dynamicSmemBytes = smem;
  VERACE_CUDA(cudaLaunchKernelEx(&cfg, lazy_cham_kernel<T, W, MF>, B, mr, mi));
  if (int rc = check_launch("lazy_cham_kernel")) return rc;
  cfg.gridDim = dim3((unsigned)((A.D + DT - 1) / DT), (unsigned)A.b);
  cfg.dynamicSmemBytes = 2 * (size_t)A.D * sizeof(float);
  VERACE_CUDA(cudaLaunchKernelEx(&cfg, lazy_out_kernel<T>, B));
  return check_launch("lazy_out_kernel");
}
template <typename T>
int launch_lazy(const LazyArgs& A, const float* h_re, const float* h_im, cudaStream_t st) {
  if (A.D % 64 != 0) return launch_lazy_w<T, 32, false>(A, h_re, h_im, st);
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    if (A.P <= LP_MAX / 2) return launch_lazy_w<T, 64, true>(A, h_re, h_im, st);
  }
  return launch_lazy_w<T, 64, false>(A, h_re, h_im, st);
}

extern "C" size_t verace_decode_lazy_workspace(int b, int D) {
  if (b <= 0 || D <= 0 || D % CWD) return 256;
  return lazy_ws_layout(b, D).total;
}

extern "C" size_t verace_decode_pending_bytes(int b, int D, int P) {
  if (b <= 0 || D <= 0 || P <= 0) return 0;
  return pending_bytes(b, D, P);
}

// The shared part of the two deferred-update entry points: A carries the step's inputs
// (q, k, v, gamma, or the projection rows y).
static int cham_lazy_run(const char* fn, LazyArgs A, float* h_re, float* h_im, void* pending, int P,
                         void* cham_out, int b, int D, int dtype, void* workspace, size_t workspace_bytes,
                         void* stream) {
  VERACE_REQUIRE(h_re && h_im && pending && cham_out, VERACE_ERR_INVALID, "%s: NULL pointer", fn);
  VERACE_REQUIRE(D % CWD == 0 && D <= MAXD, VERACE_ERR_UNSUPPORTED,
                 "%s: holographic dim %d unsupported (a multiple of %d, at most %d)", fn, D, CWD, MAXD);
  VERACE_REQUIRE((((uintptr_t)h_re | (uintptr_t)h_im | (uintptr_t)pending) & 15) == 0, VERACE_ERR_INVALID,
                 "%s: hologram and pending storage must be 16-byte aligned", fn);
  const size_t need = verace_decode_lazy_workspace(b, D);
  VERACE_REQUIRE(workspace != nullptr && workspace_bytes >= need, VERACE_ERR_WORKSPACE,
                 "%s: workspace of %zu bytes required, %zu given", fn, need, workspace ? workspace_bytes : (size_t)0);
  cudaStream_t st = (cudaStream_t)stream;
  const LazyWs L = lazy_ws_layout(b, D);
  char* base = (char*)align_up((size_t)workspace, 256);
  if (A.y != nullptr) {   // the pre-pass leaves q, k, v, gamma in the workspace for the others
    A.pq = base + L.pq; A.pk = base + L.pk; A.pv = base + L.pv; A.pg = (float*)(base + L.pg);
    A.cq = A.pq; A.ck = A.pk; A.cv = A.pv; A.gamma = A.pg;
  }
  A.hr = h_re; A.hi = h_im; A.cout = cham_out;
  pending_ptrs(pending, b, D, P, &A.pcount, &A.pa, &A.pb);
  A.g = (float*)(base + L.g);
  A.bq = (float*)(base + L.bq);
  A.part = (float*)(base + L.part);
  A.cqp = (float*)(base + L.cqp);
  A.pcold = (int*)(base + L.cnt);
  A.b = b; A.D = D; A.P = P;
  switch (dtype) {
    case VERACE_F32: return launch_lazy<float>(A, h_re, h_im, st);
    case VERACE_BF16: return launch_lazy<__nv_bfloat16>(A, h_re, h_im, st);
    default: return launch_lazy<__half>(A, h_re, h_im, st);
  }
}

extern "C" int verace_decode_cham_lazy(const void* cham_q, const void* cham_k, const void* cham_v, const float* gamma,
                                       float* h_re, float* h_im, void* pending, int P, void* cham_out, int b, int D,
                                       int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  VERACE_REQUIRE(b >= 0 && D >= 0, VERACE_ERR_INVALID, "verace_decode_cham_lazy: invalid sizes b=%d D=%d", b, D);
  VERACE_REQUIRE(dtype == VERACE_F32 || dtype == VERACE_BF16 || dtype == VERACE_F16, VERACE_ERR_INVALID,
                 "verace_decode_cham_lazy: unknown dtype %d", dtype);
  VERACE_REQUIRE(P >= 1 && P <= LP_MAX, VERACE_ERR_INVALID,
                 "verace_decode_cham_lazy: pending depth %d outside [1, %d]", P, LP_MAX);
  if (b == 0 || D == 0) return VERACE_OK;
  VERACE_REQUIRE(cham_q && cham_k && cham_v && gamma, VERACE_ERR_INVALID, "verace_decode_cham_lazy: NULL pointer");
  LazyArgs A{};
  A.cq = cham_q; A.ck = cham_k; A.cv = cham_v; A.gamma = gamma;
  return cham_lazy_run("verace_decode_cham_lazy", A, h_re, h_im, pending, P, cham_out, b, D, dtype, workspace,
                       workspace_bytes, stream);
}

extern "C" int verace_decode_cham_lazy_projected(const void* y, long long ld, float* h_re, float* h_im,
                                                 void* pending, int P, void* cham_out, int b, int D, int dtype,
                                                 void* workspace, size_t workspace_bytes, void* stream) {
  VERACE_REQUIRE(b >= 0 && D >= 0, VERACE_ERR_INVALID, "verace_decode_cham_lazy_projected: invalid sizes b=%d D=%d",
                 b, D);
  VERACE_REQUIRE(dtype == VERACE_F32 || dtype == VERACE_BF16 || dtype == VERACE_F16, VERACE_ERR_INVALID,
                 "verace_decode_cham_lazy_projected: unknown dtype %d", dtype);
  VERACE_REQUIRE(P >= 1 && P <= LP_MAX, VERACE_ERR_INVALID,
                 "verace_decode_cham_lazy_projected: pending depth %d outside [1, %d]", P, LP_MAX);
  if (b == 0 || D == 0) return VERACE_OK;
  VERACE_REQUIRE(y != nullptr, VERACE_ERR_INVALID, "verace_decode_cham_lazy_projected: NULL pointer");
  VERACE_REQUIRE(ld >= 3LL * D + 1, VERACE_ERR_INVALID,
                 "verace_decode_cham_lazy_projected: row stride %lld shorter than q | k | v | gate", ld);
  LazyArgs A{};
  A.y = y; A.yld = ld;
  return cham_lazy_run("verace_decode_cham_lazy_projected", A, h_re, h_im, pending, P, cham_out, b, D, dtype,
                       workspace, workspace_bytes, stream);
}

extern "C" int verace_decode_cham_flush(float* h_re, float* h_im, void* pending, int P, int b, int D, void* stream) {
  VERACE_REQUIRE(b >= 0 && D >= 0 && P >= 1 && P <= LP_MAX, VERACE_ERR_INVALID,
                 "verace_decode_cham_flush: invalid sizes b=%d D=%d P=%d", b, D, P);
  if (b == 0 || D == 0) return VERACE_OK;
  VERACE_REQUIRE(h_re && h_im && pending, VERACE_ERR_INVALID, "verace_decode_cham_flush: NULL pointer");
  VERACE_REQUIRE(D % CWD == 0 && D <= MAXD, VERACE_ERR_UNSUPPORTED,
                 "verace_decode_cham_flush: holographic dim %d unsupported", D);
  cudaStream_t st = (cudaStream_t)stream;
  int* cnt;
  float *pa, *pb;
  pending_ptrs(pending, b, D, P, &cnt, &pa, &pb);
  lazy_flush_kernel<<<(unsigned)(b * (D / CWD)), DT, 0, st>>>(h_re, h_im, cnt, pa, pb, D, P);
  if (int rc = check_launch("lazy_flush_kernel")) return rc;
  VERACE_CUDA(cudaMemsetAsync(cnt, 0, (size_t)b * sizeof(int), st));
  return VERACE_OK;
}
