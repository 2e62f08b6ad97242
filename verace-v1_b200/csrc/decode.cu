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
// Work split: CTA i < b·h handles SSSD (item, head) i with the whole 128 x 128 state in
// registers.  The CHAM hologram is cut into column stripes of 32; a cluster of 4 CTAs owns
// one stripe, each CTA a quarter of its rows, held in registers between the read and the
// write.  The column reductions kᵀH, vᵀH (and Hᴴu) are summed over the cluster through
// distributed shared memory, in rank order.  Each CTA writes the readout partial of its
// rows over its 32 columns; the last CTA of an (item, row quarter) to finish sums the
// stripes' partials in stripe order and writes y.  No CTA waits on another outside the
// cluster's hardware barrier.
#include "common.cuh"

#include <cooperative_groups.h>

namespace cg = cooperative_groups;

namespace verace {

__device__ unsigned int g_decode_status;

namespace {

constexpr int DT = 256;        // threads per CTA
constexpr int CWD = 32;        // CHAM stripe width (columns)
constexpr int CLU = 4;         // CTAs per CHAM cluster (row quarters of a stripe)
constexpr int MAXD = 1024;     // largest hologram dimension held in registers
constexpr int MAXHD = 128;     // largest SSSD head dimension
constexpr float DRIFT_TOL = 1e-2f;

struct DecodeArgs {
  const void* sq; const void* sk; const void* sv; const float* delta;
  float* psi; void* sout;
  const void* cq; const void* ck; const void* cv; const float* gamma;
  float* hr; float* hi; void* cout;
  const float* u;              // FIRST_ORDER: [b][2][D] (re, im) of H q
  float* part;                 // [b][D/32][D] readout partials
  unsigned int* cnt;           // [b][4] stripe counters
  float* err2;                 // [b] |E q|² accumulators
  int b, h, d, D, mode, ns_pad;
};

template <typename T>
__device__ __forceinline__ float ld1(const void* p, size_t i) {
  return to_f32(static_cast<const T*>(p)[i]);
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// ------------------------------------------------------------------------- SSSD
template <typename T>
__device__ void sssd_part(const DecodeArgs& A, int chain) {
  __shared__ float ks[MAXHD], vs[MAXHD], qs[MAXHD];
  __shared__ float red[8][MAXHD][2];
  __shared__ float fac[5];     // m00 m01 m10 m11, ok flag
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int d = A.d;
  const size_t vec = (size_t)chain * d;
  for (int i = tid; i < d; i += DT) {
    ks[i] = ld1<T>(A.sk, vec + i);
    vs[i] = ld1<T>(A.sv, vec + i);
    qs[i] = ld1<T>(A.sq, vec + i);
  }
  // state rows w + 8 m, columns 4 lane .. 4 lane + 3
  float* P = A.psi + (size_t)chain * d * d;
  const bool colok = 4 * lane < d;
  float4 ps[MAXHD / 8];
#pragma unroll
  for (int m = 0; m < MAXHD / 8; ++m) {
    const int r = w + 8 * m;
    ps[m] = (colok && r < d) ? __ldcs(reinterpret_cast<const float4*>(P + (size_t)r * d + 4 * lane))
                             : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  __syncthreads();
  if (w == 0) {
    float kk = 0.f, vv = 0.f, kv = 0.f;
    bool fin = true;
    for (int i = lane; i < d; i += 32) {
      kk += ks[i] * ks[i]; vv += vs[i] * vs[i]; kv += ks[i] * vs[i];
      fin = fin && isfinite(ks[i]) && isfinite(vs[i]);
    }
    kk = warp_sum(kk); vv = warp_sum(vv); kv = warp_sum(kv);
    fin = __all_sync(0xffffffffu, fin);
    if (lane == 0) {
      const float dl = A.delta[chain];
      const float a = 0.5f * dl;
      const float det = 1.f + a * a * (kk * vv - kv * kv);
      const float f = -2.f * a / det;
      const float m00 = f * (a * vv), m01 = f * (1.f - a * kv);
      const float m10 = f * (-1.f - a * kv), m11 = f * (a * kk);
      // Non-finite k, v, gate or factor: identity, as the reference's _solve_cayley
      // substitution does (sssd_attention.py:52-71).
      const bool ok = fin && isfinite(dl) && isfinite(m00) && isfinite(m01) && isfinite(m10) &&
                      isfinite(m11);
      fac[0] = m00; fac[1] = m01; fac[2] = m10; fac[3] = m11; fac[4] = ok ? 1.f : 0.f;
    }
  }
  // column sums kᵀΨ, vᵀΨ
  float ak[4] = {0.f, 0.f, 0.f, 0.f}, av[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int m = 0; m < MAXHD / 8; ++m) {
    const int r = w + 8 * m;
    if (r < d) {
      const float kr = ks[r], vr = vs[r];
      ak[0] += kr * ps[m].x; ak[1] += kr * ps[m].y; ak[2] += kr * ps[m].z; ak[3] += kr * ps[m].w;
      av[0] += vr * ps[m].x; av[1] += vr * ps[m].y; av[2] += vr * ps[m].z; av[3] += vr * ps[m].w;
    }
  }
  if (colok) {
#pragma unroll
    for (int j = 0; j < 4; ++j) { red[w][4 * lane + j][0] = ak[j]; red[w][4 * lane + j][1] = av[j]; }
  }
  __syncthreads();
  const bool ok = fac[4] != 0.f;
  float al[4], be[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float sa = 0.f, sb = 0.f;
    if (colok) {
#pragma unroll
      for (int ww = 0; ww < 8; ++ww) { sa += red[ww][4 * lane + j][0]; sb += red[ww][4 * lane + j][1]; }
    }
    al[j] = fac[0] * sa + fac[1] * sb;   // coefficient of k_r
    be[j] = fac[2] * sa + fac[3] * sb;   // coefficient of v_r
  }
  const float4 q4 = colok ? make_float4(qs[4 * lane], qs[4 * lane + 1], qs[4 * lane + 2], qs[4 * lane + 3])
                          : make_float4(0.f, 0.f, 0.f, 0.f);
  T* out = static_cast<T*>(A.sout) + vec;
#pragma unroll
  for (int m = 0; m < MAXHD / 8; ++m) {
    const int r = w + 8 * m;
    if (r >= d) continue;            // warp-uniform
    float4 x = ps[m];
    if (ok) {
      const float kr = ks[r], vr = vs[r];
      x.x += kr * al[0] + vr * be[0]; x.y += kr * al[1] + vr * be[1];
      x.z += kr * al[2] + vr * be[2]; x.w += kr * al[3] + vr * be[3];
    }
    float o = x.x * q4.x + x.y * q4.y + x.z * q4.z + x.w * q4.w;
    o = warp_sum(o);
    if (lane == 0) out[r] = from_f32<T>(o);
    if (colok) __stcs(reinterpret_cast<float4*>(P + (size_t)r * d + 4 * lane), x);
  }
}

// ------------------------------------------------------------------------- CHAM
// Per-column quantities summed over the stripe's rows: kᵀHr, kᵀHi, vᵀHr, vᵀHi, and for
// FIRST_ORDER (Hᴴu)re, (Hᴴu)im.
constexpr int NQ = 6;

template <typename T, int NP>
__device__ void cham_part(const DecodeArgs& A, int local) {
  __shared__ float ks[MAXD], vs[MAXD], qs[MAXD];
  __shared__ float ur[MAXD / CLU], ui[MAXD / CLU];
  __shared__ float red[8][CWD][NQ];
  __shared__ float mine[CWD][NQ];        // this CTA's sums, read by the whole cluster
  __shared__ float tot[CWD][NQ];
  __shared__ float sc[16];
  __shared__ int last_flag;
  cg::cluster_group cluster = cg::this_cluster();
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  const int D = A.D;
  const int nst = D / CWD;
  const int rank = local % CLU;
  const int sidx = local / CLU;
  const int item = sidx / nst, stripe = sidx % nst;
  const int RQ = D / CLU;               // rows of this CTA (= 32 NP)
  const int row0 = rank * RQ;
  const int cg8 = lane & 7;             // column group: columns 4 cg8 .. 4 cg8 + 3 of the stripe
  const int c0 = stripe * CWD + 4 * cg8;
  const int rp = w * 4 + (lane >> 3);   // row within a 32-row pass
  const bool fo = A.mode == VERACE_DECODE_FIRST_ORDER;

  const size_t hoff = (size_t)item * D * D;
  float* Hr = A.hr + hoff;
  float* Hi = A.hi + hoff;
  float4 xr[NP], xi[NP];
#pragma unroll
  for (int p = 0; p < NP; ++p) {
    const size_t e = (size_t)(row0 + p * 32 + rp) * D + c0;
    xr[p] = __ldcs(reinterpret_cast<const float4*>(Hr + e));
    xi[p] = __ldcs(reinterpret_cast<const float4*>(Hi + e));
  }
  const size_t voff = (size_t)item * D;
  for (int i = tid; i < D; i += DT) {
    ks[i] = ld1<T>(A.ck, voff + i);
    vs[i] = ld1<T>(A.cv, voff + i);
    qs[i] = ld1<T>(A.cq, voff + i);
  }
  if (fo) {
    for (int i = tid; i < RQ; i += DT) {
      ur[i] = A.u[(size_t)item * 2 * D + row0 + i];
      ui[i] = A.u[(size_t)item * 2 * D + D + row0 + i];
    }
  }
  __syncthreads();
  if (w == 0) {
    float kk = 0.f, vv = 0.f, kv = 0.f, qq = 0.f;
    bool fin = true;
    for (int i = lane; i < D; i += 32) {
      const float kx = ks[i], vx = vs[i], qx = qs[i];
      kk += kx * kx; vv += vx * vx; kv += kx * vx; qq += qx * qx;
      fin = fin && isfinite(kx) && isfinite(vx);
    }
    kk = warp_sum(kk); vv = warp_sum(vv); kv = warp_sum(kv); qq = warp_sum(qq);
    fin = __all_sync(0xffffffffu, fin);
    if (lane == 0) {
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
      sc[0] = n00r; sc[1] = n00i; sc[2] = n01r; sc[3] = n01i; sc[4] = n11r; sc[5] = n11i;
      sc[6] = ok ? 1.f : 0.f;
      sc[7] = qq;
    }
  }
  // per-thread partial column sums over its NP rows
  float acc[NQ][4];
#pragma unroll
  for (int qn = 0; qn < NQ; ++qn)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[qn][j] = 0.f;
#pragma unroll
  for (int p = 0; p < NP; ++p) {
    const int rl = p * 32 + rp;
    const float kr = ks[row0 + rl], vr = vs[row0 + rl];
    const float hr4[4] = {xr[p].x, xr[p].y, xr[p].z, xr[p].w};
    const float hi4[4] = {xi[p].x, xi[p].y, xi[p].z, xi[p].w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      acc[0][j] += kr * hr4[j]; acc[1][j] += kr * hi4[j];
      acc[2][j] += vr * hr4[j]; acc[3][j] += vr * hi4[j];
    }
    if (fo) {
      const float a = ur[rl], bq = ui[rl];
#pragma unroll
      for (int j = 0; j < 4; ++j) {   // conj(H) u
        acc[4][j] += hr4[j] * a + hi4[j] * bq;
        acc[5][j] += hr4[j] * bq - hi4[j] * a;
      }
    }
  }
  // lanes l, l^8, l^16, l^24 share columns
#pragma unroll
  for (int qn = 0; qn < NQ; ++qn)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float x = acc[qn][j];
      x += __shfl_xor_sync(0xffffffffu, x, 8);
      x += __shfl_xor_sync(0xffffffffu, x, 16);
      acc[qn][j] = x;
    }
  if (lane < 8) {
#pragma unroll
    for (int qn = 0; qn < NQ; ++qn)
#pragma unroll
      for (int j = 0; j < 4; ++j) red[w][4 * lane + j][qn] = acc[qn][j];
  }
  __syncthreads();
  if (tid < CWD * NQ) {
    const int c = tid / NQ, qn = tid % NQ;
    float s = 0.f;
#pragma unroll
    for (int ww = 0; ww < 8; ++ww) s += red[ww][c][qn];
    mine[c][qn] = s;
  }
  cluster.sync();
  if (tid < CWD * NQ) {
    const int c = tid / NQ, qn = tid % NQ;
    float s = 0.f;
#pragma unroll
    for (int r = 0; r < CLU; ++r) {
      const float* rem = cluster.map_shared_rank(&mine[0][0], r);
      s += rem[c * NQ + qn];
    }
    tot[c][qn] = s;
  }
  __syncthreads();
  const bool ok = sc[6] != 0.f;
  const float n00r = sc[0], n00i = sc[1], n01r = sc[2], n01i = sc[3], n11r = sc[4], n11i = sc[5];
  float alr[4], ali[4], ber[4], bei[4], zr[4], zi[4];
  float e2 = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int c = 4 * cg8 + j;
    const float akr = tot[c][0], aki = tot[c][1], bkr = tot[c][2], bki = tot[c][3];
    // α = N00 a + N01 b (coefficient of k_r), β = N01 a + N11 b (coefficient of v_r)
    alr[j] = n00r * akr - n00i * aki + n01r * bkr - n01i * bki;
    ali[j] = n00r * aki + n00i * akr + n01r * bki + n01i * bkr;
    ber[j] = n01r * akr - n01i * aki + n11r * bkr - n11i * bki;
    bei[j] = n01r * aki + n01i * akr + n11r * bki + n11i * bkr;
    const float qc = qs[c0 + j];
    if (fo) {
      const float wr = tot[c][4], wi = tot[c][5];
      zr[j] = 1.5f * qc - 0.5f * wr;
      zi[j] = -0.5f * wi;
      e2 += (wr - qc) * (wr - qc) + wi * wi;
    } else {
      zr[j] = qc;
      zi[j] = 0.f;
    }
  }
  float* part = A.part + ((size_t)item * nst + stripe) * D;
#pragma unroll
  for (int p = 0; p < NP; ++p) {
    const int rl = p * 32 + rp;
    float4 a = xr[p], bb = xi[p];
    if (ok) {
      const float kr = ks[row0 + rl], vr = vs[row0 + rl];
      a.x += kr * alr[0] + vr * ber[0]; a.y += kr * alr[1] + vr * ber[1];
      a.z += kr * alr[2] + vr * ber[2]; a.w += kr * alr[3] + vr * ber[3];
      bb.x += kr * ali[0] + vr * bei[0]; bb.y += kr * ali[1] + vr * bei[1];
      bb.z += kr * ali[2] + vr * bei[2]; bb.w += kr * ali[3] + vr * bei[3];
    }
    float o = a.x * zr[0] + a.y * zr[1] + a.z * zr[2] + a.w * zr[3];
    if (fo) o -= bb.x * zi[0] + bb.y * zi[1] + bb.z * zi[2] + bb.w * zi[3];
    o += __shfl_xor_sync(0xffffffffu, o, 1);
    o += __shfl_xor_sync(0xffffffffu, o, 2);
    o += __shfl_xor_sync(0xffffffffu, o, 4);
    if (cg8 == 0) part[row0 + rl] = o;
    const size_t e = (size_t)(row0 + rl) * D + c0;
    __stcs(reinterpret_cast<float4*>(Hr + e), a);
    __stcs(reinterpret_cast<float4*>(Hi + e), bb);
  }
  if (fo && rank == 0) {   // |E q|² of this stripe's columns (the same in every rank)
    e2 += __shfl_xor_sync(0xffffffffu, e2, 1);
    e2 += __shfl_xor_sync(0xffffffffu, e2, 2);
    e2 += __shfl_xor_sync(0xffffffffu, e2, 4);
    if (tid == 0) atomicAdd(&A.err2[item], e2);
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned int prev = atomicAdd(&A.cnt[item * CLU + rank], 1u);
    last_flag = (prev == (unsigned int)(nst - 1));
  }
  __syncthreads();
  if (last_flag) {
    __threadfence();
    const float* pb = A.part + (size_t)item * nst * D;
    T* y = static_cast<T*>(A.cout) + voff;
    for (int i = tid; i < RQ; i += DT) {
      float s = 0.f;
      for (int st = 0; st < nst; ++st) s += __ldcg(pb + (size_t)st * D + row0 + i);
      y[row0 + i] = from_f32<T>(s);
    }
    if (fo && rank == 0 && tid == 0) {
      const float err = __ldcg(&A.err2[item]);
      if (!(err <= DRIFT_TOL * DRIFT_TOL * sc[7])) atomicOr(&g_decode_status, 1u);
    }
  }
  cluster.sync();   // keep this CTA's shared memory alive until the cluster has read it
}

template <typename T, int NP>
__global__ void __launch_bounds__(DT, 2) decode_step_kernel(DecodeArgs A) {
  const int bid = blockIdx.x;
  if (bid < A.ns_pad) {
    if (bid < A.b * A.h) sssd_part<T>(A, bid);
    return;
  }
  if constexpr (NP > 0) cham_part<T, NP>(A, bid - A.ns_pad);
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
  L.cnt = off;  off = align_up(off + (size_t)b * CLU * sizeof(unsigned int), 256);
  L.err2 = off; off = align_up(off + (size_t)b * sizeof(float), 256);
  L.u = off;    off = align_up(off + (size_t)b * 2 * D * sizeof(float), 256);
  L.total = off + 256;
  return L;
}

template <typename T>
int launch_typed(const DecodeArgs& A, int np, cudaStream_t st) {
  const int ncham = (A.D > 0) ? A.b * (A.D / CWD) * CLU : 0;
  const int grid = A.ns_pad + ncham;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(DT);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CLU;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e;
  switch (np) {
    case 0: e = cudaLaunchKernelEx(&cfg, decode_step_kernel<T, 0>, A); break;
    case 1: e = cudaLaunchKernelEx(&cfg, decode_step_kernel<T, 1>, A); break;
    case 2: e = cudaLaunchKernelEx(&cfg, decode_step_kernel<T, 2>, A); break;
    case 3: e = cudaLaunchKernelEx(&cfg, decode_step_kernel<T, 3>, A); break;
    case 4: e = cudaLaunchKernelEx(&cfg, decode_step_kernel<T, 4>, A); break;
    case 5: e = cudaLaunchKernelEx(&cfg, decode_step_kernel<T, 5>, A); break;
    case 6: e = cudaLaunchKernelEx(&cfg, decode_step_kernel<T, 6>, A); break;
    case 7: e = cudaLaunchKernelEx(&cfg, decode_step_kernel<T, 7>, A); break;
    case 8: e = cudaLaunchKernelEx(&cfg, decode_step_kernel<T, 8>, A); break;
    default: set_error("verace_decode_step: unsupported D"); return VERACE_ERR_UNSUPPORTED;
  }
  if (e != cudaSuccess) {
    set_error("verace_decode_step: launch failed: %s", cudaGetErrorString(e));
    return VERACE_ERR_CUDA;
  }
  return check_launch("decode_step_kernel");
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
    VERACE_REQUIRE(D % (CWD * CLU) == 0 && D <= MAXD, VERACE_ERR_UNSUPPORTED,
                   "verace_decode_step: holographic dim %d unsupported (multiple of %d, at most %d)", D,
                   CWD * CLU, MAXD);
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
  A.ns_pad = (A.b * A.h + CLU - 1) / CLU * CLU;
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
  const int np = do_cham ? D / (CWD * CLU) : 0;
  switch (dtype) {
    case VERACE_F32: return launch_typed<float>(A, np, st);
    case VERACE_BF16: return launch_typed<__nv_bfloat16>(A, np, st);
    default: return launch_typed<__half>(A, np, st);
  }
}
