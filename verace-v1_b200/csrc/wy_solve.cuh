// Coefficient matrix of a chunk's compact-WY product, by recursive block inversion.
//
// For a chunk of 64 tokens whose factors are I + U_t N_t U_tᵀ (U_t = [k_t, v_t]), the
// product is I + W T Wᵀ with
//     T = (I - Nblk L)^-1 Nblk,   i.e.  T_t = N_t (e_t + sum_{tau < t} G_{t,tau} T_tau)
// where G = WᵀW (real, symmetric), L its strictly block-lower part and T_t the 2-row
// block of token t.  Rows are interleaved: row 2t + kv holds token t's k (kv = 0) or
// v (kv = 1), so a run of tokens is a run of rows.
//
// Splitting the tokens of any run into a first half a and a second half b,
//     T = [[T_aa, 0], [T_bb G_ba T_aa, T_bb]],
// where T_aa and T_bb are the same matrices for the halves on their own.  So T is built
// bottom-up: the 8 diagonal blocks of 8 tokens (16 rows) by forward substitution, one
// thread per column with the column in registers; then three levels that join pairs of
// 16-, 32- and 64-row blocks with two register-tiled products each,
//     X = G_ba T_aa   (written where T_ba goes: nothing reads that block yet)
//     T_ba = T_bb X   (every thread holds its 4 x 4 tile before any is stored).
// Entries above the diagonal blocks are exactly zero.  All arithmetic is fp32.
//
// The solver reads only the lower blocks of G (the diagonal blocks' lower triangles and
// the G_ba blocks), each of them for the last time in the step that writes T's entries
// at the same place, and every such step finishes its reads (a barrier) before its
// stores.  So T may overwrite G in place (Tr == G), which keeps one 128 x 128 fp32 array
// out of shared memory.
#pragma once

namespace verace {

constexpr int WY_C = 64;     // tokens per chunk
constexpr int WY_R = 128;    // rows of T

namespace wy {

__device__ __forceinline__ void fma44(float (&c)[4][4], const float4 (&a)[4], const float4 (&b)[4], float sgn) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float av[4] = {sgn * a[i].x, sgn * a[i].y, sgn * a[i].z, sgn * a[i].w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      c[i][0] = fmaf(av[k], b[k].x, c[i][0]);
      c[i][1] = fmaf(av[k], b[k].y, c[i][1]);
      c[i][2] = fmaf(av[k], b[k].z, c[i][2]);
      c[i][3] = fmaf(av[k], b[k].w, c[i][3]);
    }
  }
}

__device__ __forceinline__ void ld4(float4 (&x)[4], const float* p, int P) {
#pragma unroll
  for (int i = 0; i < 4; ++i) x[i] = *reinterpret_cast<const float4*>(p + i * P);
}

__device__ __forceinline__ void st44(float* p, int P, const float (&c)[4][4]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) *reinterpret_cast<float4*>(p + i * P) = make_float4(c[i][0], c[i][1], c[i][2], c[i][3]);
}

__device__ __forceinline__ void zero44(float (&c)[4][4]) {
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) c[i][j] = 0.f;
}

// One join level: blocks of B rows, pairs (a, b) = rows [2pB, 2pB + B), [2pB + B, 2pB + 2B).
template <int B, bool CPLX>
__device__ __forceinline__ void join_level(const float* G, int P, float* Tr, float* __restrict__ Ti, int tid) {
  constexpr int TPB = B / 4;                  // tiles per block side
  constexpr int TILES = (WY_R / (2 * B)) * TPB * TPB;
  const bool act = tid < TILES;
  const int pair = tid / (TPB * TPB), tt = tid % (TPB * TPB), tm = tt / TPB, tn = tt % TPB;
  const int a0 = 2 * B * pair, b0 = a0 + B;
  const int row = b0 + 4 * tm, col = a0 + 4 * tn;
  float cr[4][4], ci[4][4];
  // X = G_ba T_aa
  if (act) {
    zero44(cr);
    if (CPLX) zero44(ci);
    const float* ga = G + row * P + a0;
    const float* tr = Tr + a0 * P + col;
    const float* ti = CPLX ? Ti + a0 * P + col : nullptr;
#pragma unroll 4
    for (int k = 0; k < B; k += 4) {
      float4 a[4], b[4];
      ld4(a, ga + k, P);
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = *reinterpret_cast<const float4*>(tr + (k + j) * P);
      fma44(cr, a, b, 1.f);
      if (CPLX) {
#pragma unroll
        for (int j = 0; j < 4; ++j) b[j] = *reinterpret_cast<const float4*>(ti + (k + j) * P);
        fma44(ci, a, b, 1.f);
      }
    }
  }
  __syncthreads();   // every read of G_ba is done (X replaces it when Tr == G)
  if (act) {
    st44(Tr + row * P + col, P, cr);
    if (CPLX) st44(Ti + row * P + col, P, ci);
  }
  __syncthreads();
  // T_ba = T_bb X   (complex: (Tr + i Ti)(Xr + i Xi))
  if (act) {
    zero44(cr);
    if (CPLX) zero44(ci);
    const float* ar = Tr + row * P + b0;
    const float* ai = CPLX ? Ti + row * P + b0 : nullptr;
    const float* xr = Tr + b0 * P + col;
    const float* xi = CPLX ? Ti + b0 * P + col : nullptr;
#pragma unroll 2
    for (int k = 0; k < B; k += 4) {
      float4 a[4], b[4];
      ld4(a, ar + k, P);
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = *reinterpret_cast<const float4*>(xr + (k + j) * P);
      fma44(cr, a, b, 1.f);
      if (CPLX) {
        float4 a2[4], b2[4];
        ld4(a2, ai + k, P);
#pragma unroll
        for (int j = 0; j < 4; ++j) b2[j] = *reinterpret_cast<const float4*>(xi + (k + j) * P);
        fma44(cr, a2, b2, -1.f);
        fma44(ci, a, b2, 1.f);
        fma44(ci, a2, b, 1.f);
      }
    }
  }
  __syncthreads();
  if (act) {
    st44(Tr + row * P + col, P, cr);
    if (CPLX) st44(Ti + row * P + col, P, ci);
  }
  __syncthreads();
}

}  // namespace wy

// G: [128][P] fp32 Gram matrix in the interleaved row order, P a multiple of 4 and every
// array 16-byte aligned; N8: [64][8] per-token 2x2 complex blocks
// (m00r, m00i, m01r, m01i, m10r, m10i, m11r, m11i); Tr/Ti: [128][P] outputs (Ti unused
// when !CPLX).  Tr may be G itself (G is then destroyed); Ti must not overlap G.  Must be
// called by all 256 threads of the CTA; ends with a barrier.
template <bool CPLX>
__device__ __forceinline__ void wy_solve(const float* G, int P, const float* __restrict__ N8, float* Tr,
                                         float* __restrict__ Ti, int tid) {
  // zero the blocks of T above the 16-row diagonal blocks (every other entry is written
  // below; G's entries there are never read)
  for (int e = tid; e < WY_R * (WY_R / 4); e += 256) {
    const int r = e / (WY_R / 4), c4 = e % (WY_R / 4);
    if ((4 * c4) / 16 <= r / 16) continue;
    *reinterpret_cast<float4*>(Tr + r * P + 4 * c4) = make_float4(0.f, 0.f, 0.f, 0.f);
    if (CPLX) *reinterpret_cast<float4*>(Ti + r * P + 4 * c4) = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  __syncthreads();
  // diagonal blocks: leaf j = tokens [8j, 8j + 8) = rows [16j, 16j + 16); thread = one
  // of the leaf's 16 columns, the column kept in registers
  const int j = tid >> 4, c = tid & 15, r0 = 16 * j;
  float xr[16], xi[16];
  if (tid < 128) {
    const float* Gl = G + r0 * P + r0;
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      float a0r = (2 * t == c) ? 1.f : 0.f, a1r = (2 * t + 1 == c) ? 1.f : 0.f;
      float a0i = 0.f, a1i = 0.f;
#pragma unroll
      for (int tp = 0; tp < t; ++tp) {
        const float2 g0 = *reinterpret_cast<const float2*>(Gl + (2 * t) * P + 2 * tp);
        const float2 g1 = *reinterpret_cast<const float2*>(Gl + (2 * t + 1) * P + 2 * tp);
        a0r += g0.x * xr[2 * tp] + g0.y * xr[2 * tp + 1];
        a1r += g1.x * xr[2 * tp] + g1.y * xr[2 * tp + 1];
        if (CPLX) {
          a0i += g0.x * xi[2 * tp] + g0.y * xi[2 * tp + 1];
          a1i += g1.x * xi[2 * tp] + g1.y * xi[2 * tp + 1];
        }
      }
      const float* n = N8 + (8 * j + t) * 8;
      // [T_r0; T_r1] = [[m00, m01], [m10, m11]] [a0; a1]  (complex)
      xr[2 * t] = n[0] * a0r - n[1] * a0i + n[2] * a1r - n[3] * a1i;
      xr[2 * t + 1] = n[4] * a0r - n[5] * a0i + n[6] * a1r - n[7] * a1i;
      xi[2 * t] = n[0] * a0i + n[1] * a0r + n[2] * a1i + n[3] * a1r;
      xi[2 * t + 1] = n[4] * a0i + n[5] * a0r + n[6] * a1i + n[7] * a1r;
    }
  }
  __syncthreads();   // the leaf's reads of G are done (T replaces it when Tr == G)
  if (tid < 128) {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      Tr[(r0 + i) * P + r0 + c] = xr[i];
      if (CPLX) Ti[(r0 + i) * P + r0 + c] = xi[i];
    }
  }
  __syncthreads();
  wy::join_level<16, CPLX>(G, P, Tr, Ti, tid);
  wy::join_level<32, CPLX>(G, P, Tr, Ti, tid);
  wy::join_level<64, CPLX>(G, P, Tr, Ti, tid);
}

}  // namespace verace
