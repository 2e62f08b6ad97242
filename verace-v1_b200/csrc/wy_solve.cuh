// Coefficient matrix of a chunk's compact-WY product, by block forward substitution.
//
// For a chunk of 64 tokens whose factors are I + U_t N_t U_tᵀ (U_t = [k_t, v_t]), the
// product is I + W T Wᵀ with
//     T = (I - Nblk L)^-1 Nblk,   i.e.  T_t = N_t (e_t + sum_{tau < t} G_{t,tau} T_tau)
// where G = WᵀW (real) and T_t is the 2-row block of token t.  Rows and columns are
// addressed through row(t, kv) (kv = 0: k, 1: v), so callers may use any row order.
//
// The tokens are processed in 8 groups of 8.  For each group, the contribution of all
// earlier groups, ACC = sum_{tau in earlier groups} G_{t,tau} T_tau, is one small matrix
// product spread over all 256 threads; the 8-token recurrence inside the group then
// runs with one thread per column.  This replaces a 64-step dependent chain per column
// by 8 short ones.  Entries of T above the diagonal blocks come out exactly zero.
#pragma once

namespace verace {

constexpr int WY_C = 64;     // tokens per chunk
constexpr int WY_R = 128;    // rows of T
constexpr int WY_GS = 8;     // tokens per group

// G: [128][P] fp32 Gram matrix; N8: [64][8] per-token 2x2 complex blocks
// (m00r, m00i, m01r, m01i, m10r, m10i, m11r, m11i); Tr/Ti: [128][P] outputs (Ti unused
// when !CPLX); acc: scratch of 2 * 16 * 128 floats.  Must be called by all 256 threads.
template <bool CPLX, typename Row>
__device__ __forceinline__ void wy_solve(const float* __restrict__ G, int P, const float* __restrict__ N8,
                                         float* __restrict__ Tr, float* __restrict__ Ti, float* __restrict__ acc,
                                         Row row, int tid) {
  float* accr = acc;
  float* acci = acc + 2 * WY_GS * WY_R;
  const int col = tid % WY_R, rh = tid / WY_R;   // rh: which 8 of the group's 16 rows
  for (int g = 0; g < WY_C / WY_GS; ++g) {
    {
      float ar[8], ai[8];
      int grow[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int i16 = rh * 8 + u;
        grow[u] = row(g * WY_GS + (i16 >> 1), i16 & 1) * P;
        ar[u] = 0.f;
        ai[u] = 0.f;
      }
      for (int tp = 0; tp < g * WY_GS; ++tp) {
#pragma unroll
        for (int kv = 0; kv < 2; ++kv) {
          const int rr = row(tp, kv);
          const float xr = Tr[rr * P + col];
          const float xi = CPLX ? Ti[rr * P + col] : 0.f;
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const float gg = G[grow[u] + rr];
            ar[u] = fmaf(gg, xr, ar[u]);
            if (CPLX) ai[u] = fmaf(gg, xi, ai[u]);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        accr[(rh * 8 + u) * WY_R + col] = ar[u];
        if (CPLX) acci[(rh * 8 + u) * WY_R + col] = ai[u];
      }
    }
    __syncthreads();
    if (tid < WY_R) {
      for (int tt = 0; tt < WY_GS; ++tt) {
        const int t = g * WY_GS + tt;
        const int r0 = row(t, 0), r1 = row(t, 1);
        float x0r = accr[(2 * tt) * WY_R + col] + (r0 == col ? 1.f : 0.f);
        float x1r = accr[(2 * tt + 1) * WY_R + col] + (r1 == col ? 1.f : 0.f);
        float x0i = CPLX ? acci[(2 * tt) * WY_R + col] : 0.f;
        float x1i = CPLX ? acci[(2 * tt + 1) * WY_R + col] : 0.f;
        for (int tp = g * WY_GS; tp < t; ++tp) {
          const int q0 = row(tp, 0), q1 = row(tp, 1);
          const float a0r = Tr[q0 * P + col], a1r = Tr[q1 * P + col];
          const float a0i = CPLX ? Ti[q0 * P + col] : 0.f, a1i = CPLX ? Ti[q1 * P + col] : 0.f;
          const float g00 = G[r0 * P + q0], g01 = G[r0 * P + q1];
          const float g10 = G[r1 * P + q0], g11 = G[r1 * P + q1];
          x0r += g00 * a0r + g01 * a1r;
          x1r += g10 * a0r + g11 * a1r;
          if (CPLX) {
            x0i += g00 * a0i + g01 * a1i;
            x1i += g10 * a0i + g11 * a1i;
          }
        }
        const float* n = N8 + t * 8;
        // [T_r0; T_r1] = [[m00, m01], [m10, m11]] [x0; x1]  (complex)
        Tr[r0 * P + col] = n[0] * x0r - n[1] * x0i + n[2] * x1r - n[3] * x1i;
        Tr[r1 * P + col] = n[4] * x0r - n[5] * x0i + n[6] * x1r - n[7] * x1i;
        if (CPLX) {
          Ti[r0 * P + col] = n[0] * x0i + n[1] * x0r + n[2] * x1i + n[3] * x1r;
          Ti[r1 * P + col] = n[4] * x0i + n[5] * x0r + n[6] * x1i + n[7] * x1r;
        }
      }
    }
    __syncthreads();
  }
}

}  // namespace verace
