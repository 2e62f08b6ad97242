// CHAM scan on the tcgen05 tensor cores (sm_100a), for holographic widths D that are
// multiples of 128 and a fresh hologram (H_0 = I, so the readout vectors are y_t = q_t).
//
// Same chunked compact-WY recurrence as cham_scan.cu (see the derivation there), with
// chunks of C = 64 tokens so that the chunk rank 2C = 128 is one tensor-core tile:
//     Z = Wᵀ S,  [P1 | P2] = [Tr | Ti] Z,  Cm = (P1_re - P2_im) + i (P1_im + P2_re)
//     S_next = S + W Cm,   E = Re(Cm) Y (reduced over column blocks),
//     rec_t = Re(S y_t) + sum_{tau<=t} U_tau E_tau,t
// fp32 operands enter the bf16 tensor cores as hi + lo bf16 pairs (x = hi + lo to 16
// significant bits); products that need it take hi*hi + hi*lo + lo*hi, accumulated in
// fp32 in tensor memory.  bf16 q/k/v (the model's dtype) are exact in bf16 and need
// no split; fp32 q/k/v are split too.  The state stays fp32 in global memory.
//
// Kernels (per call: one prep launch, then per chunk one colpass + one readout):
//   cham_tc_prep     T (complex 128x128) for every chunk, written as bf16 hi/lo tiles
//                    in the tensor-core operand layout; zeroes the chunk's E block.
//   cham_tc_colpass  one CTA per (item, 32 complex columns): Z, Cm, E partial, and
//                    that column block of S_next.  TMEM: 320 of 512 columns.
//   cham_tc_readout  one CTA per (item, 128 rows): Re(S Y) + W mask(E).
#include "common.cuh"

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include "tc.cuh"
#include "wy_solve.cuh"

#include "tmap.cuh"

namespace verace {
namespace {

constexpr int C2 = 64;          // tokens per chunk
constexpr int R2 = 128;         // chunk rank (k and v of 64 tokens)
constexpr int NB2 = 32;         // complex columns per colpass CTA
constexpr int N2 = 2 * NB2;     // real columns (re | im) per colpass CTA
constexpr int KT = 128;         // rows of S per K tile
constexpr int THR = 256;
constexpr uint32_t MAX_POLLS = 1u << 22;
constexpr int PREP_DT = 32;

__device__ int g_tc_status = 0;  // non-zero after a bounded wait gave up

// tile sizes in bytes
constexpr int W_TILE = R2 * KT * 2;        // 32 KB: 128 vectors x 128 elements, bf16
constexpr int H_TILE = KT * N2 * 2;        // 16 KB: 128 rows x 64 columns, bf16
constexpr int T_TILE = R2 * R2 * 2;        // 32 KB: 128 x 128 bf16
constexpr int Z_TILE = R2 * N2 * 2;        // 16 KB: 128 x 64 bf16
constexpr int CA_TILE = R2 * NB2 * 2;      //  8 KB: 128 x 32 bf16
constexpr int Y_TILE = C2 * NB2 * 2;       //  4 KB: 64 tokens x 32 columns bf16

constexpr int RING = 12;         // chunks per column-pass group; the ring keeps two groups' end states

struct TcWs {
  unsigned char* T;          // [b][nch][4][T_TILE]: Tr_hi, Tr_lo, Ti_hi, Ti_lo
  float* E;                  // [b][nch][R2][C2]
  unsigned long long* bad;   // [b][nch]
  float* Hre;
  float* Him;
  float* ring;               // [min(nch, 2 RING)][b][D][D]: real parts of chunk end states (fp32 rows,
                             // or in the batched schedule the readout's bf16 operand images, half a slot)
  int nring;
  unsigned char* cm;         // [2][b][D/64][64 KB]: fused schedule, Cm operands between launches
};

size_t tc_ws_layout(int b, int s, int D, TcWs* w, char* base) {
  const size_t nch = ((size_t)s + C2 - 1) / C2;
  size_t off = 0;
  auto take = [&](size_t bytes) { size_t o = off; off += align_up(bytes, 256); return base ? (void*)(base + o) : nullptr; };
  TcWs t;
  t.T = (unsigned char*)take((size_t)b * nch * 4 * T_TILE);
  t.E = (float*)take((size_t)b * nch * R2 * C2 * sizeof(float));
  t.bad = (unsigned long long*)take((size_t)b * nch * sizeof(unsigned long long));
  const bool ping = nch >= 2;
  t.Hre = (float*)take(ping ? (size_t)b * D * D * sizeof(float) : 0);
  t.Him = (float*)take(ping ? (size_t)b * D * D * sizeof(float) : 0);
  t.nring = (int)std::min<size_t>(nch, 2 * RING);
  t.ring = (float*)take((size_t)t.nring * b * D * D * sizeof(float));
  t.cm = (unsigned char*)take((size_t)2 * b * (D / 64) * (64 * 1024));
  if (w) *w = t;
  return off + 256;
}

__device__ __forceinline__ void record_timeout() { atomicExch(&g_tc_status, 1); }

// byte offset of element (r, k) in a K-major tile with R rows
__device__ __forceinline__ int kmaj(int r, int k, int R) { return ((k >> 3) * R + r) * 16 + (k & 7) * 2; }
// byte offset of element (k, n) in a directly built MN-major tile with NG = N/8 groups
__device__ __forceinline__ int mnmaj(int k, int n, int NG) { return (((k >> 3) * NG + (n >> 3)) * 128) + (k & 7) * 16 + (n & 7) * 2; }

__device__ __forceinline__ void load8(const __nv_bfloat16* p, float* x) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&u);
#pragma unroll
  for (int i = 0; i < 8; ++i) x[i] = __bfloat162float(h[i]);
}
__device__ __forceinline__ void load8(const float* p, float* x) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  const float4 b = *reinterpret_cast<const float4*>(p + 4);
  x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}

// Stage 8 consecutive input elements as one 16-byte bf16 chunk (hi) and, for fp32
// inputs, the matching lo chunk.  Non-finite or padded tokens are staged as zeros.
template <typename T>
__device__ __forceinline__ void stage8(const T* src, bool valid, unsigned char* hi, unsigned char* lo) {
  if (sizeof(T) == 2) {
    uint4 u = make_uint4(0, 0, 0, 0);
    if (valid) u = *reinterpret_cast<const uint4*>(src);
    *reinterpret_cast<uint4*>(hi) = u;
  } else {
    float x[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (valid) load8(src, x);
    uint4 h, l;
    tc::split8(x, h, l);
    *reinterpret_cast<uint4*>(hi) = h;
    *reinterpret_cast<uint4*>(lo) = l;
  }
}

// Row order of the chunk's W = [k_1 .. k_64, v_1 .. v_64]: row r holds token tok(r) = r % 64,
// the k vector for r < 64 and the v vector for r >= 64 (so that k and v rows each form
// one contiguous 64-row block, the shape a TMA box delivers).  T, Z, Cm and E use it too.
__device__ __forceinline__ int tok(int r) { return r & (C2 - 1); }
// split-order row r (k block 0..63, v block 64..127) -> interleaved row 2 * token + kv
__device__ __forceinline__ int ilv(int r) { return 2 * (r & (C2 - 1)) + (r >> 6); }
__device__ __forceinline__ bool is_v(int r) { return r >= C2; }

// Stage the chunk's k/v vectors, elements [i0, i0+KT), as a K-major tile with rows = r.
template <typename T>
__device__ __forceinline__ void stage_w(unsigned char* sw_hi, unsigned char* sw_lo,
                                        const T* __restrict__ k, const T* __restrict__ v,
                                        int item, int S, int D, int t0, int nt, unsigned long long bad,
                                        int i0, int tid) {
  for (int e = tid; e < R2 * (KT / 8); e += THR) {
    const int r = e % R2, g = e / R2;  // consecutive threads -> consecutive vectors
    const int tau = tok(r);
    const bool valid = tau < nt && !((bad >> tau) & 1ull);
    const T* src = (is_v(r) ? v : k) + ((size_t)item * S + t0 + (valid ? tau : 0)) * D + i0 + g * 8;
    stage8(src, valid, sw_hi + kmaj(r, g * 8, R2), sw_lo + kmaj(r, g * 8, R2));
  }
}

// ---------------------------------------------------------------------------------
// prep: W Gram matrix, N_t, complex T by block forward substitution (fp32 SIMT), then
// T written as bf16 hi/lo K-major 128x128 tiles.  smem: Wt [DT][R2+1], Gs/Tr/Ti [R2][R2+1]
template <typename T>
__global__ void __launch_bounds__(THR)
cham_tc_prep(const T* __restrict__ k, const T* __restrict__ v, const float* __restrict__ gamma,
             unsigned char* __restrict__ Tws, float* __restrict__ Ews, unsigned long long* __restrict__ badws,
             int S, int D, int nch) {
  extern __shared__ float sm[];
  constexpr int P = R2 + 1;
  float* Wt = sm;
  float* Gs = Wt + PREP_DT * P;
  float* Tr = Gs + R2 * P;
  float* Ti = Tr + R2 * P;
  __shared__ float Ns[C2 * 6];
  __shared__ unsigned long long bad_bits;
  const int c = blockIdx.x, item = blockIdx.y, tid = threadIdx.x;
  const int t0 = c * C2, nt = min(C2, S - t0);
  if (tid == 0) bad_bits = 0ull;
  for (int e = tid; e < R2 * P; e += THR) Gs[e] = 0.f;
  for (int i0 = 0; i0 < D; i0 += PREP_DT) {
    __syncthreads();
    for (int e = tid; e < PREP_DT * R2; e += THR) {
      const int i = e / R2, r = e % R2, tau = r >> 1;
      float val = 0.f;
      if (tau < nt && i0 + i < D) {
        const size_t off = ((size_t)item * S + t0 + tau) * D + i0 + i;
        val = to_f32((r & 1) ? v[off] : k[off]);
      }
      Wt[i * P + r] = val;
      if (!isfinite(val)) atomicOr(&bad_bits, 1ull << tau);
    }
    __syncthreads();
    if (bad_bits) {
      for (int e = tid; e < PREP_DT * R2; e += THR)
        if ((bad_bits >> ((e % R2) >> 1)) & 1ull) Wt[(e / R2) * P + e % R2] = 0.f;
      __syncthreads();
    }
    smem_gemm<4, 4, true>(R2, R2, PREP_DT, Wt, 1, P, Wt, P, 1, Gs, P, 1, tid, THR);
  }
  __syncthreads();
  if (tid < C2 && tid < nt && !isfinite(gamma[(size_t)item * S + t0 + tid])) atomicOr(&bad_bits, 1ull << tid);
  __syncthreads();
  if (tid < C2) {
    const int tau = tid;
    float n00r = 0.f, n00i = 0.f, n01r = 0.f, n01i = 0.f, n11r = 0.f, n11i = 0.f;
    bool flagged = (bad_bits >> tau) & 1ull;
    if (tau < nt && !flagged) {
      const float kk = Gs[(2 * tau) * P + 2 * tau];
      const float vv = Gs[(2 * tau + 1) * P + 2 * tau + 1];
      const float kv = Gs[(2 * tau) * P + 2 * tau + 1];
      const float g = gamma[(size_t)item * S + t0 + tau];
      const float cc = 0.5f * g;
      const float dr = 1.f + cc * cc * (kk * vv - kv * kv);
      const float di = -2.f * cc * kv;
      const float m2 = dr * dr + di * di;
      const float fr = 2.f * cc * dr / m2;
      const float fi = -2.f * cc * di / m2;
      n00r = fr * (-cc * vv); n00i = fi * (-cc * vv);
      n11r = fr * (-cc * kk); n11i = fi * (-cc * kk);
      n01r = fr * (cc * kv) - fi; n01i = fr + fi * (cc * kv);
      const bool ok = isfinite(kk) && isfinite(vv) && isfinite(kv) && isfinite(n00r) && isfinite(n00i) &&
                      isfinite(n01r) && isfinite(n01i) && isfinite(n11r) && isfinite(n11i);
      if (!ok) {
        n00r = n00i = n01r = n01i = n11r = n11i = 0.f;
        atomicOr(&bad_bits, 1ull << tau);
        flagged = true;
      }
    }
    if (flagged) {
      for (int r = 0; r < R2; ++r) {
        Gs[(2 * tau) * P + r] = 0.f; Gs[(2 * tau + 1) * P + r] = 0.f;
        Gs[r * P + 2 * tau] = 0.f; Gs[r * P + 2 * tau + 1] = 0.f;
      }
    }
    float* n = Ns + tau * 6;
    n[0] = n00r; n[1] = n00i; n[2] = n01r; n[3] = n01i; n[4] = n11r; n[5] = n11i;
  }
  __syncthreads();
  if (tid < R2) {
    const int sg = tid, blk = sg >> 1;
    for (int r = 0; r < 2 * blk; ++r) { Tr[r * P + sg] = 0.f; Ti[r * P + sg] = 0.f; }
    for (int t = blk; t < C2; ++t) {
      float x0r = (sg == 2 * t) ? 1.f : 0.f, x0i = 0.f;
      float x1r = (sg == 2 * t + 1) ? 1.f : 0.f, x1i = 0.f;
      for (int tp = blk; tp < t; ++tp) {
        const float a0r = Tr[(2 * tp) * P + sg], a0i = Ti[(2 * tp) * P + sg];
        const float a1r = Tr[(2 * tp + 1) * P + sg], a1i = Ti[(2 * tp + 1) * P + sg];
        const float g00 = Gs[(2 * t) * P + 2 * tp], g01 = Gs[(2 * t) * P + 2 * tp + 1];
        const float g10 = Gs[(2 * t + 1) * P + 2 * tp], g11 = Gs[(2 * t + 1) * P + 2 * tp + 1];
        x0r += g00 * a0r + g01 * a1r; x0i += g00 * a0i + g01 * a1i;
        x1r += g10 * a0r + g11 * a1r; x1i += g10 * a0i + g11 * a1i;
      }
      const float* n = Ns + t * 6;
      Tr[(2 * t) * P + sg] = n[0] * x0r - n[1] * x0i + n[2] * x1r - n[3] * x1i;
      Ti[(2 * t) * P + sg] = n[0] * x0i + n[1] * x0r + n[2] * x1i + n[3] * x1r;
      Tr[(2 * t + 1) * P + sg] = n[2] * x0r - n[3] * x0i + n[4] * x1r - n[5] * x1i;
      Ti[(2 * t + 1) * P + sg] = n[2] * x0i + n[3] * x0r + n[4] * x1i + n[5] * x1r;
    }
  }
  __syncthreads();
  const size_t chunk = (size_t)item * nch + c;
  unsigned char* To = Tws + chunk * 4 * T_TILE;
  // K-major tiles: A(m = r, k = r') = T[r][r'] in the kernels' row order (k block, v
  // block); T was formed with rows interleaved (2*tau + {k, v}).
  auto src_idx = [](int ro) { return 2 * tok(ro) + (is_v(ro) ? 1 : 0); };
  for (int e = tid; e < R2 * (R2 / 8); e += THR) {
    const int r = e % R2, g = e / R2;
    const int rs = src_idx(r);
    float xr[8], xi[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int cs = src_idx(g * 8 + j);
      xr[j] = Tr[rs * P + cs];
      xi[j] = Ti[rs * P + cs];
    }
    uint4 h, l;
    const int off = kmaj(r, g * 8, R2);
    tc::split8(xr, h, l);
    *reinterpret_cast<uint4*>(To + 0 * T_TILE + off) = h;
    *reinterpret_cast<uint4*>(To + 1 * T_TILE + off) = l;
    tc::split8(xi, h, l);
    *reinterpret_cast<uint4*>(To + 2 * T_TILE + off) = h;
    *reinterpret_cast<uint4*>(To + 3 * T_TILE + off) = l;
  }
  float* Eo = Ews + chunk * R2 * C2;
  for (int e = tid; e < R2 * C2; e += THR) Eo[e] = 0.f;
  if (tid == 0) badws[chunk] = bad_bits;
}

// ---------------------------------------------------------------------------------
// colpass.  Shared memory (bytes), bf16 inputs (two-stage pipeline over the K tiles):
//   U [0,128K)     phases A/B: stage s at s*64K = W (32K) | H hi (16K) | H lo (16K)
//                  phase T:    Tr hi | Tr lo | Ti hi | Ti lo (4 x 32K)
//                  phase E:    Re(Cm) as the A operand (hi 8K | lo 8K) | Y block (4K)
//   Zs [128K,160K) Z as the B operand of T Z (MN-major, hi 16K | lo 16K)
//   Cs [160K,192K) Cm as the B operand of W Cm (MN-major, hi 16K | lo 16K)
//   barriers, TMEM slot
// fp32 inputs need the lo halves of W and Y as well and run single-buffered:
//   U [0,128K) = W hi | H hi | H lo | W lo; Ca at 192K, Y at 208K (hi | lo).
// TMEM columns: Z [0,64) P1 [64,128) P2 [128,192) E [192,256) dH0 [256,320) dH1 [320,384)
constexpr int SM_Z = 128 * 1024, SM_C = 160 * 1024;
constexpr int SM_CA_F32 = 192 * 1024, SM_Y_F32 = 208 * 1024;
constexpr int SM_BAR_BF16 = 192 * 1024, SM_BAR_F32 = 216 * 1024;
constexpr int STAGE = 64 * 1024;
constexpr int colpass_smem(bool f32) { return (f32 ? SM_BAR_F32 : SM_BAR_BF16) + 128; }

template <typename T>
__global__ void __launch_bounds__(THR, 1)
cham_tc_colpass(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                const unsigned char* __restrict__ Tws, float* __restrict__ Ews,
                const unsigned long long* __restrict__ badws,
                const float* __restrict__ src_r, const float* __restrict__ src_i,
                float* __restrict__ dst_r, float* __restrict__ dst_i, int S, int D, int nch, int c) {
  extern __shared__ __align__(1024) unsigned char smc[];
  constexpr bool F32IN = sizeof(T) == 4;
  unsigned char* sT = smc;
  unsigned char* sZh = smc + SM_Z;
  unsigned char* sZl = sZh + Z_TILE;
  unsigned char* sCh = smc + SM_C;
  unsigned char* sCl = sCh + Z_TILE;
  unsigned char* sAh = F32IN ? smc + SM_CA_F32 : smc;
  unsigned char* sAl = sAh + CA_TILE;
  unsigned char* sYh = F32IN ? smc + SM_Y_F32 : smc + 2 * CA_TILE;
  unsigned char* sYl = sYh + Y_TILE;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smc + (F32IN ? SM_BAR_F32 : SM_BAR_BF16));
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 8);
  // barrier roles: 0,1 = K-tile stages of phases A and B, 2 = single-shot phases
  auto stage_w_ptr = [&](int st) { return F32IN ? smc : smc + st * STAGE; };
  auto stage_hh_ptr = [&](int st) { return F32IN ? smc + W_TILE : smc + st * STAGE + W_TILE; };
  unsigned char* sWl = smc + W_TILE + 2 * H_TILE;   // fp32 inputs only

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int item = blockIdx.y, j0 = blockIdx.x * NB2;
  const int t0 = c * C2, nt = min(C2, S - t0);
  const size_t chunk = (size_t)item * nch + c;
  const unsigned long long bad = badws[chunk];
  const size_t soff = (size_t)item * D * D;
  const float* sr = src_r ? src_r + soff : nullptr;
  const float* si = src_i ? src_i + soff : nullptr;

  if (warp == 0) tc::tmem_alloc(tslot, 512);
  if (tid == 0) {
    for (int i = 0; i < 3; ++i) tc::mbar_init(&bars[i], 1);
    tc::fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = *tslot;
  const uint32_t tZ = tbase, tP1 = tbase + 64, tP2 = tbase + 128, tE = tbase + 192, tDH = tbase + 256;
  const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
  const int row = 32 * (warp & 3) + lane;   // TMEM lane == accumulator row of this thread
  const int half = warp >> 2;               // which half of the accumulator columns
  uint32_t ph[3] = {0u, 0u, 0u};
  bool failed = false;

  auto wait_bar = [&](int b) -> bool {
    const bool ok = tc::mbar_wait(&bars[b], ph[b], MAX_POLLS);
    ph[b] ^= 1u;
    if (__syncthreads_or(!ok)) { if (tid == 0) record_timeout(); return false; }
    tc::fence_after_sync();
    return true;
  };
  const int NT = D / KT;

  // W tile of K tile kt into stage st: bf16 by cp.async, fp32 through registers (split)
  auto stage_w_tile = [&](int kt, int st) {
    if constexpr (F32IN) {
      stage_w<T>(stage_w_ptr(st), sWl, k, v, item, S, D, t0, nt, bad, kt * KT, tid);
    } else {
      unsigned char* sw = stage_w_ptr(st);
#pragma unroll
      for (int u = 0; u < (R2 * KT / 8) / THR; ++u) {
        const int e = tid + THR * u;
        const int r = e % R2, g = e / R2, tau = tok(r);
        const bool valid = tau < nt && !((bad >> tau) & 1ull);
        const T* src = (is_v(r) ? v : k) + ((size_t)item * S + t0 + (valid ? tau : 0)) * D + kt * KT + g * 8;
        tc::cp_async16(sw + kmaj(r, g * 8, R2), src, valid);
      }
      tc::cp_async_commit();
    }
  };
  // H tile (rows [kt*KT, +KT), columns re|im of this block) into stage st, split hi/lo.
  // All global loads of the thread are issued before any conversion.
  auto stage_h_tile = [&](int kt, int st) {
    unsigned char* hh = stage_hh_ptr(st);
    unsigned char* hl = hh + H_TILE;
    constexpr int PER = (KT * (N2 / 8)) / THR;   // 4 chunks of 8 columns per thread
    float4 buf[PER][2];
#pragma unroll
    for (int u = 0; u < PER; ++u) {
      const int e = tid + THR * u;
      const int g = e % (N2 / 8), i = e / (N2 / 8);
      const int col = j0 + (g & 3) * 8, gi = kt * KT + i;
      if (sr) {
        const float* p = ((g < 4) ? sr : si) + (size_t)gi * D + col;
        buf[u][0] = *reinterpret_cast<const float4*>(p);
        buf[u][1] = *reinterpret_cast<const float4*>(p + 4);
      } else {
        float x[8];
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) x[jj] = (g < 4 && gi == col + jj) ? 1.f : 0.f;
        buf[u][0] = make_float4(x[0], x[1], x[2], x[3]);
        buf[u][1] = make_float4(x[4], x[5], x[6], x[7]);
      }
    }
#pragma unroll
    for (int u = 0; u < PER; ++u) {
      const int e = tid + THR * u;
      const int g = e % (N2 / 8), i = e / (N2 / 8);
      const float x[8] = {buf[u][0].x, buf[u][0].y, buf[u][0].z, buf[u][0].w,
                          buf[u][1].x, buf[u][1].y, buf[u][1].z, buf[u][1].w};
      uint4 h, l;
      tc::split8(x, h, l);
      *reinterpret_cast<uint4*>(hh + mnmaj(i, g * 8, N2 / 8)) = h;
      *reinterpret_cast<uint4*>(hl + mnmaj(i, g * 8, N2 / 8)) = l;
    }
  };

  // ---------------- phase A: Z = Wᵀ S[:, block], pipelined over K tiles
  constexpr uint32_t ID_Z = tc::idesc_bf16(128, N2, false, true);
  {
    int outstanding[2] = {0, 0};
    for (int kt = 0; kt < NT && !failed; ++kt) {
      const int st = F32IN ? 0 : (kt & 1);
      if (outstanding[st]) { failed = !wait_bar(st); outstanding[st] = 0; if (failed) break; }
      stage_w_tile(kt, st);
      stage_h_tile(kt, st);
      if constexpr (!F32IN) tc::cp_async_wait_all();
      tc::fence_proxy_async();
      __syncthreads();
      if (tid == 0) {
        tc::fence_after_sync();
        const uint32_t aw = tc::smem_addr(stage_w_ptr(st)), awl = tc::smem_addr(sWl);
        const uint32_t bh = tc::smem_addr(stage_hh_ptr(st)), bl = bh + H_TILE;
#pragma unroll 1
        for (int ks = 0; ks < KT / 16; ++ks) {
          const uint64_t a = tc::sdesc(aw + ks * 2 * R2 * 16, R2 * 16, 128);
          const uint64_t b_hi = tc::sdesc(bh + ks * 2 * (N2 / 8) * 128, (N2 / 8) * 128, 128);
          const uint64_t b_lo = tc::sdesc(bl + ks * 2 * (N2 / 8) * 128, (N2 / 8) * 128, 128);
          tc::mma_bf16(tZ, a, b_hi, ID_Z, (kt > 0 || ks > 0) ? 1u : 0u);
          tc::mma_bf16(tZ, a, b_lo, ID_Z, 1u);
          if (F32IN) tc::mma_bf16(tZ, tc::sdesc(awl + ks * 2 * R2 * 16, R2 * 16, 128), b_hi, ID_Z, 1u);
        }
        tc::commit(&bars[st]);
      }
      outstanding[st] = 1;
    }
    for (int st = 0; st < 2 && !failed; ++st)
      if (outstanding[st]) { failed = !wait_bar(st); outstanding[st] = 0; }
  }

  // ---------------- phase T: P1 = Tr Z, P2 = Ti Z  (Z split hi/lo, T split hi/lo)
  if (!failed) {
    const uint4* Tin = reinterpret_cast<const uint4*>(Tws + chunk * 4 * T_TILE);
    if constexpr (!F32IN) {
#pragma unroll 4
      for (int e = tid; e < 4 * T_TILE / 16; e += THR) tc::cp_async16(sT + 16 * e, Tin + e, true);
      tc::cp_async_commit();
    } else {
      for (int e = tid; e < 4 * T_TILE / 16; e += THR) reinterpret_cast<uint4*>(sT)[e] = Tin[e];
    }
    float z[32];
    tc::tmem_ld16(tZ + lane_base + 32 * half, z);
    tc::tmem_ld16(tZ + lane_base + 32 * half + 16, z + 16);
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      uint4 h, l;
      tc::split8(z + 8 * g, h, l);
      const int off = mnmaj(row, 32 * half + 8 * g, N2 / 8);
      *reinterpret_cast<uint4*>(sZh + off) = h;
      *reinterpret_cast<uint4*>(sZl + off) = l;
    }
    if constexpr (!F32IN) tc::cp_async_wait_all();
    tc::fence_proxy_async();
    tc::fence_before_sync();
    __syncthreads();
    if (tid == 0) {
      tc::fence_after_sync();
      constexpr uint32_t ID_T = tc::idesc_bf16(128, N2, false, true);
      const uint32_t t_base = tc::smem_addr(sT);
      const uint32_t zh = tc::smem_addr(sZh), zl = tc::smem_addr(sZl);
#pragma unroll 1
      for (int part = 0; part < 2; ++part) {       // 0: Tr -> P1, 1: Ti -> P2
        const uint32_t th = t_base + (2 * part) * T_TILE, tl = th + T_TILE;
        const uint32_t td = part ? tP2 : tP1;
#pragma unroll 1
        for (int ks = 0; ks < R2 / 16; ++ks) {
          const uint64_t ah = tc::sdesc(th + ks * 2 * R2 * 16, R2 * 16, 128);
          const uint64_t al = tc::sdesc(tl + ks * 2 * R2 * 16, R2 * 16, 128);
          const uint64_t bh = tc::sdesc(zh + ks * 2 * (N2 / 8) * 128, (N2 / 8) * 128, 128);
          const uint64_t bl = tc::sdesc(zl + ks * 2 * (N2 / 8) * 128, (N2 / 8) * 128, 128);
          tc::mma_bf16(td, ah, bh, ID_T, ks > 0 ? 1u : 0u);
          tc::mma_bf16(td, ah, bl, ID_T, 1u);
          tc::mma_bf16(td, al, bh, ID_T, 1u);
        }
      }
      tc::commit(&bars[2]);
    }
    failed = !wait_bar(2);
  }

  // ---------------- Cm, then E = Re(Cm) Y_block
  if (!failed) {
    float p1r[16], p1i[16], p2r[16], p2i[16];
    tc::tmem_ld16(tP1 + lane_base + 16 * half, p1r);
    tc::tmem_ld16(tP1 + lane_base + 32 + 16 * half, p1i);
    tc::tmem_ld16(tP2 + lane_base + 16 * half, p2r);
    tc::tmem_ld16(tP2 + lane_base + 32 + 16 * half, p2i);
    float cr[16], ci[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) { cr[j] = p1r[j] - p2i[j]; ci[j] = p1i[j] + p2r[j]; }
    // the T tiles are dead once P1/P2 are in TMEM, so Ca and Y may reuse region U
#pragma unroll
    for (int g = 0; g < 2; ++g) {
      uint4 h, l;
      const int jc = 16 * half + 8 * g;
      tc::split8(cr + 8 * g, h, l);
      *reinterpret_cast<uint4*>(sCh + mnmaj(row, jc, N2 / 8)) = h;
      *reinterpret_cast<uint4*>(sCl + mnmaj(row, jc, N2 / 8)) = l;
      *reinterpret_cast<uint4*>(sAh + kmaj(row, jc, R2)) = h;
      *reinterpret_cast<uint4*>(sAl + kmaj(row, jc, R2)) = l;
      tc::split8(ci + 8 * g, h, l);
      *reinterpret_cast<uint4*>(sCh + mnmaj(row, NB2 + jc, N2 / 8)) = h;
      *reinterpret_cast<uint4*>(sCl + mnmaj(row, NB2 + jc, N2 / 8)) = l;
    }
    for (int e = tid; e < C2 * (NB2 / 8); e += THR) {
      const int t = e % C2, g = e / C2;
      const bool valid = t < nt;
      const T* src = q + ((size_t)item * S + t0 + (valid ? t : 0)) * D + j0 + g * 8;
      stage8(src, valid, sYh + kmaj(t, g * 8, C2), sYl + kmaj(t, g * 8, C2));
    }
    tc::fence_proxy_async();
    tc::fence_before_sync();
    __syncthreads();
    if (tid == 0) {
      tc::fence_after_sync();
      constexpr uint32_t ID_E = tc::idesc_bf16(128, C2, false, false);
      const uint32_t ah = tc::smem_addr(sAh), al = tc::smem_addr(sAl);
      const uint32_t yh = tc::smem_addr(sYh), yl = tc::smem_addr(sYl);
#pragma unroll 1
      for (int ks = 0; ks < NB2 / 16; ++ks) {
        const uint64_t a_h = tc::sdesc(ah + ks * 2 * R2 * 16, R2 * 16, 128);
        const uint64_t a_l = tc::sdesc(al + ks * 2 * R2 * 16, R2 * 16, 128);
        const uint64_t b_h = tc::sdesc(yh + ks * 2 * C2 * 16, C2 * 16, 128);
        tc::mma_bf16(tE, a_h, b_h, ID_E, ks > 0 ? 1u : 0u);
        tc::mma_bf16(tE, a_l, b_h, ID_E, 1u);
        if (F32IN) tc::mma_bf16(tE, a_h, tc::sdesc(yl + ks * 2 * C2 * 16, C2 * 16, 128), ID_E, 1u);
      }
      tc::commit(&bars[2]);
    }
    failed = !wait_bar(2);
  }
  if (!failed) {
    float e[32];
    tc::tmem_ld16(tE + lane_base + 32 * half, e);
    tc::tmem_ld16(tE + lane_base + 32 * half + 16, e + 16);
    float* Eo = Ews + chunk * R2 * C2 + (size_t)row * C2 + 32 * half;
#pragma unroll
    for (int t = 0; t < 32; ++t) atomicAdd(Eo + t, e[t]);
  }

  // ---------------- phase B: S_next[:, block] = S[:, block] + W Cm, pipelined:
  // tile kt's MMAs (into dH[kt&1]) overlap tile kt-1's epilogue and tile kt+1's W load.
  constexpr uint32_t ID_H = tc::idesc_bf16(128, N2, true, true);
  auto issue_b = [&](int kt, int st) {
    if (tid == 0) {
      tc::fence_after_sync();
      const uint32_t aw = tc::smem_addr(stage_w_ptr(st)), awl = tc::smem_addr(sWl);
      const uint32_t ch = tc::smem_addr(sCh), cl = tc::smem_addr(sCl);
      const uint32_t td = tDH + 64 * (F32IN ? 0 : st);
#pragma unroll 1
      for (int ks = 0; ks < R2 / 16; ++ks) {
        // A = W viewed MN-major: M = element index i, K = vector index r
        const uint64_t a = tc::sdesc(aw + ks * 256, 128, R2 * 16);
        const uint64_t b_h = tc::sdesc(ch + ks * 2 * (N2 / 8) * 128, (N2 / 8) * 128, 128);
        const uint64_t b_l = tc::sdesc(cl + ks * 2 * (N2 / 8) * 128, (N2 / 8) * 128, 128);
        tc::mma_bf16(td, a, b_h, ID_H, ks > 0 ? 1u : 0u);
        tc::mma_bf16(td, a, b_l, ID_H, 1u);
        if (F32IN) tc::mma_bf16(td, tc::sdesc(awl + ks * 256, 128, R2 * 16), b_h, ID_H, 1u);
      }
      tc::commit(&bars[st]);
    }
  };
  // epilogue of tile kt: row kt*KT + row, columns [32*half, +32) = re (half 0) / im (half 1)
  auto epilogue_b = [&](int kt, int st) -> bool {
    const int gi = kt * KT + row;
    const size_t o = soff + (size_t)gi * D + j0;
    float4 hv[8];
    if (sr) {
      const float* src = (half ? src_i : src_r) + o;
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) hv[jj] = *reinterpret_cast<const float4*>(src + 4 * jj);
    } else {
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        float a[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) a[u] = (!half && gi == j0 + 4 * jj + u) ? 1.f : 0.f;
        hv[jj] = make_float4(a[0], a[1], a[2], a[3]);
      }
    }
    if (!wait_bar(st)) return false;
    float dh[32];
    const uint32_t td = tDH + 64 * (F32IN ? 0 : st);
    tc::tmem_ld16(td + lane_base + 32 * half, dh);
    tc::tmem_ld16(td + lane_base + 32 * half + 16, dh + 16);
    float* dst = (half ? dst_i : dst_r) + o;
#pragma unroll
    for (int jj = 0; jj < 8; ++jj)
      *reinterpret_cast<float4*>(dst + 4 * jj) =
          make_float4(hv[jj].x + dh[4 * jj], hv[jj].y + dh[4 * jj + 1], hv[jj].z + dh[4 * jj + 2],
                      hv[jj].w + dh[4 * jj + 3]);
    return true;
  };
  if (!failed) {
    // the epilogue of tile kt-1 runs after tile kt's MMAs are issued; tile kt+1's W
    // stage (kt+1)&1 is free once tile kt-1's MMAs completed (waited in its epilogue)
    for (int kt = 0; kt < NT && !failed; ++kt) {
      const int st = F32IN ? 0 : (kt & 1);
      if (F32IN && kt > 0) { if (!epilogue_b(kt - 1, 0)) { failed = true; break; } }
      tc::fence_before_sync();
      __syncthreads();   // previous readers of this stage and of dH[st] are done
      stage_w_tile(kt, st);
      if constexpr (!F32IN) tc::cp_async_wait_all();
      tc::fence_proxy_async();
      __syncthreads();
      issue_b(kt, st);
      if (!F32IN && kt > 0) { if (!epilogue_b(kt - 1, st ^ 1)) { failed = true; break; } }
    }
    if (!failed) failed = !epilogue_b(NT - 1, F32IN ? 0 : ((NT - 1) & 1));
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tbase, 512);
}

// ---------------------------------------------------------------------------------
// readout: rec[t][i0 + i] = Re(S y_t)_i + sum_r W[i][r] E[r][t] (token block of r <= t)
// smem: A (S rows, K-major hi/lo 2 x 32K) | Y (K-major, 64 rows, hi/lo 2 x 16K) |
//       W (32K, + lo 32K for fp32) | E (MN-major hi/lo 2 x 16K) | bar, slot
constexpr int RD_A = 0, RD_Y = 64 * 1024, RD_W = 96 * 1024, RD_E = 160 * 1024, RD_BAR = 192 * 1024;
constexpr int READOUT_SMEM = RD_BAR + 64;

template <typename T>
__global__ void __launch_bounds__(THR, 1)
cham_tc_readout(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                const float* __restrict__ Ews, const unsigned long long* __restrict__ badws,
                const float* __restrict__ src_r, T* __restrict__ out, int S, int D, int nch, int c) {
  extern __shared__ __align__(1024) unsigned char smr[];
  constexpr bool F32IN = sizeof(T) == 4;
  unsigned char* sAh = smr + RD_A;
  unsigned char* sAl = sAh + R2 * KT * 2;
  unsigned char* sYh = smr + RD_Y;
  unsigned char* sYl = sYh + C2 * KT * 2;
  unsigned char* sW = smr + RD_W;
  unsigned char* sWl = sW + W_TILE;
  unsigned char* sEh = smr + RD_E;
  unsigned char* sEl = sEh + R2 * C2 * 2;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smr + RD_BAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smr + RD_BAR + 16);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int item = blockIdx.y, i0 = blockIdx.x * R2;
  const int t0 = c * C2, nt = min(C2, S - t0);
  const size_t chunk = (size_t)item * nch + c;
  const unsigned long long bad = badws[chunk];
  const float* sr = src_r ? src_r + (size_t)item * D * D : nullptr;

  if (warp == 0) tc::tmem_alloc(tslot, 64);
  if (tid == 0) { tc::mbar_init(bar, 1); tc::fence_mbar_init(); }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tO = *tslot;
  const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
  const int row = 32 * (warp & 3) + lane, half = warp >> 2;
  uint32_t phase = 0;
  bool failed = false;
  auto wait_mma = [&]() -> bool {
    const bool ok = tc::mbar_wait(bar, phase, MAX_POLLS);
    phase ^= 1u;
    if (__syncthreads_or(!ok)) { if (tid == 0) record_timeout(); return false; }
    tc::fence_after_sync();
    return true;
  };
  constexpr uint32_t ID_O = tc::idesc_bf16(128, C2, false, false);

  // Re(S y_t): A = S rows [i0, i0+128) (K-major over columns j), B = Y (n = t, k = j)
  for (int j0 = 0; j0 < D && !failed; j0 += KT) {
    if (j0 > 0) { tc::fence_before_sync(); __syncthreads(); }
    for (int e = tid; e < R2 * (KT / 8); e += THR) {
      const int g = e % (KT / 8), i = e / (KT / 8);
      float x[8];
      if (sr) load8(sr + (size_t)(i0 + i) * D + j0 + g * 8, x);
      else {
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) x[jj] = (i0 + i == j0 + g * 8 + jj) ? 1.f : 0.f;
      }
      uint4 h, l;
      tc::split8(x, h, l);
      *reinterpret_cast<uint4*>(sAh + kmaj(i, g * 8, R2)) = h;
      *reinterpret_cast<uint4*>(sAl + kmaj(i, g * 8, R2)) = l;
    }
    for (int e = tid; e < C2 * (KT / 8); e += THR) {
      const int t = e % C2, g = e / C2;
      const bool valid = t < nt;
      const T* src = q + ((size_t)item * S + t0 + (valid ? t : 0)) * D + j0 + g * 8;
      stage8(src, valid, sYh + kmaj(t, g * 8, C2), sYl + kmaj(t, g * 8, C2));
    }
    tc::fence_proxy_async();
    __syncthreads();
    if (tid == 0) {
      tc::fence_after_sync();
      const uint32_t ah = tc::smem_addr(sAh), al = tc::smem_addr(sAl);
      const uint32_t yh = tc::smem_addr(sYh), yl = tc::smem_addr(sYl);
#pragma unroll 1
      for (int ks = 0; ks < KT / 16; ++ks) {
        const uint64_t a_h = tc::sdesc(ah + ks * 2 * R2 * 16, R2 * 16, 128);
        const uint64_t a_l = tc::sdesc(al + ks * 2 * R2 * 16, R2 * 16, 128);
        const uint64_t b_h = tc::sdesc(yh + ks * 2 * C2 * 16, C2 * 16, 128);
        tc::mma_bf16(tO, a_h, b_h, ID_O, (j0 > 0 || ks > 0) ? 1u : 0u);
        tc::mma_bf16(tO, a_l, b_h, ID_O, 1u);
        if (F32IN) tc::mma_bf16(tO, a_h, tc::sdesc(yl + ks * 2 * C2 * 16, C2 * 16, 128), ID_O, 1u);
      }
      tc::commit(bar);
    }
    failed = !wait_mma();
  }
  // + W E:  A = W rows [i0, i0+128) viewed MN-major (M = i, K = r), B = mask(E) (k = r, n = t)
  if (!failed) {
    tc::fence_before_sync();
    __syncthreads();
    stage_w<T>(sW, sWl, k, v, item, S, D, t0, nt, bad, i0, tid);
    const float* Ein = Ews + chunk * R2 * C2;
    for (int e = tid; e < R2 * (C2 / 8); e += THR) {
      const int g = e % (C2 / 8), r = e / (C2 / 8);
      float x[8];
      load8(Ein + (size_t)r * C2 + g * 8, x);
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) if (tok(r) > g * 8 + jj) x[jj] = 0.f;
      uint4 h, l;
      tc::split8(x, h, l);
      *reinterpret_cast<uint4*>(sEh + mnmaj(r, g * 8, C2 / 8)) = h;
      *reinterpret_cast<uint4*>(sEl + mnmaj(r, g * 8, C2 / 8)) = l;
    }
    tc::fence_proxy_async();
    __syncthreads();
    if (tid == 0) {
      tc::fence_after_sync();
      constexpr uint32_t ID_W = tc::idesc_bf16(128, C2, true, true);
      const uint32_t aw = tc::smem_addr(sW), awl = tc::smem_addr(sWl);
      const uint32_t eh = tc::smem_addr(sEh), el = tc::smem_addr(sEl);
#pragma unroll 1
      for (int ks = 0; ks < R2 / 16; ++ks) {
        const uint64_t a = tc::sdesc(aw + ks * 256, 128, R2 * 16);
        const uint64_t b_h = tc::sdesc(eh + ks * 2 * (C2 / 8) * 128, (C2 / 8) * 128, 128);
        const uint64_t b_l = tc::sdesc(el + ks * 2 * (C2 / 8) * 128, (C2 / 8) * 128, 128);
        tc::mma_bf16(tO, a, b_h, ID_W, 1u);
        tc::mma_bf16(tO, a, b_l, ID_W, 1u);
        if (F32IN) tc::mma_bf16(tO, tc::sdesc(awl + ks * 256, 128, R2 * 16), b_h, ID_W, 1u);
      }
      tc::commit(bar);
    }
    failed = !wait_mma();
  }
  if (!failed) {
    float o[32];
    tc::tmem_ld16(tO + lane_base + 32 * half, o);
    tc::tmem_ld16(tO + lane_base + 32 * half + 16, o + 16);
#pragma unroll
    for (int u = 0; u < 32; ++u) {
      const int t = 32 * half + u;
      if (t < nt) out[((size_t)item * S + t0 + t) * D + i0 + row] = from_f32<T>(o[u]);
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tO, 64);
}

// ---------------------------------------------------------------------------------
// Warp-specialised colpass for bf16 inputs.  Warp 8 (one thread) is the producer: it
// issues the TMA loads (k/v tiles straight into the tensor-core layout, fp32 state tiles
// with 128-byte swizzle, T tiles as bulk copies) and every tcgen05.mma; warps 0-7 are
// the consumers: they split fp32 state tiles into bf16 hi/lo operands, turn Z and Cm
// into operands, and run the state-update epilogue.  Producer and consumers hand over
// through mbarriers; every wait is bounded.  Same arithmetic as cham_tc_colpass.
//
// smem: U [0,128K)   stage s = (W 32K | state re 16K | state im 16K) at s*64K
//                    phase T: T tiles (4 x 32K); phase E: Ca (16K) | Y (4K)
//       HS[2] [128K,192K)  split state tiles (hi 16K | lo 16K); phase T: Z split in
//                          HS[0]; phases E/B: Cm split in HS[1]
//       barriers, TMEM slot, failure flag at 192K
// TMEM: Z [0,64) P1 [64,128) P2 [128,192) E [192,256) dH[2] [256,384)
constexpr int CONS = 256;                 // consumer threads
constexpr int WS_THREADS = CONS + 32;     // + producer warp
constexpr int WS_HS = 128 * 1024, WS_BAR = 192 * 1024;
constexpr int WS_SMEM = WS_BAR + 256;
enum { B_TFULL = 0, B_SFULL = 2, B_MDONE = 4, B_EDONE = 6, B_WFIX = 8, B_TT = 10, B_ZREADY = 11,
       B_MT = 12, B_CREADY = 13, B_ME = 14, B_DFREE = 15, N_BARS = 17 };

__device__ __forceinline__ bool consumers_all(bool ok) {
  int r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, 2, 256, p;\n\t"
      "selp.s32 %0, 1, 0, q;\n\t}\n"
      : "=r"(r)
      : "r"((int)ok)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void
colpass_ws_body(const CUtensorMap& tm_k, const CUtensorMap& tm_v, const CUtensorMap& tm_sr,
                const CUtensorMap& tm_si, const CUtensorMap& tm_dr, const CUtensorMap& tm_di,
                const __nv_bfloat16* __restrict__ q, const unsigned char* __restrict__ Tws,
                float* __restrict__ Ews, const unsigned long long* __restrict__ badws, int src_identity,
                float* __restrict__ dst_r, float* __restrict__ dst_i, int S, int D, int nch, int c, int bx) {
  extern __shared__ __align__(1024) unsigned char smw[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smw + WS_BAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smw + WS_BAR + 8 * N_BARS);
  volatile int* fail = reinterpret_cast<volatile int*>(smw + WS_BAR + 8 * N_BARS + 16);
  auto stageW = [&](int s) { return smw + s * STAGE; };
  auto stageHr = [&](int s) { return smw + s * STAGE + W_TILE; };
  auto stageHi = [&](int s) { return smw + s * STAGE + W_TILE + 16 * 1024; };
  auto splitH = [&](int s) { return smw + WS_HS + s * 32 * 1024; };
  unsigned char* sZh = splitH(0);
  unsigned char* sZl = sZh + Z_TILE;
  unsigned char* sO = splitH(0);   // phase B: updated state tile (re 16K | im 16K, swizzled) for TMA stores
  unsigned char* sCh = splitH(1);
  unsigned char* sCl = sCh + Z_TILE;
  unsigned char* sAh = smw;
  unsigned char* sAl = smw + CA_TILE;
  unsigned char* sY = smw + 2 * CA_TILE;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int item = blockIdx.y, j0 = bx * NB2;
  const int t0 = c * C2, nt = min(C2, S - t0);
  const size_t chunk = (size_t)item * nch + c;
  const unsigned long long bad = badws[chunk];
  const bool patch_w = bad != 0ull;   // padded rows come back zero from the TMA bounds
  const int NT = D / KT;

  if (warp == 0) tc::tmem_alloc(tslot, 512);
  if (tid == 0) {
    for (int i = 0; i < N_BARS; ++i) tc::mbar_init(&bars[i], 1);
    *fail = 0;
    tc::fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = *tslot;
  const uint32_t tZ = tbase, tP1 = tbase + 64, tP2 = tbase + 128, tE = tbase + 192, tDH = tbase + 256;

  if (warp == 8) {
    // ======================= producer (one thread) =======================
    if (lane == 0) {
      bool ok = true;
      auto pwait = [&](int b, uint32_t par) {
        if (!ok) return false;
        if (*fail || !tc::mbar_wait(&bars[b], par, MAX_POLLS)) { ok = false; *fail = 1; record_timeout(); }
        return ok;
      };
      auto issue_tiles = [&](int g, int kt) {   // K tile kt of global tile counter g
        const int s = g & 1;
        tc::mbar_expect_tx(&bars[B_TFULL + s], W_TILE + (src_identity ? 0 : 2 * 16 * 1024));
        unsigned char* w = stageW(s);
        // W tile in the 128-byte-swizzled K-major layout: [element block of 64][row r][128 B],
        // rows 0-63 = k of the chunk's tokens, 64-127 = v
#pragma unroll
        for (int kb = 0; kb < KT / 64; ++kb) {
          tc::tma_load_3d(w + kb * 16384, &tm_k, kt * KT + kb * 64, t0, item, &bars[B_TFULL + s]);
          tc::tma_load_3d(w + kb * 16384 + 8192, &tm_v, kt * KT + kb * 64, t0, item, &bars[B_TFULL + s]);
        }
        if (!src_identity) {
          tc::tma_load_2d(stageHr(s), &tm_sr, j0, item * D + kt * KT, &bars[B_TFULL + s]);
          tc::tma_load_2d(stageHi(s), &tm_si, j0, item * D + kt * KT, &bars[B_TFULL + s]);
        }
      };
      constexpr uint32_t ID_Z = tc::idesc_bf16(128, N2, false, true);
      constexpr uint32_t ID_H = tc::idesc_bf16(128, N2, true, true);
      // ---- phase A
      issue_tiles(0, 0);
      if (NT > 1) issue_tiles(1, 1);
      for (int kt = 0; kt < NT && ok; ++kt) {
        const int g = kt, s = g & 1;
        if (!pwait(B_TFULL + s, (g >> 1) & 1) || !pwait(B_SFULL + s, (kt >> 1) & 1)) break;
        tc::fence_after_sync();
        const uint32_t aw = tc::smem_addr(stageW(s));
        const uint32_t bh = tc::smem_addr(splitH(s)), bl = bh + H_TILE;
#pragma unroll 1
        for (int ks = 0; ks < KT / 16; ++ks) {
          const uint64_t a = tc::sdesc_sw128(aw + (ks >> 2) * 16384 + (ks & 3) * 32, 16, 1024);
          tc::mma_bf16(tZ, a, tc::sdesc(bh + ks * 2 * (N2 / 8) * 128, (N2 / 8) * 128, 128), ID_Z,
                       (kt > 0 || ks > 0) ? 1u : 0u);
          tc::mma_bf16(tZ, a, tc::sdesc(bl + ks * 2 * (N2 / 8) * 128, (N2 / 8) * 128, 128), ID_Z, 1u);
        }
        tc::commit(&bars[B_MDONE + s]);
        if (kt + 2 < NT) {
          if (!pwait(B_MDONE + s, (g >> 1) & 1)) break;
          issue_tiles(g + 2, kt + 2);
        }
      }
      // ---- phase T: bring in T once every phase-A MMA is done, then P1 = Tr Z, P2 = Ti Z
      if (ok && pwait(B_MDONE + ((NT - 1) & 1), ((NT - 1) >> 1) & 1)) {
        tc::mbar_expect_tx(&bars[B_TT], 4 * T_TILE);
        const unsigned char* tsrc = Tws + chunk * 4 * T_TILE;
        for (int p4 = 0; p4 < 4; ++p4) tc::bulk_load(smw + p4 * T_TILE, tsrc + p4 * T_TILE, T_TILE, &bars[B_TT]);
        if (pwait(B_ZREADY, 0) && pwait(B_TT, 0)) {
          tc::fence_after_sync();
          constexpr uint32_t ID_T = tc::idesc_bf16(128, N2, false, true);
          const uint32_t zh = tc::smem_addr(sZh), zl = tc::smem_addr(sZl);
#pragma unroll 1
          for (int part = 0; part < 2; ++part) {
            const uint32_t th = tc::smem_addr(smw) + (2 * part) * T_TILE, tl = th + T_TILE;
            const uint32_t td = part ? tP2 : tP1;
#pragma unroll 1
            for (int ks = 0; ks < R2 / 16; ++ks) {
              const uint64_t ah = tc::sdesc(th + ks * 2 * R2 * 16, R2 * 16, 128);
              const uint64_t al = tc::sdesc(tl + ks * 2 * R2 * 16, R2 * 16, 128);
              const uint64_t b_h = tc::sdesc(zh + ks * 2 * (N2 / 8) * 128, (N2 / 8) * 128, 128);
              const uint64_t b_l = tc::sdesc(zl + ks * 2 * (N2 / 8) * 128, (N2 / 8) * 128, 128);
              tc::mma_bf16(td, ah, b_h, ID_T, ks > 0 ? 1u : 0u);
              tc::mma_bf16(td, ah, b_l, ID_T, 1u);
              tc::mma_bf16(td, al, b_h, ID_T, 1u);
            }
          }
          tc::commit(&bars[B_MT]);
        }
      }
      // ---- phase E: E = Re(Cm) Y
      if (ok && pwait(B_CREADY, 0)) {
        tc::fence_after_sync();
        constexpr uint32_t ID_E = tc::idesc_bf16(128, C2, false, false);
        const uint32_t ah = tc::smem_addr(sAh), al = tc::smem_addr(sAl), yh = tc::smem_addr(sY);
#pragma unroll 1
        for (int ks = 0; ks < NB2 / 16; ++ks) {
          const uint64_t b_h = tc::sdesc(yh + ks * 2 * C2 * 16, C2 * 16, 128);
          tc::mma_bf16(tE, tc::sdesc(ah + ks * 2 * R2 * 16, R2 * 16, 128), b_h, ID_E, ks > 0 ? 1u : 0u);
          tc::mma_bf16(tE, tc::sdesc(al + ks * 2 * R2 * 16, R2 * 16, 128), b_h, ID_E, 1u);
        }
        tc::commit(&bars[B_ME]);
      }
      // ---- phase B: dH = W Cm per K tile, overlapped with the consumers' epilogues
      if (ok && pwait(B_ME, 0)) {
        auto mma_b = [&](int kt) {
          const int g = NT + kt, s = g & 1, d = kt & 1;
          if (!pwait(B_TFULL + s, (g >> 1) & 1)) return false;
          if (patch_w && !pwait(B_WFIX + d, (kt >> 1) & 1)) return false;
          if (kt >= 2 && !pwait(B_DFREE + d, ((kt - 2) >> 1) & 1)) return false;
          tc::fence_after_sync();
          const uint32_t aw = tc::smem_addr(stageW(s));
          const uint32_t ch = tc::smem_addr(sCh), cl = tc::smem_addr(sCl);
#pragma unroll 1
          for (int ks = 0; ks < R2 / 16; ++ks) {
            const uint64_t a = tc::sdesc_sw128(aw + ks * 2048, 16384, 1024);
            tc::mma_bf16(tDH + 64 * d, a, tc::sdesc(ch + ks * 2 * (N2 / 8) * 128, (N2 / 8) * 128, 128), ID_H,
                         ks > 0 ? 1u : 0u);
            tc::mma_bf16(tDH + 64 * d, a, tc::sdesc(cl + ks * 2 * (N2 / 8) * 128, (N2 / 8) * 128, 128), ID_H, 1u);
          }
          tc::commit(&bars[B_MDONE + s]);
          return true;
        };
        issue_tiles(NT, 0);
        if (NT > 1) issue_tiles(NT + 1, 1);
        if (mma_b(0)) {
          for (int kt = 0; kt < NT && ok; ++kt) {
            if (kt + 1 < NT && !mma_b(kt + 1)) break;
            if (kt + 2 < NT) {
              if (!pwait(B_EDONE + (kt & 1), (kt >> 1) & 1)) break;
              issue_tiles(NT + kt + 2, kt + 2);
            }
          }
        }
      }
    }
  } else {
    // ======================= consumers (warps 0-7) =======================
    const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
    const int row = 32 * (warp & 3) + lane, half = warp >> 2;
    bool ok = true;
    auto cwait = [&](int b, uint32_t par) {
      bool mine = ok && !*fail && tc::mbar_wait(&bars[b], par, MAX_POLLS);
      const bool all = consumers_all(mine);
      if (!all) { if (ok && tid == 0) record_timeout(); ok = false; *fail = 1; }
      return ok;
    };
    auto zero_bad_rows = [&](unsigned char* w) {   // swizzled W tile
      for (int e = tid; e < R2 * (KT / 8); e += CONS) {
        const int r = e % R2, cc = e / R2;             // 16-byte chunk cc of row r
        if ((bad >> tok(r)) & 1ull)
          *reinterpret_cast<uint4*>(w + (cc >> 3) * 16384 + r * 128 + (((cc & 7) ^ (r & 7)) << 4)) =
              make_uint4(0, 0, 0, 0);
      }
    };
    // ---- phase A: split the state tiles
    for (int kt = 0; kt < NT && ok; ++kt) {
      const int g = kt, s = g & 1;
      if (!cwait(B_TFULL + s, (g >> 1) & 1)) break;
      if (kt >= 2 && !cwait(B_MDONE + s, ((g - 2) >> 1) & 1)) break;
      if (patch_w) zero_bad_rows(stageW(s));
      unsigned char* hh = splitH(s);
      unsigned char* hl = hh + H_TILE;
      const unsigned char* hr = stageHr(s);
      const unsigned char* hi = stageHi(s);
#pragma unroll
      for (int u = 0; u < (KT * (N2 / 8)) / CONS; ++u) {
        const int e = tid + CONS * u;
        const int i = e % KT, gg = e / KT;        // row i, 8-column group gg (0-3 re, 4-7 im)
        float x[8];
        if (src_identity) {
          const int gi = kt * KT + i, col = j0 + (gg & 3) * 8;
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) x[jj] = (gg < 4 && gi == col + jj) ? 1.f : 0.f;
        } else {
          const unsigned char* box = gg < 4 ? hr : hi;
          const int c0 = 2 * (gg & 3);
          const float4 a = *reinterpret_cast<const float4*>(box + i * 128 + (((c0) ^ (i & 7)) << 4));
          const float4 b = *reinterpret_cast<const float4*>(box + i * 128 + (((c0 + 1) ^ (i & 7)) << 4));
          x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
        }
        uint4 h, l;
        tc::split8(x, h, l);
        *reinterpret_cast<uint4*>(hh + mnmaj(i, gg * 8, N2 / 8)) = h;
        *reinterpret_cast<uint4*>(hl + mnmaj(i, gg * 8, N2 / 8)) = l;
      }
      tc::fence_proxy_async();
      tc::named_sync(1, CONS);
      if (tid == 0) tc::mbar_arrive(&bars[B_SFULL + s]);
    }
    // ---- phase T: Z -> operand
    if (ok && cwait(B_MDONE + ((NT - 1) & 1), ((NT - 1) >> 1) & 1)) {
      tc::fence_after_sync();
      float z[32];
      tc::tmem_ld16(tZ + lane_base + 32 * half, z);
      tc::tmem_ld16(tZ + lane_base + 32 * half + 16, z + 16);
#pragma unroll
      for (int g4 = 0; g4 < 4; ++g4) {
        uint4 h, l;
        tc::split8(z + 8 * g4, h, l);
        const int off = mnmaj(row, 32 * half + 8 * g4, N2 / 8);
        *reinterpret_cast<uint4*>(sZh + off) = h;
        *reinterpret_cast<uint4*>(sZl + off) = l;
      }
      tc::fence_proxy_async();
      tc::fence_before_sync();
      tc::named_sync(1, CONS);
      if (tid == 0) tc::mbar_arrive(&bars[B_ZREADY]);
    }
    // ---- phase E: Cm -> operands, Y, then E partial
    if (ok && cwait(B_MT, 0)) {
      tc::fence_after_sync();
      float p1r[16], p1i[16], p2r[16], p2i[16];
      tc::tmem_ld16(tP1 + lane_base + 16 * half, p1r);
      tc::tmem_ld16(tP1 + lane_base + 32 + 16 * half, p1i);
      tc::tmem_ld16(tP2 + lane_base + 16 * half, p2r);
      tc::tmem_ld16(tP2 + lane_base + 32 + 16 * half, p2i);
      float cr[16], ci[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) { cr[j] = p1r[j] - p2i[j]; ci[j] = p1i[j] + p2r[j]; }
#pragma unroll
      for (int g2 = 0; g2 < 2; ++g2) {
        uint4 h, l;
        const int jc = 16 * half + 8 * g2;
        tc::split8(cr + 8 * g2, h, l);
        *reinterpret_cast<uint4*>(sCh + mnmaj(row, jc, N2 / 8)) = h;
        *reinterpret_cast<uint4*>(sCl + mnmaj(row, jc, N2 / 8)) = l;
        *reinterpret_cast<uint4*>(sAh + kmaj(row, jc, R2)) = h;
        *reinterpret_cast<uint4*>(sAl + kmaj(row, jc, R2)) = l;
        tc::split8(ci + 8 * g2, h, l);
        *reinterpret_cast<uint4*>(sCh + mnmaj(row, NB2 + jc, N2 / 8)) = h;
        *reinterpret_cast<uint4*>(sCl + mnmaj(row, NB2 + jc, N2 / 8)) = l;
      }
      {
        const int t = tid % C2, gq = tid / C2;   // 64 tokens x 4 groups of 8 columns
        uint4 u = make_uint4(0, 0, 0, 0);
        if (t < nt) u = *reinterpret_cast<const uint4*>(q + ((size_t)item * S + t0 + t) * D + j0 + gq * 8);
        *reinterpret_cast<uint4*>(sY + kmaj(t, gq * 8, C2)) = u;
      }
      tc::fence_proxy_async();
      tc::fence_before_sync();
      tc::named_sync(1, CONS);
      if (tid == 0) tc::mbar_arrive(&bars[B_CREADY]);
    }
    if (ok && cwait(B_ME, 0)) {
      tc::fence_after_sync();
      float e[32];
      tc::tmem_ld16(tE + lane_base + 32 * half, e);
      tc::tmem_ld16(tE + lane_base + 32 * half + 16, e + 16);
      float4* Eo = reinterpret_cast<float4*>(Ews + chunk * R2 * C2 + (size_t)row * C2 + 32 * half);
#pragma unroll
      for (int t = 0; t < 8; ++t) atomicAdd(Eo + t, make_float4(e[4 * t], e[4 * t + 1], e[4 * t + 2], e[4 * t + 3]));
    }
    // ---- phase B: epilogues; results go back into the (swizzled) state stage and leave by
    // TMA stores; a stage is released (edone) once its store has read it
    for (int kt = 0; kt < NT && ok; ++kt) {
      const int g = NT + kt, s = g & 1, d = kt & 1;
      if (!cwait(B_TFULL + s, (g >> 1) & 1)) break;
      if (patch_w) {
        zero_bad_rows(stageW(s));
        tc::fence_proxy_async();
        tc::named_sync(1, CONS);
        if (tid == 0) tc::mbar_arrive(&bars[B_WFIX + d]);
      }
      if (!cwait(B_MDONE + s, (g >> 1) & 1)) break;
      tc::fence_after_sync();
      const int gi = kt * KT + row;
      float hv[32];
      if (src_identity) {
#pragma unroll
        for (int jj = 0; jj < 32; ++jj) hv[jj] = (!half && gi == j0 + jj) ? 1.f : 0.f;
      } else {
        const unsigned char* box = half ? stageHi(s) : stageHr(s);
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
          const float4 a = *reinterpret_cast<const float4*>(box + row * 128 + ((cc ^ (row & 7)) << 4));
          hv[4 * cc] = a.x; hv[4 * cc + 1] = a.y; hv[4 * cc + 2] = a.z; hv[4 * cc + 3] = a.w;
        }
      }
      float dh[32];
      tc::tmem_ld16(tDH + 64 * d + lane_base + 32 * half, dh);
      tc::tmem_ld16(tDH + 64 * d + lane_base + 32 * half + 16, dh + 16);
      tc::fence_before_sync();
      tc::named_sync(1, CONS);
      if (tid == 0) {                            // input stage and dH[d] are free again
        tc::mbar_arrive(&bars[B_DFREE + d]);
        tc::mbar_arrive(&bars[B_EDONE + d]);
        tc::bulk_wait_read<0>();                 // the previous tile's store has read sO
      }
      tc::named_sync(1, CONS);
      unsigned char* obox = sO + half * 16 * 1024;
#pragma unroll
      for (int cc = 0; cc < 8; ++cc)
        *reinterpret_cast<float4*>(obox + row * 128 + ((cc ^ (row & 7)) << 4)) =
            make_float4(hv[4 * cc] + dh[4 * cc], hv[4 * cc + 1] + dh[4 * cc + 1], hv[4 * cc + 2] + dh[4 * cc + 2],
                        hv[4 * cc + 3] + dh[4 * cc + 3]);
      tc::fence_proxy_async();
      tc::named_sync(1, CONS);
      if (tid == 0) {
        tc::tma_store_2d(&tm_dr, j0, item * D + kt * KT, sO);
        tc::tma_store_2d(&tm_di, j0, item * D + kt * KT, sO + 16 * 1024);
        tc::bulk_commit();
      }
    }
    if (tid == 0) tc::bulk_wait<0>();            // all state writes performed
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tbase, 512);
}

// ---------------------------------------------------------------------------------
// Warp-specialised readout for bf16 inputs, run in the same launch as the next chunk's
// colpass.  It reads the chunk's END state S_end (the next colpass's source) and uses
//     rec_t = Re(S_end y_t) - sum_{tau > t} U_tau E[tau, t]
// (S_t = S_end minus the later tokens' rank-2 terms).  One CTA per (item, 128 rows):
// producer = TMA (state rows as swizzled fp32 boxes, Y and W as swizzled bf16 boxes) +
// tcgen05 issue; consumers = fp32 -> bf16 hi/lo split of the state rows, the masked E
// operand and the output epilogue.
// smem: stage s at s*48K = state rows [128][64] fp32 (2 boxes, 32K) | Y [64 tok][64] (8K)
//       A split [2] at 96K (hi 16K | lo 16K each); phase 2: W (32K) at 0, E split at 160K
// TMEM: O [0,64)
constexpr int RW_STAGE = 48 * 1024, RW_AS = 96 * 1024, RW_E = 160 * 1024;
constexpr int RKT = 64;   // state columns per K tile

__device__ __forceinline__ void
readout_ws_body(const CUtensorMap& tm_k, const CUtensorMap& tm_v, const CUtensorMap& tm_q,
                const CUtensorMap& tm_sr, const float* __restrict__ Ews,
                const unsigned long long* __restrict__ badws, __nv_bfloat16* __restrict__ out,
                int S, int D, int nch, int c, int bx, int item, int srow) {
  extern __shared__ __align__(1024) unsigned char smw[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smw + WS_BAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smw + WS_BAR + 8 * N_BARS);
  volatile int* fail = reinterpret_cast<volatile int*>(smw + WS_BAR + 8 * N_BARS + 16);
  auto stA = [&](int s) { return smw + s * RW_STAGE; };
  auto stY = [&](int s) { return smw + s * RW_STAGE + 32 * 1024; };
  auto splitA = [&](int s) { return smw + RW_AS + s * 32 * 1024; };
  unsigned char* sW = smw;
  unsigned char* sEh = smw + RW_E;
  unsigned char* sEl = sEh + 16 * 1024;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int i0 = bx * R2;
  const int t0 = c * C2, nt = min(C2, S - t0);
  const size_t chunk = (size_t)item * nch + c;
  const unsigned long long bad = badws[chunk];
  const int NTR = D / RKT;

  if (warp == 0) tc::tmem_alloc(tslot, 64);
  if (tid == 0) {
    for (int i = 0; i < N_BARS; ++i) tc::mbar_init(&bars[i], 1);
    *fail = 0;
    tc::fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tO = *tslot;

  if (warp == 8) {
    if (lane == 0) {
      bool ok = true;
      auto pwait = [&](int b, uint32_t par) {
        if (!ok) return false;
        if (*fail || !tc::mbar_wait(&bars[b], par, MAX_POLLS)) { ok = false; *fail = 1; record_timeout(); }
        return ok;
      };
      auto issue = [&](int kt) {
        const int s = kt & 1;
        tc::mbar_expect_tx(&bars[B_TFULL + s], 32 * 1024 + 8 * 1024);
        tc::tma_load_2d(stA(s), &tm_sr, kt * RKT, srow + i0, &bars[B_TFULL + s]);
        tc::tma_load_2d(stA(s) + 16 * 1024, &tm_sr, kt * RKT + 32, srow + i0, &bars[B_TFULL + s]);
        tc::tma_load_3d(stY(s), &tm_q, kt * RKT, t0, item, &bars[B_TFULL + s]);
      };
      constexpr uint32_t ID_O = tc::idesc_bf16(128, C2, false, false);
      issue(0);
      if (NTR > 1) issue(1);
      for (int kt = 0; kt < NTR && ok; ++kt) {
        const int s = kt & 1;
        if (!pwait(B_TFULL + s, (kt >> 1) & 1) || !pwait(B_SFULL + s, (kt >> 1) & 1)) break;
        tc::fence_after_sync();
        const uint32_t ah = tc::smem_addr(splitA(s)), al = ah + 16 * 1024;
        const uint32_t y = tc::smem_addr(stY(s));
#pragma unroll 1
        for (int ks = 0; ks < RKT / 16; ++ks) {
          const uint64_t b = tc::sdesc_sw128(y + ks * 32, 16, 1024);
          tc::mma_bf16(tO, tc::sdesc(ah + ks * 2 * R2 * 16, R2 * 16, 128), b, ID_O, (kt > 0 || ks > 0) ? 1u : 0u);
          tc::mma_bf16(tO, tc::sdesc(al + ks * 2 * R2 * 16, R2 * 16, 128), b, ID_O, 1u);
        }
        tc::commit(&bars[B_MDONE + s]);
        if (kt + 2 < NTR) {
          if (!pwait(B_MDONE + s, (kt >> 1) & 1)) break;
          issue(kt + 2);
        }
      }
      // W rows [i0, i0+128) of the chunk (k block, v block), then O -= W mask(E)
      if (ok && pwait(B_MDONE + ((NTR - 1) & 1), ((NTR - 1) >> 1) & 1)) {
        tc::mbar_expect_tx(&bars[B_TT], W_TILE);
#pragma unroll
        for (int kb = 0; kb < R2 / 64; ++kb) {
          tc::tma_load_3d(sW + kb * 16384, &tm_k, i0 + kb * 64, t0, item, &bars[B_TT]);
          tc::tma_load_3d(sW + kb * 16384 + 8192, &tm_v, i0 + kb * 64, t0, item, &bars[B_TT]);
        }
        if (pwait(B_TT, 0) && pwait(B_CREADY, 0)) {
          tc::fence_after_sync();
          constexpr uint32_t ID_W = tc::idesc_bf16(128, C2, true, true);
          const uint32_t aw = tc::smem_addr(sW), eh = tc::smem_addr(sEh), el = tc::smem_addr(sEl);
#pragma unroll 1
          for (int ks = 0; ks < R2 / 16; ++ks) {
            const uint64_t a = tc::sdesc_sw128(aw + ks * 2048, 16384, 1024);
            tc::mma_bf16(tO, a, tc::sdesc(eh + ks * 2 * (C2 / 8) * 128, (C2 / 8) * 128, 128), ID_W, 1u);
            tc::mma_bf16(tO, a, tc::sdesc(el + ks * 2 * (C2 / 8) * 128, (C2 / 8) * 128, 128), ID_W, 1u);
          }
          tc::commit(&bars[B_ME]);
        }
      }
    }
  } else {
    const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
    const int row = 32 * (warp & 3) + lane, half = warp >> 2;
    bool ok = true;
    auto cwait = [&](int b, uint32_t par) {
      bool mine = ok && !*fail && tc::mbar_wait(&bars[b], par, MAX_POLLS);
      const bool all = consumers_all(mine);
      if (!all) { if (ok && tid == 0) record_timeout(); ok = false; *fail = 1; }
      return ok;
    };
    for (int kt = 0; kt < NTR && ok; ++kt) {
      const int s = kt & 1;
      if (!cwait(B_TFULL + s, (kt >> 1) & 1)) break;
      if (kt >= 2 && !cwait(B_MDONE + s, ((kt - 2) >> 1) & 1)) break;
      unsigned char* ah = splitA(s);
      unsigned char* al = ah + 16 * 1024;
      const unsigned char* a = stA(s);
#pragma unroll
      for (int u = 0; u < (R2 * (RKT / 8)) / CONS; ++u) {
        const int e = tid + CONS * u;
        const int i = e % R2, gg = e / R2;                 // row i, columns 8*gg .. 8*gg+7
        const unsigned char* box = a + (gg >> 2) * 16384;
        const int c0 = 2 * (gg & 3);
        const float4 x0 = *reinterpret_cast<const float4*>(box + i * 128 + ((c0 ^ (i & 7)) << 4));
        const float4 x1 = *reinterpret_cast<const float4*>(box + i * 128 + (((c0 + 1) ^ (i & 7)) << 4));
        const float x[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
        uint4 h, l;
        tc::split8(x, h, l);
        *reinterpret_cast<uint4*>(ah + kmaj(i, gg * 8, R2)) = h;
        *reinterpret_cast<uint4*>(al + kmaj(i, gg * 8, R2)) = l;
      }
      tc::fence_proxy_async();
      tc::named_sync(1, CONS);
      if (tid == 0) tc::mbar_arrive(&bars[B_SFULL + s]);
    }
    if (ok) {
      // -mask(E): keep later tokens (tok(r) > t), zero tokens that are non-finite
      const float* Ein = Ews + chunk * R2 * C2;
#pragma unroll
      for (int u = 0; u < (R2 * (C2 / 8)) / CONS; ++u) {
        const int e = tid + CONS * u;
        const int gq = e % (C2 / 8), r = e / (C2 / 8);
        float x[8];
        load8(Ein + (size_t)r * C2 + gq * 8, x);
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) x[jj] = (tok(r) > gq * 8 + jj) ? -x[jj] : 0.f;
        uint4 h, l;
        tc::split8(x, h, l);
        *reinterpret_cast<uint4*>(sEh + mnmaj(r, gq * 8, C2 / 8)) = h;
        *reinterpret_cast<uint4*>(sEl + mnmaj(r, gq * 8, C2 / 8)) = l;
      }
      // rows of non-finite tokens must not reach the product (their E rows are 0, and
      // 0 x inf is NaN): zero them in the W tile once it has landed
      if (cwait(B_TT, 0) && bad) {
        for (int e = tid; e < R2 * (R2 / 8); e += CONS) {
          const int r = e % R2, cc = e / R2;
          if ((bad >> tok(r)) & 1ull)
            *reinterpret_cast<uint4*>(sW + (cc >> 3) * 16384 + r * 128 + (((cc & 7) ^ (r & 7)) << 4)) =
                make_uint4(0, 0, 0, 0);
        }
      }
      tc::fence_proxy_async();
      tc::named_sync(1, CONS);
      if (ok && tid == 0) tc::mbar_arrive(&bars[B_CREADY]);
    }
    if (ok && cwait(B_ME, 0)) {
      tc::fence_after_sync();
      float o[32];
      tc::tmem_ld16(tO + lane_base + 32 * half, o);
      tc::tmem_ld16(tO + lane_base + 32 * half + 16, o + 16);
#pragma unroll
      for (int u = 0; u < 32; ++u) {
        const int t = 32 * half + u;
        if (t < nt) out[((size_t)item * S + t0 + t) * D + i0 + row] = __float2bfloat16_rn(o[u]);
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tO, 64);
}

// ---------------------------------------------------------------------------------
// Readout for the batched schedule, two CTAs per SM: readout_ws_body with the fp32
// state rows split in place (no separate split buffers), or, given `pre`, the rows
// already split by the column pass: per K tile one 32 KB image (bf16 hi 16K | lo 16K,
// K-major core matrices, rows i0 .. i0+127) taken by one bulk copy, with no split step.
// smem: stage s at s*40K = state rows [128][64] fp32 (2 boxes, 32K; split in place into
//       bf16 hi 16K | lo 16K) | Y [64 tok][64] (8K); phase 2: W (32K) at 0, E split at 40K
// TMEM: O [0,64)
constexpr int RW2_STAGE = 40 * 1024, RW2_BAR = 80 * 1024;
constexpr int RW2_SMEM = RW2_BAR + 256;

__device__ __forceinline__ void
readout2_body(const CUtensorMap& tm_k, const CUtensorMap& tm_v, const CUtensorMap& tm_q,
                const CUtensorMap& tm_sr, const float* __restrict__ Ews,
                const unsigned long long* __restrict__ badws, __nv_bfloat16* __restrict__ out,
                int S, int D, int nch, int c, int bx, int item, int srow, const unsigned char* __restrict__ pre) {
  extern __shared__ __align__(1024) unsigned char smw[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smw + RW2_BAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smw + RW2_BAR + 8 * N_BARS);
  volatile int* fail = reinterpret_cast<volatile int*>(smw + RW2_BAR + 8 * N_BARS + 16);
  auto stA = [&](int s) { return smw + s * RW2_STAGE; };
  auto stY = [&](int s) { return smw + s * RW2_STAGE + 32 * 1024; };
  auto splitA = [&](int s) { return smw + s * RW2_STAGE; };   // in place of the fp32 rows
  unsigned char* sW = smw;
  unsigned char* sEh = smw + RW2_STAGE;
  unsigned char* sEl = sEh + 16 * 1024;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int i0 = bx * R2;
  const int t0 = c * C2, nt = min(C2, S - t0);
  const size_t chunk = (size_t)item * nch + c;
  const unsigned long long bad = badws[chunk];
  const int NTR = D / RKT;

  if (warp == 0) tc::tmem_alloc(tslot, 64);
  if (tid == 0) {
    for (int i = 0; i < N_BARS; ++i) tc::mbar_init(&bars[i], 1);
    *fail = 0;
    tc::fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tO = *tslot;

  if (warp == 8) {
    if (lane == 0) {
      bool ok = true;
      auto pwait = [&](int b, uint32_t par) {
        if (!ok) return false;
        if (*fail || !tc::mbar_wait(&bars[b], par, MAX_POLLS)) { ok = false; *fail = 1; record_timeout(); }
        return ok;
      };
      auto issue = [&](int kt) {
        const int s = kt & 1;
        tc::mbar_expect_tx(&bars[B_TFULL + s], (pre != nullptr ? 16 : 32) * 1024 + 8 * 1024);
        if (pre != nullptr) {   // the image's bf16 tile (the real part rounded once)
          tc::bulk_load_hint(stA(s), pre + (size_t)(bx * NTR + kt) * (16 * 1024), 16 * 1024, &bars[B_TFULL + s],
                             tc::policy_evict_first());
        } else {
          tc::tma_load_2d(stA(s), &tm_sr, kt * RKT, srow + i0, &bars[B_TFULL + s]);
          tc::tma_load_2d(stA(s) + 16 * 1024, &tm_sr, kt * RKT + 32, srow + i0, &bars[B_TFULL + s]);
        }
        tc::tma_load_3d(stY(s), &tm_q, kt * RKT, t0, item, &bars[B_TFULL + s]);
      };
      constexpr uint32_t ID_O = tc::idesc_bf16(128, C2, false, false);
      issue(0);
      if (NTR > 1) issue(1);
      for (int kt = 0; kt < NTR && ok; ++kt) {
        const int s = kt & 1;
        if (!pwait(B_TFULL + s, (kt >> 1) & 1) || (pre == nullptr && !pwait(B_SFULL + s, (kt >> 1) & 1))) break;
        tc::fence_after_sync();
        const uint32_t ah = tc::smem_addr(splitA(s)), al = ah + 16 * 1024;
        const uint32_t y = tc::smem_addr(stY(s));
#pragma unroll 1
        for (int ks = 0; ks < RKT / 16; ++ks) {
          const uint64_t b = tc::sdesc_sw128(y + ks * 32, 16, 1024);
          tc::mma_bf16(tO, tc::sdesc(ah + ks * 2 * R2 * 16, R2 * 16, 128), b, ID_O, (kt > 0 || ks > 0) ? 1u : 0u);
          if (pre == nullptr) tc::mma_bf16(tO, tc::sdesc(al + ks * 2 * R2 * 16, R2 * 16, 128), b, ID_O, 1u);
        }
        tc::commit(&bars[B_MDONE + s]);
        if (kt + 2 < NTR) {
          if (!pwait(B_MDONE + s, (kt >> 1) & 1)) break;
          issue(kt + 2);
        }
        if (kt == NTR - 1) tc::commit(&bars[B_EDONE]);   // every main-loop MMA done (phase 0)
      }
      // W rows [i0, i0+128) of the chunk (k block, v block), then O -= W mask(E)
      if (ok && pwait(B_MDONE + ((NTR - 1) & 1), ((NTR - 1) >> 1) & 1)) {
        tc::mbar_expect_tx(&bars[B_TT], W_TILE);
#pragma unroll
        for (int kb = 0; kb < R2 / 64; ++kb) {
          tc::tma_load_3d(sW + kb * 16384, &tm_k, i0 + kb * 64, t0, item, &bars[B_TT]);
          tc::tma_load_3d(sW + kb * 16384 + 8192, &tm_v, i0 + kb * 64, t0, item, &bars[B_TT]);
        }
        if (pwait(B_TT, 0) && pwait(B_CREADY, 0)) {
          tc::fence_after_sync();
          constexpr uint32_t ID_W = tc::idesc_bf16(128, C2, true, true);
          const uint32_t aw = tc::smem_addr(sW), eh = tc::smem_addr(sEh), el = tc::smem_addr(sEl);
#pragma unroll 1
          for (int ks = 0; ks < R2 / 16; ++ks) {
            const uint64_t a = tc::sdesc_sw128(aw + ks * 2048, 16384, 1024);
            tc::mma_bf16(tO, a, tc::sdesc(eh + ks * 2 * (C2 / 8) * 128, (C2 / 8) * 128, 128), ID_W, 1u);
            tc::mma_bf16(tO, a, tc::sdesc(el + ks * 2 * (C2 / 8) * 128, (C2 / 8) * 128, 128), ID_W, 1u);
          }
          tc::commit(&bars[B_ME]);
        }
      }
    }
  } else if (warp < 8) {   // (a launch shared with the column pass has a tenth, idle warp)
    const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
    const int row = 32 * (warp & 3) + lane, half = warp >> 2;
    bool ok = true;
    auto cwait = [&](int b, uint32_t par) {
      bool mine = ok && !*fail && tc::mbar_wait(&bars[b], par, MAX_POLLS);
      const bool all = consumers_all(mine);
      if (!all) { if (ok && tid == 0) record_timeout(); ok = false; *fail = 1; }
      return ok;
    };
    for (int kt = 0; kt < NTR && ok && pre == nullptr; ++kt) {
      const int s = kt & 1;
      if (!cwait(B_TFULL + s, (kt >> 1) & 1)) break;
      unsigned char* ah = splitA(s);
      unsigned char* al = ah + 16 * 1024;
      const unsigned char* a = stA(s);
      constexpr int UN = (R2 * (RKT / 8)) / CONS;
      float x[UN][8];
#pragma unroll
      for (int u = 0; u < UN; ++u) {
        const int e = tid + CONS * u;
        const int i = e % R2, gg = e / R2;                 // row i, columns 8*gg .. 8*gg+7
        const unsigned char* box = a + (gg >> 2) * 16384;
        const int c0 = 2 * (gg & 3);
        const float4 x0 = *reinterpret_cast<const float4*>(box + i * 128 + ((c0 ^ (i & 7)) << 4));
        const float4 x1 = *reinterpret_cast<const float4*>(box + i * 128 + (((c0 + 1) ^ (i & 7)) << 4));
        x[u][0] = x0.x; x[u][1] = x0.y; x[u][2] = x0.z; x[u][3] = x0.w;
        x[u][4] = x1.x; x[u][5] = x1.y; x[u][6] = x1.z; x[u][7] = x1.w;
      }
      tc::named_sync(1, CONS);   // every fp32 value read before the split overwrites it
#pragma unroll
      for (int u = 0; u < UN; ++u) {
        const int e = tid + CONS * u;
        const int i = e % R2, gg = e / R2;
        uint4 h, l;
        tc::split8(x[u], h, l);
        *reinterpret_cast<uint4*>(ah + kmaj(i, gg * 8, R2)) = h;
        *reinterpret_cast<uint4*>(al + kmaj(i, gg * 8, R2)) = l;
      }
      tc::fence_proxy_async();
      tc::named_sync(1, CONS);
      if (tid == 0) tc::mbar_arrive(&bars[B_SFULL + s]);
    }
    // the E operand goes into stage 1: wait until the last main-loop MMA has read it (a
    // barrier of its own: consumers that skip the split loop would otherwise meet the
    // stage barriers at an ambiguous phase)
    if (ok && cwait(B_EDONE, 0)) {
      // -mask(E): keep later tokens (tok(r) > t), zero tokens that are non-finite
      const float* Ein = Ews + chunk * R2 * C2;
#pragma unroll
      for (int u = 0; u < (R2 * (C2 / 8)) / CONS; ++u) {
        const int e = tid + CONS * u;
        const int gq = e % (C2 / 8), r = e / (C2 / 8);
        float x[8];
        load8(Ein + (size_t)r * C2 + gq * 8, x);
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) x[jj] = (tok(r) > gq * 8 + jj) ? -x[jj] : 0.f;
        uint4 h, l;
        tc::split8(x, h, l);
        *reinterpret_cast<uint4*>(sEh + mnmaj(r, gq * 8, C2 / 8)) = h;
        *reinterpret_cast<uint4*>(sEl + mnmaj(r, gq * 8, C2 / 8)) = l;
      }
      // rows of non-finite tokens must not reach the product (their E rows are 0, and
      // 0 x inf is NaN): zero them in the W tile once it has landed
      if (cwait(B_TT, 0) && bad) {
        for (int e = tid; e < R2 * (R2 / 8); e += CONS) {
          const int r = e % R2, cc = e / R2;
          if ((bad >> tok(r)) & 1ull)
            *reinterpret_cast<uint4*>(sW + (cc >> 3) * 16384 + r * 128 + (((cc & 7) ^ (r & 7)) << 4)) =
                make_uint4(0, 0, 0, 0);
        }
      }
      tc::fence_proxy_async();
      tc::named_sync(1, CONS);
      if (ok && tid == 0) tc::mbar_arrive(&bars[B_CREADY]);
    }
    if (ok && cwait(B_ME, 0)) {
      tc::fence_after_sync();
      float o[32];
      tc::tmem_ld16(tO + lane_base + 32 * half, o);
      tc::tmem_ld16(tO + lane_base + 32 * half + 16, o + 16);
#pragma unroll
      for (int u = 0; u < 32; ++u) {
        const int t = 32 * half + u;
        if (t < nt) out[((size_t)item * S + t0 + t) * D + i0 + row] = __float2bfloat16_rn(o[u]);
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tO, 64);
}

// ---------------------------------------------------------------------------------
// prep for bf16 inputs: the Gram matrix G = W Wᵀ on the tensor cores (W tiles by TMA in
// the kernels' row order, k block then v block; bf16 inputs are exact, so one product),
// then N_t, T by block forward substitution (fp32 SIMT) directly in that row order.
// smem: Gs [128][132] fp32 | W stages (2 x 32K, 1024-aligned) aliased later by Tr | Ti
constexpr int PW_P = 132;   // row pitch of Gs / Tr / Ti in floats (a multiple of 4: float4 rows)
constexpr int PW_TR = 67584, PW_TI = PW_TR + R2 * PW_P * 4;
constexpr int PREP_WS_END = PW_TI + R2 * PW_P * 4;
static_assert(R2 * PW_P * 4 <= PW_TR, "Gs overlaps the W stages");
constexpr int PREP_WS_SMEM = PREP_WS_END;

__global__ void __launch_bounds__(THR, 1)
cham_tc_prep_ws(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                const float* __restrict__ gamma, unsigned char* __restrict__ Tws, float* __restrict__ Ews,
                unsigned long long* __restrict__ badws, int S, int D, int nch) {
  extern __shared__ __align__(1024) unsigned char smp[];
  constexpr int P = PW_P;
  float* Gs = reinterpret_cast<float*>(smp);
  float* Tr = reinterpret_cast<float*>(smp + PW_TR);
  float* Ti = reinterpret_cast<float*>(smp + PW_TI);
  auto stW = [&](int s) { return smp + PW_TR + s * W_TILE; };
  __shared__ float Ns[C2 * 8];
  __shared__ unsigned long long bad_bits;
  __shared__ __align__(8) uint64_t bars[5];   // tfull[2], mdone[2], done
  __shared__ uint32_t tslot;
  __shared__ int pfail;
  const int c = blockIdx.x, item = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int t0 = c * C2, nt = min(C2, S - t0);
  const int NT = D / KT;
  if (warp == 0) tc::tmem_alloc(&tslot, 128);
  if (tid == 0) {
    bad_bits = 0ull;
    pfail = 0;
    for (int i = 0; i < 5; ++i) tc::mbar_init(&bars[i], 1);
    tc::fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tG = tslot;
  if (tid == 0) {
    bool ok = true;
    auto issue = [&](int kt) {
      const int s = kt & 1;
      tc::mbar_expect_tx(&bars[s], W_TILE);
#pragma unroll
      for (int kb = 0; kb < KT / 64; ++kb) {
        tc::tma_load_3d(stW(s) + kb * 16384, &tm_k, kt * KT + kb * 64, t0, item, &bars[s]);
        tc::tma_load_3d(stW(s) + kb * 16384 + 8192, &tm_v, kt * KT + kb * 64, t0, item, &bars[s]);
      }
    };
    constexpr uint32_t ID_G = tc::idesc_bf16(128, 128, false, false);
    issue(0);
    if (NT > 1) issue(1);
    for (int kt = 0; kt < NT && ok; ++kt) {
      const int s = kt & 1;
      if (!tc::mbar_wait(&bars[s], (kt >> 1) & 1, MAX_POLLS)) { ok = false; break; }
      tc::fence_after_sync();
      const uint32_t w = tc::smem_addr(stW(s));
#pragma unroll 1
      for (int ks = 0; ks < KT / 16; ++ks) {
        const uint64_t d = tc::sdesc_sw128(w + (ks >> 2) * 16384 + (ks & 3) * 32, 16, 1024);
        tc::mma_bf16(tG, d, d, ID_G, (kt > 0 || ks > 0) ? 1u : 0u);
      }
      tc::commit(&bars[2 + s]);
      if (kt + 2 < NT) {
        if (!tc::mbar_wait(&bars[2 + s], (kt >> 1) & 1, MAX_POLLS)) { ok = false; break; }
        issue(kt + 2);
      }
    }
    if (ok) tc::commit(&bars[4]);
    else { pfail = 1; record_timeout(); }
  }
  const bool got = tc::mbar_wait(&bars[4], 0, MAX_POLLS);
  if (__syncthreads_or(!got || pfail)) {
    if (tid == 0) record_timeout();
  } else {
    tc::fence_after_sync();
    {  // G -> Gs in the solver's interleaved order (row 2t + kv): thread = TMEM lane
       // (split-order row), 64 columns per warp half (the k half or the v half)
      const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
      const int row = 32 * (warp & 3) + lane, half = warp >> 2;
      float* grow = Gs + ilv(row) * P + half;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        float x[16];
        tc::tmem_ld16(tG + lane_base + 64 * half + 16 * u, x);
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) grow[2 * (16 * u + jj)] = x[jj];
      }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (tid < C2) {
      const int tau = tid;
      float n00r = 0.f, n00i = 0.f, n01r = 0.f, n01i = 0.f, n11r = 0.f, n11i = 0.f;
      bool flagged = false;
      if (tau < nt) {
        const float kk = Gs[(2 * tau) * P + 2 * tau];
        const float vv = Gs[(2 * tau + 1) * P + 2 * tau + 1];
        const float kv = Gs[(2 * tau) * P + 2 * tau + 1];
        const float g = gamma[(size_t)item * S + t0 + tau];
        const float cc = 0.5f * g;
        const float dr = 1.f + cc * cc * (kk * vv - kv * kv);
        const float di = -2.f * cc * kv;
        const float m2 = dr * dr + di * di;
        const float fr = 2.f * cc * dr / m2;
        const float fi = -2.f * cc * di / m2;
        n00r = fr * (-cc * vv); n00i = fi * (-cc * vv);
        n11r = fr * (-cc * kk); n11i = fi * (-cc * kk);
        n01r = fr * (cc * kv) - fi; n01i = fr + fi * (cc * kv);
        // a non-finite k or v makes its diagonal Gram entries non-finite
        flagged = !(isfinite(kk) && isfinite(vv) && isfinite(kv) && isfinite(g) && isfinite(n00r) &&
                    isfinite(n00i) && isfinite(n01r) && isfinite(n01i) && isfinite(n11r) && isfinite(n11i));
        if (flagged) {
          n00r = n00i = n01r = n01i = n11r = n11i = 0.f;
          atomicOr(&bad_bits, 1ull << tau);
        }
      }
      float* n = Ns + tau * 8;   // [[n00, n01], [n01, n11]]
      n[0] = n00r; n[1] = n00i; n[2] = n01r; n[3] = n01i; n[4] = n01r; n[5] = n01i; n[6] = n11r; n[7] = n11i;
    }
    __syncthreads();
    if (bad_bits) {   // clear the Gram rows/columns of non-finite tokens
      for (int e = tid; e < R2 * R2; e += THR) {
        const int r = e / R2, cl = e % R2;
        if (((bad_bits >> (r >> 1)) & 1ull) || ((bad_bits >> (cl >> 1)) & 1ull)) Gs[r * P + cl] = 0.f;
      }
      __syncthreads();
    }
    wy_solve<true>(Gs, P, Ns, Tr, Ti, tid);
    const size_t chunk = (size_t)item * nch + c;
    unsigned char* To = Tws + chunk * 4 * T_TILE;
    for (int e = tid; e < R2 * (R2 / 8); e += THR) {
      const int r = e % R2, g = e / R2;
      // T in the kernels' split order: element (r, c) is the solver's (ilv(r), ilv(c))
      float xr[8], xi[8];
      const int ro = ilv(r) * P, c0 = ilv(g * 8);
#pragma unroll
      for (int j = 0; j < 8; ++j) { xr[j] = Tr[ro + c0 + 2 * j]; xi[j] = Ti[ro + c0 + 2 * j]; }
      uint4 h, l;
      const int off = kmaj(r, g * 8, R2);
      tc::split8(xr, h, l);
      *reinterpret_cast<uint4*>(To + 0 * T_TILE + off) = h;
      *reinterpret_cast<uint4*>(To + 1 * T_TILE + off) = l;
      tc::split8(xi, h, l);
      *reinterpret_cast<uint4*>(To + 2 * T_TILE + off) = h;
      *reinterpret_cast<uint4*>(To + 3 * T_TILE + off) = l;
    }
    float* Eo = Ews + chunk * R2 * C2;
    for (int e = tid; e < R2 * C2; e += THR) Eo[e] = 0.f;
    if (tid == 0) badws[chunk] = bad_bits;
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tG, 128);
}

// One launch per chunk step c: colpass of chunk c (blocks [0, ncol)) and readout of chunk
// c-1 (the remaining blocks); both read the state at the start of chunk c.
__global__ void __launch_bounds__(WS_THREADS, 1)
cham_tc_step_ws(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_sr,
                const __grid_constant__ CUtensorMap tm_si, const __grid_constant__ CUtensorMap tm_dr,
                const __grid_constant__ CUtensorMap tm_di, const __nv_bfloat16* __restrict__ q,
                const unsigned char* __restrict__ Tws, float* __restrict__ Ews,
                const unsigned long long* __restrict__ badws, int src_identity, float* __restrict__ dst_r,
                float* __restrict__ dst_i, __nv_bfloat16* __restrict__ out, int S, int D, int nch, int c,
                int ncol) {
  if ((int)blockIdx.x < ncol)
    colpass_ws_body(tm_k, tm_v, tm_sr, tm_si, tm_dr, tm_di, q, Tws, Ews, badws, src_identity, dst_r, dst_i, S, D,
                    nch, c, blockIdx.x);
  else
    readout_ws_body(tm_k, tm_v, tm_q, tm_sr, Ews, badws, out, S, D, nch, c - 1, blockIdx.x - ncol, blockIdx.y,
                    blockIdx.y * D);
}

// ---------------------------------------------------------------------------------
// Column pass, two CTAs per SM (bf16 inputs).  Same arithmetic as colpass_ws_body, laid
// out so that 96 KB of shared memory and 256 TMEM columns suffice: at b = 8, D = 1024
// all 256 column blocks of a chunk are resident at once (the 320-CTA merged launch took
// three CTA generations per SM).  The readout runs in separate launches over batches of
// chunks (cham_tc_readout_batch), from the chunks' end states kept in a ring of buffers.
//
// smem: ring [0, 64K) = 2 slots of 32 KB
//         phase A: three slots (the two ring slots and ZC, idle until phase T);
//                  slot = W half tile (64 state rows x 128 vectors: k box 8K | v box 8K)
//                  | state half tile (re 8K | im 8K, fp32 SW128), split in place into
//                  one bf16 MN-major operand [64 rows][hi 64 | lo 64] (16K)
//         phase T: Tr (hi | lo) across both slots, then Ti (hi | lo)
//         phase E: Ca hi/lo (16K) | Y (4K) in slot 0
//         phase B: slot = W tile (128 state rows x 128 vectors, 32K); once the tile's
//                  MMA is done, the same slot takes dH (re 16K | im 16K, fp32 SW128),
//                  which TMA adds onto the state
//       ZC [64K, 96K): Z as [128][hi 64 | lo 64] bf16, then Cm the same way
//       barriers, TMEM slot, failure flag at 96K
// Each hi/lo operand pair is one N = 128 operand, so an A tile is read once per K step
// (the MMAs are bound by shared-memory operand bandwidth); the accumulator halves are
// summed by the consumers.
// TMEM (256 columns): phase A Z [0,128); phase T P1 [0,128) P2 [128,256); phase E E [0,64);
// phase B dH[2] at [0,128) and [128,256).
constexpr int CP2_SLOT = 32 * 1024, CP2_ZC = 64 * 1024, CP2_BAR = 96 * 1024;
constexpr int CP2_SMEM = CP2_BAR + 256;
constexpr int KH = 64;   // state rows per phase-A half tile
constexpr int CP2_THREADS = CONS + 64;    // consumers + producer warp (MMAs, phases T/E/B) + phase-A loader warp
enum { B2_FULL = 0, B2_SPL = 3, B2_MD = 6, B2_TT = 9, B2_ZR = 10, B2_P1 = 11, B2_MT = 12, B2_CR = 13, B2_ME = 14,
       B2_DH = 15, B2_DF = 17, B2_ER = 19, B2_SR = 21, N_BARS2 = 23 };

__device__ __forceinline__ void
colpass2_body(const CUtensorMap& tm_k, const CUtensorMap& tm_v, const CUtensorMap& tm_hr64, const CUtensorMap& tm_hi64,
              const CUtensorMap& tm_hr128, const CUtensorMap& tm_hi128, unsigned char* __restrict__ ring, int nring, int b,
              const __nv_bfloat16* __restrict__ q, const unsigned char* __restrict__ Tws, float* __restrict__ Ews,
              const unsigned long long* __restrict__ badws, int S, int D, int nch, int c0, int c1, int item, int jb,
              int h0) {
  extern __shared__ __align__(1024) unsigned char smc[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smc + CP2_BAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smc + CP2_BAR + 8 * N_BARS2);
  volatile int* fail = reinterpret_cast<volatile int*>(smc + CP2_BAR + 8 * N_BARS2 + 16);
  auto slot = [&](int s) { return smc + s * CP2_SLOT; };   // slot 2 = the ZC region, phase A only
  unsigned char* sZ = smc + CP2_ZC;       // Z, then Cm: [128][hi 64 | lo 64] bf16 MN-major (32K)
  constexpr int NGW = 2 * N2 / 8;          // core-matrix columns of an N = 128 operand
  unsigned char* sAh = smc;               // phase E: Re(Cm) K-major hi/lo, Y
  unsigned char* sAl = smc + CA_TILE;
  unsigned char* sY = smc + 2 * CA_TILE;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int j0 = jb * NB2;
  const int NH = D / KH, NT = D / KT;

  if (warp == 0) tc::tmem_alloc(tslot, 256);
  if (tid == 0) {
    for (int i = 0; i < N_BARS2; ++i) tc::mbar_init(&bars[i], 1);
    *fail = 0;
    tc::fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = *tslot;
  const uint32_t tZ = tbase, tP1 = tbase, tP2 = tbase + 128, tE = tbase, tDH = tbase;

  // The chunks [c0, c1) one after another: a column block depends only on its own
  // column block of the previous chunk, so the CTAs never wait for one another.
  for (int c = c0; c < c1; ++c) {
    const int t0 = c * C2, nt = min(C2, S - t0);
    const size_t chunk = (size_t)item * nch + c;
    const unsigned long long bad = badws[chunk];
    const bool patch_w = bad != 0ull;       // padded rows come back zero from the TMA bounds
    const int src_identity = c == 0 && !h0;   // with a carried hologram the planes start as H0
    // The state is updated in place in the output planes (phase A reads its column
    // block, phase B adds dH with TMA reductions); phase A also stores the real part it
    // reads (the end state of chunk c-1), rounded to bf16, to that chunk's ring slot as
    // the readout's K-major operand images: row r, column j of an item's D x D real plane
    // at ((r / 128) (D / 64) + j / 64) 16K + kmaj(r % 128, j % 64).  (The readout's state
    // operand is the one place the bf16 path rounds the state: Re(H) q with Re(H) to 2^-9
    // relative, the readout itself rounded to bf16 after; the state and everything
    // carried from chunk to chunk stay fp32-accurate.)
    const CUtensorMap* tm_sr = &tm_hr64;
    const CUtensorMap* tm_si = &tm_hi64;
    const CUtensorMap* tm_dr = &tm_hr128;
    const CUtensorMap* tm_di = &tm_hi128;
    const int src_row_re = 0, src_row_im = 0, dst_row_re = 0, dst_row_im = 0;
    unsigned char* ring_img = c > 0 ? ring + (((size_t)((c - 1) % nring) * b + item) * D) * D * sizeof(float) : nullptr;

    auto issue_a = [&](int h) {   // phase-A half tile h into slot h % 3
      const int s = h % 3;
      unsigned char* w = slot(s);
      tc::mbar_expect_tx(&bars[B2_FULL + s], 16 * 1024 + (src_identity ? 0 : 16 * 1024));
      tc::tma_load_3d(w, &tm_k, h * KH, t0, item, &bars[B2_FULL + s]);
      tc::tma_load_3d(w + 8192, &tm_v, h * KH, t0, item, &bars[B2_FULL + s]);
      if (!src_identity) {   // the state stays in L2 from chunk to chunk (b D^2 x 8 B)
        const uint64_t keep = tc::policy_evict_last();
        tc::tma_load_2d_hint(w + 16384, tm_sr, j0, (src_row_re + item) * D + h * KH, &bars[B2_FULL + s], keep);
        tc::tma_load_2d_hint(w + 24576, tm_si, j0, (src_row_im + item) * D + h * KH, &bars[B2_FULL + s], keep);
      }
    };
    if (warp == 9) {
      // ============ phase-A loader (one thread): refill each slot once its MMAs are done ============
      if (lane == 0) {
        for (int h = 0; h + 3 < NH; ++h) {
          if (*fail || !tc::mbar_wait(&bars[B2_MD + h % 3], (h / 3) & 1, MAX_POLLS)) {
            *fail = 1;
            record_timeout();
            break;
          }
          issue_a(h + 3);
        }
      }
    } else if (warp == 8) {
      // ======================= producer (one thread) =======================
      if (lane == 0) {
        bool ok = true;
        // Barrier parities are closed forms of the tile indices (no counters indexed by a
        // runtime slot, which would live in local memory): phase-A half tile h is use h / 3
        // of slot h % 3; phase-B tile kt is use a_uses(s) + kt / 2 of slot s = (kt + 1) & 1.
        auto pwait = [&](int b, uint32_t par) {
          if (!ok) return false;
          if (*fail || !tc::mbar_wait(&bars[b], par, MAX_POLLS)) { ok = false; *fail = 1; record_timeout(); }
          return ok;
        };
        auto issue_b = [&](int kt) {  // phase-B W tile kt into slot (kt + 1) & 1
          const int s = (kt + 1) & 1;
          unsigned char* w = slot(s);
          tc::mbar_expect_tx(&bars[B2_FULL + s], W_TILE);
#pragma unroll
          for (int kb = 0; kb < KT / 64; ++kb) {
            tc::tma_load_3d(w + kb * 16384, &tm_k, kt * KT + kb * 64, t0, item, &bars[B2_FULL + s]);
            tc::tma_load_3d(w + kb * 16384 + 8192, &tm_v, kt * KT + kb * 64, t0, item, &bars[B2_FULL + s]);
          }
        };
        constexpr uint32_t ID_Z = tc::idesc_bf16(128, 2 * N2, false, true);
        constexpr uint32_t ID_H = tc::idesc_bf16(128, 2 * N2, true, true);
        // ---- phase A: Z = Wᵀ S over 64-row half tiles (the loader warp refills the slots)
        for (int h = 0; h < 3 && h < NH; ++h) issue_a(h);
        for (int h = 0; h < NH && ok; ++h) {
          const int s = h % 3;
          if (!pwait(B2_FULL + s, (h / 3) & 1) || !pwait(B2_SPL + s, (h / 3) & 1)) break;
          tc::fence_after_sync();
          const uint32_t aw = tc::smem_addr(slot(s));
          const uint32_t bb = aw + 16384;
#pragma unroll 1
          for (int ks = 0; ks < KH / 16; ++ks) {
            const uint64_t a = tc::sdesc_sw128(aw + ks * 32, 16, 1024);
            tc::mma_bf16(tZ, a, tc::sdesc(bb + ks * 2 * NGW * 128, NGW * 128, 128), ID_Z, (h > 0 || ks > 0) ? 1u : 0u);
          }
          tc::commit(&bars[B2_MD + s]);
        }
        // ---- phase T: P1 = Tr Z, then P2 = Ti Z, T halves through the ring
        const int sl = (NH - 1) % 3;
        const unsigned char* tsrc = Tws + chunk * 4 * T_TILE;
        constexpr uint32_t ID_T = tc::idesc_bf16(128, 2 * N2, false, true);
        constexpr uint32_t ID_T64 = tc::idesc_bf16(128, N2, false, true);
        auto t_mmas = [&](uint32_t td) {
          const uint32_t th = tc::smem_addr(slot(0)), tl = tc::smem_addr(slot(1));
          const uint32_t z = tc::smem_addr(sZ);
#pragma unroll 1
          for (int ks = 0; ks < R2 / 16; ++ks) {
            const uint64_t ah = tc::sdesc(th + ks * 2 * R2 * 16, R2 * 16, 128);
            const uint64_t al = tc::sdesc(tl + ks * 2 * R2 * 16, R2 * 16, 128);
            const uint64_t bz = tc::sdesc(z + ks * 2 * NGW * 128, NGW * 128, 128);   // [Z_hi | Z_lo]
            tc::mma_bf16(td, ah, bz, ID_T, ks > 0 ? 1u : 0u);
            tc::mma_bf16(td, al, bz, ID_T64, 1u);                                    // Tr_lo Z_hi
          }
        };
        if (ok && pwait(B2_MD + sl, ((NH - 1) / 3) & 1)) {   // every phase-A MMA done: ring free
          tc::mbar_expect_tx(&bars[B2_TT], 2 * T_TILE);
          tc::bulk_load(slot(0), tsrc, T_TILE, &bars[B2_TT]);
          tc::bulk_load(slot(1), tsrc + T_TILE, T_TILE, &bars[B2_TT]);
          if (pwait(B2_ZR, 0) && pwait(B2_TT, 0)) {
            tc::fence_after_sync();
            t_mmas(tP1);
            tc::commit(&bars[B2_P1]);
            if (pwait(B2_P1, 0)) {
              tc::mbar_expect_tx(&bars[B2_TT], 2 * T_TILE);
              tc::bulk_load(slot(0), tsrc + 2 * T_TILE, T_TILE, &bars[B2_TT]);
              tc::bulk_load(slot(1), tsrc + 3 * T_TILE, T_TILE, &bars[B2_TT]);
              if (pwait(B2_TT, 1)) {
                tc::fence_after_sync();
                t_mmas(tP2);
                tc::commit(&bars[B2_MT]);
              }
            }
          }
        }
        // ---- phase E: E = Re(Cm) Y (slot 0); the first phase-B W tile goes to slot 1
        if (ok && pwait(B2_MT, 0)) {
          issue_b(0);
          if (pwait(B2_CR, 0)) {
            tc::fence_after_sync();
            constexpr uint32_t ID_E = tc::idesc_bf16(128, C2, false, false);
            const uint32_t ah = tc::smem_addr(sAh), al = tc::smem_addr(sAl), yh = tc::smem_addr(sY);
#pragma unroll 1
            for (int ks = 0; ks < NB2 / 16; ++ks) {
              const uint64_t b_h = tc::sdesc(yh + ks * 2 * C2 * 16, C2 * 16, 128);
              tc::mma_bf16(tE, tc::sdesc(ah + ks * 2 * R2 * 16, R2 * 16, 128), b_h, ID_E, ks > 0 ? 1u : 0u);
              tc::mma_bf16(tE, tc::sdesc(al + ks * 2 * R2 * 16, R2 * 16, 128), b_h, ID_E, 1u);
            }
            tc::commit(&bars[B2_ME]);
          }
        }
        // ---- phase B: per 128-row tile: W tile -> dH = W Cm (TMEM, double-buffered) ->
        // the state tile into the same slot -> consumers' epilogue -> TMA store -> slot free
        if (ok && pwait(B2_ME, 0)) {
          if (NT > 1) issue_b(1);
          for (int kt = 0; kt < NT && ok; ++kt) {
            const int s = (kt + 1) & 1, d = kt & 1;
            const uint32_t use = (uint32_t)((NH + 2 - s) / 3 + (kt >> 1));   // use of slot s
            if (!pwait(B2_FULL + s, use & 1)) break;
            if (patch_w && !pwait(B2_SPL + s, use & 1)) break;
            if (kt == 0 && !pwait(B2_ER, 0)) break;   // dH[0] overlaps E: the consumers have read it
            if (kt >= 2 && !pwait(B2_DF + d, ((kt - 2) >> 1) & 1)) break;
            tc::fence_after_sync();
            const uint32_t aw = tc::smem_addr(slot(s));
            const uint32_t cm = tc::smem_addr(sZ);
#pragma unroll 1
            for (int ks = 0; ks < R2 / 16; ++ks) {
              const uint64_t a = tc::sdesc_sw128(aw + ks * 2048, 16384, 1024);
              tc::mma_bf16(tDH + 128 * d, a, tc::sdesc(cm + ks * 2 * NGW * 128, NGW * 128, 128), ID_H, ks > 0 ? 1u : 0u);
            }
            tc::commit(&bars[B2_DH + d]);
            // tile kt-1's slot, once its store has read it, takes W tile kt+1
            if (kt >= 1 && kt + 1 < NT) {
              const int sp = kt & 1;
              if (!pwait(B2_SR + sp, ((kt - 1) >> 1) & 1)) break;
              issue_b(kt + 1);
            }
          }
        }
      }
    } else {
      // ======================= consumers (warps 0-7) =======================
      const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
      const int row = 32 * (warp & 3) + lane, half = warp >> 2;
      bool ok = true;
      auto cwait = [&](int b, uint32_t par) {
        bool mine = ok && !*fail && tc::mbar_wait(&bars[b], par, MAX_POLLS);
        const bool all = consumers_all(mine);
        if (!all) { if (ok && tid == 0) record_timeout(); ok = false; *fail = 1; }
        return ok;
      };
      auto zero_bad_rows = [&](unsigned char* w, int nblk) {   // swizzled W (half) tile, nblk blocks of 16K
        for (int e = tid; e < R2 * 8 * nblk; e += CONS) {
          const int r = e % R2, cc = e / R2;                    // 16-byte chunk cc of row r
          if ((bad >> tok(r)) & 1ull)
            *reinterpret_cast<uint4*>(w + (cc >> 3) * 16384 + r * 128 + (((cc & 7) ^ (r & 7)) << 4)) =
                make_uint4(0, 0, 0, 0);
        }
      };
      // ---- phase A: split each state half tile in place
      const uint64_t stream_once = tc::policy_evict_first();
      for (int h = 0; h < NH && ok; ++h) {
        const int s = h % 3;
        if (!cwait(B2_FULL + s, (h / 3) & 1)) break;
        unsigned char* w = slot(s);
        if (patch_w) zero_bad_rows(w, 1);
        float x[2][8];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int e = tid + CONS * u;
          const int i = e % KH, gg = e / KH;        // row i, 8-column group gg (0-3 re, 4-7 im)
          if (src_identity) {
            const int gi = h * KH + i, col = j0 + (gg & 3) * 8;
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) x[u][jj] = (gg < 4 && gi == col + jj) ? 1.f : 0.f;
          } else {
            const unsigned char* box = w + (gg < 4 ? 16384 : 24576);
            const int c0 = 2 * (gg & 3);
            const float4 a = *reinterpret_cast<const float4*>(box + i * 128 + ((c0 ^ (i & 7)) << 4));
            const float4 b = *reinterpret_cast<const float4*>(box + i * 128 + (((c0 + 1) ^ (i & 7)) << 4));
            x[u][0] = a.x; x[u][1] = a.y; x[u][2] = a.z; x[u][3] = a.w;
            x[u][4] = b.x; x[u][5] = b.y; x[u][6] = b.z; x[u][7] = b.w;
          }
        }
        tc::named_sync(1, CONS);   // every fp32 value read before the split overwrites it
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int e = tid + CONS * u;
          const int i = e % KH, gg = e / KH;
          uint4 hv, lv;
          tc::split8(x[u], hv, lv);
          *reinterpret_cast<uint4*>(w + 16384 + mnmaj(i, gg * 8, NGW)) = hv;
          *reinterpret_cast<uint4*>(w + 16384 + mnmaj(i, N2 + gg * 8, NGW)) = lv;
          if (gg < 4 && ring_img != nullptr) {   // the real half as read: chunk c-1's end state
            const int r = h * KH + i, j = j0 + gg * 8;
            unsigned char* img = ring_img + (size_t)((r >> 7) * (D / RKT) + (j >> 6)) * (16 * 1024) + kmaj(r & 127, j & 63, R2);
            tc::st_global_hint(img, hv, stream_once);   // read once, by the readout
          }
        }
        tc::fence_proxy_async();
        tc::named_sync(1, CONS);
        if (tid == 0) tc::mbar_arrive(&bars[B2_SPL + s]);
      }
      // ---- phase T: Z -> operand (MD of the last half tile: every phase-A MMA done)
      const int sl = (NH - 1) % 3;
      if (ok && cwait(B2_MD + sl, ((NH - 1) / 3) & 1)) {
        tc::fence_after_sync();
        float z[32], zl[32];
        tc::tmem_ld16(tZ + lane_base + 32 * half, z);
        tc::tmem_ld16(tZ + lane_base + 32 * half + 16, z + 16);
        tc::tmem_ld16(tZ + lane_base + N2 + 32 * half, zl);
        tc::tmem_ld16(tZ + lane_base + N2 + 32 * half + 16, zl + 16);
#pragma unroll
        for (int j = 0; j < 32; ++j) z[j] += zl[j];
#pragma unroll
        for (int g4 = 0; g4 < 4; ++g4) {
          uint4 hv, lv;
          tc::split8(z + 8 * g4, hv, lv);
          *reinterpret_cast<uint4*>(sZ + mnmaj(row, 32 * half + 8 * g4, NGW)) = hv;
          *reinterpret_cast<uint4*>(sZ + mnmaj(row, N2 + 32 * half + 8 * g4, NGW)) = lv;
        }
        tc::fence_proxy_async();
        tc::fence_before_sync();
        tc::named_sync(1, CONS);
        if (tid == 0) tc::mbar_arrive(&bars[B2_ZR]);
      }
      // ---- phase E: Cm -> operands (ZC: MN-major re | im; slot 0: Re(Cm) K-major, Y)
      if (ok && cwait(B2_MT, 0)) {
        tc::fence_after_sync();
        // Cm = P1 - i P2 term by term (Re = P1r - P2i, Im = P1i + P2r), each product's two
        // accumulator halves (hi-operand and lo-operand parts) summed; real part first
#pragma unroll
        for (int part = 0; part < 2; ++part) {
          const int c1 = part == 0 ? 0 : 32, c2 = part == 0 ? 32 : 0;
          const float sg = part == 0 ? -1.f : 1.f;
          float cv[16], a[16], b2[16];
          tc::tmem_ld16(tP1 + lane_base + c1 + 16 * half, a);
          tc::tmem_ld16(tP1 + lane_base + N2 + c1 + 16 * half, b2);
#pragma unroll
          for (int j = 0; j < 16; ++j) cv[j] = a[j] + b2[j];
          tc::tmem_ld16(tP2 + lane_base + c2 + 16 * half, a);
          tc::tmem_ld16(tP2 + lane_base + N2 + c2 + 16 * half, b2);
#pragma unroll
          for (int j = 0; j < 16; ++j) cv[j] += sg * (a[j] + b2[j]);
#pragma unroll
          for (int g2 = 0; g2 < 2; ++g2) {
            uint4 hv, lv;
            const int jc = 16 * half + 8 * g2;
            tc::split8(cv + 8 * g2, hv, lv);
            *reinterpret_cast<uint4*>(sZ + mnmaj(row, c1 + jc, NGW)) = hv;
            *reinterpret_cast<uint4*>(sZ + mnmaj(row, N2 + c1 + jc, NGW)) = lv;
            if (part == 0) {
              *reinterpret_cast<uint4*>(sAh + kmaj(row, jc, R2)) = hv;
              *reinterpret_cast<uint4*>(sAl + kmaj(row, jc, R2)) = lv;
            }
          }
        }
        {
          const int t = tid % C2, gq = tid / C2;   // 64 tokens x 4 groups of 8 columns
          uint4 u = make_uint4(0, 0, 0, 0);
          if (t < nt) u = *reinterpret_cast<const uint4*>(q + ((size_t)item * S + t0 + t) * D + j0 + gq * 8);
          *reinterpret_cast<uint4*>(sY + kmaj(t, gq * 8, C2)) = u;
        }
        tc::fence_proxy_async();
        tc::fence_before_sync();
        tc::named_sync(1, CONS);
        if (tid == 0) tc::mbar_arrive(&bars[B2_CR]);
      }
      if (ok && cwait(B2_ME, 0)) {
        tc::fence_after_sync();
        float e[32];
        tc::tmem_ld16(tE + lane_base + 32 * half, e);
        tc::tmem_ld16(tE + lane_base + 32 * half + 16, e + 16);
        tc::fence_before_sync();
        tc::named_sync(1, CONS);
        if (tid == 0) tc::mbar_arrive(&bars[B2_ER]);   // E read: the first dH may overwrite it
        float4* Eo = reinterpret_cast<float4*>(Ews + chunk * R2 * C2 + (size_t)row * C2 + 32 * half);
#pragma unroll
        for (int t = 0; t < 8; ++t) atomicAdd(Eo + t, make_float4(e[4 * t], e[4 * t + 1], e[4 * t + 2], e[4 * t + 3]));
      }
      // ---- phase B: S_next = S + dH in the slot (thread: one row of one plane), TMA store
      for (int kt = 0; kt < NT && ok; ++kt) {
        const int s = (kt + 1) & 1, d = kt & 1;
        unsigned char* w = slot(s);
        if (patch_w) {
          if (!cwait(B2_FULL + s, ((NH + 2 - s) / 3 + (kt >> 1)) & 1)) break;
          zero_bad_rows(w, 2);
          tc::fence_proxy_async();
          tc::named_sync(1, CONS);
          if (tid == 0) tc::mbar_arrive(&bars[B2_SPL + s]);
        }
        if (!cwait(B2_DH + d, (kt >> 1) & 1)) break;
        tc::fence_after_sync();
        float dh[32], dl[32];
        tc::tmem_ld16(tDH + 128 * d + lane_base + 32 * half, dh);
        tc::tmem_ld16(tDH + 128 * d + lane_base + 32 * half + 16, dh + 16);
        tc::tmem_ld16(tDH + 128 * d + lane_base + N2 + 32 * half, dl);
        tc::tmem_ld16(tDH + 128 * d + lane_base + N2 + 32 * half + 16, dl + 16);
#pragma unroll
        for (int j = 0; j < 32; ++j) dh[j] += dl[j];
        tc::fence_before_sync();
        tc::named_sync(1, CONS);
        if (tid == 0) tc::mbar_arrive(&bars[B2_DF + d]);   // dH[d] may be overwritten
        // the slot (its W tile read) takes dH, which TMA adds onto the state in place; the
        // first chunk stores I + dH instead
        unsigned char* box = w + half * 16384;
        const int gi = kt * KT + row;
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
          float v4[4];
#pragma unroll
          for (int jj = 0; jj < 4; ++jj)
            v4[jj] = dh[4 * cc + jj] + ((src_identity && !half && gi == j0 + 4 * cc + jj) ? 1.f : 0.f);
          *reinterpret_cast<float4*>(box + row * 128 + ((cc ^ (row & 7)) << 4)) = make_float4(v4[0], v4[1], v4[2], v4[3]);
        }
        tc::fence_proxy_async();
        tc::named_sync(1, CONS);
        if (tid == 0) {
          const uint64_t keep = tc::policy_evict_last();
          if (src_identity) {
            tc::tma_store_2d_hint(tm_dr, j0, (dst_row_re + item) * D + kt * KT, w, keep);
            tc::tma_store_2d_hint(tm_di, j0, (dst_row_im + item) * D + kt * KT, w + 16384, keep);
          } else {
            tc::tma_reduce_add_2d_hint(tm_dr, j0, (dst_row_re + item) * D + kt * KT, w, keep);
            tc::tma_reduce_add_2d_hint(tm_di, j0, (dst_row_im + item) * D + kt * KT, w + 16384, keep);
          }
          tc::bulk_commit();
          tc::bulk_wait_read<0>();                 // the store has read the slot
          tc::mbar_arrive(&bars[B2_SR + s]);
        }
      }
      if (tid == 0) {
        tc::bulk_wait<0>();                        // all state writes performed
        tc::fence_proxy_async_global();            // before the next chunk's loads read them
      }
    }
    // chunk done: every load consumed, every MMA waited for, every store performed
    tc::fence_before_sync();
    __syncthreads();
    if (*fail) break;
    if (c + 1 < c1) {
      if (tid == 0) {
        for (int i = 0; i < N_BARS2; ++i) {
          tc::mbar_inval(&bars[i]);
          tc::mbar_init(&bars[i], 1);
        }
        tc::fence_mbar_init();
      }
      __syncthreads();
      tc::fence_after_sync();
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tbase, 256);
}

// One launch per group of chunks: CTAs [0, D/32 * b) run the column pass of chunks
// [c0, c1) (item-major); the rest run the readouts of chunks [r0, r0 + nr), whose end
// states the previous group left in the ring, on the SM slots the column pass leaves free.
__global__ void __launch_bounds__(CP2_THREADS, 2)
cham_tc_colpass2(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                 const __grid_constant__ CUtensorMap tm_hr64, const __grid_constant__ CUtensorMap tm_hi64,
                 const __grid_constant__ CUtensorMap tm_hr128, const __grid_constant__ CUtensorMap tm_hi128,
                 const __grid_constant__ CUtensorMap tm_q, unsigned char* __restrict__ ring, int nring, int b,
                 const __nv_bfloat16* __restrict__ q,
                 const unsigned char* __restrict__ Tws, float* __restrict__ Ews,
                 const unsigned long long* __restrict__ badws, __nv_bfloat16* __restrict__ out, int S, int D, int nch,
                 int c0, int c1, int r0, int nr, int h0) {
  const int ncol = D / NB2, nrb = D / R2;
  const int bid = blockIdx.x;
  if (bid < ncol * b) {
    colpass2_body(tm_k, tm_v, tm_hr64, tm_hi64, tm_hr128, tm_hi128, ring, nring, b, q, Tws, Ews, badws, S, D, nch,
                  c0, c1, bid / ncol, bid % ncol, h0);
  } else {
    const int r = bid - ncol * b, item = r / (nrb * nr), c = r0 + (r % (nrb * nr)) / nrb, bx = r % nrb;
    // (the fp32 state map is not read: the ring slot holds the pre-split images)
    readout2_body(tm_k, tm_v, tm_q, tm_hr128, Ews, badws, out, S, D, nch, c, bx, item, 0,
                  ring + (((size_t)(c % nring) * b + item) * D) * D * sizeof(float));
  }
}

// ---------------------------------------------------------------------------------
// Fused column pass (bf16 inputs): launch c makes ONE pass over the state rows that
// finishes chunk c-1 and starts chunk c,
//     S_c = S_{c-1} + W_{c-1} Cm_{c-1}        (stored: re -> ring[c-1], im -> ping)
//     Z_c = W_cᵀ S_c                          (accumulated tile by tile in TMEM)
// then Cm_c = T_c Z_c (written to global as the next launch's MMA operand) and the E
// partial of chunk c.  Launch 0 starts from the identity; launch nch only finishes.
// The state is read once and written once per chunk.  One CTA per (item, 64 complex
// columns), one per SM; rows in tiles of 64 (dH = W_{c-1} Cm_{c-1} with M = 64: row r of
// the tile in TMEM lane (r mod 16) + 32 (r / 16)).
//
// smem: stage s (2) at s*64K = W_{c-1} half (16K) | W_c half (16K) | state tile (64 rows
//       x (re 64 | im 64) fp32: four 32-column SW128 boxes of 8K; after the store, split in
//       place into bf16 hi 16K | lo 16K); phase T: T tiles (4 x 32K) over both stages,
//       then Re(Cm) K-major hi/lo (32K) | Y (8K)
//       CZ [128K, 192K): Cm_{c-1} operand (hi 32K | lo 32K), then Z_c operand
//       barriers, TMEM slot, failure flag at 192K
// TMEM (512 columns): Z [0,128)  dH[2] [128,384) (M = 64)  P1 [128,256) P2 [256,384)
//       E [384,448)
constexpr int NB3 = 64, N3 = 2 * NB3, KH3 = 64;
constexpr int CP3_STAGE = 64 * 1024, CP3_CZ = 128 * 1024, CP3_BAR = 192 * 1024;
constexpr int CP3_SMEM = CP3_BAR + 256;
constexpr int CM3_BYTES = 64 * 1024;   // Cm operand per CTA (hi | lo), MN-major K = 128, N = 128
enum { B3_FULL = 0, B3_WFIX = 2, B3_DH = 4, B3_DF = 6, B3_SPL = 8, B3_MD = 10, B3_CMF = 12, B3_TT = 13,
       B3_ZR = 14, B3_MT = 15, B3_CR = 16, B3_ME = 17, N_BARS3 = 18 };

__global__ void __launch_bounds__(WS_THREADS, 1)
cham_tc_colpass3(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                 const __grid_constant__ CUtensorMap tm_sr, const __grid_constant__ CUtensorMap tm_si,
                 const __grid_constant__ CUtensorMap tm_dr, const __grid_constant__ CUtensorMap tm_di,
                 int src_row_re, int src_row_im, int dst_row_re, int dst_row_im,
                 const unsigned char* __restrict__ cm_in, unsigned char* __restrict__ cm_out,
                 const __nv_bfloat16* __restrict__ q, const unsigned char* __restrict__ Tws,
                 float* __restrict__ Ews, const unsigned long long* __restrict__ badws, int S, int D, int nch,
                 int c) {
  extern __shared__ __align__(1024) unsigned char smf[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smf + CP3_BAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(smf + CP3_BAR + 8 * N_BARS3);
  volatile int* fail = reinterpret_cast<volatile int*>(smf + CP3_BAR + 8 * N_BARS3 + 16);
  auto stage = [&](int s) { return smf + s * CP3_STAGE; };
  unsigned char* sCZ = smf + CP3_CZ;
  unsigned char* sAh = smf;                      // phase E: Re(Cm) K-major hi/lo, Y
  unsigned char* sAl = smf + 16384;
  unsigned char* sY = smf + 32768;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int item = blockIdx.y, j0 = blockIdx.x * NB3;
  const bool has_prev = c > 0, has_next = c < nch;
  const bool prev_identity = c == 1;             // S_0 = I is not in memory
  const int tp = (c - 1) * C2, tc0 = c * C2;     // first tokens of chunks c-1 and c
  const unsigned long long bad_prev = has_prev ? badws[(size_t)item * nch + c - 1] : 0ull;
  const unsigned long long bad_next = has_next ? badws[(size_t)item * nch + c] : 0ull;
  const bool patch_w = (bad_prev | bad_next) != 0ull;
  const int NH = D / KH3;
  const size_t cm_off = ((size_t)item * (D / NB3) + blockIdx.x) * CM3_BYTES;

  if (warp == 0) tc::tmem_alloc(tslot, 512);
  if (tid == 0) {
    for (int i = 0; i < N_BARS3; ++i) tc::mbar_init(&bars[i], 1);
    *fail = 0;
    tc::fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = *tslot;
  const uint32_t tZ = tbase, tDH = tbase + 128, tP1 = tbase + 128, tP2 = tbase + 256, tE = tbase + 384;

  if (warp == 8) {
    // ======================= producer (one thread) =======================
    if (lane == 0) {
      bool ok = true;
      auto pwait = [&](int b, uint32_t par) {
        if (!ok) return false;
        if (*fail || !tc::mbar_wait(&bars[b], par, MAX_POLLS)) { ok = false; *fail = 1; record_timeout(); }
        return ok;
      };
      auto issue = [&](int i) {   // tile i into stage i & 1
        const int s = i & 1;
        unsigned char* st = stage(s);
        tc::mbar_expect_tx(&bars[B3_FULL + s], (has_prev ? 16384 + (prev_identity ? 0 : 32768) : 0) +
                                                     (has_next ? 16384 : 0));
        if (has_prev) {
          tc::tma_load_3d(st, &tm_k, i * KH3, tp, item, &bars[B3_FULL + s]);
          tc::tma_load_3d(st + 8192, &tm_v, i * KH3, tp, item, &bars[B3_FULL + s]);
#pragma unroll
          for (int bx = 0; bx < 2 && !prev_identity; ++bx) {
            tc::tma_load_2d(st + 32768 + bx * 8192, &tm_sr, j0 + 32 * bx, (src_row_re + item) * D + i * KH3,
                            &bars[B3_FULL + s]);
            tc::tma_load_2d(st + 49152 + bx * 8192, &tm_si, j0 + 32 * bx, (src_row_im + item) * D + i * KH3,
                            &bars[B3_FULL + s]);
          }
        }
        if (has_next) {
          tc::tma_load_3d(st + 16384, &tm_k, i * KH3, tc0, item, &bars[B3_FULL + s]);
          tc::tma_load_3d(st + 16384 + 8192, &tm_v, i * KH3, tc0, item, &bars[B3_FULL + s]);
        }
      };
      constexpr uint32_t ID_H = tc::idesc_bf16(64, N3, true, true);
      constexpr uint32_t ID_Z = tc::idesc_bf16(128, N3, false, true);
      auto do_dh = [&](int i) {   // dH[i & 1] = W_{c-1} rows of tile i x Cm_{c-1}
        const int s = i & 1, d = i & 1;
        if (!pwait(B3_FULL + s, (i >> 1) & 1)) return false;
        if (patch_w && !pwait(B3_WFIX + s, (i >> 1) & 1)) return false;
        if (i == 0 && !pwait(B3_CMF, 0)) return false;
        if (i >= 2 && !pwait(B3_DF + d, ((i - 2) >> 1) & 1)) return false;
        tc::fence_after_sync();
        const uint32_t aw = tc::smem_addr(stage(s));
        const uint32_t ch = tc::smem_addr(sCZ), cl = ch + 32768;
#pragma unroll 1
        for (int ks = 0; ks < R2 / 16; ++ks) {
          const uint64_t a = tc::sdesc_sw128(aw + ks * 2048, 16384, 1024);
          tc::mma_bf16(tDH + 128 * d, a, tc::sdesc(ch + ks * 2 * (N3 / 8) * 128, (N3 / 8) * 128, 128), ID_H,
                       ks > 0 ? 1u : 0u);
          tc::mma_bf16(tDH + 128 * d, a, tc::sdesc(cl + ks * 2 * (N3 / 8) * 128, (N3 / 8) * 128, 128), ID_H, 1u);
        }
        tc::commit(&bars[B3_DH + d]);
        return true;
      };
      if (has_prev) {
        tc::mbar_expect_tx(&bars[B3_CMF], CM3_BYTES);
        tc::bulk_load(sCZ, cm_in + cm_off, CM3_BYTES / 2, &bars[B3_CMF]);
        tc::bulk_load(sCZ + CM3_BYTES / 2, cm_in + cm_off + CM3_BYTES / 2, CM3_BYTES / 2, &bars[B3_CMF]);
      }
      issue(0);
      if (NH > 1) issue(1);
      if (has_prev && !do_dh(0)) ok = false;
      for (int i = 0; i < NH && ok; ++i) {
        const int s = i & 1;
        if (has_prev && i + 1 < NH && !do_dh(i + 1)) break;
        if (!has_prev) {
          if (!pwait(B3_FULL + s, (i >> 1) & 1)) break;
          if (patch_w && !pwait(B3_WFIX + s, (i >> 1) & 1)) break;
        }
        if (!pwait(B3_SPL + s, (i >> 1) & 1)) break;   // stored (and split) by the consumers
        if (has_next) {
          tc::fence_after_sync();
          const uint32_t aw = tc::smem_addr(stage(s)) + 16384;
          const uint32_t bh = tc::smem_addr(stage(s)) + 32768, bl = bh + 16384;
#pragma unroll 1
          for (int ks = 0; ks < KH3 / 16; ++ks) {
            const uint64_t a = tc::sdesc_sw128(aw + ks * 32, 16, 1024);
            tc::mma_bf16(tZ, a, tc::sdesc(bh + ks * 2 * (N3 / 8) * 128, (N3 / 8) * 128, 128), ID_Z,
                         (i > 0 || ks > 0) ? 1u : 0u);
            tc::mma_bf16(tZ, a, tc::sdesc(bl + ks * 2 * (N3 / 8) * 128, (N3 / 8) * 128, 128), ID_Z, 1u);
          }
          tc::commit(&bars[B3_MD + s]);
          if (!pwait(B3_MD + s, (i >> 1) & 1)) break;
        }
        if (i + 2 < NH) issue(i + 2);
      }
      // ---- phase T (chunk c): Cm_c = T_c Z_c; stages are free, CZ is free (every MMA done)
      if (ok && has_next) {
        const unsigned char* tsrc = Tws + ((size_t)item * nch + c) * 4 * T_TILE;
        tc::mbar_expect_tx(&bars[B3_TT], 4 * T_TILE);
        for (int p4 = 0; p4 < 4; ++p4) tc::bulk_load(smf + p4 * T_TILE, tsrc + p4 * T_TILE, T_TILE, &bars[B3_TT]);
        if (pwait(B3_ZR, 0) && pwait(B3_TT, 0)) {
          tc::fence_after_sync();
          constexpr uint32_t ID_T = tc::idesc_bf16(128, N3, false, true);
          const uint32_t zh = tc::smem_addr(sCZ), zl = zh + 32768;
#pragma unroll 1
          for (int part = 0; part < 2; ++part) {
            const uint32_t th = tc::smem_addr(smf) + (2 * part) * T_TILE, tl = th + T_TILE;
            const uint32_t td = part ? tP2 : tP1;
#pragma unroll 1
            for (int ks = 0; ks < R2 / 16; ++ks) {
              const uint64_t ah = tc::sdesc(th + ks * 2 * R2 * 16, R2 * 16, 128);
              const uint64_t al = tc::sdesc(tl + ks * 2 * R2 * 16, R2 * 16, 128);
              const uint64_t b_h = tc::sdesc(zh + ks * 2 * (N3 / 8) * 128, (N3 / 8) * 128, 128);
              const uint64_t b_l = tc::sdesc(zl + ks * 2 * (N3 / 8) * 128, (N3 / 8) * 128, 128);
              tc::mma_bf16(td, ah, b_h, ID_T, ks > 0 ? 1u : 0u);
              tc::mma_bf16(td, ah, b_l, ID_T, 1u);
              tc::mma_bf16(td, al, b_h, ID_T, 1u);
            }
          }
          tc::commit(&bars[B3_MT]);
        }
        // ---- phase E: E = Re(Cm_c) Y_c
        if (ok && pwait(B3_CR, 0)) {
          tc::fence_after_sync();
          constexpr uint32_t ID_E = tc::idesc_bf16(128, C2, false, false);
          const uint32_t ah = tc::smem_addr(sAh), al = tc::smem_addr(sAl), yh = tc::smem_addr(sY);
#pragma unroll 1
          for (int ks = 0; ks < NB3 / 16; ++ks) {
            const uint64_t b_h = tc::sdesc(yh + ks * 2 * C2 * 16, C2 * 16, 128);
            tc::mma_bf16(tE, tc::sdesc(ah + ks * 2 * R2 * 16, R2 * 16, 128), b_h, ID_E, ks > 0 ? 1u : 0u);
            tc::mma_bf16(tE, tc::sdesc(al + ks * 2 * R2 * 16, R2 * 16, 128), b_h, ID_E, 1u);
          }
          tc::commit(&bars[B3_ME]);
        }
      }
    }
  } else {
    // ======================= consumers (warps 0-7) =======================
    const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
    const int row = 32 * (warp & 3) + lane, half = warp >> 2;
    const int hrow = 16 * (warp & 3) + lane;     // dH row of this thread (lanes 0-15)
    bool ok = true;
    auto cwait = [&](int b, uint32_t par) {
      bool mine = ok && !*fail && tc::mbar_wait(&bars[b], par, MAX_POLLS);
      const bool all = consumers_all(mine);
      if (!all) { if (ok && tid == 0) record_timeout(); ok = false; *fail = 1; }
      return ok;
    };
    auto zero_rows = [&](unsigned char* w, unsigned long long bad) {   // swizzled W half tile
      for (int e = tid; e < R2 * 8; e += CONS) {
        const int r = e % R2, cc = e / R2;
        if ((bad >> tok(r)) & 1ull)
          *reinterpret_cast<uint4*>(w + r * 128 + ((cc ^ (r & 7)) << 4)) = make_uint4(0, 0, 0, 0);
      }
    };
    for (int i = 0; i < NH && ok; ++i) {
      const int s = i & 1, d = i & 1;
      unsigned char* st = stage(s);
      unsigned char* sbox = st + 32768;
      bool waited_full = false;
      if (patch_w) {
        if (!cwait(B3_FULL + s, (i >> 1) & 1)) break;
        waited_full = true;
        if (bad_prev) zero_rows(st, bad_prev);
        if (bad_next) zero_rows(st + 16384, bad_next);
        tc::fence_proxy_async();
        tc::named_sync(1, CONS);
        if (tid == 0) tc::mbar_arrive(&bars[B3_WFIX + s]);
      }
      if (has_prev) {
        if (!cwait(B3_DH + d, (i >> 1) & 1)) break;
        tc::fence_after_sync();
        float dh[64];
#pragma unroll
        for (int u = 0; u < 4; ++u) tc::tmem_ld16(tDH + 128 * d + lane_base + 64 * half + 16 * u, dh + 16 * u);
        tc::fence_before_sync();
        tc::named_sync(1, CONS);
        if (tid == 0) tc::mbar_arrive(&bars[B3_DF + d]);
        if (!waited_full && !cwait(B3_FULL + s, (i >> 1) & 1)) break;
        if (lane < 16) {   // S_c = S_{c-1} + dH for row hrow, plane `half` (two 32-column boxes)
          const int gi = i * KH3 + hrow;
#pragma unroll
          for (int bx = 0; bx < 2; ++bx) {
            unsigned char* box = sbox + half * 16384 + bx * 8192;
#pragma unroll
            for (int cc = 0; cc < 8; ++cc) {
              float4* p4 = reinterpret_cast<float4*>(box + hrow * 128 + ((cc ^ (hrow & 7)) << 4));
              const int gc = j0 + 32 * bx + 4 * cc;
              const float4 a = prev_identity ? make_float4(!half && gi == gc ? 1.f : 0.f, !half && gi == gc + 1 ? 1.f : 0.f,
                                                           !half && gi == gc + 2 ? 1.f : 0.f, !half && gi == gc + 3 ? 1.f : 0.f)
                                             : *p4;
              const float* x = dh + 32 * bx + 4 * cc;
              *p4 = make_float4(a.x + x[0], a.y + x[1], a.z + x[2], a.w + x[3]);
            }
          }
        }
        tc::fence_proxy_async();
        tc::named_sync(1, CONS);
        if (tid == 0) {
#pragma unroll
          for (int bx = 0; bx < 2; ++bx) {
            tc::tma_store_2d(&tm_dr, j0 + 32 * bx, (dst_row_re + item) * D + i * KH3, sbox + bx * 8192);
            tc::tma_store_2d(&tm_di, j0 + 32 * bx, (dst_row_im + item) * D + i * KH3, sbox + 16384 + bx * 8192);
          }
          tc::bulk_commit();
          tc::bulk_wait_read<0>();               // the stores have read the tile
        }
        tc::named_sync(1, CONS);
      } else if (!waited_full) {
        if (!cwait(B3_FULL + s, (i >> 1) & 1)) break;
      }
      if (has_next) {
        // split S_c (or the identity for c == 0) in place: MN-major B operand, K = 64 rows
        float x[4][8];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int e = tid + CONS * u;
          const int ri = e % KH3, gg = e / KH3;   // row ri, 8-column group gg (0-7 re, 8-15 im)
          if (!has_prev) {
            const int gi = i * KH3 + ri, col = j0 + (gg & 7) * 8;
#pragma unroll
            for (int jj = 0; jj < 8; ++jj) x[u][jj] = (gg < 8 && gi == col + jj) ? 1.f : 0.f;
          } else {
            const unsigned char* box = sbox + (gg >> 3) * 16384 + ((gg >> 2) & 1) * 8192;
            const int q0 = 2 * (gg & 3);
            const float4 a = *reinterpret_cast<const float4*>(box + ri * 128 + ((q0 ^ (ri & 7)) << 4));
            const float4 b = *reinterpret_cast<const float4*>(box + ri * 128 + (((q0 + 1) ^ (ri & 7)) << 4));
            x[u][0] = a.x; x[u][1] = a.y; x[u][2] = a.z; x[u][3] = a.w;
            x[u][4] = b.x; x[u][5] = b.y; x[u][6] = b.z; x[u][7] = b.w;
          }
        }
        tc::named_sync(1, CONS);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int e = tid + CONS * u;
          const int ri = e % KH3, gg = e / KH3;
          uint4 hv, lv;
          tc::split8(x[u], hv, lv);
          *reinterpret_cast<uint4*>(sbox + mnmaj(ri, gg * 8, N3 / 8)) = hv;
          *reinterpret_cast<uint4*>(sbox + 16384 + mnmaj(ri, gg * 8, N3 / 8)) = lv;
        }
        tc::fence_proxy_async();
      }
      tc::named_sync(1, CONS);
      if (tid == 0) tc::mbar_arrive(&bars[B3_SPL + s]);
    }
    if (tid == 0) tc::bulk_wait<0>();            // this launch's state writes performed
    // ---- phase T: Z -> operand in CZ (the last tile's Z MMA done: every MMA done)
    if (ok && has_next) {
      const int sl = (NH - 1) & 1;
      if (cwait(B3_MD + sl, ((NH - 1) >> 1) & 1)) {
        tc::fence_after_sync();
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          float z[16];
          tc::tmem_ld16(tZ + lane_base + 64 * half + 16 * u, z);
#pragma unroll
          for (int g2 = 0; g2 < 2; ++g2) {
            uint4 hv, lv;
            tc::split8(z + 8 * g2, hv, lv);
            const int off = mnmaj(row, 64 * half + 16 * u + 8 * g2, N3 / 8);
            *reinterpret_cast<uint4*>(sCZ + off) = hv;
            *reinterpret_cast<uint4*>(sCZ + 32768 + off) = lv;
          }
        }
        tc::fence_proxy_async();
        tc::fence_before_sync();
        tc::named_sync(1, CONS);
        if (tid == 0) tc::mbar_arrive(&bars[B3_ZR]);
      }
      // ---- Cm_c -> global operand (next launch), Re(Cm_c) K-major + Y -> smem (phase E)
      if (ok && cwait(B3_MT, 0)) {
        tc::fence_after_sync();
        unsigned char* cmg = cm_out + cm_off;
#pragma unroll
        for (int u = 0; u < 2; ++u) {   // complex columns 32 * half + 16 * u .. + 15
          float p1r[16], p1i[16], p2r[16], p2i[16];
          const int jc = 32 * half + 16 * u;
          tc::tmem_ld16(tP1 + lane_base + jc, p1r);
          tc::tmem_ld16(tP1 + lane_base + NB3 + jc, p1i);
          tc::tmem_ld16(tP2 + lane_base + jc, p2r);
          tc::tmem_ld16(tP2 + lane_base + NB3 + jc, p2i);
          float cr[16], ci[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) { cr[j] = p1r[j] - p2i[j]; ci[j] = p1i[j] + p2r[j]; }
#pragma unroll
          for (int g2 = 0; g2 < 2; ++g2) {
            uint4 hv, lv;
            const int jj = jc + 8 * g2;
            tc::split8(cr + 8 * g2, hv, lv);
            *reinterpret_cast<uint4*>(cmg + mnmaj(row, jj, N3 / 8)) = hv;
            *reinterpret_cast<uint4*>(cmg + 32768 + mnmaj(row, jj, N3 / 8)) = lv;
            *reinterpret_cast<uint4*>(sAh + kmaj(row, jj, R2)) = hv;
            *reinterpret_cast<uint4*>(sAl + kmaj(row, jj, R2)) = lv;
            tc::split8(ci + 8 * g2, hv, lv);
            *reinterpret_cast<uint4*>(cmg + mnmaj(row, NB3 + jj, N3 / 8)) = hv;
            *reinterpret_cast<uint4*>(cmg + 32768 + mnmaj(row, NB3 + jj, N3 / 8)) = lv;
          }
        }
        {
          const int nt = min(C2, S - tc0);
          const int t = tid % C2, gq = tid / C2;   // 64 tokens x 4 groups of 8 columns, twice
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int g8 = gq + 4 * u;
            uint4 w = make_uint4(0, 0, 0, 0);
            if (t < nt) w = *reinterpret_cast<const uint4*>(q + ((size_t)item * S + tc0 + t) * D + j0 + g8 * 8);
            *reinterpret_cast<uint4*>(sY + kmaj(t, g8 * 8, C2)) = w;
          }
        }
        tc::fence_proxy_async();
        tc::fence_before_sync();
        tc::named_sync(1, CONS);
        if (tid == 0) tc::mbar_arrive(&bars[B3_CR]);
      }
      if (ok && cwait(B3_ME, 0)) {
        tc::fence_after_sync();
        float e[32];
        tc::tmem_ld16(tE + lane_base + 32 * half, e);
        tc::tmem_ld16(tE + lane_base + 32 * half + 16, e + 16);
        float4* Eo = reinterpret_cast<float4*>(Ews + ((size_t)item * nch + c) * R2 * C2 + (size_t)row * C2 +
                                               32 * half);
#pragma unroll
        for (int t = 0; t < 8; ++t) atomicAdd(Eo + t, make_float4(e[4 * t], e[4 * t + 1], e[4 * t + 2], e[4 * t + 3]));
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tbase, 512);
}

// Readout of a batch of chunks from their end states (rows of a ring of state buffers):
// CTA (x, y) = (chunk c0 + x / (D/128), item y, rows 128 (x % (D/128)) ...).
__global__ void __launch_bounds__(WS_THREADS, 2)
cham_tc_readout_batch(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                      const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_ring,
                      const __grid_constant__ CUtensorMap tm_last, const float* __restrict__ Ews,
                      const unsigned long long* __restrict__ badws, __nv_bfloat16* __restrict__ out, int S, int D,
                      int nch, int c0, int nring, int b, int c_last, const unsigned char* __restrict__ pre_ring) {
  const int nrb = D / R2;
  const int c = c0 + (int)blockIdx.x / nrb, bx = (int)blockIdx.x % nrb;
  const int item = blockIdx.y;
  // chunk c's end state: its ring slot (fp32 rows, or with pre_ring the pre-split images),
  // or for chunk c_last (if any) tm_last, a [b*D] fp32 plane
  const bool last = c == c_last;
  const unsigned char* pre =
      (last || pre_ring == nullptr) ? nullptr : pre_ring + (((size_t)(c % nring) * b + item) * D) * D * sizeof(float);
  readout2_body(tm_k, tm_v, tm_q, last ? tm_last : tm_ring, Ews, badws, out, S, D, nch, c, bx, item,
                last ? item * D : ((c % nring) * b + item) * D, pre);
}

// k or v as a [b][S][D] bf16 tensor, boxes of 64 elements x 64 tokens with 128-byte swizzle
// (rows past S read as 0)
int make_kv_map(CUtensorMap* m, const void* base, int b, int S, int D) {
  auto enc = tmap_encoder();
  VERACE_REQUIRE(enc != nullptr, VERACE_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  const cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)b};
  const cuuint64_t strides[2] = {(cuuint64_t)D * 2, (cuuint64_t)S * D * 2};
  const cuuint32_t box[3] = {64, (cuuint32_t)C2, 1};
  const cuuint32_t es[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  VERACE_REQUIRE(r == CUDA_SUCCESS, VERACE_ERR_CUDA, "cuTensorMapEncodeTiled (k/v) failed: %d", (int)r);
  return VERACE_OK;
}

// one plane of a [b][D][D] fp32 state as [b*D rows][D], boxes of 32 columns x 128 rows, 128B swizzle
int make_state_map(CUtensorMap* m, const float* base, int b, int D, int rows = KT) {
  auto enc = tmap_encoder();
  VERACE_REQUIRE(enc != nullptr, VERACE_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  const cuuint64_t dims[2] = {(cuuint64_t)D, (cuuint64_t)b * D};
  const cuuint64_t strides[1] = {(cuuint64_t)D * 4};
  const cuuint32_t box[2] = {32, (cuuint32_t)rows};
  const cuuint32_t es[2] = {1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  VERACE_REQUIRE(r == CUDA_SUCCESS, VERACE_ERR_CUDA, "cuTensorMapEncodeTiled (state) failed: %d", (int)r);
  return VERACE_OK;
}

// Schedule of the bf16 path.
//   merged:  one column-pass + readout launch per chunk, one CTA per SM.
//   batched: column passes two CTAs per SM, readouts batched over up to RING chunks.
//   fused:   one pass over the state per chunk (finish chunk c-1, start chunk c), one CTA
//            per 64 columns, readouts batched as above.
// VERACE_CHAM_SCHEDULE=merged|batched|fused forces one; all are tested against each other.
enum Schedule { SCHED_MERGED, SCHED_BATCHED, SCHED_FUSED };
Schedule cham_schedule(int b, int D) {
  const char* e = getenv("VERACE_CHAM_SCHEDULE");
  if (e != nullptr) {
    if (!strcmp(e, "merged")) return SCHED_MERGED;
    if (!strcmp(e, "batched")) return SCHED_BATCHED;
    if (!strcmp(e, "fused")) return SCHED_FUSED;
  }
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return (long long)b * (D / NB2 + D / R2) <= sms ? SCHED_MERGED : SCHED_BATCHED;
}

size_t tc_prep_smem() { return sizeof(float) * (PREP_DT * (R2 + 1) + 3 * R2 * (R2 + 1)); }

template <typename T>
int launch_cham_tc(const void* q, const void* k, const void* v, const float* gamma, const float* h0r,
                   const float* h0i, void* out, float* hr, float* hi, int b, int s, int D, const TcWs& w,
                   cudaStream_t st) {
  const int nch = (s + C2 - 1) / C2;
  int rc;
  const size_t ps = tc_prep_smem();
  VERACE_CUDA(cudaFuncSetAttribute(cham_tc_prep<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ps));
  VERACE_CUDA(cudaFuncSetAttribute(cham_tc_prep_ws, cudaFuncAttributeMaxDynamicSharedMemorySize, PREP_WS_SMEM));
  constexpr int CPS = colpass_smem(sizeof(T) == 4);
  VERACE_CUDA(cudaFuncSetAttribute(cham_tc_colpass<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, CPS));
  VERACE_CUDA(cudaFuncSetAttribute(cham_tc_readout<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, READOUT_SMEM));
  constexpr bool BF = sizeof(T) == 2;
  CUtensorMap pk, pv;
  if (BF) {
    if ((rc = make_kv_map(&pk, k, b, s, D)) || (rc = make_kv_map(&pv, v, b, s, D))) return rc;
    cham_tc_prep_ws<<<dim3(nch, b), THR, PREP_WS_SMEM, st>>>(pk, pv, gamma, w.T, w.E, w.bad, s, D, nch);
    if ((rc = check_launch("cham_tc_prep_ws"))) return rc;
  } else {
    cham_tc_prep<T><<<dim3(nch, b), THR, ps, st>>>((const T*)k, (const T*)v, gamma, w.T, w.E, w.bad, s, D, nch);
    if ((rc = check_launch("cham_tc_prep"))) return rc;
  }
  const dim3 gc(D / NB2, b), gr(D / R2, b);
  const float* cur_r = h0r;   // state at the start of the chunk: nullptr = the identity
  const float* cur_i = h0i;
  constexpr bool WS = sizeof(T) == 2;   // bf16: warp-specialised TMA colpass
  CUtensorMap mk, mv, m_out_r, m_out_i, m_ping_r, m_ping_i;
  if (WS) {
    if ((rc = make_kv_map(&mk, k, b, s, D)) || (rc = make_kv_map(&mv, v, b, s, D)) ||
        (rc = make_state_map(&m_out_r, hr, b, D)) || (rc = make_state_map(&m_out_i, hi, b, D)))
      return rc;
    if (nch >= 2 && ((rc = make_state_map(&m_ping_r, w.Hre, b, D)) || (rc = make_state_map(&m_ping_i, w.Him, b, D))))
      return rc;
    if (nch < 2) { m_ping_r = m_out_r; m_ping_i = m_out_i; }
  }
  Schedule sched = WS ? cham_schedule(b, D) : SCHED_MERGED;
  if (h0r != nullptr && sched == SCHED_FUSED) sched = SCHED_BATCHED;   // the fused schedule starts from I
  if (sched == SCHED_FUSED) {
    CUtensorMap mq, m_ring, m_ring64, m_him64, m_hi64;
    const size_t plane = (size_t)b * D * D;
    if ((rc = make_kv_map(&mq, q, b, s, D)) || (rc = make_state_map(&m_ring, w.ring, w.nring * b, D)) ||
        (rc = make_state_map(&m_ring64, w.ring, w.nring * b, D, KH3)) ||
        (rc = make_state_map(&m_hi64, hi, b, D, KH3)))
      return rc;
    if (nch >= 2 && (rc = make_state_map(&m_him64, w.Him, b, D, KH3))) return rc;
    if (nch < 2) m_him64 = m_hi64;
    VERACE_CUDA(cudaFuncSetAttribute(cham_tc_colpass3, cudaFuncAttributeMaxDynamicSharedMemorySize, CP3_SMEM));
    VERACE_CUDA(cudaFuncSetAttribute(cham_tc_readout_batch, cudaFuncAttributeMaxDynamicSharedMemorySize, RW2_SMEM));
    auto im_buf = [&](int j) { return ((nch - 1 - j) % 2 == 0) ? hi : w.Him; };   // im of S_{j+1}
    const size_t cm_half = (size_t)b * (D / 64) * (64 * 1024);
    for (int c = 0; c <= nch; ++c) {
      // launch c finishes chunk c-1 (S_c into ring[(c-1) % RING] and im_buf(c-1)) and starts chunk c
      const int rs = c >= 2 ? (c - 2) % w.nring : 0, rd = c >= 1 ? (c - 1) % w.nring : 0;
      float* si = c >= 2 ? im_buf(c - 2) : hi;
      float* di = c >= 1 ? im_buf(c - 1) : hi;
      cham_tc_colpass3<<<dim3(D / 64, b), WS_THREADS, CP3_SMEM, st>>>(
          mk, mv, m_ring64, si == hi ? m_hi64 : m_him64, m_ring64, di == hi ? m_hi64 : m_him64, rs * b, 0, rd * b, 0,
          w.cm + ((c + 1) & 1) * cm_half, w.cm + (c & 1) * cm_half, (const __nv_bfloat16*)q, w.T, w.E, w.bad, s, D,
          nch, c);
      if ((rc = check_launch("cham_tc_colpass3"))) return rc;
      if (c >= 1 && (c % w.nring == 0 || c == nch)) {
        const int cb = ((c - 1) / w.nring) * w.nring;
        cham_tc_readout_batch<<<dim3((D / R2) * (c - cb), b), WS_THREADS, RW2_SMEM, st>>>(
            mk, mv, mq, m_ring, m_ring, w.E, w.bad, (__nv_bfloat16*)out, s, D, nch, cb, w.nring, b, -1, nullptr);
        if ((rc = check_launch("cham_tc_readout_batch"))) return rc;
      }
    }
    VERACE_CUDA(cudaMemcpyAsync(hr, w.ring + ((nch - 1) % w.nring) * plane, plane * sizeof(float),
                                cudaMemcpyDeviceToDevice, st));
    return VERACE_OK;
  }
  if (sched == SCHED_BATCHED) {
    // Column passes two CTAs per SM over groups of RING chunks, the state in place in
    // hr / hi.  Chunk c's end state is copied into the ring by chunk c+1's column pass
    // (the last chunk's is hr), so group g's launch also runs the readouts of the chunks
    // group g-1 completed, in the SM slots its column pass leaves free; one readout
    // launch finishes the sequence.  The ring holds two groups, so the two never meet.
    // The ring slots hold the end states' real parts as the readout's bf16 operand images
    // (half the bytes of fp32), written by phase A.
    CUtensorMap mq, m_hr64, m_hi64, m_hr128, m_hi128;
    unsigned char* ring = reinterpret_cast<unsigned char*>(w.ring);
    if ((rc = make_kv_map(&mq, q, b, s, D)) ||
        (rc = make_state_map(&m_hr64, hr, b, D, KH)) || (rc = make_state_map(&m_hi64, hi, b, D, KH)) ||
        (rc = make_state_map(&m_hr128, hr, b, D)) || (rc = make_state_map(&m_hi128, hi, b, D)))
      return rc;
    VERACE_CUDA(cudaFuncSetAttribute(cham_tc_colpass2, cudaFuncAttributeMaxDynamicSharedMemorySize, CP2_SMEM));
    VERACE_CUDA(cudaFuncSetAttribute(cham_tc_readout_batch, cudaFuncAttributeMaxDynamicSharedMemorySize, RW2_SMEM));
    if (h0r != nullptr) {   // the planes are updated in place: start them as H0
      const size_t plane = (size_t)b * D * D * sizeof(float);
      VERACE_CUDA(cudaMemcpyAsync(hr, h0r, plane, cudaMemcpyDeviceToDevice, st));
      VERACE_CUDA(cudaMemcpyAsync(hi, h0i, plane, cudaMemcpyDeviceToDevice, st));
    }
    int r0 = 0;   // first chunk not read out yet
    for (int cb = 0; cb < nch; cb += RING) {
      const int ce = std::min(nch, cb + RING);
      const int nr = std::max(cb - 1, 0) - r0;   // chunks [r0, cb - 1) have their end states in the ring
      cham_tc_colpass2<<<(D / NB2) * b + (D / R2) * nr * b, CP2_THREADS, CP2_SMEM, st>>>(
          mk, mv, m_hr64, m_hi64, m_hr128, m_hi128, mq, ring, w.nring, b, (const __nv_bfloat16*)q, w.T, w.E, w.bad,
          (__nv_bfloat16*)out, s, D, nch, cb, ce, r0, nr, h0r != nullptr ? 1 : 0);
      if ((rc = check_launch("cham_tc_colpass2"))) return rc;
      r0 += nr;
    }
    // (chunks before the last read their pre-split ring images; the fp32 map serves the last)
    cham_tc_readout_batch<<<dim3((D / R2) * (nch - r0), b), WS_THREADS, RW2_SMEM, st>>>(
        mk, mv, mq, m_hr128, m_hr128, w.E, w.bad, (__nv_bfloat16*)out, s, D, nch, r0, w.nring, b, nch - 1, ring);
    if ((rc = check_launch("cham_tc_readout_batch"))) return rc;
    return VERACE_OK;
  }
  if (WS) {
    CUtensorMap mq, m_h0r, m_h0i;
    if ((rc = make_kv_map(&mq, q, b, s, D))) return rc;
    if (h0r != nullptr && ((rc = make_state_map(&m_h0r, h0r, b, D)) || (rc = make_state_map(&m_h0i, h0i, b, D))))
      return rc;
    VERACE_CUDA(cudaFuncSetAttribute(cham_tc_step_ws, cudaFuncAttributeMaxDynamicSharedMemorySize, WS_SMEM));
    for (int c = 0; c <= nch; ++c) {
      const bool to_out = ((nch - 1 - c) % 2) == 0;
      float* dr = to_out ? hr : w.Hre;
      float* di = to_out ? hi : w.Him;
      // state at the start of chunk c: identity (c == 0) or the buffer chunk c-1 wrote
      const bool src_out = c > 0 && ((nch - c) % 2) == 0;
      const int ncol = c < nch ? D / NB2 : 0;
      const int nread = c > 0 ? D / R2 : 0;
      const bool from_h0 = c == 0 && h0r != nullptr;   // chunk 0 reads the carried hologram
      cham_tc_step_ws<<<dim3(ncol + nread, b), WS_THREADS, WS_SMEM, st>>>(
          mk, mv, mq, from_h0 ? m_h0r : (src_out ? m_out_r : m_ping_r), from_h0 ? m_h0i : (src_out ? m_out_i : m_ping_i),
          to_out ? m_out_r : m_ping_r, to_out ? m_out_i : m_ping_i, (const __nv_bfloat16*)q, w.T,
          w.E, w.bad, (c == 0 && h0r == nullptr) ? 1 : 0, dr, di, (__nv_bfloat16*)out, s, D, nch, c, ncol);
      if ((rc = check_launch("cham_tc_step_ws"))) return rc;
    }
    return VERACE_OK;
  }
  if constexpr (!WS) {
    for (int c = 0; c < nch; ++c) {
      const bool to_out = ((nch - 1 - c) % 2) == 0;
      float* dr = to_out ? hr : w.Hre;
      float* di = to_out ? hi : w.Him;
      cham_tc_colpass<T><<<gc, THR, CPS, st>>>((const T*)q, (const T*)k, (const T*)v, w.T, w.E, w.bad, cur_r, cur_i,
                                               dr, di, s, D, nch, c);
      if ((rc = check_launch("cham_tc_colpass"))) return rc;
      cham_tc_readout<T><<<gr, THR, READOUT_SMEM, st>>>((const T*)q, (const T*)k, (const T*)v, w.E, w.bad, cur_r,
                                                        (T*)out, s, D, nch, c);
      if ((rc = check_launch("cham_tc_readout"))) return rc;
      cur_r = dr;
      cur_i = di;
    }
  }
  return VERACE_OK;
}

}  // namespace

// The tensor-core scan reads out Re(H_t q_t): the exact Newton-Schulz readout for a fresh
// hologram, and for a carried one only where the caller has established that H0 is unitary
// (verace_cham_scan_unitary).  Exact readouts of a carried hologram take the SIMT path.
bool cham_tc_supported(int D, int dtype, bool has_h0) {
  return !has_h0 && D >= 128 && D % 128 == 0 && (dtype == VERACE_BF16 || dtype == VERACE_F32);
}
bool cham_tc_supported_unitary(int D, int dtype) {
  return D >= 128 && D % 128 == 0 && (dtype == VERACE_BF16 || dtype == VERACE_F32);
}

size_t cham_tc_workspace(int b, int s, int D) { return tc_ws_layout(b, s, D, nullptr, nullptr); }

int cham_tc_scan(const void* q, const void* k, const void* v, const float* gamma, const float* h0r,
                 const float* h0i, void* out, float* hr, float* hi, int b, int s, int D, int dtype, void* workspace,
                 cudaStream_t st) {
  TcWs w;
  char* base = (char*)align_up((size_t)workspace, 256);
  tc_ws_layout(b, s, D, &w, base);
  if (dtype == VERACE_BF16)
    return launch_cham_tc<__nv_bfloat16>(q, k, v, gamma, h0r, h0i, out, hr, hi, b, s, D, w, st);
  return launch_cham_tc<float>(q, k, v, gamma, h0r, h0i, out, hr, hi, b, s, D, w, st);
}

int tc_read_status(cudaStream_t st, int* status) {
  int h = 0;
  VERACE_CUDA(cudaMemcpyFromSymbolAsync(&h, g_tc_status, sizeof(int), 0, cudaMemcpyDeviceToHost, st));
  VERACE_CUDA(cudaStreamSynchronize(st));
  if (h) {
    const int zero = 0;
    VERACE_CUDA(cudaMemcpyToSymbolAsync(g_tc_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice, st));
    VERACE_CUDA(cudaStreamSynchronize(st));
  }
  *status = h;
  return VERACE_OK;
}

}  // namespace verace
