// SSSD scan on the tcgen05 tensor cores (sm_100a) for head_dim 128: one CTA per
// (batch, head) chain with the 128x128 fp32 state resident in tensor memory for the
// whole sequence.
//
// Same chunked compact-WY recurrence as sssd_scan.cu (derivation there), with chunks of
// C = 64 tokens (chunk rank 128 = one tensor-core tile).  Per chunk, starting from S:
//     Z = Wᵀ S,  Y = S Q,  Cm = T Z,  E = mask(Cm Q),  S += W Cm,  O = Y + W E
// Every product runs as tcgen05.mma (kind::f16) with fp32 accumulation in TMEM; fp32
// operands (the state, Z, Cm, E, T, and fp32 inputs) enter as bf16 hi + lo pairs and
// products take hi*hi + hi*lo + lo*hi.  The state update accumulates straight into
// the TMEM copy of S, which is read back to global memory only after the last chunk.
// T for every chunk comes from sssd_tc_prep (all chunks in parallel, fp32 SIMT).
#include <mutex>

#include "common.cuh"
#include "tc.cuh"
#include "tmap.cuh"
#include "wy_solve.cuh"

namespace verace {
namespace {

constexpr int C3 = 64;     // tokens per chunk
constexpr int R3 = 128;    // chunk rank
constexpr int HD = 128;    // head_dim handled by this path
constexpr int THR3 = 256;
constexpr uint32_t POLLS3 = 1u << 22;
constexpr int TILE3 = 128 * 128 * 2;  // 32 KB bf16 128 x 128

__device__ int g_sssd_tc_status = 0;

__device__ __forceinline__ int kmaj3(int r, int k, int R) { return ((k >> 3) * R + r) * 16 + (k & 7) * 2; }
// 128 x 128 "X" layout: element (i, j) at (j/8)*2048 + (i/8)*128 + (i%8)*16 + (j%8)*2
//   K-major view (rows i, k = j): SBO 128, LBO 2048, K step of 16 -> +4096
//   MN-major view (n = j, k = i): SBO 2048, LBO 128, K step of 16 -> +256
__device__ __forceinline__ int xoff(int i, int j) { return kmaj3(i, j, 128); }
__device__ __forceinline__ int mnmaj3(int k, int n, int NG) { return (((k >> 3) * NG + (n >> 3)) * 128) + (k & 7) * 16 + (n & 7) * 2; }
// Row orders of a chunk's 128 vectors: interleaved (row 2t + kv: the solver's, and the
// fp32 scan's) and split (row t for k_t, 64 + t for v_t: the bf16 scan's, whose W tiles
// arrive as one TMA box of k rows and one of v rows).  ilv3 maps split -> interleaved.
__device__ __forceinline__ int ilv3(int r) { return 2 * (r & (C3 - 1)) + (r >> 6); }

template <typename T>
__device__ __forceinline__ void stage8_3(const T* src, bool valid, unsigned char* hi, unsigned char* lo) {
  if (sizeof(T) == 2) {
    uint4 u = make_uint4(0, 0, 0, 0);
    if (valid) u = *reinterpret_cast<const uint4*>(src);
    *reinterpret_cast<uint4*>(hi) = u;
  } else {
    float x[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (valid) {
      const float4 a = *reinterpret_cast<const float4*>(src);
      const float4 b = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(src) + 4);
      x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
    }
    uint4 h, l;
    tc::split8(x, h, l);
    *reinterpret_cast<uint4*>(hi) = h;
    *reinterpret_cast<uint4*>(lo) = l;
  }
}

// ---------------------------------------------------------------------------------
// prep: Gram, M_t, T (fp32 SIMT), T written as bf16 hi/lo K-major 128x128 tiles (split
// row order for bf16 inputs, interleaved for fp32).
// smem: [Ws [128][129] fp32, fp32 inputs only] | Gs [128][132] (row pitch a multiple of 4:
// the solver reads G rows as float4), overwritten in place by T.  For bf16 inputs the bf16
// W tile (32 KB) sits in the front of Gs: the Gram product has completed (its commit
// barrier) before G is read out of TMEM into Gs, so 68 KB suffice and three CTAs share an
// SM.
template <typename T>
constexpr int prep_ctas() { return sizeof(T) == 2 ? 3 : 1; }

template <typename T>
__global__ void __launch_bounds__(THR3, prep_ctas<T>())
sssd_tc_prep(const T* __restrict__ k, const T* __restrict__ v, const float* __restrict__ delta,
             unsigned char* __restrict__ Tws, unsigned long long* __restrict__ badws, int S, int H, int nch,
             int c_base) {
  extern __shared__ __align__(16) float sm3[];
  constexpr int PW = R3 + 1, P = 132;
  constexpr bool BF = sizeof(T) == 2;   // bf16 inputs: G on the tensor cores (W is exact in bf16)
  float* Ws = sm3;
  float* Gs = BF ? sm3 : Ws + HD * PW;
  float* Ts = Gs;
  __shared__ float Ms[C3 * 8];   // per token [[m00, m01], [m10, m11]] as complex with zero imaginary parts
  __shared__ unsigned long long bad_bits;
  __shared__ __align__(8) uint64_t gbar;
  __shared__ uint32_t gslot;
  const int c = c_base + blockIdx.x, chain = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int bi = chain / H, hi = chain % H;
  const int t0 = c * C3, nt = min(C3, S - t0);
  if (BF && warp == 0) tc::tmem_alloc(&gslot, 128);
  if (tid == 0) {
    bad_bits = 0ull;
    if (BF) { tc::mbar_init(&gbar, 1); tc::fence_mbar_init(); }
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if constexpr (BF) {
    // W as a bf16 K-major tile (rows r = 2*tau + {k, v}) in the front of Ws
    unsigned char* Wb = reinterpret_cast<unsigned char*>(Ws);
    constexpr int PER = (R3 * (HD / 8)) / THR3;
    uint4 raw[PER];
#pragma unroll
    for (int u = 0; u < PER; ++u) {
      const int e = tid + THR3 * u, r = e % R3, g = e / R3, tau = r >> 1;
      raw[u] = make_uint4(0, 0, 0, 0);
      if (tau < nt)
        raw[u] = *reinterpret_cast<const uint4*>(((r & 1) ? v : k) +
                                                 ((size_t)(bi * (size_t)S + t0 + tau) * H + hi) * HD + g * 8);
    }
#pragma unroll
    for (int u = 0; u < PER; ++u) {
      const int e = tid + THR3 * u, r = e % R3, g = e / R3;
      const __nv_bfloat16* hb = reinterpret_cast<const __nv_bfloat16*>(&raw[u]);
      bool fin = true;
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) fin = fin && isfinite(__bfloat162float(hb[jj]));
      if (!fin) atomicOr(&bad_bits, 1ull << (r >> 1));
      *reinterpret_cast<uint4*>(Wb + kmaj3(r, g * 8, R3)) = raw[u];
    }
    __syncthreads();
    if (tid < C3 && tid < nt && !isfinite(delta[(size_t)(bi * (size_t)S + t0 + tid) * H + hi]))
      atomicOr(&bad_bits, 1ull << tid);
    __syncthreads();
    if (bad_bits) {
      for (int e = tid; e < R3 * (HD / 8); e += THR3) {
        const int r = e % R3, g = e / R3;
        if ((bad_bits >> (r >> 1)) & 1ull) *reinterpret_cast<uint4*>(Wb + kmaj3(r, g * 8, R3)) = make_uint4(0, 0, 0, 0);
      }
    }
    tc::fence_proxy_async();
    __syncthreads();
    const uint32_t tG = gslot;
    if (tid == 0) {
      tc::fence_after_sync();
      constexpr uint32_t ID_G = tc::idesc_bf16(128, 128, false, false);
      const uint32_t w = tc::smem_addr(Wb);
#pragma unroll 1
      for (int ks = 0; ks < HD / 16; ++ks) {
        const uint64_t d = tc::sdesc(w + ks * 4096, 2048, 128);
        tc::mma_bf16(tG, d, d, ID_G, ks > 0 ? 1u : 0u);
      }
      tc::commit(&gbar);
    }
    const bool ok = tc::mbar_wait(&gbar, 0, POLLS3);
    if (__syncthreads_or(!ok)) {
      if (tid == 0) atomicExch(&g_sssd_tc_status, 1);
    } else {
      tc::fence_after_sync();
      const uint32_t lb = (uint32_t)(32 * (warp & 3)) << 16;
      const int row = 32 * (warp & 3) + lane, half = warp >> 2;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        float x[16];
        tc::tmem_ld16(tG + lb + 64 * half + 16 * u, x);
#pragma unroll
        for (int jj = 0; jj < 16; jj += 4)
          *reinterpret_cast<float4*>(Gs + row * P + 64 * half + 16 * u + jj) =
              make_float4(x[jj], x[jj + 1], x[jj + 2], x[jj + 3]);
      }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) tc::tmem_dealloc(tG, 128);
  } else {
    // W^T into Ws[i][r]: each thread takes 8 (vector r, 8 consecutive elements) chunks;
    // all global loads are issued before any use so their latencies overlap
    constexpr int PER = (R3 * (HD / 8)) / THR3;
    float x[PER][8];
#pragma unroll
    for (int u = 0; u < PER; ++u) {
      const int e = tid + THR3 * u, r = e % R3, g = e / R3, tau = r >> 1;
      if (tau < nt) {
        const T* src = ((r & 1) ? v : k) + ((size_t)(bi * (size_t)S + t0 + tau) * H + hi) * HD + g * 8;
        if (sizeof(T) == 2) {
          const uint4 w = *reinterpret_cast<const uint4*>(src);
          const __nv_bfloat16* hb = reinterpret_cast<const __nv_bfloat16*>(&w);
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) x[u][jj] = __bfloat162float(hb[jj]);
        } else {
          const float4 a = *reinterpret_cast<const float4*>(src);
          const float4 b = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(src) + 4);
          x[u][0] = a.x; x[u][1] = a.y; x[u][2] = a.z; x[u][3] = a.w;
          x[u][4] = b.x; x[u][5] = b.y; x[u][6] = b.z; x[u][7] = b.w;
        }
      } else {
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) x[u][jj] = 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < PER; ++u) {
      const int e = tid + THR3 * u, r = e % R3, g = e / R3;
      bool fin = true;
#pragma unroll
      for (int jj = 0; jj < 8; ++jj) {
        Ws[(g * 8 + jj) * PW + r] = x[u][jj];
        fin = fin && isfinite(x[u][jj]);
      }
      if (!fin) atomicOr(&bad_bits, 1ull << (r >> 1));
    }
  __syncthreads();
  if (tid < C3 && tid < nt && !isfinite(delta[(size_t)(bi * (size_t)S + t0 + tid) * H + hi]))
    atomicOr(&bad_bits, 1ull << tid);
  __syncthreads();
  if (bad_bits) {
    for (int e = tid; e < HD * R3; e += THR3)
      if ((bad_bits >> ((e % R3) >> 1)) & 1ull) Ws[(e / R3) * PW + e % R3] = 0.f;
    __syncthreads();
  }
  smem_gemm<4, 4, false>(R3, R3, HD, Ws, 1, PW, Ws, PW, 1, Gs, P, 1, tid, THR3);
  __syncthreads();
  }
  if (tid < C3) {
    const int tau = tid;
    float m00 = 0.f, m01 = 0.f, m10 = 0.f, m11 = 0.f;
    bool flagged = (bad_bits >> tau) & 1ull;
    if (tau < nt && !flagged) {
      const float kk = Gs[(2 * tau) * P + 2 * tau];
      const float vv = Gs[(2 * tau + 1) * P + 2 * tau + 1];
      const float kv = Gs[(2 * tau) * P + 2 * tau + 1];
      const float a = 0.5f * delta[(size_t)(bi * (size_t)S + t0 + tau) * H + hi];
      const float det = 1.f + a * a * (kk * vv - kv * kv);
      const float f = -2.f * a / det;
      m00 = f * (a * vv); m01 = f * (1.f - a * kv);
      m10 = f * (-1.f - a * kv); m11 = f * (a * kk);
      if (!(isfinite(kk) && isfinite(vv) && isfinite(kv) && isfinite(m00) && isfinite(m01) &&
            isfinite(m10) && isfinite(m11))) {
        m00 = m01 = m10 = m11 = 0.f;
        atomicOr(&bad_bits, 1ull << tau);
        flagged = true;
      }
    }
    if (flagged) {
      for (int r = 0; r < R3; ++r) {
        Gs[(2 * tau) * P + r] = 0.f; Gs[(2 * tau + 1) * P + r] = 0.f;
        Gs[r * P + 2 * tau] = 0.f; Gs[r * P + 2 * tau + 1] = 0.f;
      }
    }
    float* n = Ms + tau * 8;
    n[0] = m00; n[1] = 0.f; n[2] = m01; n[3] = 0.f; n[4] = m10; n[5] = 0.f; n[6] = m11; n[7] = 0.f;
  }
  __syncthreads();
  wy_solve<false>(Gs, P, Ms, Ts, nullptr, tid);   // T overwrites G
  const size_t chunk = (size_t)chain * nch + c;
  unsigned char* To = Tws + chunk * 2 * TILE3;
  for (int e = tid; e < R3 * (R3 / 8); e += THR3) {
    const int r = e % R3, g = e / R3;
    float x[8];
    if constexpr (BF) {
      // the bf16 scan's split row order: element (r, c) is the solver's (ilv3(r), ilv3(c))
      const float* src = Ts + ilv3(r) * P + ilv3(g * 8);
#pragma unroll
      for (int j = 0; j < 8; ++j) x[j] = src[2 * j];
    } else {
      const float4 a = *reinterpret_cast<const float4*>(Ts + r * P + g * 8);
      const float4 b = *reinterpret_cast<const float4*>(Ts + r * P + g * 8 + 4);
      x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w; x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
    }
    uint4 h, l;
    tc::split8(x, h, l);
    *reinterpret_cast<uint4*>(To + kmaj3(r, g * 8, R3)) = h;
    *reinterpret_cast<uint4*>(To + TILE3 + kmaj3(r, g * 8, R3)) = l;
  }
  if (tid == 0) badws[chunk] = bad_bits;
}

// ---------------------------------------------------------------------------------
// scan.  smem (bytes): W hi [0,32K) | W lo [32K,64K) | Q hi [64K,80K) | Q lo [80K,96K) |
//   T hi/lo [96K,160K) (later: E as an MN-major B operand, hi/lo 2 x 16K) |
//   X hi/lo [160K,224K): S, then Z, then Cm, as bf16 pairs in the "X" layout | bar
// TMEM columns: S [0,128) Z [128,256) Cm [256,384) Y/O [384,448) E [448,512)
constexpr int X_W = 0, X_WL = 32 * 1024, X_Q = 64 * 1024, X_QL = 80 * 1024, X_T = 96 * 1024;
constexpr int X_X = 160 * 1024, X_BAR = 224 * 1024;
constexpr int SSSD_TC_SMEM = X_BAR + 64;

template <typename T>
__global__ void __launch_bounds__(THR3, 1)
sssd_tc_scan(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
             const float* __restrict__ psi0, T* __restrict__ out, float* __restrict__ psi_out,
             const unsigned char* __restrict__ Tws, const unsigned long long* __restrict__ badws,
             int S, int H, int nch) {
  extern __shared__ __align__(1024) unsigned char sx[];
  constexpr bool F32IN = sizeof(T) == 4;
  unsigned char* sW = sx + X_W;
  unsigned char* sWl = sx + X_WL;
  unsigned char* sQ = sx + X_Q;
  unsigned char* sQl = sx + X_QL;
  unsigned char* sT = sx + X_T;
  unsigned char* sEh = sx + X_T;
  unsigned char* sEl = sx + X_T + 16 * 1024;
  unsigned char* sXh = sx + X_X;
  unsigned char* sXl = sx + X_X + TILE3;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sx + X_BAR);
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sx + X_BAR + 16);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int chain = blockIdx.x, bi = chain / H, hi = chain % H;
  if (warp == 0) tc::tmem_alloc(tslot, 512);
  if (tid == 0) { tc::mbar_init(bar, 1); tc::fence_mbar_init(); }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tb = *tslot;
  const uint32_t tS = tb, tZ = tb + 128, tC = tb + 256, tO = tb + 384, tE = tb + 448;
  const uint32_t lb = (uint32_t)(32 * (warp & 3)) << 16;
  const int row = 32 * (warp & 3) + lane, half = warp >> 2;
  uint32_t phase = 0;
  bool failed = false;
  auto wait_mma = [&]() -> bool {
    const bool ok = tc::mbar_wait(bar, phase, POLLS3);
    phase ^= 1u;
    if (__syncthreads_or(!ok)) { if (tid == 0) atomicExch(&g_sssd_tc_status, 1); return false; }
    tc::fence_after_sync();
    return true;
  };
  // this thread's 64 columns [64*half, 64*half+64) of a 128-column TMEM matrix -> X layout
  auto tmem_to_x = [&](uint32_t tm) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float x[16];
      tc::tmem_ld16(tm + lb + 64 * half + 16 * u, x);
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        uint4 h, l;
        tc::split8(x + 8 * g, h, l);
        const int off = xoff(row, 64 * half + 16 * u + 8 * g);
        *reinterpret_cast<uint4*>(sXh + off) = h;
        *reinterpret_cast<uint4*>(sXl + off) = l;
      }
    }
  };

  {  // initial state into TMEM
    const float* p0 = psi0 ? psi0 + (size_t)chain * HD * HD + (size_t)row * HD : nullptr;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float x[16];
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) {
        const int j = 64 * half + 16 * u + jj;
        x[jj] = p0 ? p0[j] : (row == j ? 1.f : 0.f);
      }
      tc::tmem_st16(tS + lb + 64 * half + 16 * u, x);
    }
  }

  constexpr uint32_t ID_Z = tc::idesc_bf16(128, 128, false, true);
  constexpr uint32_t ID_Y = tc::idesc_bf16(128, 64, false, false);
  constexpr uint32_t ID_C = tc::idesc_bf16(128, 128, false, true);
  constexpr uint32_t ID_E = tc::idesc_bf16(128, 64, false, false);
  constexpr uint32_t ID_S = tc::idesc_bf16(128, 128, true, true);
  constexpr uint32_t ID_O = tc::idesc_bf16(128, 64, true, true);

  for (int c = 0; c < nch && !failed; ++c) {
    const int t0 = c * C3, nt = min(C3, S - t0);
    const size_t chunk = (size_t)chain * nch + c;
    const unsigned long long bad = badws[chunk];
    // ---- stage W (rows = vector r), Q (rows = token t), T (hi | lo)
    for (int e = tid; e < R3 * (HD / 8); e += THR3) {
      const int r = e % R3, g = e / R3, tau = r >> 1;
      const bool valid = tau < nt && !((bad >> tau) & 1ull);
      const T* src = ((r & 1) ? v : k) + ((size_t)(bi * (size_t)S + t0 + (valid ? tau : 0)) * H + hi) * HD + g * 8;
      stage8_3(src, valid, sW + kmaj3(r, g * 8, R3), sWl + kmaj3(r, g * 8, R3));
    }
    for (int e = tid; e < C3 * (HD / 8); e += THR3) {
      const int t = e % C3, g = e / C3;
      const bool valid = t < nt;
      const T* src = q + ((size_t)(bi * (size_t)S + t0 + (valid ? t : 0)) * H + hi) * HD + g * 8;
      stage8_3(src, valid, sQ + kmaj3(t, g * 8, C3), sQl + kmaj3(t, g * 8, C3));
    }
    {
      const uint4* Tin = reinterpret_cast<const uint4*>(Tws + chunk * 2 * TILE3);
      for (int e = tid; e < 2 * TILE3 / 16; e += THR3) reinterpret_cast<uint4*>(sT)[e] = Tin[e];
    }
    tmem_to_x(tS);
    tc::fence_proxy_async();
    tc::fence_before_sync();
    __syncthreads();
    // ---- Z = Wᵀ S  and  Y = S Q
    if (tid == 0) {
      tc::fence_after_sync();
      const uint32_t w = tc::smem_addr(sW), wl = tc::smem_addr(sWl);
      const uint32_t xh = tc::smem_addr(sXh), xl = tc::smem_addr(sXl);
      const uint32_t qh = tc::smem_addr(sQ), ql = tc::smem_addr(sQl);
#pragma unroll 1
      for (int ks = 0; ks < 8; ++ks) {
        const uint64_t a_w = tc::sdesc(w + ks * 4096, 2048, 128);
        const uint64_t b_sh = tc::sdesc(xh + ks * 256, 128, 2048);
        const uint64_t b_sl = tc::sdesc(xl + ks * 256, 128, 2048);
        tc::mma_bf16(tZ, a_w, b_sh, ID_Z, ks > 0 ? 1u : 0u);
        tc::mma_bf16(tZ, a_w, b_sl, ID_Z, 1u);
        if (F32IN) tc::mma_bf16(tZ, tc::sdesc(wl + ks * 4096, 2048, 128), b_sh, ID_Z, 1u);
        const uint64_t a_sh = tc::sdesc(xh + ks * 4096, 2048, 128);
        const uint64_t a_sl = tc::sdesc(xl + ks * 4096, 2048, 128);
        const uint64_t b_q = tc::sdesc(qh + ks * 2048, 1024, 128);
        tc::mma_bf16(tO, a_sh, b_q, ID_Y, ks > 0 ? 1u : 0u);
        tc::mma_bf16(tO, a_sl, b_q, ID_Y, 1u);
        if (F32IN) tc::mma_bf16(tO, a_sh, tc::sdesc(ql + ks * 2048, 1024, 128), ID_Y, 1u);
      }
      tc::commit(bar);
    }
    if (!(failed = !wait_mma())) {
      // ---- Cm = T Z
      tmem_to_x(tZ);
      tc::fence_proxy_async();
      tc::fence_before_sync();
      __syncthreads();
      if (tid == 0) {
        tc::fence_after_sync();
        const uint32_t th = tc::smem_addr(sT), tl = th + TILE3;
        const uint32_t xh = tc::smem_addr(sXh), xl = tc::smem_addr(sXl);
#pragma unroll 1
        for (int ks = 0; ks < 8; ++ks) {
          const uint64_t ah = tc::sdesc(th + ks * 4096, 2048, 128);
          const uint64_t al = tc::sdesc(tl + ks * 4096, 2048, 128);
          const uint64_t bh = tc::sdesc(xh + ks * 256, 128, 2048);
          const uint64_t bl = tc::sdesc(xl + ks * 256, 128, 2048);
          tc::mma_bf16(tC, ah, bh, ID_C, ks > 0 ? 1u : 0u);
          tc::mma_bf16(tC, ah, bl, ID_C, 1u);
          tc::mma_bf16(tC, al, bh, ID_C, 1u);
        }
        tc::commit(bar);
      }
      failed = !wait_mma();
    }
    if (!failed) {
      // ---- E = Cm Q ; S += W Cm
      tmem_to_x(tC);
      tc::fence_proxy_async();
      tc::fence_before_sync();
      __syncthreads();
      if (tid == 0) {
        tc::fence_after_sync();
        const uint32_t w = tc::smem_addr(sW), wl = tc::smem_addr(sWl);
        const uint32_t xh = tc::smem_addr(sXh), xl = tc::smem_addr(sXl);
        const uint32_t qh = tc::smem_addr(sQ), ql = tc::smem_addr(sQl);
#pragma unroll 1
        for (int ks = 0; ks < 8; ++ks) {
          const uint64_t a_ch = tc::sdesc(xh + ks * 4096, 2048, 128);
          const uint64_t a_cl = tc::sdesc(xl + ks * 4096, 2048, 128);
          const uint64_t b_q = tc::sdesc(qh + ks * 2048, 1024, 128);
          tc::mma_bf16(tE, a_ch, b_q, ID_E, ks > 0 ? 1u : 0u);
          tc::mma_bf16(tE, a_cl, b_q, ID_E, 1u);
          if (F32IN) tc::mma_bf16(tE, a_ch, tc::sdesc(ql + ks * 2048, 1024, 128), ID_E, 1u);
          const uint64_t a_w = tc::sdesc(w + ks * 256, 128, 2048);
          const uint64_t b_ch = tc::sdesc(xh + ks * 256, 128, 2048);
          const uint64_t b_cl = tc::sdesc(xl + ks * 256, 128, 2048);
          tc::mma_bf16(tS, a_w, b_ch, ID_S, 1u);
          tc::mma_bf16(tS, a_w, b_cl, ID_S, 1u);
          if (F32IN) tc::mma_bf16(tS, tc::sdesc(wl + ks * 256, 128, 2048), b_ch, ID_S, 1u);
        }
        tc::commit(bar);
      }
      failed = !wait_mma();
    }
    if (!failed) {
      // ---- O = Y + W mask(E)
      {
        float e[32];
        tc::tmem_ld16(tE + lb + 32 * half, e);
        tc::tmem_ld16(tE + lb + 32 * half + 16, e + 16);
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          float x[8];
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
            const int t = 32 * half + 8 * g + jj;
            x[jj] = ((row >> 1) <= t) ? e[8 * g + jj] : 0.f;
          }
          uint4 h, l;
          tc::split8(x, h, l);
          const int off = mnmaj3(row, 32 * half + 8 * g, C3 / 8);
          *reinterpret_cast<uint4*>(sEh + off) = h;
          *reinterpret_cast<uint4*>(sEl + off) = l;
        }
      }
      tc::fence_proxy_async();
      tc::fence_before_sync();
      __syncthreads();
      if (tid == 0) {
        tc::fence_after_sync();
        const uint32_t w = tc::smem_addr(sW), wl = tc::smem_addr(sWl);
        const uint32_t eh = tc::smem_addr(sEh), el = tc::smem_addr(sEl);
#pragma unroll 1
        for (int ks = 0; ks < 8; ++ks) {
          const uint64_t a_w = tc::sdesc(w + ks * 256, 128, 2048);
          const uint64_t b_eh = tc::sdesc(eh + ks * 2048, 1024, 128);
          const uint64_t b_el = tc::sdesc(el + ks * 2048, 1024, 128);
          tc::mma_bf16(tO, a_w, b_eh, ID_O, 1u);
          tc::mma_bf16(tO, a_w, b_el, ID_O, 1u);
          if (F32IN) tc::mma_bf16(tO, tc::sdesc(wl + ks * 256, 128, 2048), b_eh, ID_O, 1u);
        }
        tc::commit(bar);
      }
      failed = !wait_mma();
    }
    if (!failed) {
      float o[32];
      tc::tmem_ld16(tO + lb + 32 * half, o);
      tc::tmem_ld16(tO + lb + 32 * half + 16, o + 16);
#pragma unroll 4
      for (int u = 0; u < 32; ++u) {
        const int t = 32 * half + u;
        if (t < nt) out[((size_t)(bi * (size_t)S + t0 + t) * H + hi) * HD + row] = from_f32<T>(o[u]);
      }
      tc::fence_before_sync();
      __syncthreads();
    }
  }
  if (!failed) {
    float* po = psi_out + (size_t)chain * HD * HD + (size_t)row * HD;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float x[16];
      tc::tmem_ld16(tS + lb + 64 * half + 16 * u, x);
#pragma unroll
      for (int jj = 0; jj < 16; jj += 4)
        *reinterpret_cast<float4*>(po + 64 * half + 16 * u + jj) = make_float4(x[jj], x[jj + 1], x[jj + 2], x[jj + 3]);
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tb, 512);
}

// ---------------------------------------------------------------------------------
// scan for bf16 inputs, chunk inputs prefetched: W (k rows | v rows) and Q of chunk c + 1
// arrive by TMA in a second buffer while chunk c runs, and T of chunk c + 1 by one bulk
// copy as soon as chunk c's Cm product has read T(c).  Rows in the split order; same
// products as sssd_tc_scan.
// smem (bytes): W[2] [0, 64K), 128B-swizzled K-major (per 64-element K block 128 rows x
//   128 B; rows 0-63 k, 64-127 v) | Q[2] [64K, 96K) (per K block 64 token rows x 128 B) |
//   T hi/lo [96K, 160K) | X hi/lo [160K, 224K): S, Z, Cm as bf16 pairs in the "X" layout,
//   then E (MN-major hi/lo) | barriers.  O leaves through the chunk's W slot (free once
//   the O product is done) as [64 tokens][128] bf16 rows, for 16-byte coalesced stores.
constexpr int Y_W = 0, Y_Q = 64 * 1024, Y_T = 96 * 1024, Y_X = 160 * 1024, Y_BAR = 224 * 1024;
constexpr int SSSD_TC2_SMEM = Y_BAR + 64;
constexpr int Q_TILE = 64 * 128 * 2;   // 16 KB bf16 64 x 128

__global__ void __launch_bounds__(THR3, 1)
sssd_tc_scan_bf16(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                  const __grid_constant__ CUtensorMap tm_v, const float* __restrict__ psi0,
                  __nv_bfloat16* __restrict__ out, float* __restrict__ psi_out,
                  const unsigned char* __restrict__ Tws, const unsigned long long* __restrict__ badws,
                  int S, int H, int nch, int c_begin, int c_end) {
  extern __shared__ __align__(1024) unsigned char sx[];
  auto sW = [&](int s) { return sx + Y_W + s * TILE3; };
  auto sQ = [&](int s) { return sx + Y_Q + s * Q_TILE; };
  unsigned char* sT = sx + Y_T;
  unsigned char* sXh = sx + Y_X;
  unsigned char* sXl = sx + Y_X + TILE3;
  unsigned char* sEh = sx + Y_X;
  unsigned char* sEl = sx + Y_X + 16 * 1024;
  uint64_t* bar = reinterpret_cast<uint64_t*>(sx + Y_BAR);   // [0] MMA, [1 + s] W/Q slot s, [3] T
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sx + Y_BAR + 32);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int chain = blockIdx.x, bi = chain / H, hi = chain % H;
  if (warp == 0) tc::tmem_alloc(tslot, 512);
  if (tid == 0) {
    for (int i = 0; i < 4; ++i) tc::mbar_init(&bar[i], 1);
    tc::fence_mbar_init();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tb = *tslot;
  const uint32_t tS = tb, tZ = tb + 128, tC = tb + 256, tO = tb + 384, tE = tb + 448;
  const uint32_t lb = (uint32_t)(32 * (warp & 3)) << 16;
  const int row = 32 * (warp & 3) + lane, half = warp >> 2;

  // The launch runs chunks [c_begin, c_end) (the state enters as psi0 and leaves as
  // psi_out); j below counts chunks from c_begin, which sets the slots and barrier phases.
  // chunk j's W and Q into slot j & 1; chunk j's T into the T buffer (thread 0)
  const int ncl = c_end - c_begin;
  auto issue_wq = [&](int j) {
    const int s = j & 1, cg = c_begin + j;
    tc::mbar_expect_tx(&bar[1 + s], TILE3 + Q_TILE);
#pragma unroll
    for (int kb = 0; kb < 2; ++kb) {
      tc::tma_load_4d(sW(s) + kb * 16384, &tm_k, 64 * kb, hi, cg * C3, bi, &bar[1 + s]);
      tc::tma_load_4d(sW(s) + kb * 16384 + 8192, &tm_v, 64 * kb, hi, cg * C3, bi, &bar[1 + s]);
      tc::tma_load_4d(sQ(s) + kb * 8192, &tm_q, 64 * kb, hi, cg * C3, bi, &bar[1 + s]);
    }
  };
  auto issue_t = [&](int j) {
    tc::mbar_expect_tx(&bar[3], 2 * TILE3);
    tc::bulk_load(sT, Tws + ((size_t)chain * nch + c_begin + j) * 2 * TILE3, 2 * TILE3, &bar[3]);
  };
  int wq_issued = min(ncl, 2), wq_done = 0, t_issued = ncl > 0 ? 1 : 0, t_done = 0;
  if (tid == 0 && ncl > 0) {
    issue_wq(0);
    if (ncl > 1) issue_wq(1);
    issue_t(0);
  }

  uint32_t phase = 0;
  bool failed = false;
  auto wait_all = [&](uint64_t* b, uint32_t parity) -> bool {
    const bool ok = tc::mbar_wait(b, parity, POLLS3);
    if (__syncthreads_or(!ok)) {
      if (tid == 0) atomicExch(&g_sssd_tc_status, 1);
      return false;
    }
    tc::fence_after_sync();
    return true;
  };
  auto wait_mma = [&]() -> bool {
    const bool ok = wait_all(&bar[0], phase);
    phase ^= 1u;
    return ok;
  };
  // this thread's 64 columns [64*half, 64*half+64) of a 128-column TMEM matrix -> X layout
  auto tmem_to_x = [&](uint32_t tm) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float x[16];
      tc::tmem_ld16(tm + lb + 64 * half + 16 * u, x);
#pragma unroll
      for (int g = 0; g < 2; ++g) {
        uint4 h, l;
        tc::split8(x + 8 * g, h, l);
        const int off = xoff(row, 64 * half + 16 * u + 8 * g);
        *reinterpret_cast<uint4*>(sXh + off) = h;
        *reinterpret_cast<uint4*>(sXl + off) = l;
      }
    }
  };
  auto sync_for_mma = [&]() {
    tc::fence_proxy_async();
    tc::fence_before_sync();
    __syncthreads();
  };

  {  // initial state into TMEM
    const float* p0 = psi0 ? psi0 + (size_t)chain * HD * HD + (size_t)row * HD : nullptr;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float x[16];
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) {
        const int j = 64 * half + 16 * u + jj;
        x[jj] = p0 ? p0[j] : (row == j ? 1.f : 0.f);
      }
      tc::tmem_st16(tS + lb + 64 * half + 16 * u, x);
    }
  }

  constexpr uint32_t ID_Z = tc::idesc_bf16(128, 128, false, true);
  constexpr uint32_t ID_Y = tc::idesc_bf16(128, 64, false, false);
  constexpr uint32_t ID_C = tc::idesc_bf16(128, 128, false, true);
  constexpr uint32_t ID_S = tc::idesc_bf16(128, 128, true, true);
  constexpr uint32_t ID_O = tc::idesc_bf16(128, 64, true, true);

  for (int j = 0; j < ncl; ++j) {
    const int c = c_begin + j;
    const int s = j & 1, t0 = c * C3, nt = min(C3, S - t0);
    const unsigned long long bad = badws[(size_t)chain * nch + c];
    tmem_to_x(tS);
    if (!wait_all(&bar[1 + s], (j >> 1) & 1)) { failed = true; break; }
    wq_done = j + 1;
    if (bad) {   // zero the k and v rows of non-finite tokens (both K blocks)
      for (int e = tid; e < C3 * 32; e += THR3) {
        const int tau = e >> 5, kv = (e >> 4) & 1, kb = (e >> 3) & 1, ch = e & 7;
        if ((bad >> tau) & 1ull)
          *reinterpret_cast<uint4*>(sW(s) + kb * 16384 + (kv * C3 + tau) * 128 + ch * 16) = make_uint4(0, 0, 0, 0);
      }
    }
    sync_for_mma();
    // ---- Z = Wᵀ S  and  Y = S Q
    if (tid == 0) {
      tc::fence_after_sync();
      const uint32_t w = tc::smem_addr(sW(s)), q = tc::smem_addr(sQ(s));
      const uint32_t xh = tc::smem_addr(sXh), xl = tc::smem_addr(sXl);
#pragma unroll 1
      for (int ks = 0; ks < 8; ++ks) {
        const uint64_t a_w = tc::sdesc_sw128(w + (ks >> 2) * 16384 + (ks & 3) * 32, 16, 1024);
        tc::mma_bf16(tZ, a_w, tc::sdesc(xh + ks * 256, 128, 2048), ID_Z, ks > 0 ? 1u : 0u);
        tc::mma_bf16(tZ, a_w, tc::sdesc(xl + ks * 256, 128, 2048), ID_Z, 1u);
        const uint64_t b_q = tc::sdesc_sw128(q + (ks >> 2) * 8192 + (ks & 3) * 32, 16, 1024);
        tc::mma_bf16(tO, tc::sdesc(xh + ks * 4096, 2048, 128), b_q, ID_Y, ks > 0 ? 1u : 0u);
        tc::mma_bf16(tO, tc::sdesc(xl + ks * 4096, 2048, 128), b_q, ID_Y, 1u);
      }
      tc::commit(&bar[0]);
    }
    if (!wait_mma()) { failed = true; break; }
    // ---- Cm = T Z
    tmem_to_x(tZ);
    sync_for_mma();
    if (!wait_all(&bar[3], j & 1)) { failed = true; break; }
    t_done = j + 1;
    if (tid == 0) {
      const uint32_t th = tc::smem_addr(sT), tl = th + TILE3;
      const uint32_t xh = tc::smem_addr(sXh), xl = tc::smem_addr(sXl);
#pragma unroll 1
      for (int ks = 0; ks < 8; ++ks) {
        const uint64_t ah = tc::sdesc(th + ks * 4096, 2048, 128);
        const uint64_t al = tc::sdesc(tl + ks * 4096, 2048, 128);
        const uint64_t bh = tc::sdesc(xh + ks * 256, 128, 2048);
        const uint64_t bl = tc::sdesc(xl + ks * 256, 128, 2048);
        tc::mma_bf16(tC, ah, bh, ID_C, ks > 0 ? 1u : 0u);
        tc::mma_bf16(tC, ah, bl, ID_C, 1u);
        tc::mma_bf16(tC, al, bh, ID_C, 1u);
      }
      tc::commit(&bar[0]);
    }
    if (!wait_mma()) { failed = true; break; }
    if (j + 1 < ncl) {   // T(c) has been read
      if (tid == 0) issue_t(j + 1);
      t_issued = j + 2;
    }
    // ---- E = Cm Q ; S += W Cm
    tmem_to_x(tC);
    sync_for_mma();
    if (tid == 0) {
      tc::fence_after_sync();
      const uint32_t w = tc::smem_addr(sW(s)), q = tc::smem_addr(sQ(s));
      const uint32_t xh = tc::smem_addr(sXh), xl = tc::smem_addr(sXl);
#pragma unroll 1
      for (int ks = 0; ks < 8; ++ks) {
        const uint64_t b_q = tc::sdesc_sw128(q + (ks >> 2) * 8192 + (ks & 3) * 32, 16, 1024);
        tc::mma_bf16(tE, tc::sdesc(xh + ks * 4096, 2048, 128), b_q, ID_Y, ks > 0 ? 1u : 0u);
        tc::mma_bf16(tE, tc::sdesc(xl + ks * 4096, 2048, 128), b_q, ID_Y, 1u);
        const uint64_t a_w = tc::sdesc_sw128(w + ks * 2048, 16384, 1024);
        tc::mma_bf16(tS, a_w, tc::sdesc(xh + ks * 256, 128, 2048), ID_S, 1u);
        tc::mma_bf16(tS, a_w, tc::sdesc(xl + ks * 256, 128, 2048), ID_S, 1u);
      }
      tc::commit(&bar[0]);
    }
    if (!wait_mma()) { failed = true; break; }
    // ---- O = Y + W mask(E); E goes where Cm was
    {
      float e[32];
      tc::tmem_ld16(tE + lb + 32 * half, e);
      tc::tmem_ld16(tE + lb + 32 * half + 16, e + 16);
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        float x[8];
#pragma unroll
        for (int jj = 0; jj < 8; ++jj) {
          const int t = 32 * half + 8 * g + jj;
          x[jj] = ((row & (C3 - 1)) <= t) ? e[8 * g + jj] : 0.f;
        }
        uint4 h, l;
        tc::split8(x, h, l);
        const int off = mnmaj3(row, 32 * half + 8 * g, C3 / 8);
        *reinterpret_cast<uint4*>(sEh + off) = h;
        *reinterpret_cast<uint4*>(sEl + off) = l;
      }
    }
    sync_for_mma();
    if (tid == 0) {
      tc::fence_after_sync();
      const uint32_t w = tc::smem_addr(sW(s));
      const uint32_t eh = tc::smem_addr(sEh), el = tc::smem_addr(sEl);
#pragma unroll 1
      for (int ks = 0; ks < 8; ++ks) {
        const uint64_t a_w = tc::sdesc_sw128(w + ks * 2048, 16384, 1024);
        tc::mma_bf16(tO, a_w, tc::sdesc(eh + ks * 2048, 1024, 128), ID_O, 1u);
        tc::mma_bf16(tO, a_w, tc::sdesc(el + ks * 2048, 1024, 128), ID_O, 1u);
      }
      tc::commit(&bar[0]);
    }
    if (!wait_mma()) { failed = true; break; }
    // ---- O -> [token][dim] bf16 rows in the W slot -> 16-byte coalesced stores
    {
      __nv_bfloat16* stg = reinterpret_cast<__nv_bfloat16*>(sW(s));
      float o[32];
      tc::tmem_ld16(tO + lb + 32 * half, o);
      tc::tmem_ld16(tO + lb + 32 * half + 16, o + 16);
#pragma unroll
      for (int u = 0; u < 32; ++u) stg[(32 * half + u) * HD + row] = __float2bfloat16_rn(o[u]);
      tc::fence_before_sync();
      __syncthreads();
      for (int e = tid; e < C3 * (HD / 8); e += THR3) {
        const int t = e >> 4, part = e & 15;
        if (t < nt)
          *reinterpret_cast<uint4*>(out + ((size_t)(bi * (size_t)S + t0 + t) * H + hi) * HD + part * 8) =
              *reinterpret_cast<const uint4*>(stg + t * HD + part * 8);
      }
    }
    // the slot is free again: chunk c + 2's W and Q go there
    tc::fence_proxy_async();
    __syncthreads();
    if (j + 2 < ncl) {
      if (tid == 0) issue_wq(j + 2);
      wq_issued = j + 3;
    }
  }
  if (failed) {
    // let copies still in flight land before the CTA's shared memory is released
    if (tid == 0) {
      for (int j = wq_done; j < wq_issued; ++j) tc::mbar_wait(&bar[1 + (j & 1)], (j >> 1) & 1, POLLS3);
      if (t_done < t_issued) tc::mbar_wait(&bar[3], (t_issued - 1) & 1, POLLS3);
    }
  } else {
    float* po = psi_out + (size_t)chain * HD * HD + (size_t)row * HD;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float x[16];
      tc::tmem_ld16(tS + lb + 64 * half + 16 * u, x);
#pragma unroll
      for (int jj = 0; jj < 16; jj += 4)
        *reinterpret_cast<float4*>(po + 64 * half + 16 * u + jj) = make_float4(x[jj], x[jj + 1], x[jj + 2], x[jj + 3]);
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tb, 512);
}

// q, k or v as a [b][S][H][128] bf16 tensor; boxes of 64 elements x 1 head x 64 tokens with
// 128-byte swizzle (tokens past S read as 0)
int make_head_map(CUtensorMap* m, const void* base, int b, int S, int H) {
  auto enc = tmap_encoder();
  VERACE_REQUIRE(enc != nullptr, VERACE_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  const cuuint64_t dims[4] = {(cuuint64_t)HD, (cuuint64_t)H, (cuuint64_t)S, (cuuint64_t)b};
  const cuuint64_t strides[3] = {(cuuint64_t)HD * 2, (cuuint64_t)H * HD * 2, (cuuint64_t)S * H * HD * 2};
  const cuuint32_t box[4] = {64, 1, (cuuint32_t)C3, 1};
  const cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, es,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  VERACE_REQUIRE(r == CUDA_SUCCESS, VERACE_ERR_CUDA, "cuTensorMapEncodeTiled (q/k/v heads) failed: %d", (int)r);
  return VERACE_OK;
}

template <typename T>
size_t sssd_tc_prep_smem() { return sizeof(float) * ((sizeof(T) == 2 ? 0 : HD * (R3 + 1)) + R3 * 132); }

// Split launch (bf16): the scan runs one chain per CTA, so b*h chains busy at most b*h SMs
// and the prep of every chunk (many short CTAs) runs first on the whole GPU.  When the
// chains fill no more than half of the SMs, the call is cut into SSSD_PARTS chunk ranges:
// the prep of range p + 1 runs on a side stream while the scan of range p runs on the
// caller's stream (events order them; no kernel waits on another), and the state passes
// from one range to the next through psi_out.  Streams and events are created once per
// device; a capturing caller stream takes the single-launch path.
constexpr int SSSD_PARTS = 3;
struct SplitRes {
  cudaStream_t side = nullptr;
  cudaEvent_t ev[1 + SSSD_PARTS] = {};
  bool ready = false;
};
constexpr int SPLIT_MAX_DEVICES = 64;
SplitRes g_split[SPLIT_MAX_DEVICES];
std::mutex g_split_mutex;

int split_resources(int dev, SplitRes** out) {
  SplitRes& r = g_split[dev];
  if (!r.ready) {
    VERACE_CUDA(cudaStreamCreateWithFlags(&r.side, cudaStreamNonBlocking));
    for (auto& e : r.ev) VERACE_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    r.ready = true;
  }
  *out = &r;
  return VERACE_OK;
}

template <typename T>
int launch_prep(const void* k, const void* v, const float* delta, unsigned char* Tws, unsigned long long* badws,
                int s, int h, int chains, int nch, int c0, int c1, cudaStream_t st) {
  const size_t ps = sssd_tc_prep_smem<T>();
  VERACE_CUDA(cudaFuncSetAttribute(sssd_tc_prep<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ps));
  sssd_tc_prep<T><<<dim3(c1 - c0, chains), THR3, ps, st>>>((const T*)k, (const T*)v, delta, Tws, badws, s, h, nch,
                                                           c0);
  return check_launch("sssd_tc_prep");
}

template <typename T>
int launch_sssd_tc(const void* q, const void* k, const void* v, const float* delta, const float* psi0,
                   void* out, float* psi_out, int b, int s, int h, unsigned char* Tws,
                   unsigned long long* badws, cudaStream_t st) {
  const int chains = b * h;
  const int nch = (s + C3 - 1) / C3;
  int rc;
  if constexpr (sizeof(T) == 2) {
    // (an empty sequence issues no copies; its maps only need valid extents)
    const int sm = s > 0 ? s : 1;
    CUtensorMap mq, mk, mv;
    if ((rc = make_head_map(&mq, q, b, sm, h)) || (rc = make_head_map(&mk, k, b, sm, h)) ||
        (rc = make_head_map(&mv, v, b, sm, h)))
      return rc;
    VERACE_CUDA(cudaFuncSetAttribute(sssd_tc_scan_bf16, cudaFuncAttributeMaxDynamicSharedMemorySize, SSSD_TC2_SMEM));
    int dev = 0, sms = 0;
    VERACE_CUDA(cudaGetDevice(&dev));
    VERACE_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    VERACE_CUDA(cudaStreamIsCapturing(st, &cap));
    if (nch >= 2 * SSSD_PARTS && 2 * chains <= sms && cap == cudaStreamCaptureStatusNone &&
        dev < SPLIT_MAX_DEVICES) {
      std::lock_guard<std::mutex> lock(g_split_mutex);
      SplitRes* r = nullptr;
      if ((rc = split_resources(dev, &r))) return rc;
      VERACE_CUDA(cudaEventRecord(r->ev[0], st));             // the inputs are ready
      VERACE_CUDA(cudaStreamWaitEvent(r->side, r->ev[0], 0));
      for (int p = 0; p < SSSD_PARTS; ++p) {
        const int c0 = p * nch / SSSD_PARTS, c1 = (p + 1) * nch / SSSD_PARTS;
        if ((rc = launch_prep<T>(k, v, delta, Tws, badws, s, h, chains, nch, c0, c1, r->side))) return rc;
        VERACE_CUDA(cudaEventRecord(r->ev[1 + p], r->side));
      }
      for (int p = 0; p < SSSD_PARTS; ++p) {
        const int c0 = p * nch / SSSD_PARTS, c1 = (p + 1) * nch / SSSD_PARTS;
        VERACE_CUDA(cudaStreamWaitEvent(st, r->ev[1 + p], 0));
        sssd_tc_scan_bf16<<<chains, THR3, SSSD_TC2_SMEM, st>>>(mq, mk, mv, p == 0 ? psi0 : psi_out,
                                                              (__nv_bfloat16*)out, psi_out, Tws, badws, s, h, nch,
                                                              c0, c1);
        if ((rc = check_launch("sssd_tc_scan_bf16"))) return rc;
      }
      return VERACE_OK;
    }
    if (nch > 0 && (rc = launch_prep<T>(k, v, delta, Tws, badws, s, h, chains, nch, 0, nch, st))) return rc;
    sssd_tc_scan_bf16<<<chains, THR3, SSSD_TC2_SMEM, st>>>(mq, mk, mv, psi0, (__nv_bfloat16*)out, psi_out, Tws, badws,
                                                          s, h, nch, 0, nch);
    return check_launch("sssd_tc_scan_bf16");
  } else {
    if (nch > 0 && (rc = launch_prep<T>(k, v, delta, Tws, badws, s, h, chains, nch, 0, nch, st))) return rc;
    VERACE_CUDA(cudaFuncSetAttribute(sssd_tc_scan<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, SSSD_TC_SMEM));
    sssd_tc_scan<T><<<chains, THR3, SSSD_TC_SMEM, st>>>((const T*)q, (const T*)k, (const T*)v, psi0, (T*)out,
                                                       psi_out, Tws, badws, s, h, nch);
    return check_launch("sssd_tc_scan");
  }
}

}  // namespace

bool sssd_tc_supported(int d, int dtype) { return d == HD && (dtype == VERACE_BF16 || dtype == VERACE_F32); }

size_t sssd_tc_workspace(int b, int s, int h) {
  const size_t chains = (size_t)b * h, nch = ((size_t)s + C3 - 1) / C3;
  return align_up(chains * nch * 2 * TILE3, 256) + align_up(chains * nch * sizeof(unsigned long long), 256) + 256;
}

int sssd_tc_scan_launch(const void* q, const void* k, const void* v, const float* delta, const float* psi0,
                        void* out, float* psi_out, int b, int s, int h, int dtype, void* workspace,
                        cudaStream_t st) {
  const size_t chains = (size_t)b * h, nch = ((size_t)s + C3 - 1) / C3;
  unsigned char* Tws = (unsigned char*)align_up((size_t)workspace, 256);
  unsigned long long* badws = (unsigned long long*)(Tws + align_up(chains * nch * 2 * TILE3, 256));
  if (dtype == VERACE_BF16)
    return launch_sssd_tc<__nv_bfloat16>(q, k, v, delta, psi0, out, psi_out, b, s, h, Tws, badws, st);
  return launch_sssd_tc<float>(q, k, v, delta, psi0, out, psi_out, b, s, h, Tws, badws, st);
}

int sssd_tc_read_status(int* status) {
  int h = 0;
  VERACE_CUDA(cudaMemcpyFromSymbol(&h, g_sssd_tc_status, sizeof(int)));
  if (h) {
    const int zero = 0;
    VERACE_CUDA(cudaMemcpyToSymbol(g_sssd_tc_status, &zero, sizeof(int)));
  }
  *status = h;
  return VERACE_OK;
}

}  // namespace verace
