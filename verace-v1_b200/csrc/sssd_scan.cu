// SSSD Cayley-rotation scan (fp32 state, chunked compact-WY form).
//
// Per token the reference forms R_t = (I + X_t)^-1 (I - X_t), X_t = (d_t/2)(k vᵀ - v kᵀ)
// (verace_v1/modules/sssd_attention.py:154-166) and the state Psi_t = R_t Psi_{t-1}
// (:169-175).  With U_t = [k_t, v_t] the factor is a rank-2 perturbation of I:
//     R_t = I + U_t M_t U_tᵀ,   M_t = -(2a/det) [[a vv, 1 - a kv], [-1 - a kv, a kk]],
//     a = d_t / 2,  det = 1 + a² (kk vv - kv²)
// (exact; continuous at d_t -> 0, where M_t -> 0 and R_t -> I).  A chunk of C tokens
// composes to  R_C ... R_1 = I + W T Wᵀ  with W = [U_1 .. U_C] (d x 2C) and the block
// lower-triangular T = (I - Mblk L)^-1 Mblk, L the strictly block-lower part of WᵀW.
// For a chunk starting from state S:
//     Z = Wᵀ S,  Cm = T Z,  S_t = S + sum_{tau<=t} U_tau Cm_tau,  S_next = S + W Cm
//     o_t = S_t q_t = (S Q)_t + W mask(Cm Q)_t      (mask keeps token blocks tau <= t)
// Two kernels: sssd_prep (T for every chunk, all chunks in parallel, no state
// dependency) and sssd_scan (one CTA per (batch, head) chain; the 128x128 state
// stays in shared memory for the whole sequence; chunks are processed in order).
#include "common.cuh"

#include <mutex>
#include <stdlib.h>

namespace verace {

// tcgen05 path for head_dim 128 (sssd_tc.cu)
bool sssd_tc_supported(int d, int dtype);
size_t sssd_tc_workspace(int b, int s, int h);
int sssd_tc_scan_launch(const void* q, const void* k, const void* v, const float* delta, const float* psi0,
                        void* out, float* psi_out, int b, int s, int h, int dtype, void* workspace,
                        cudaStream_t st);

namespace {

// VERACE_SSSD_SIMT=1 forces the fp32 SIMT kernels (used to compare the two paths).
bool sssd_force_simt() {
  const char* e = getenv("VERACE_SSSD_SIMT");
  return e && e[0] && e[0] != '0';
}

constexpr int SC = 32;       // tokens per chunk
constexpr int SR = 2 * SC;   // rank of a chunk transform
constexpr int SSSD_MAX_D = 128;
constexpr int PREP_THREADS = 256;
constexpr int SCAN_THREADS = 512;

struct SssdWs {
  float* T;                  // [chains][nch][SR][SR]
  unsigned long long* bad;   // [chains][nch] bit tau set: token's factor is non-finite
};

__host__ __device__ inline size_t sssd_t_bytes(size_t chains, size_t nch) {
  return chains * nch * SR * SR * sizeof(float);
}

// ---------------------------------------------------------------------------------
// prep: W = [k_1, v_1, ..., k_C, v_C], G = WᵀW, per-token M_t, T by block forward
// substitution (column sigma of T is owned by one thread).
// smem: Ws [d][SR+1], Gs [SR][SR+1], Ts [SR][SR+1], Ms [SC][4]
template <typename T>
__global__ void __launch_bounds__(PREP_THREADS)
sssd_prep_kernel(const T* __restrict__ k, const T* __restrict__ v,
                 const float* __restrict__ delta, float* __restrict__ Tws,
                 unsigned long long* __restrict__ badws, int S, int H, int d, int nch) {
  extern __shared__ float sm[];
  float* Ws = sm;
  float* Gs = Ws + d * (SR + 1);
  float* Ts = Gs + SR * (SR + 1);
  float* Ms = Ts + SR * (SR + 1);
  __shared__ unsigned long long bad_bits;

  const int c = blockIdx.x;
  const int chain = blockIdx.y;
  const int bi = chain / H, hi = chain % H;
  const int t0 = c * SC;
  const int nt = min(SC, S - t0);
  const int tid = threadIdx.x;
  if (tid == 0) bad_bits = 0ull;

  for (int e = tid; e < d * SR; e += blockDim.x) {
    const int r = e % SR, i = e / SR;
    const int tau = r >> 1;
    float val = 0.f;
    if (tau < nt) {
      const size_t off = ((size_t)(bi * (size_t)S + t0 + tau) * H + hi) * d + i;
      val = to_f32((r & 1) ? v[off] : k[off]);
    }
    Ws[i * (SR + 1) + r] = val;
  }
  __syncthreads();
  // Tokens with a non-finite k, v or gate get the identity factor (the reference's
  // _solve_cayley substitution, sssd_attention.py:52-71): their W columns are zeroed
  // before the Gram matrix is formed so that nothing non-finite reaches T.
  if (tid < SC && tid < nt) {
    bool ok = isfinite(delta[(size_t)(bi * (size_t)S + t0 + tid) * H + hi]);
    for (int i = 0; i < d && ok; ++i)
      ok = isfinite(Ws[i * (SR + 1) + 2 * tid]) && isfinite(Ws[i * (SR + 1) + 2 * tid + 1]);
    if (!ok) atomicOr(&bad_bits, 1ull << tid);
  }
  __syncthreads();
  if (bad_bits) {
    for (int e = tid; e < d * SR; e += blockDim.x)
      if ((bad_bits >> ((e % SR) >> 1)) & 1ull) Ws[(e / SR) * (SR + 1) + e % SR] = 0.f;
    __syncthreads();
  }
  // G = Wᵀ W  (A(m=r, k=i) = Ws[i][r], B(k=i, n=r') = Ws[i][r'])
  smem_gemm<4, 4, false>(SR, SR, d, Ws, 1, SR + 1, Ws, SR + 1, 1, Gs, SR + 1, 1, tid, blockDim.x);
  __syncthreads();
  if (tid < SC) {
    const int tau = tid;
    float m00 = 0.f, m01 = 0.f, m10 = 0.f, m11 = 0.f;
    if (tau < nt && !((bad_bits >> tau) & 1ull)) {
      const float kk = Gs[(2 * tau) * (SR + 1) + 2 * tau];
      const float vv = Gs[(2 * tau + 1) * (SR + 1) + 2 * tau + 1];
      const float kv = Gs[(2 * tau) * (SR + 1) + 2 * tau + 1];
      const float dl = delta[(size_t)(bi * (size_t)S + t0 + tau) * H + hi];
      const float a = 0.5f * dl;
      const float det = 1.f + a * a * (kk * vv - kv * kv);
      const float f = -2.f * a / det;
      m00 = f * (a * vv);
      m01 = f * (1.f - a * kv);
      m10 = f * (-1.f - a * kv);
      m11 = f * (a * kk);
      const bool ok = isfinite(kk) && isfinite(vv) && isfinite(kv) &&
                      isfinite(m00) && isfinite(m01) && isfinite(m10) && isfinite(m11);
      if (!ok) {  // overflowing factor: identity, and its Gram rows/columns cleared
        m00 = m01 = m10 = m11 = 0.f;
        atomicOr(&bad_bits, 1ull << tau);
        for (int r = 0; r < SR; ++r) {
          Gs[(2 * tau) * (SR + 1) + r] = 0.f; Gs[(2 * tau + 1) * (SR + 1) + r] = 0.f;
          Gs[r * (SR + 1) + 2 * tau] = 0.f; Gs[r * (SR + 1) + 2 * tau + 1] = 0.f;
        }
      }
    }
    Ms[tau * 4 + 0] = m00; Ms[tau * 4 + 1] = m01;
    Ms[tau * 4 + 2] = m10; Ms[tau * 4 + 3] = m11;
  }
  __syncthreads();
  if (tid < SR) {
    const int sg = tid;          // column of T
    const int blk = sg >> 1;
    for (int r = 0; r < 2 * blk; ++r) Ts[r * (SR + 1) + sg] = 0.f;
    for (int t = blk; t < SC; ++t) {
      float x0 = (sg == 2 * t) ? 1.f : 0.f;
      float x1 = (sg == 2 * t + 1) ? 1.f : 0.f;
      for (int tp = blk; tp < t; ++tp) {
        const float t0v = Ts[(2 * tp) * (SR + 1) + sg];
        const float t1v = Ts[(2 * tp + 1) * (SR + 1) + sg];
        x0 += Gs[(2 * t) * (SR + 1) + 2 * tp] * t0v + Gs[(2 * t) * (SR + 1) + 2 * tp + 1] * t1v;
        x1 += Gs[(2 * t + 1) * (SR + 1) + 2 * tp] * t0v + Gs[(2 * t + 1) * (SR + 1) + 2 * tp + 1] * t1v;
      }
      Ts[(2 * t) * (SR + 1) + sg] = Ms[t * 4 + 0] * x0 + Ms[t * 4 + 1] * x1;
      Ts[(2 * t + 1) * (SR + 1) + sg] = Ms[t * 4 + 2] * x0 + Ms[t * 4 + 3] * x1;
    }
  }
  __syncthreads();
  float* Tout = Tws + ((size_t)chain * nch + c) * SR * SR;
  for (int e = tid; e < SR * SR; e += blockDim.x) Tout[e] = Ts[(e / SR) * (SR + 1) + e % SR];
  if (tid == 0) badws[(size_t)chain * nch + c] = bad_bits;
}

// ---------------------------------------------------------------------------------
// scan: one CTA per chain.  smem (pitches padded by one):
//   Ss [d][d+1]  Ws [d][SR+1]  Qs [d][SC+1]  Ts [SR][SR+1]
//   Zs [SR][d+1] Cs [SR][d+1]  Ys [d][SC+1]  Es [SR][SC+1]
template <typename T>
__global__ void __launch_bounds__(SCAN_THREADS, 1)
sssd_scan_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                 const float* __restrict__ psi0, T* __restrict__ out, float* __restrict__ psi_out,
                 const float* __restrict__ Tws, const unsigned long long* __restrict__ badws,
                 int S, int H, int d, int nch) {
  extern __shared__ float sm[];
  const int pd = d + 1;
  float* Ss = sm;
  float* Ws = Ss + d * pd;
  float* Qs = Ws + d * (SR + 1);
  float* Ts = Qs + d * (SC + 1);
  float* Zs = Ts + SR * (SR + 1);
  float* Cs = Zs + SR * pd;
  float* Ys = Cs + SR * pd;
  float* Es = Ys + d * (SC + 1);

  const int chain = blockIdx.x;
  const int bi = chain / H, hi = chain % H;
  const int tid = threadIdx.x, nthr = blockDim.x;
  const float* p0 = psi0 ? psi0 + (size_t)chain * d * d : nullptr;
  for (int e = tid; e < d * d; e += nthr) {
    const int i = e / d, j = e % d;
    Ss[i * pd + j] = p0 ? p0[e] : (i == j ? 1.f : 0.f);
  }

  for (int c = 0; c < nch; ++c) {
    const int t0 = c * SC;
    const int nt = min(SC, S - t0);
    const unsigned long long bad = badws[(size_t)chain * nch + c];
    // W (zero columns of padded / non-finite tokens) and Q
    for (int e = tid; e < d * SR; e += nthr) {
      const int i = e / SR, r = e % SR, tau = r >> 1;
      float val = 0.f;
      if (tau < nt && !((bad >> tau) & 1ull)) {
        const size_t off = ((size_t)(bi * (size_t)S + t0 + tau) * H + hi) * d + i;
        val = to_f32((r & 1) ? v[off] : k[off]);
      }
      Ws[i * (SR + 1) + r] = val;
    }
    for (int e = tid; e < d * SC; e += nthr) {
      const int t = e / d, j = e % d;
      float val = 0.f;
      if (t < nt) val = to_f32(q[((size_t)(bi * (size_t)S + t0 + t) * H + hi) * d + j]);
      Qs[j * (SC + 1) + t] = val;
    }
    const float* Tin = Tws + ((size_t)chain * nch + c) * SR * SR;
    for (int e = tid; e < SR * SR; e += nthr) Ts[(e / SR) * (SR + 1) + e % SR] = Tin[e];
    __syncthreads();
    // Z = Wᵀ S ; Y = S Q
    smem_gemm<4, 4, false>(SR, d, d, Ws, 1, SR + 1, Ss, pd, 1, Zs, pd, 1, tid, nthr);
    smem_gemm<4, 4, false>(d, SC, d, Ss, pd, 1, Qs, SC + 1, 1, Ys, SC + 1, 1, tid, nthr);
    __syncthreads();
    // Cm = T Z
    smem_gemm<4, 4, false>(SR, d, SR, Ts, SR + 1, 1, Zs, pd, 1, Cs, pd, 1, tid, nthr);
    __syncthreads();
    // E = Cm Q, then causal mask (token block of r must be <= t)
    smem_gemm<4, 4, false>(SR, SC, d, Cs, pd, 1, Qs, SC + 1, 1, Es, SC + 1, 1, tid, nthr);
    __syncthreads();
    for (int e = tid; e < SR * SC; e += nthr) {
      const int r = e / SC, t = e % SC;
      if ((r >> 1) > t) Es[r * (SC + 1) + t] = 0.f;
    }
    __syncthreads();
    // O = Y + W E ; S += W Cm
    smem_gemm<4, 4, true>(d, SC, SR, Ws, SR + 1, 1, Es, SC + 1, 1, Ys, SC + 1, 1, tid, nthr);
    smem_gemm<4, 4, true>(d, d, SR, Ws, SR + 1, 1, Cs, pd, 1, Ss, pd, 1, tid, nthr);
    __syncthreads();
    for (int e = tid; e < nt * d; e += nthr) {
      const int t = e / d, i = e % d;
      out[((size_t)(bi * (size_t)S + t0 + t) * H + hi) * d + i] = from_f32<T>(Ys[i * (SC + 1) + t]);
    }
    // the next chunk's loads only overwrite Ws/Qs/Ts, which this write-out does not read
  }
  __syncthreads();
  float* po = psi_out + (size_t)chain * d * d;
  for (int e = tid; e < d * d; e += nthr) po[e] = Ss[(e / d) * pd + e % d];
}

size_t prep_smem(int d) { return sizeof(float) * (d * (SR + 1) + 2 * SR * (SR + 1) + SC * 4); }
size_t scan_smem(int d) {
  return sizeof(float) * (d * (d + 1) + d * (SR + 1) + d * (SC + 1) + SR * (SR + 1) +
                          2 * SR * (d + 1) + d * (SC + 1) + SR * (SC + 1));
}

template <typename T>
int launch_sssd(const void* q, const void* k, const void* v, const float* delta,
                const float* psi0, void* out, float* psi_out, int b, int s, int h, int d,
                float* Tws, unsigned long long* badws, cudaStream_t st) {
  const int chains = b * h;
  const int nch = (s + SC - 1) / SC;
  if (nch > 0) {
    const size_t ps = prep_smem(d);
    VERACE_CUDA(cudaFuncSetAttribute(sssd_prep_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ps));
    sssd_prep_kernel<T><<<dim3(nch, chains), PREP_THREADS, ps, st>>>(
        (const T*)k, (const T*)v, delta, Tws, badws, s, h, d, nch);
    int rc = check_launch("sssd_prep_kernel");
    if (rc) return rc;
  }
  const size_t ss = scan_smem(d);
  VERACE_CUDA(cudaFuncSetAttribute(sssd_scan_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ss));
  sssd_scan_kernel<T><<<chains, SCAN_THREADS, ss, st>>>(
      (const T*)q, (const T*)k, (const T*)v, psi0, (T*)out, psi_out, Tws, badws, s, h, d, nch);
  return check_launch("sssd_scan_kernel");
}

}  // namespace
}  // namespace verace

using namespace verace;

namespace verace {
namespace {
size_t simt_workspace(int b, int s, int h) {
  const size_t chains = (size_t)b * h;
  const size_t nch = ((size_t)s + SC - 1) / SC;
  return align_up(sssd_t_bytes(chains, nch), 256) + align_up(chains * nch * sizeof(unsigned long long), 256);
}
}  // namespace
}  // namespace verace

extern "C" size_t verace_sssd_scan_workspace(int b, int s, int h, int d) {
  if (b <= 0 || s <= 0 || h <= 0) return 256;
  size_t n = simt_workspace(b, s, h);
  if (d == 128) {
    const size_t t = sssd_tc_workspace(b, s, h);
    if (t > n) n = t;
  }
  return n;
}

extern "C" int verace_sssd_scan(const void* q, const void* k, const void* v, const float* delta,
                                const float* psi0, void* out, float* psi_out, int b, int s, int h,
                                int d, int dtype, void* workspace, size_t workspace_bytes,
                                void* stream) {
  VERACE_REQUIRE(b >= 0 && s >= 0 && h >= 1 && d >= 1, VERACE_ERR_INVALID,
                 "verace_sssd_scan: invalid sizes b=%d s=%d h=%d d=%d", b, s, h, d);
  VERACE_REQUIRE(d <= SSSD_MAX_D, VERACE_ERR_UNSUPPORTED,
                 "verace_sssd_scan: head_dim %d > %d is not supported", d, SSSD_MAX_D);
  VERACE_REQUIRE(dtype == VERACE_F32 || dtype == VERACE_BF16 || dtype == VERACE_F16,
                 VERACE_ERR_INVALID, "verace_sssd_scan: unknown dtype %d", dtype);
  if (b == 0) return VERACE_OK;
  VERACE_REQUIRE(psi_out != nullptr, VERACE_ERR_INVALID, "verace_sssd_scan: psi_out is NULL");
  VERACE_REQUIRE(s == 0 || (q && k && v && delta && out), VERACE_ERR_INVALID,
                 "verace_sssd_scan: NULL input/output pointer");
  const size_t need = s > 0 ? verace_sssd_scan_workspace(b, s, h, d) : 0;
  VERACE_REQUIRE(need == 0 || (workspace != nullptr && workspace_bytes >= need), VERACE_ERR_WORKSPACE,
                 "verace_sssd_scan: workspace of %zu bytes required, %zu given", need,
                 workspace ? workspace_bytes : (size_t)0);
  const size_t chains = (size_t)b * h;
  const size_t nch = ((size_t)s + SC - 1) / SC;
  cudaStream_t st = (cudaStream_t)stream;
  if (s > 0 && sssd_tc_supported(d, dtype) && !sssd_force_simt())
    return sssd_tc_scan_launch(q, k, v, delta, psi0, out, psi_out, b, s, h, dtype, workspace, st);
  float* Tws = (float*)workspace;
  unsigned long long* badws =
      (unsigned long long*)((char*)workspace + align_up(sssd_t_bytes(chains, nch), 256));
  switch (dtype) {
    case VERACE_F32: return launch_sssd<float>(q, k, v, delta, psi0, out, psi_out, b, s, h, d, Tws, badws, st);
    case VERACE_BF16: return launch_sssd<__nv_bfloat16>(q, k, v, delta, psi0, out, psi_out, b, s, h, d, Tws, badws, st);
    default: return launch_sssd<__half>(q, k, v, delta, psi0, out, psi_out, b, s, h, d, Tws, badws, st);
  }
}

// ---------------------------------------------------------------------------------
// Allocation-free variant.  Some hosts cannot call cudaMalloc on the path that runs
// this scan: plugin / FFI runtimes that own every byte of device memory and hand the
// library only its inputs and outputs, and memory-budgeted serving loops where an
// allocation (which may synchronise the device) is not allowed.  For them the scan's
// scratch (the per-chunk transforms T and the non-finite-token masks) lives in the
// fixed device array below, which every GPU that loads this library holds until the
// process exits.  Host code never uses the array's name as a device address: the
// address is looked up with cudaGetSymbolAddress once per device (by the first call
// on that device, with that device current) and passed to the kernels.
namespace verace {
namespace {

constexpr size_t SSSD_NOALLOC_SCRATCH_BYTES = size_t(16) << 20;  // 16 MiB
static __device__ __align__(256) unsigned char g_sssd_noalloc_scratch[SSSD_NOALLOC_SCRATCH_BYTES];

constexpr int MAX_DEVICES = 64;
std::mutex g_noalloc_mutex;
void* g_noalloc_ptr[MAX_DEVICES] = {};

int noalloc_scratch(void** out, cudaStream_t stream) {
  int dev = 0;
  VERACE_CUDA(cudaGetDevice(&dev));
  VERACE_REQUIRE(dev >= 0 && dev < MAX_DEVICES, VERACE_ERR_UNSUPPORTED,
                 "verace_sssd_scan_noalloc: device ordinal %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_ptr[dev] == nullptr) {
    // the address lookup is a runtime call that must not be recorded into a graph
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    VERACE_CUDA(cudaStreamIsCapturing(stream, &cap));
    VERACE_REQUIRE(cap == cudaStreamCaptureStatusNone, VERACE_ERR_INVALID,
                   "verace_sssd_scan_noalloc: the first call on device %d came while its stream is "
                   "being captured; make one call on this device before any capture", dev);
    void* p = nullptr;
    VERACE_CUDA(cudaGetSymbolAddress(&p, g_sssd_noalloc_scratch));
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return VERACE_OK;
}

}  // namespace
}  // namespace verace

extern "C" int verace_sssd_scan_noalloc(const void* q, const void* k, const void* v,
                                        const float* delta, const float* psi0, void* out,
                                        float* psi_out, int b, int s, int h, int d, int dtype,
                                        void* stream) {
  VERACE_REQUIRE(b >= 0 && s >= 0 && h >= 1 && d >= 1, VERACE_ERR_INVALID,
                 "verace_sssd_scan_noalloc: invalid sizes b=%d s=%d h=%d d=%d", b, s, h, d);
  VERACE_REQUIRE(d <= SSSD_MAX_D, VERACE_ERR_UNSUPPORTED,
                 "verace_sssd_scan_noalloc: head_dim %d > %d is not supported", d, SSSD_MAX_D);
  VERACE_REQUIRE(dtype == VERACE_F32 || dtype == VERACE_BF16 || dtype == VERACE_F16,
                 VERACE_ERR_INVALID, "verace_sssd_scan_noalloc: unknown dtype %d", dtype);
  if (b == 0) return VERACE_OK;
  // the size limit first: a size that does not fit is refused before any pointer is looked at
  const size_t need = s > 0 ? simt_workspace(b, s, h) : 0;
  VERACE_REQUIRE(need <= SSSD_NOALLOC_SCRATCH_BYTES, VERACE_ERR_UNSUPPORTED,
                 "verace_sssd_scan_noalloc: this size needs %zu bytes of scratch, more than the "
                 "fixed %zu-byte device array; use verace_sssd_scan with a workspace",
                 need, SSSD_NOALLOC_SCRATCH_BYTES);
  VERACE_REQUIRE(psi_out != nullptr, VERACE_ERR_INVALID, "verace_sssd_scan_noalloc: psi_out is NULL");
  VERACE_REQUIRE(s == 0 || (q && k && v && delta && out), VERACE_ERR_INVALID,
                 "verace_sssd_scan_noalloc: NULL input/output pointer");
  void* scratch = nullptr;
  const int rc = noalloc_scratch(&scratch, (cudaStream_t)stream);
  if (rc != VERACE_OK) return rc;
  const size_t chains = (size_t)b * h;
  const size_t nch = ((size_t)s + SC - 1) / SC;
  float* Tws = (float*)scratch;
  unsigned long long* badws =
      (unsigned long long*)((char*)scratch + align_up(sssd_t_bytes(chains, nch), 256));
  cudaStream_t st = (cudaStream_t)stream;
  switch (dtype) {
    case VERACE_F32: return launch_sssd<float>(q, k, v, delta, psi0, out, psi_out, b, s, h, d, Tws, badws, st);
    case VERACE_BF16: return launch_sssd<__nv_bfloat16>(q, k, v, delta, psi0, out, psi_out, b, s, h, d, Tws, badws, st);
    default: return launch_sssd<__half>(q, k, v, delta, psi0, out, psi_out, b, s, h, d, Tws, badws, st);
  }
}
