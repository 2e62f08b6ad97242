/*
 * verace_b200.h -- C ABI of the B200-native (sm_100a) Verace V1 sequence-mixing path.
 *
 * Plain pointers and sizes only; no framework types.  All tensor arguments are
 * DEVICE pointers to dense row-major (C-contiguous) arrays.  Every entry point
 * enqueues its kernels on `stream` (a cudaStream_t passed as void*; NULL = the
 * legacy default stream) and returns without synchronising.  Return value: 0 on
 * success, otherwise one of VERACE_ERR_*, with a message from verace_last_error().
 * Inputs are never modified; outputs are written, never read.
 *
 * Element types: `dtype` selects the type of q/k/v and of the sequence output
 * (VERACE_F32, VERACE_BF16, VERACE_F16).  Gates (delta, gamma) are fp32, and every
 * recurrent state (SSSD Psi, CHAM H = Hr + i Hi) is fp32, as in the reference.
 *
 * Scratch: the scan entry points take a caller-allocated device `workspace` of at
 * least the size returned by the matching *_workspace() query (256-byte aligned).
 *
 * The reference these entry points replace is Python (Verace-Pvt-Ltd/Verace-V1,
 * package verace_v1); each declaration cites the reference function it stands in for.
 */
#ifndef VERACE_B200_H_
#define VERACE_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define VERACE_API __attribute__((visibility("default")))
#else
#define VERACE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
  VERACE_OK = 0,
  VERACE_ERR_INVALID = 1,     /* bad argument (null pointer, negative size, ...) */
  VERACE_ERR_UNSUPPORTED = 2, /* valid but unsupported shape (e.g. head_dim > 128) */
  VERACE_ERR_CUDA = 3,        /* a CUDA runtime call or kernel launch failed */
  VERACE_ERR_WORKSPACE = 4,   /* workspace missing or smaller than required */
  VERACE_ERR_TIMEOUT = 5,     /* a bounded device-side wait gave up */
  VERACE_ERR_STATE = 6        /* a decode step met a hologram too far from unitary */
};

enum { VERACE_F32 = 0, VERACE_BF16 = 1, VERACE_F16 = 2 };

/* Version of this ABI (major*10000 + minor*100 + patch). */
VERACE_API int verace_version(void);

/* Message describing the last error returned on the calling host thread. */
VERACE_API const char* verace_last_error(void);

/* Synchronises `stream`, then reports (and clears) the device-side status words of
 * this library: VERACE_ERR_TIMEOUT if a kernel gave up waiting for a tensor-core
 * completion since the last call, else VERACE_ERR_STATE if a VERACE_DECODE_FIRST_ORDER
 * decode step found |(H^H H - I) q| > 1e-2 |q| for some item, else 0.  No reference
 * counterpart: the reference has no device-side waits and no decode precondition. */
VERACE_API int verace_device_status(void* stream);

/* Number of kernels this library has launched in the process so far (all devices,
 * all host threads).  Lets a caller count the library's own launches in a region. */
VERACE_API unsigned long long verace_kernel_launches(void);

/* ------------------------------------------------------------------------------
 * SSSD Cayley-rotation scan.
 * Replaces launch_sssd_triton_scan (verace_v1/serving/triton_kernels.py:603-636),
 * the kernel behind SSSDAttention.forward (verace_v1/modules/sssd_attention.py:129-136),
 * with the eager path's semantics (sssd_attention.py:144-181):
 *   R_t = (I + d_t A_t / 2)^-1 (I - d_t A_t / 2),  A_t = k_t v_t^T - v_t k_t^T
 *   Psi_t = R_t Psi_{t-1},  o_t = Psi_t q_t
 * q, k, v, out : [b, s, h, d] (dtype)       delta : [b, s, h] fp32
 * psi0         : [b, h, d, d] fp32, or NULL for the identity
 * psi_out      : [b, h, d, d] fp32 (state after the last token; = psi0 when s == 0)
 * Supports 1 <= d <= 128.
 * ---------------------------------------------------------------------------- */
VERACE_API size_t verace_sssd_scan_workspace(int b, int s, int h, int d);
VERACE_API int verace_sssd_scan(const void* q, const void* k, const void* v, const float* delta,
                     const float* psi0, void* out, float* psi_out,
                     int b, int s, int h, int d, int dtype,
                     void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------------
 * Allocation-free SSSD scan.  No counterpart in the reference: it exists for hosts
 * that cannot allocate device memory on the path that runs the scan (plugin or FFI
 * runtimes that own all device memory and pass only inputs and outputs; serving
 * loops with a fixed memory budget, where an allocation may synchronise the device).
 * Same arguments as verace_sssd_scan without the workspace: the scratch is a fixed
 * 16 MiB device array inside this library, which every GPU that loads the library holds
 * until the process exits.  It always runs the fp32 SIMT scan kernels (32-token chunk
 * transforms), whatever the head size, so its results equal verace_sssd_scan's to the
 * fp32 parity tolerance (1e-4 relative), not bit for bit where verace_sssd_scan takes
 * the tensor-core path (head_dim 128).  Limit: the scratch holds b*h*ceil(s/32) chunk
 * transforms of 16 KiB each plus one 8-byte mask word per transform (each part rounded
 * up to 256 bytes); sizes beyond 16 MiB return VERACE_ERR_UNSUPPORTED before any pointer
 * is looked at (b*h*ceil(s/32) <= 1023, e.g. b = 2, h = 8, s = 2016).
 * The first call on a device looks the array's device address up (once per device,
 * with that device current); it returns VERACE_ERR_INVALID if `stream` is being
 * captured at that moment, so make that first call before any stream capture.
 * All calls in a process share the one array per device: calls that overlap on the
 * GPU (issued on concurrent streams, or from several host threads) race on it and
 * give undefined results, so serialise them (one stream, or an event between calls).
 * Each call rewrites the scratch it reads, so nothing in it needs to start at zero.
 * ---------------------------------------------------------------------------- */
VERACE_API int verace_sssd_scan_noalloc(const void* q, const void* k, const void* v,
                                        const float* delta, const float* psi0, void* out,
                                        float* psi_out, int b, int s, int h, int d, int dtype,
                                        void* stream);

/* ------------------------------------------------------------------------------
 * CHAM holographic-memory scan with Newton-Schulz readout retraction.
 * Replaces launch_cham_triton_update / launch_cham_triton_tiled
 * (verace_v1/serving/triton_kernels.py:639-685, :552-597), the kernels behind
 * ContinuousHolographicMemory.forward (verace_v1/modules/cham_memory.py:164-168),
 * with the eager path's semantics (cham_memory.py:177-243):
 *   U_t = (I - i G_t / 2)^-1 (I + i G_t / 2),  G_t = g_t (k_t v_t^T + v_t k_t^T)
 *   H_t = U_t H_{t-1}  (raw, never retracted; exported)
 *   rec_t = Re(NS3(H_t)) q_t          (3 Newton-Schulz steps, cham_memory.py:296-315)
 * q, k, v, out : [b, s, D] (dtype)          gamma : [b, s] fp32
 * h0_re, h0_im : [b, D, D] fp32, or both NULL for (I, 0)
 * h_re, h_im   : [b, D, D] fp32 raw state after the last token
 * ---------------------------------------------------------------------------- */
VERACE_API size_t verace_cham_scan_workspace(int b, int s, int D, int has_h0);
VERACE_API int verace_cham_scan(const void* q, const void* k, const void* v, const float* gamma,
                     const float* h0_re, const float* h0_im, void* out,
                     float* h_re, float* h_im, int b, int s, int D, int dtype,
                     void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------------
 * Continuing a CHAM scan from a carried hologram H0 (initial_hologram of
 * ContinuousHolographicMemory.forward, cham_memory.py:117-122 and :229-239; the
 * launchers' initial_hologram argument, triton_kernels.py:639-685, :552-597).
 * Every U_t is unitary, so NS3(H_t) = H_t p(A) with A = H0^H H0 for the Newton-Schulz
 * polynomial p, and p(I + E) = I - E/2 + O(E^2).
 * verace_cham_unitarity: eps [b] fp32 (device) = max over 4 fixed +-1 probe vectors r of
 *   |(H^H H - I) r| / |r| per item, in fp64 (three launches; workspace
 *   verace_cham_unitarity_workspace(b, D) bytes).  It estimates the RMS action of E; for a
 *   worst-case (rank-one) E the readout error of the unitary scan is up to sqrt(D) eps / 2.
 * verace_cham_scan_unitary: verace_cham_scan with the readout Re(H_t q_t), i.e. p(A) = I,
 *   exact when H0 is unitary and within |E q_t| / 2 + O(|E|^2) of the Newton-Schulz
 *   readout otherwise; runs on the tensor cores for D % 128 == 0 (bf16 / fp32), else on
 *   the SIMT scan without the readout polynomial.  Workspace as verace_cham_scan with
 *   has_h0 = 1.  A caller picks it over verace_cham_scan when eps shows H0 unitary to
 *   within its tolerance (the Python launcher does: tensor-core speed for holograms grown
 *   by these scans, the exact polynomial readout for any other).
 * ---------------------------------------------------------------------------- */
VERACE_API size_t verace_cham_unitarity_workspace(int b, int D);
VERACE_API int verace_cham_unitarity(const float* h_re, const float* h_im, int b, int D, float* eps,
                                     void* workspace, size_t workspace_bytes, void* stream);
VERACE_API int verace_cham_scan_unitary(const void* q, const void* k, const void* v, const float* gamma,
                                        const float* h0_re, const float* h0_im, void* out, float* h_re,
                                        float* h_im, int b, int s, int D, int dtype, void* workspace,
                                        size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------------
 * Dense Newton-Schulz unitary retraction, `steps` iterations of H <- H (3I - H^H H) / 2.
 * Replaces newton_schulz_unitary_retraction (verace_v1/modules/cham_memory.py:21-51).
 * h_re, h_im, out_re, out_im : [b, D, D] fp32 (out may not alias the input).
 * ---------------------------------------------------------------------------- */
VERACE_API size_t verace_cham_retract_workspace(int b, int D);
VERACE_API int verace_cham_retract(const float* h_re, const float* h_im, float* out_re, float* out_im,
                        int b, int D, int steps, void* workspace, size_t workspace_bytes,
                        void* stream);

/* ------------------------------------------------------------------------------
 * Fused single-token decode step of one layer for a batch: SSSD state rotation and
 * CHAM hologram update with both readouts, states updated IN PLACE.
 * Replaces, for all b items at once, what one incremental-decode step runs per layer
 * and per item through layer_states (verace_v1/serving/hyper_generate.py:58-77,
 * verace_v1/modules/backbone.py:53-101): SSSDAttention.forward with s = 1 and
 * initial_state (sssd_attention.py:103-182, launcher triton_kernels.py:603-636) and
 * ContinuousHolographicMemory.forward with s = 1 and initial_hologram
 * (cham_memory.py:117-243, launcher triton_kernels.py:639-685 / _cham_tiled_step :477-549).
 *   SSSD:  Psi <- R Psi,  sssd_out = Psi q           (per item and head)
 *   CHAM:  H <- U H,      cham_out = Re(NS3(H) q)    (per item; H = h_re + i h_im)
 * sssd_q, sssd_k, sssd_v, sssd_out : [b, h, d] (dtype)   delta : [b, h] fp32
 * psi                              : [b, h, d, d] fp32, read and overwritten
 * cham_q, cham_k, cham_v, cham_out : [b, D] (dtype)      gamma : [b] fp32
 * h_re, h_im                       : [b, D, D] fp32, read and overwritten
 * The readout retraction NS3 uses that U is unitary: NS3(U H) = U H p(H^H H) for the
 * Newton-Schulz polynomial p, and p(I + E) = I - E/2 + O(E^2).
 *   mode VERACE_DECODE_UNITARY:     cham_out = Re(H q) (p = I); exact for H^H H = I,
 *                                   which holds to fp32 rounding for every state grown
 *                                   from an identity start.  One launch.
 *   mode VERACE_DECODE_FIRST_ORDER: cham_out = Re(H (q - E q / 2)), an O(|E|^2)
 *                                   difference; one extra pass over H (two launches);
 *                                   flags |E q| > 1e-2 |q| (see verace_device_status).
 * h == 0 or d == 0 skips SSSD (its pointers may be NULL); D == 0 skips CHAM.
 * Supports d % 4 == 0, d <= 128; D % 32 == 0, D <= 2048.  Workspace (CHAM only):
 * verace_decode_workspace(b, D) bytes; calls sharing a workspace must not overlap.
 * ---------------------------------------------------------------------------- */
/* ------------------------------------------------------------------------------
 * Mixer prologue: the elementwise tail of the q/k/v/gate projections of both mixers,
 * fused into one pass over one concatenated projection (the GEMM itself stays with the
 * caller's BLAS).  Replaces the normalisation and gate code of SSSDAttention.project
 * (verace_v1/modules/sssd_attention.py:116-126) and ContinuousHolographicMemory.project
 * (verace_v1/modules/cham_memory.py:129-153).
 * y      : [n, ld] (dtype), row = q | k | v (each heads*head_dim) | gate (gate_cols)
 * q, k, v: [n, heads*head_dim] (dtype): F.normalize(., p=2, dim=-1) per head (eps 1e-12),
 *          v first through SiLU when silu_v != 0 (CHAM)
 * gate   : [n, gate_cols] fp32: 0.1 * sigmoid(.) * mask[row] (mask [n] bytes, or NULL)
 * Supports head_dim % 8 == 0, head_dim <= 2048; ld % 8 == 0.
 * ---------------------------------------------------------------------------- */
VERACE_API int verace_mixer_prologue(const void* y, long long ld, void* q, void* k, void* v, float* gate,
                                     const unsigned char* mask, long long n, int heads, int head_dim,
                                     int gate_cols, int silu_v, int dtype, void* stream);

/* ------------------------------------------------------------------------------
 * Lazy CHAM decode (unitary readout): the hologram's rank-2 step updates are kept as
 * pending factors, H = S + sum_j [k_j v_j] B_j with S the stored planes, and folded
 * into S every P steps, so that a step reads S once instead of reading it twice and
 * writing it.  Same step and readout as verace_decode_step with
 * VERACE_DECODE_UNITARY, up to fp32 rounding order.
 * pending: verace_decode_pending_bytes(b, D, P) bytes per layer, zero-filled before the
 *          first step (an empty list); S is the true state only after
 *          verace_decode_cham_flush.  P in [1, 16].
 * Supports D % 32 == 0, D <= 2048; calls sharing a workspace must not overlap.
 * ---------------------------------------------------------------------------- */
VERACE_API size_t verace_decode_lazy_workspace(int b, int D);
VERACE_API size_t verace_decode_pending_bytes(int b, int D, int P);
VERACE_API int verace_decode_cham_lazy(const void* cham_q, const void* cham_k, const void* cham_v,
                                       const float* gamma, float* h_re, float* h_im, void* pending, int P,
                                       void* cham_out, int b, int D, int dtype, void* workspace,
                                       size_t workspace_bytes, void* stream);
VERACE_API int verace_decode_cham_flush(float* h_re, float* h_im, void* pending, int P, int b, int D,
                                        void* stream);
/* The same step from the layer's raw projection rows, with the projection epilogue of
 * ContinuousHolographicMemory.project (verace_v1/modules/cham_memory.py:129-153: SiLU on v,
 * q, k, v L2-normalised, gamma = 0.1 * sigmoid) folded into the step's first kernel: one
 * launch fewer than verace_mixer_prologue + verace_decode_cham_lazy, the same arithmetic
 * (SiLU rounded to dtype as the reference's SiLU output is; normalised values rounded to
 * dtype).  y: [b, ld] (dtype), row = q | k | v (D each) | gate; ld >= 3 D + 1. */
VERACE_API int verace_decode_cham_lazy_projected(const void* y, long long ld, float* h_re, float* h_im,
                                                 void* pending, int P, void* cham_out, int b, int D, int dtype,
                                                 void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------------
 * Block glue: the RMSNorms and residual adds around the two mixers
 * (verace_v1/modules/backbone.py: h <- h + SSSD(RMSNorm(h)); h <- h + CHAM(RMSNorm(h));
 * SSSDAttention's per-head RMSNorm, sssd_attention.py:177-182; CHAM's output RMSNorm,
 * cham_memory.py:241).  RMSNorm as torch.nn.RMSNorm: x * rsqrt(mean(x^2) + eps) in fp32,
 * rounded to the dtype, then times the weight (rounded); no weight when weight is NULL.
 * Rows of `cols` contiguous elements; cols % 8 == 0, cols <= 2048.
 * verace_rmsnorm:     y = RMSNorm(x)                   (x and y may alias)
 * verace_add_rmsnorm: h <- h + (norm_y ? RMSNorm(y; y_weight, y_eps) : y), in place;
 *                     then n = RMSNorm(h; n_weight, n_eps) when n is not NULL.
 * ---------------------------------------------------------------------------- */
VERACE_API int verace_rmsnorm(const void* x, const void* weight, void* y, long long rows, int cols, float eps,
                              int dtype, void* stream);
VERACE_API int verace_add_rmsnorm(void* h, const void* y, int norm_y, const void* y_weight, float y_eps,
                                  const void* n_weight, float n_eps, void* n, long long rows, int cols, int dtype,
                                  void* stream);

/* ------------------------------------------------------------------------------
 * M-CMoE (Manifold Continuous Mixture-of-Experts), ManifoldContinuousMoE.forward
 * (verace_v1/modules/mcmoe.py:58-120).
 * verace_mcmoe_route: the router's top-K and gate weights (mcmoe.py:91-96): for each of
 *   n rows of C logits, the K largest (descending; NaN ranks first, ties to the lower
 *   index) as int64 indices [n][K] and softmax over those K logits [n][K] in `dtype`.
 *   C <= 256, K <= min(C, 16).
 * verace_mcmoe_projection: replaces launch_mcmoe_triton_projection
 *   (verace_v1/serving/triton_kernels.py:688-723; kernel :313-353):
 *   out[t] = sum_k w[t,k] U[c] (sigma[t,c,:] * (V[c] x_t)),  c = idx[t,k], with x [n][d],
 *   u_basis [C][d][r], v_basis [C][r][d], idx/w [n][K], sigma [n][C][r], out [n][d], all
 *   in `dtype` except idx (int64).  sigma_is_logits != 0: sigma holds the hyper-network's
 *   pre-activation and sigmoid (rounded to dtype) is applied inside.  bf16 with
 *   d % 128 == 0 and C*r % 128 == 0 runs on the tensor cores and needs
 *   verace_mcmoe_workspace bytes of workspace; other cases need none.
 * verace_situ_glu: SiTUGLU.forward's activation (verace_v1/modules/activations.py):
 *   out = [b1 tanh(g/b1) sigmoid(g)] * [b2 tanh(u/b2)] elementwise over [n][cols], g and
 *   u with row stride ld (e.g. the two halves of one [n][2 cols] projection), out dense.
 * ---------------------------------------------------------------------------- */
VERACE_API size_t verace_mcmoe_workspace(long long n, int d, int C, int r, int dtype);
VERACE_API int verace_mcmoe_route(const void* logits, long long n, int C, int K, long long* idx, void* weights,
                                  int dtype, void* stream);
VERACE_API int verace_mcmoe_projection(const void* x, const void* u_basis, const void* v_basis, const long long* idx,
                                       const void* weights, const void* sigma, int sigma_is_logits, void* out,
                                       long long n, int d, int C, int r, int K, int dtype, void* workspace,
                                       size_t workspace_bytes, void* stream);
VERACE_API int verace_situ_glu(const void* gate, const void* up, long long ld, void* out, long long n, int cols,
                               float beta1, float beta2, int dtype, void* stream);

enum { VERACE_DECODE_UNITARY = 0, VERACE_DECODE_FIRST_ORDER = 1 };
VERACE_API size_t verace_decode_workspace(int b, int D);
VERACE_API int verace_decode_step(const void* sssd_q, const void* sssd_k, const void* sssd_v,
                                  const float* delta, float* psi, void* sssd_out,
                                  const void* cham_q, const void* cham_k, const void* cham_v,
                                  const float* gamma, float* h_re, float* h_im, void* cham_out,
                                  int b, int h, int d, int D, int dtype, int mode,
                                  void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* VERACE_B200_H_ */
