"""numpy restatement of the reference's eager (pure-PyTorch) SSSD and CHAM algorithms.

TEST INFRASTRUCTURE ONLY -- the parity checker for the CUDA path and the timed CPU
baseline.  The product package never imports it.

Every function follows the reference's *eager* path (the path the reference trains
with, and the one its tests treat as ground truth), not its Triton kernels:

* SSSD  -- ``verace_v1/modules/sssd_attention.py``
    projections / L2-normalise / delta gate      :116-126
    Cayley factor R = solve(I + X, I - X), X=δA/2 :154-166  (``_solve_cayley`` :21-72)
    prefix product P_t = R_t ... R_1 (newest left):169      (``parallel_prefix_scan`` :185-217)
    Ψ_t = P_t Ψ_0,  o_t = Ψ_t q_t                  :173-175
    head RMSNorm + w_out, state = Ψ_s              :177-181
* CHAM  -- ``verace_v1/modules/cham_memory.py``
    projections, v = normalize(silu(.)), γ gate    :129-153
    U = solve(I - iG/2, I + iG/2), G=γ(kvᵀ+vkᵀ)   :211-218  (``_solve_cham_cayley`` :54-96)
    prefix product P_t = U_t ... U_1               :222     (``parallel_complex_prefix_scan`` :246-293)
    H_t = P_t H_0 (H_0 on the right)               :229-230
    per-position Newton-Schulz x3                  :236     (``parallel_newton_schulz_retraction`` :296-315)
    (``cham_scan_rank2``: the same scan in O(D^2) per token by the reference Triton
    kernel's Woodbury form, triton_kernels.py:152-306, for long sequences at D = 1024)
    rec_t = Re(NS(H_t)) q_t, y = RMSNorm(w_out rec):239-241
    exported state = raw H_s (never retracted)     :243
* ``newton_schulz_unitary_retraction``             cham_memory.py:21-51
* M-CMoE -- ``verace_v1/modules/mcmoe.py``, ``verace_v1/modules/activations.py``
    base FFN w_down(SiTU-GLU(x))                  :66   (``SiTUGLU.forward``)
    router top-K, softmax over the kept logits     :91-96
    sigma = sigmoid(hyper_sigma x)                 :98
    manifold = sum_k w_k U_c (sigma_c * (V_c x))   :108-117 (eager loop)
    y = base + RMSNorm(manifold)                   :119

The prefix products are formed sequentially (P_t = R_t P_{t-1}); the reference's
Blelloch scan forms the same products in a different association order, which only
changes fp rounding.  Non-finite Cayley factors are replaced by the identity, as the
reference's ``_solve_cayley`` / ``_solve_cham_cayley`` do (sssd_attention.py:52-71,
cham_memory.py:76-96).

``dtype`` selects the arithmetic: ``np.float32`` mirrors the reference's fp32 eager
path (complex64 for CHAM); ``np.float64`` is the fp64 gold in the style of
``tests/test_triton_kernels.py:35-83`` (``_cham_fp64_reference``).
"""

from __future__ import annotations

import numpy as np

__all__ = [
    "l2_normalize", "sigmoid", "silu", "rms_norm",
    "sssd_cayley_factors", "sssd_scan", "sssd_forward",
    "cham_cayley_factors", "cham_scan", "cham_forward", "cham_scan_rank2", "cham_scan_rank2_c", "ns_polynomial",
    "newton_schulz_unitary_retraction", "sssd_projections", "cham_projections",
    "situ_glu", "mcmoe_route", "mcmoe_projection", "mcmoe_forward",
]


# --------------------------------------------------------------------------------------
# elementwise helpers (torch semantics)
# --------------------------------------------------------------------------------------
def l2_normalize(x, eps=1e-12):
    """``F.normalize(x, p=2, dim=-1)``: x / max(||x||_2, eps)."""
    n = np.sqrt(np.sum(x * x, axis=-1, keepdims=True))
    return x / np.maximum(n, eps)


def sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


def silu(x):
    return x * sigmoid(x)


def rms_norm(x, weight, eps=None):
    """``nn.RMSNorm``: eps=None means ``finfo(dtype).eps`` (torch's default)."""
    if eps is None:
        eps = np.finfo(x.dtype).eps
    ms = np.mean(x * x, axis=-1, keepdims=True)
    return (x / np.sqrt(ms + eps)) * weight


def _linear(x, w):
    return x @ w.T


# --------------------------------------------------------------------------------------
# SSSD
# --------------------------------------------------------------------------------------
def sssd_projections(p, x, num_heads, head_dim, active_mask=None):
    """sssd_attention.py:116-126 -> q, k, v [b,s,h,d], delta [b,s,h]."""
    b, s, _ = x.shape
    q = l2_normalize(_linear(x, p["w_q.weight"]).reshape(b, s, num_heads, head_dim))
    k = l2_normalize(_linear(x, p["w_k.weight"]).reshape(b, s, num_heads, head_dim))
    v = l2_normalize(_linear(x, p["w_v.weight"]).reshape(b, s, num_heads, head_dim))
    delta = 0.1 * sigmoid(_linear(x, p["w_delta.weight"]))  # [b,s,h]
    if active_mask is not None:
        delta = delta * active_mask[..., None].astype(delta.dtype)
    return q, k, v, delta


def sssd_cayley_factors(k, v, delta):
    """R = solve(I + δA/2, I - δA/2), A = k vᵀ - v kᵀ  (sssd_attention.py:154-166).

    k, v: [..., d]; delta: [...].  Returns R: [..., d, d]."""
    d = k.shape[-1]
    eye = np.eye(d, dtype=k.dtype)
    A = k[..., :, None] * v[..., None, :] - v[..., :, None] * k[..., None, :]
    X = 0.5 * delta[..., None, None] * A
    R = np.linalg.solve(eye + X, eye - X)
    bad = ~np.isfinite(R).all(axis=(-1, -2))
    if bad.any():  # _solve_cayley's identity substitution (sssd_attention.py:52-71)
        R[bad] = eye
    return R


def sssd_scan(q, k, v, delta, initial_state=None, dtype=np.float64):
    """Launcher-level SSSD scan (the contract of ``launch_sssd_triton_scan``,
    triton_kernels.py:603-636), computed by the eager algorithm.

    q, k, v: [b,s,h,d]; delta: [b,s,h]; initial_state: [b,h,d,d] or None (identity).
    Returns (o [b,s,h,d], psi [b,h,d,d])."""
    q, k, v, delta = (np.asarray(a, dtype=dtype) for a in (q, k, v, delta))
    b, s, h, d = q.shape
    if initial_state is None:
        psi0 = np.broadcast_to(np.eye(d, dtype=dtype), (b, h, d, d)).copy()
    else:
        psi0 = np.asarray(initial_state, dtype=dtype)
    o = np.zeros((b, s, h, d), dtype=dtype)
    P = np.broadcast_to(np.eye(d, dtype=dtype), (b, h, d, d)).copy()
    psi = psi0.copy()
    for t in range(s):
        R = sssd_cayley_factors(k[:, t], v[:, t], delta[:, t])  # [b,h,d,d]
        P = R @ P                                              # P_t = R_t P_{t-1}
        psi = P @ psi0                                         # Ψ_t = P_t Ψ_0
        o[:, t] = (psi @ q[:, t, :, :, None])[..., 0]
    return o, psi


def sssd_forward(p, x, num_heads, head_dim, initial_state=None, return_state=False,
                 active_mask=None, dtype=np.float64, norm_eps=None):
    """``SSSDAttention.forward`` (sssd_attention.py:103-182), eager path.  ``norm_eps``: the
    head RMSNorm's eps (None: the machine epsilon of ``dtype``, as torch.nn.RMSNorm(eps=None)
    does for its input's dtype; a model run in bf16 uses bf16's)."""
    x = np.asarray(x, dtype=dtype)
    p = {n: np.asarray(w, dtype=dtype) for n, w in p.items()}
    b, s, _ = x.shape
    q, k, v, delta = sssd_projections(p, x, num_heads, head_dim, active_mask)
    o, psi = sssd_scan(q, k, v, delta, initial_state, dtype=dtype)
    o_norm = rms_norm(o, p["head_rmsnorm.weight"], norm_eps).reshape(b, s, num_heads * head_dim)
    out = _linear(o_norm, p["w_out.weight"])
    return out, (psi if return_state else None)


# --------------------------------------------------------------------------------------
# CHAM
# --------------------------------------------------------------------------------------
def cham_projections(p, x, active_mask=None):
    """cham_memory.py:129-153 -> q, k, v [b,s,D], gamma [b,s]."""
    q = l2_normalize(_linear(x, p["w_q.weight"]))
    k = l2_normalize(_linear(x, p["w_k.weight"]))
    v = l2_normalize(silu(_linear(x, p["w_v.weight"])))
    gamma = 0.1 * sigmoid(_linear(x, p["w_gamma.weight"]))[..., 0]
    if active_mask is not None:
        gamma = gamma * active_mask.astype(gamma.dtype)
    return q, k, v, gamma


def _cdtype(dtype):
    return np.complex128 if np.dtype(dtype) == np.float64 else np.complex64


def cham_cayley_factors(k, v, gamma):
    """U = solve(I - iG/2, I + iG/2), G = γ(k vᵀ + v kᵀ)  (cham_memory.py:211-218)."""
    D = k.shape[-1]
    cd = _cdtype(k.dtype)
    eye = np.eye(D, dtype=cd)
    G = gamma[..., None, None] * (k[..., :, None] * v[..., None, :] + v[..., :, None] * k[..., None, :])
    G = G.astype(cd)
    U = np.linalg.solve(eye - 0.5j * G, eye + 0.5j * G)
    bad = ~np.isfinite(U).all(axis=(-1, -2))
    if bad.any():  # _solve_cham_cayley's identity substitution (cham_memory.py:76-96)
        U[bad] = eye
    return U


def newton_schulz_unitary_retraction(H_real, H_imag, steps=3):
    """cham_memory.py:21-51: H <- 0.5 H (3I - Hᴴ H), both parts from the same pre-update H."""
    H = np.asarray(H_real) + 1j * np.asarray(H_imag)
    D = H.shape[-1]
    eye = np.eye(D, dtype=H.dtype)
    for _ in range(steps):
        HH = np.conj(np.swapaxes(H, -1, -2)) @ H
        H = 0.5 * (H @ (3.0 * eye - HH))
    return H.real.copy(), H.imag.copy()


def cham_scan(q, k, v, gamma, initial_hologram=None, dtype=np.float64, ns_steps=3):
    """Launcher-level CHAM scan (contract of ``launch_cham_triton_update``,
    triton_kernels.py:639-685) computed by the eager algorithm, including the
    per-position Newton-Schulz retraction of the readout.

    q, k, v: [b,s,D]; gamma: [b,s]; initial_hologram: (Hr, Hi) [b,D,D] or None (I, 0).
    Returns (rec [b,s,D], (Hr_raw, Hi_raw) [b,D,D])."""
    q, k, v, gamma = (np.asarray(a, dtype=dtype) for a in (q, k, v, gamma))
    b, s, D = q.shape
    cd = _cdtype(dtype)
    if initial_hologram is None:
        H0 = np.broadcast_to(np.eye(D, dtype=cd), (b, D, D)).copy()
    else:
        H0 = (np.asarray(initial_hologram[0], dtype=dtype)
              + 1j * np.asarray(initial_hologram[1], dtype=dtype)).astype(cd)
    P = np.broadcast_to(np.eye(D, dtype=cd), (b, D, D)).copy()
    Hraw = H0.copy()
    rec = np.zeros((b, s, D), dtype=dtype)
    for t in range(s):
        U = cham_cayley_factors(k[:, t], v[:, t], gamma[:, t])  # [b,D,D]
        P = U @ P                       # P_t = U_t P_{t-1}
        Hraw = P @ H0                   # H_t = P_t H_0
        Hr, _ = newton_schulz_unitary_retraction(Hraw.real, Hraw.imag, ns_steps)
        rec[:, t] = (Hr @ q[:, t, :, None])[..., 0]
    return rec, (Hraw.real.astype(dtype), Hraw.imag.astype(dtype))


def ns_polynomial(H0, steps=3):
    """p(A) with A = H0ᴴ H0 such that NS^steps(H) = H p(A) for every H with Hᴴ H = A.

    One Newton-Schulz step (cham_memory.py:21-51) maps H to H g(A), g(X) = (3I - X)/2, and
    then (H g(A))ᴴ (H g(A)) = A g(A)^2 (g(A) commutes with A), so three steps give
    H g(A0) g(A1) g(A2) with A_{j+1} = A_j g(A_j)^2."""
    D = H0.shape[-1]
    eye = np.eye(D, dtype=H0.dtype)
    A = np.conj(np.swapaxes(H0, -1, -2)) @ H0
    poly = np.broadcast_to(eye, A.shape).copy()
    for _ in range(steps):
        g = 0.5 * (3.0 * eye - A)
        poly = poly @ g
        A = A @ g @ g
    return poly


def cham_scan_rank2(q, k, v, gamma, initial_hologram=None, dtype=np.float64, ns_steps=3, dense_ns_at=()):
    """The CHAM scan of ``cham_scan`` in O(D^2) per token, for long sequences at D = 1024.

    State update: the reference's own Woodbury form of the exact Cayley factor
    (triton_kernels.py:152-306, the per-token comment there): U_t = (I - iG/2)^-1 (I + iG/2)
    with G = γ W J Wᵀ, W = [k v], J = [[0, 1], [1, 0]], so with B = (iγ/2) J and
    K = (I2 - B WᵀW)^-1 B (Sherman-Morrison-Woodbury, no 1/γ):
        Y = H + W (B (Wᵀ H)),   U_t H = Y + W (K (Wᵀ Y)).
    H_t = U_t H_{t-1} from H_0 (the same product as P_t H_0 of cham_memory.py:222-230, in
    sequential order).  A non-finite factor leaves the state unchanged (the identity
    substitution of cham_memory.py:76-96).

    Readout: rec_t = Re(NS^3(H_t) q_t) (cham_memory.py:236-239) evaluated as
    Re(H_t p(A) q_t) with p = ``ns_polynomial`` of A = H_0ᴴ H_0: every U_t is unitary, so
    H_tᴴ H_t = A for all t and NS^3(H_t) = H_t p(A) exactly in exact arithmetic.  For the
    positions in ``dense_ns_at`` the readout is also formed by the dense retraction of H_t
    (``newton_schulz_unitary_retraction``) and returned in a dict, so a caller can check
    the identity on its own inputs.

    Returns (rec [b,s,D], (Hr, Hi) [b,D,D], {t: dense rec_t [b,D]})."""
    q, k, v, gamma = (np.asarray(a, dtype=dtype) for a in (q, k, v, gamma))
    b, s, D = q.shape
    cd = _cdtype(dtype)
    if initial_hologram is None:
        H = np.broadcast_to(np.eye(D, dtype=cd), (b, D, D)).copy()
    else:
        H = (np.asarray(initial_hologram[0], dtype=dtype)
             + 1j * np.asarray(initial_hologram[1], dtype=dtype)).astype(cd)
    poly = ns_polynomial(H, ns_steps)
    J = np.array([[0.0, 1.0], [1.0, 0.0]], dtype=cd)
    I2 = np.eye(2, dtype=cd)
    rec = np.zeros((b, s, D), dtype=dtype)
    dense = {}
    want = set(int(t) for t in dense_ns_at)
    for t in range(s):
        for i in range(b):
            W = np.stack([k[i, t], v[i, t]], axis=1).astype(cd)          # [D, 2]
            B = 0.5j * gamma[i, t] * J
            with np.errstate(all="ignore"):
                K = np.linalg.solve(I2 - B @ (W.T @ W), B)
                Y = H[i] + W @ (B @ (W.T @ H[i]))
                Hn = Y + W @ (K @ (W.T @ Y))
            if np.isfinite(Hn).all():
                H[i] = Hn
        rec[:, t] = np.real(H @ (poly @ q[:, t, :, None].astype(cd)))[..., 0]
        if t in want:
            Hr, _ = newton_schulz_unitary_retraction(H.real, H.imag, ns_steps)
            dense[t] = (Hr @ q[:, t, :, None])[..., 0]
    return rec, (H.real.astype(dtype), H.imag.astype(dtype)), dense


_CLIB = None


def _clib():
    """oracle/_liboracle.so (``cham_rank2.c``), built on first use."""
    global _CLIB
    if _CLIB is None:
        import ctypes
        import importlib.util
        import os
        here = os.path.dirname(os.path.abspath(__file__))
        spec = importlib.util.spec_from_file_location("oracle_build", os.path.join(here, "build.py"))
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        L = ctypes.CDLL(mod.build())
        dp = ctypes.c_void_p
        L.cham_rank2_scan.restype = None
        L.cham_rank2_scan.argtypes = [ctypes.c_int] * 3 + [dp] * 9
        _CLIB = L
    return _CLIB


def cham_scan_rank2_c(q, k, v, gamma, initial_hologram=None, ns_steps=3):
    """``cham_scan_rank2`` (fp64) computed by ``cham_rank2.c``: same arguments and results,
    without the dense check.  Returns (rec [b,s,D], (Hr, Hi) [b,D,D])."""
    q, k, v, gamma = (np.ascontiguousarray(a, dtype=np.float64) for a in (q, k, v, gamma))
    b, s, D = q.shape
    if initial_hologram is None:
        Hr = np.ascontiguousarray(np.broadcast_to(np.eye(D), (b, D, D)))
        Hi = np.zeros((b, D, D))
        pr = pi = None
    else:
        Hr = np.array(initial_hologram[0], dtype=np.float64, order="C")
        Hi = np.array(initial_hologram[1], dtype=np.float64, order="C")
        poly = ns_polynomial(Hr + 1j * Hi, ns_steps)
        pr, pi = np.ascontiguousarray(poly.real), np.ascontiguousarray(poly.imag)
    rec = np.zeros((b, s, D))
    ptr = lambda a: None if a is None else a.ctypes.data
    _clib().cham_rank2_scan(b, s, D, ptr(q), ptr(k), ptr(v), ptr(gamma), ptr(Hr), ptr(Hi), ptr(pr), ptr(pi),
                            ptr(rec))
    return rec, (Hr, Hi)


def cham_forward(p, x, initial_hologram=None, active_mask=None, dtype=np.float64, norm_eps=None, rank2=False):
    """``ContinuousHolographicMemory.forward`` (cham_memory.py:117-243), eager path."""
    x = np.asarray(x, dtype=dtype)
    p = {n: np.asarray(w, dtype=dtype) for n, w in p.items()}
    q, k, v, gamma = cham_projections(p, x, active_mask)
    if rank2:   # the same scan in O(D^2) per token (fp64, cham_rank2.c)
        rec, H = cham_scan_rank2_c(q, k, v, gamma, initial_hologram)
    else:
        rec, H = cham_scan(q, k, v, gamma, initial_hologram, dtype=dtype)
    y = rms_norm(_linear(rec, p["w_out.weight"]), p["norm.weight"], norm_eps)
    return y, H


# --------------------------------------------------------------------------------------
# M-CMoE
# --------------------------------------------------------------------------------------
def situ_glu(p, x, beta1=4.0, beta2=25.0, prefix="base_situ_glu."):
    """``SiTUGLU.forward`` (activations.py): [b1 tanh(g/b1) sigmoid(g)] * [b2 tanh(u/b2)]."""
    g = _linear(x, p[prefix + "w_gate.weight"])
    u = _linear(x, p[prefix + "w_up.weight"])
    return (beta1 * np.tanh(g / beta1) * sigmoid(g)) * (beta2 * np.tanh(u / beta2))


def mcmoe_route(logits, k):
    """Top-k of each row (descending; ties to the lower index) and the softmax over the
    kept logits, i.e. softmax of the row with the others masked to -inf (mcmoe.py:91-96).
    Returns (indices [n, k], weights [n, k])."""
    logits = np.asarray(logits)
    idx = np.argsort(-logits, axis=-1, kind="stable")[:, :k]
    top = np.take_along_axis(logits, idx, -1)
    e = np.exp(top - top[:, :1])
    return idx, e / e.sum(-1, keepdims=True)


def mcmoe_projection(x, u_basis, v_basis, idx, w, sigma):
    """The eager loop of mcmoe.py:108-117 (and the reference kernel's formula):
    out[t] = sum_k w[t,k] U[c] (sigma[t,c,:] * (V[c] x_t)),  c = idx[t,k].
    x [n,d], u_basis [C,d,r], v_basis [C,r,d], idx/w [n,K], sigma [n,C,r]."""
    n, d = x.shape
    out = np.zeros((n, d), dtype=np.result_type(x, u_basis))
    rows = np.arange(n)
    for k in range(idx.shape[1]):
        c = idx[:, k]
        vp = np.einsum("nrd,nd->nr", v_basis[c], x) * sigma[rows, c]
        out += w[:, k:k + 1] * np.einsum("ndr,nr->nd", u_basis[c], vp)
    return out


def mcmoe_forward(p, x, rank, num_components, top_k, beta1=4.0, beta2=25.0, dtype=np.float64, norm_eps=None):
    """``ManifoldContinuousMoE.forward`` (mcmoe.py:58-120), eager path.  norm_eps None means
    the fp32 machine epsilon (torch.nn.RMSNorm(eps=None) on fp32 activations)."""
    x = np.asarray(x, dtype=dtype)
    p = {n: np.asarray(w, dtype=dtype) for n, w in p.items()}
    b, s, d = x.shape
    xf = x.reshape(b * s, d)
    base = _linear(situ_glu(p, xf, beta1, beta2), p["base_w_down.weight"])
    k = min(top_k, num_components)
    idx, w = mcmoe_route(_linear(xf, p["router.weight"]), k)
    sig = sigmoid(_linear(xf, p["hyper_sigma.weight"])).reshape(b * s, num_components, rank)
    m = mcmoe_projection(xf, p["u_basis"], p["v_basis"], idx, w, sig)
    eps = np.finfo(np.float32).eps if norm_eps is None else norm_eps
    y = base + rms_norm(m, p["norm.weight"], eps)
    return y.reshape(b, s, d)
