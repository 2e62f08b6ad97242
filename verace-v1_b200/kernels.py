"""Launchers for the sm_100a SSSD / CHAM kernels, with the reference launchers' contracts.

``launch_sssd_scan`` and ``launch_cham_update`` take and return exactly what the
reference's ``launch_sssd_triton_scan`` / ``launch_cham_triton_update``
(verace_v1/serving/triton_kernels.py:603-636, :639-685) take and return, so they are
drop-ins for them; both names are exported as aliases too.  Differences in behaviour:

* the CHAM readout applies the Newton-Schulz retraction of the eager path
  (cham_memory.py:236-239) for every holographic width (the reference's D > 128
  Triton fallback loops on the host per token);
* non-CUDA inputs raise ``AssertionError("This kernel requires CUDA tensors")``, as
  the reference launchers do (triton_kernels.py:616, 652).

Outputs are freshly allocated; inputs are never modified; states are fp32.  Kernels
are enqueued on torch's current CUDA stream.
"""
from typing import Optional, Tuple

import torch

from ._lib import BF16, F16, F32, check, lib

_DTYPE = {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16}


def _prep(x: torch.Tensor) -> torch.Tensor:
    if x.dtype not in _DTYPE:
        x = x.float()
    return x.contiguous()


def _stream(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _workspace(nbytes: int, device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 1), dtype=torch.uint8, device=device)


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def launch_sssd_scan(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, delta: torch.Tensor,
                     initial_state: Optional[torch.Tensor] = None, *, _ranges: bool = True
                     ) -> Tuple[torch.Tensor, torch.Tensor]:
    """q, k, v: [b, s, h, d] (L2-normalised); delta: [b, s, h]; initial_state:
    optional [b, h, d, d] (identity when None).
    Returns (out [b, s, h, d] in q's dtype, final_state [b, h, d, d] fp32).
    Long sequences on few chains run as parallel sequence ranges (ranges.py)."""
    assert q.is_cuda, "This kernel requires CUDA tensors"
    b, s, h, d = q.shape
    if _ranges and b * h > 0 and not torch.cuda.is_current_stream_capturing():
        from .ranges import pick_ranges, sssd_scan_ranges
        R = pick_ranges(b * h, s, q.device, per_sm=1)
        if R > 1:
            return sssd_scan_ranges(q, k, v, delta, initial_state, R)
    q_c = _prep(q)
    dt = q_c.dtype
    k_c = k.to(dt).contiguous()
    v_c = v.to(dt).contiguous()
    delta_c = delta.reshape(b, s, h).float().contiguous()
    psi0 = None if initial_state is None else initial_state.float().contiguous()
    out = torch.empty_like(q_c)
    psi_out = torch.empty(b, h, d, d, device=q.device, dtype=torch.float32)
    L = lib()
    nbytes = L.verace_sssd_scan_workspace(b, s, h, d)
    ws = _workspace(nbytes, q.device)
    with torch.cuda.device(q.device):
        rc = L.verace_sssd_scan(q_c.data_ptr(), k_c.data_ptr(), v_c.data_ptr(), delta_c.data_ptr(),
                                _ptr(psi0), out.data_ptr(), psi_out.data_ptr(), b, s, h, d,
                                _DTYPE[dt], ws.data_ptr(), ws.numel(), _stream(q.device))
    check(rc, "verace_sssd_scan")
    return out, psi_out


# A carried hologram H0 whose unitarity probe (hologram_unitarity) is at most this continues
# on the scan that reads out Re(H_t q_t) (verace_cham_scan_unitary, the tensor cores at
# D % 128 == 0); that readout differs from the Newton-Schulz one by |(H0ᴴH0 - I) q| / 2
# (+ O(|E|^2)), i.e. by about the probe value, and at most sqrt(D) times it for a rank-one
# drift.  Holograms grown by these scans are unitary to ~1e-5 in bf16 runs.  Above it, the
# exact readout polynomial runs (verace_cham_scan).
UNITARY_TOL = {torch.float32: 2e-6, torch.bfloat16: 5e-4, torch.float16: 5e-4}
# One-token continuations take the decode kernel's first-order readout Re(U H (q - E q / 2)),
# which differs from the Newton-Schulz one by O(|E|^2): far looser probes qualify.
FIRST_ORDER_TOL = {torch.float32: 1e-4, torch.bfloat16: 1e-3, torch.float16: 1e-3}
# which path the last launch_cham_update call with a carried hologram took: "unitary",
# "first_order" or "exact" (for tests and diagnostics)
last_carried_path = None


def hologram_unitarity(H_real: torch.Tensor, H_imag: torch.Tensor) -> torch.Tensor:
    """eps [b] fp32 on the device: max over four fixed +-1 probe vectors r of
    |(Hᴴ H - I) r| / |r| per item, computed in fp64 (verace_cham_unitarity)."""
    assert H_real.is_cuda, "This kernel requires CUDA tensors"
    hr = H_real.float().contiguous()
    hi = H_imag.float().contiguous()
    b, D = hr.shape[0], hr.shape[-1]
    eps = torch.empty(b, device=hr.device, dtype=torch.float32)
    L = lib()
    ws = _workspace(L.verace_cham_unitarity_workspace(b, D), hr.device)
    with torch.cuda.device(hr.device):
        rc = L.verace_cham_unitarity(hr.data_ptr(), hi.data_ptr(), b, D, eps.data_ptr(), ws.data_ptr(), ws.numel(),
                                     _stream(hr.device))
    check(rc, "verace_cham_unitarity")
    return eps


def _carried_path(h0r: torch.Tensor, h0i: torch.Tensor, s: int, D: int, dt: torch.dtype) -> str:
    """Pick the continuation for a carried hologram: one host read of its unitarity probe
    (no read while the stream is being captured: the exact path then)."""
    if torch.cuda.is_current_stream_capturing():
        return "exact"
    eps = float(hologram_unitarity(h0r, h0i).max())
    if s == 1 and D % 32 == 0 and D <= 2048 and eps <= FIRST_ORDER_TOL[dt]:
        return "first_order"
    return "unitary" if eps <= UNITARY_TOL[dt] else "exact"


def launch_cham_update(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, gamma: torch.Tensor,
                       initial_hologram: Optional[Tuple[torch.Tensor, torch.Tensor]] = None, *,
                       _ranges: bool = True
                       ) -> Tuple[torch.Tensor, Tuple[torch.Tensor, torch.Tensor]]:
    """q, k, v: [b, s, D]; gamma: [b, s]; initial_hologram: optional (H_real, H_imag)
    [b, D, D] ((I, 0) when None).
    Returns (out [b, s, D] in q's dtype, (H_real, H_imag) [b, D, D] fp32 raw state).

    A carried hologram is checked for unitarity first (one host read): a unitary one
    continues on the tensor-core scan (one token: the fused decode kernel), any other on
    the exact Newton-Schulz readout polynomial; see UNITARY_TOL.  Long sequences on few
    holograms run as parallel sequence ranges (ranges.py)."""
    global last_carried_path
    assert q.is_cuda, "This kernel requires CUDA tensors"
    b, s, D = q.shape
    if _ranges and b > 0 and D % 32 == 0 and not torch.cuda.is_current_stream_capturing():
        from .ranges import cham_scan_ranges, pick_ranges
        R = pick_ranges(b * (D // 32), s, q.device, per_sm=2)
        if R > 1:
            return cham_scan_ranges(q, k, v, gamma, initial_hologram, R)
    q_c = _prep(q)
    dt = q_c.dtype
    k_c = k.to(dt).contiguous()
    v_c = v.to(dt).contiguous()
    g_c = gamma.reshape(b, s).float().contiguous()
    path = None
    if initial_hologram is None:
        h0r = h0i = None
    else:
        h0r = initial_hologram[0].float().contiguous()
        h0i = initial_hologram[1].float().contiguous()
        if s > 0 and b > 0:
            path = last_carried_path = _carried_path(h0r, h0i, s, D, dt)
    if path == "first_order":
        from .decode import launch_decode_step
        hr, hi = h0r.clone(), h0i.clone()
        _, out = launch_decode_step(None, (q_c.view(b, D), k_c.view(b, D), v_c.view(b, D), g_c.view(b), hr, hi),
                                    mode="first_order")
        return out.view(b, 1, D), (hr, hi)
    out = torch.empty(b, s, D, device=q.device, dtype=dt)
    hr = torch.empty(b, D, D, device=q.device, dtype=torch.float32)
    hi = torch.empty(b, D, D, device=q.device, dtype=torch.float32)
    L = lib()
    nbytes = L.verace_cham_scan_workspace(b, s, D, 0 if h0r is None else 1)
    ws = _workspace(nbytes, q.device)
    entry = L.verace_cham_scan_unitary if path == "unitary" else L.verace_cham_scan
    with torch.cuda.device(q.device):
        rc = entry(q_c.data_ptr(), k_c.data_ptr(), v_c.data_ptr(), g_c.data_ptr(),
                   _ptr(h0r), _ptr(h0i), out.data_ptr(), hr.data_ptr(), hi.data_ptr(),
                   b, s, D, _DTYPE[dt], ws.data_ptr(), ws.numel(), _stream(q.device))
    check(rc, "verace_cham_scan_unitary" if path == "unitary" else "verace_cham_scan")
    return out, (hr, hi)


def cham_retract(H_real: torch.Tensor, H_imag: torch.Tensor, steps: int = 3
                 ) -> Tuple[torch.Tensor, torch.Tensor]:
    """Dense Newton-Schulz retraction on CUDA (the contract of
    newton_schulz_unitary_retraction, cham_memory.py:21-51).  [b, D, D] fp32."""
    assert H_real.is_cuda, "This kernel requires CUDA tensors"
    hr = H_real.float().contiguous()
    hi = H_imag.float().contiguous()
    b, D, _ = hr.shape
    out_r = torch.empty_like(hr)
    out_i = torch.empty_like(hi)
    L = lib()
    ws = _workspace(L.verace_cham_retract_workspace(b, D), hr.device)
    with torch.cuda.device(hr.device):
        rc = L.verace_cham_retract(hr.data_ptr(), hi.data_ptr(), out_r.data_ptr(), out_i.data_ptr(),
                                   b, D, int(steps), ws.data_ptr(), ws.numel(), _stream(hr.device))
    check(rc, "verace_cham_retract")
    return out_r, out_i


def mixer_prologue(y: torch.Tensor, heads: int, head_dim: int, gate_cols: int, silu_v: bool,
                   active_mask: Optional[torch.Tensor] = None
                   ) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    """One pass over a concatenated projection y [n, ld] (row = q | k | v | gate): q, k, v
    [n, heads*head_dim] L2-normalised per head (v through SiLU first when `silu_v`), and
    gate [n, gate_cols] fp32 = 0.1 sigmoid(.) * mask.  The elementwise tail of
    sssd_attention.py:116-126 and cham_memory.py:129-153."""
    assert y.is_cuda, "This kernel requires CUDA tensors"
    y = _prep(y)
    n, ld = y.shape
    hd = heads * head_dim
    q = torch.empty(n, hd, device=y.device, dtype=y.dtype)
    k = torch.empty_like(q)
    v = torch.empty_like(q)
    gate = torch.empty(n, gate_cols, device=y.device, dtype=torch.float32)
    m = None
    if active_mask is not None:
        m = active_mask.reshape(n).to(torch.uint8).contiguous()
    with torch.cuda.device(y.device):
        rc = lib().verace_mixer_prologue(y.data_ptr(), ld, q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                         gate.data_ptr(), _ptr(m), n, heads, head_dim, gate_cols,
                                         1 if silu_v else 0, _DTYPE[y.dtype], _stream(y.device))
    check(rc, "verace_mixer_prologue")
    return q, k, v, gate


def concat_weights(module: torch.nn.Module, weights) -> torch.Tensor:
    """[W_q; W_k; W_v; W_gate] with zero rows up to a multiple of 8, cached on `module`
    and rebuilt whenever one of the weights is replaced or modified in place."""
    key = tuple((w.data_ptr(), w._version, w.dtype, w.device) for w in weights)
    cached = getattr(module, "_verace_cat", None)
    if cached is not None and cached[0] == key:
        return cached[1]
    with torch.no_grad():
        W = torch.cat([w.detach() for w in weights], dim=0)
        pad = (-W.shape[0]) % 8
        if pad:
            W = torch.cat([W, W.new_zeros(pad, W.shape[1])], dim=0)
    module._verace_cat = (key, W.contiguous())
    return module._verace_cat[1]


# drop-in aliases with the reference's launcher names
launch_sssd_triton_scan = launch_sssd_scan
launch_cham_triton_update = launch_cham_update


def _norm_args(norm: Optional[torch.nn.Module], x: torch.Tensor):
    """(weight pointer, eps) of a torch.nn.RMSNorm over x's last dimension (eps None means
    torch.finfo(x.dtype).eps, as torch.nn.RMSNorm does)."""
    if norm is None:
        return 0, 0.0
    assert tuple(norm.normalized_shape) == (x.shape[-1],), "RMSNorm must normalise the last dimension"
    eps = norm.eps if norm.eps is not None else torch.finfo(x.dtype).eps
    w = norm.weight
    if w is None:
        return 0, float(eps)
    assert w.dtype == x.dtype and w.is_contiguous() and w.device == x.device, \
        "RMSNorm weight must be contiguous, on the input's device and in its dtype"
    return w.data_ptr(), float(eps)


def fused_norm_supported(x: torch.Tensor) -> bool:
    """Whether rmsnorm / add_rmsnorm take rows of x's last dimension."""
    c = x.shape[-1]
    return x.dtype in _DTYPE and c % 8 == 0 and c <= 2048


def rmsnorm(x: torch.Tensor, norm: torch.nn.Module) -> torch.Tensor:
    """`norm` (a torch.nn.RMSNorm over the last dimension) applied to x in one pass."""
    assert x.is_cuda, "This kernel requires CUDA tensors"
    x = x.contiguous()
    y = torch.empty_like(x)
    w, eps = _norm_args(norm, x)
    cols = x.shape[-1]
    with torch.cuda.device(x.device):
        rc = lib().verace_rmsnorm(x.data_ptr(), w, y.data_ptr(), x.numel() // cols, cols, eps,
                                  _DTYPE[x.dtype], _stream(x.device))
    check(rc, "verace_rmsnorm")
    return y


def add_rmsnorm(h: torch.Tensor, y: torch.Tensor, y_norm: Optional[torch.nn.Module] = None,
                out_norm: Optional[torch.nn.Module] = None) -> Optional[torch.Tensor]:
    """A block's residual step in one pass: h <- h + (y_norm(y) if y_norm else y) in place
    (h contiguous), then out_norm(h) is returned (None without out_norm)."""
    assert h.is_cuda and h.is_contiguous(), "h must be a contiguous CUDA tensor (updated in place)"
    assert y.shape == h.shape and y.dtype == h.dtype, "h and y must match"
    y = y.contiguous()
    wy, ey = _norm_args(y_norm, h)
    wn, en = _norm_args(out_norm, h)
    n = torch.empty_like(h) if out_norm is not None else None
    cols = h.shape[-1]
    with torch.cuda.device(h.device):
        rc = lib().verace_add_rmsnorm(h.data_ptr(), y.data_ptr(), 1 if y_norm is not None else 0, wy, ey, wn, en,
                                      _ptr(n), h.numel() // cols, cols, _DTYPE[h.dtype], _stream(h.device))
    check(rc, "verace_add_rmsnorm")
    return n


def apply_rmsnorm(norm: torch.nn.Module, x: torch.Tensor) -> torch.Tensor:
    """norm(x) through the fused kernel where it applies (CUDA input, the weight in x's
    dtype, rows of a multiple of 8 up to 2048), else through the module itself."""
    w = getattr(norm, "weight", None)
    if (x.is_cuda and fused_norm_supported(x) and tuple(norm.normalized_shape) == (x.shape[-1],)
            and (w is None or (w.dtype == x.dtype and w.device == x.device))):
        return rmsnorm(x, norm)
    return norm(x)
