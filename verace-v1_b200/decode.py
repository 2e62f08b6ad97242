"""Batched incremental decode: one fused launch per layer and token for all items.

The reference decodes one token at a time through ``layer_states``
(verace_v1/serving/hyper_generate.py:58-77): every step calls each layer's
SSSDAttention.forward with ``initial_state`` and ContinuousHolographicMemory.forward
with ``initial_hologram`` (verace_v1/modules/backbone.py:53-101), per batch item inside
the ACDE loop (verace_v1/modules/acd_engine.py:94-156), and gets freshly allocated state
tensors back.  Here the states of all layers and items live in one resident container,
:class:`DecodeState`, and :func:`launch_decode_step` advances one layer of it by one
token for the whole batch, in place, with ``verace_decode_step``.

The per-item state tuples of the reference, ``(Psi [1, h, d, d], (H_re [1, D, D],
H_im [1, D, D]))`` per layer (acd_engine.py:46-60), convert both ways with
:meth:`DecodeState.from_layer_states` and :meth:`DecodeState.layer_states`.

Readout modes (the CHAM readout is Re(NS3(H) q), cham_memory.py:233-241):

* ``"unitary"``: Re(H q), exact when Hᴴ H = I.  Every state grown from an identity
  start (prefill with ``initial_hologram=None``, then decode) is unitary to fp32
  rounding.  One launch per layer.
* ``"first_order"``: Re(H (q - E q / 2)) with E = Hᴴ H - I, which leaves an O(|E|²)
  difference to NS3; one extra pass over H.  It also raises the device status
  (``device_status()``) when |E q| > 1e-2 |q|.

The default is ``"first_order"`` for fp32 inputs and ``"unitary"`` for bf16 / fp16.

Lazy hologram updates (unitary readout, :func:`launch_decode_cham_lazy`,
``DecodeState(pending_depth=P)``): the rank-2 step updates are kept as pending factors,
H = S + sum_j [k_j v_j] B_j, and folded into the stored planes S every P steps, so that a
step reads S once instead of reading it twice and writing it.  The stored planes are
the true state only after a flush (:func:`flush_pending`, ``DecodeState.flush``).
"""
from typing import List, Optional, Sequence, Tuple

import torch

from ._lib import BF16, F16, F32, check, lib

_DTYPE = {torch.float32: F32, torch.bfloat16: BF16, torch.float16: F16}
_MODE = {"unitary": 0, "first_order": 1}

_ws_cache = {}


def _workspace(b: int, D: int, device) -> torch.Tensor:
    n = int(lib().verace_decode_workspace(b, D))
    key = (torch.device(device), n)
    ws = _ws_cache.get(key)
    if ws is None:
        ws = torch.empty(n, dtype=torch.uint8, device=device)
        _ws_cache[key] = ws
    return ws


def _mode(mode: Optional[str], dt: torch.dtype) -> int:
    if mode is None:
        mode = "first_order" if dt == torch.float32 else "unitary"
    if mode not in _MODE:
        raise ValueError(f"unknown decode readout mode {mode!r} (expected one of {sorted(_MODE)})")
    return _MODE[mode]


def _vec(x: torch.Tensor, dt: torch.dtype) -> torch.Tensor:
    return x.to(dt).contiguous()


def launch_decode_step(sssd: Optional[Sequence[torch.Tensor]],
                       cham: Optional[Sequence[torch.Tensor]],
                       mode: Optional[str] = None,
                       workspace: Optional[torch.Tensor] = None
                       ) -> Tuple[Optional[torch.Tensor], Optional[torch.Tensor]]:
    """Advance one layer's SSSD and CHAM states by one token for every item, in place.

    sssd: (q, k, v, delta, psi) with q/k/v [b, h, d] (or [b, 1, h, d]), delta [b, h]
          (or [b, 1, h]) and psi [b, h, d, d] fp32 contiguous, overwritten; or None.
    cham: (q, k, v, gamma, H_real, H_imag) with q/k/v [b, D] (or [b, 1, D]), gamma [b]
          (or [b, 1]) and H_real/H_imag [b, D, D] fp32 contiguous, overwritten; or None.
    Returns (sssd_out [b, h, d], cham_out [b, D]) in the q dtype (None where skipped).
    """
    if sssd is None and cham is None:
        return None, None
    ref = (sssd or cham)[0]
    assert ref.is_cuda, "This kernel requires CUDA tensors"
    dt = ref.dtype if ref.dtype in _DTYPE else torch.float32
    dev = ref.device
    null = 0
    b = ref.shape[0]
    h = d = D = 0
    sp = [None] * 6
    cp = [None] * 7
    sout = cout = None
    keep = []
    if sssd is not None:
        q, k, v, delta, psi = sssd
        b, h, d = q.shape[0], q.shape[-2], q.shape[-1]
        assert psi.dtype == torch.float32 and psi.is_contiguous() and tuple(psi.shape) == (b, h, d, d), \
            "psi must be a contiguous fp32 [b, h, d, d] tensor (updated in place)"
        qs, ks, vs = (_vec(x.reshape(b, h, d), dt) for x in (q, k, v))
        ds = delta.reshape(b, h).float().contiguous()
        sout = torch.empty(b, h, d, device=dev, dtype=dt)
        keep += [qs, ks, vs, ds]
        sp = [qs.data_ptr(), ks.data_ptr(), vs.data_ptr(), ds.data_ptr(), psi.data_ptr(), sout.data_ptr()]
    if cham is not None:
        q, k, v, gamma, hr, hi = cham
        D = q.shape[-1]
        assert q.shape[0] == b, "SSSD and CHAM inputs must have the same batch"
        for H in (hr, hi):
            assert H.dtype == torch.float32 and H.is_contiguous() and tuple(H.shape) == (b, D, D), \
                "H_real / H_imag must be contiguous fp32 [b, D, D] tensors (updated in place)"
        qc, kc, vc = (_vec(x.reshape(b, D), dt) for x in (q, k, v))
        gc = gamma.reshape(b).float().contiguous()
        cout = torch.empty(b, D, device=dev, dtype=dt)
        keep += [qc, kc, vc, gc]
        cp = [qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), gc.data_ptr(), hr.data_ptr(), hi.data_ptr(),
              cout.data_ptr()]
    if workspace is None:
        workspace = _workspace(b, max(D, 1), dev)
    L = lib()
    with torch.cuda.device(dev):
        rc = L.verace_decode_step(*(p if p is not None else null for p in sp),
                                  *(p if p is not None else null for p in cp),
                                  b, h, d, D, _DTYPE[dt], _mode(mode, dt),
                                  workspace.data_ptr(), workspace.numel(),
                                  torch.cuda.current_stream(dev).cuda_stream)
    check(rc, "verace_decode_step")
    return sout, cout


def pending_storage(b: int, D: int, P: int, device="cuda") -> torch.Tensor:
    """Zero-filled pending-factor storage for one layer's holograms (an empty list)."""
    return torch.zeros(int(lib().verace_decode_pending_bytes(b, D, P)), dtype=torch.uint8, device=device)


_lazy_ws_cache = {}


def _lazy_workspace(b: int, D: int, device) -> torch.Tensor:
    n = int(lib().verace_decode_lazy_workspace(b, D))
    key = (torch.device(device), n)
    ws = _lazy_ws_cache.get(key)
    if ws is None:
        ws = torch.empty(n, dtype=torch.uint8, device=device)
        _lazy_ws_cache[key] = ws
    return ws


def launch_decode_cham_lazy(q, k, v, gamma, H_real, H_imag, pending: torch.Tensor, P: int,
                            workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One unitary-readout CHAM decode step with deferred hologram updates.

    q/k/v [b, D] (or [b, 1, D]), gamma [b] (or [b, 1]); H_real/H_imag [b, D, D] fp32, the
    stored planes; pending: storage from :func:`pending_storage` for these planes and P.
    Returns the readout [b, D] in q's dtype; the planes and the pending list are updated
    in place (the planes change only on the steps that fold the list into them)."""
    assert q.is_cuda, "This kernel requires CUDA tensors"
    dt = q.dtype if q.dtype in _DTYPE else torch.float32
    b, D = q.shape[0], q.shape[-1]
    for H in (H_real, H_imag):
        assert H.dtype == torch.float32 and H.is_contiguous() and tuple(H.shape) == (b, D, D), \
            "H_real / H_imag must be contiguous fp32 [b, D, D] tensors (updated in place)"
    assert pending.dtype == torch.uint8 and pending.numel() >= lib().verace_decode_pending_bytes(b, D, P), \
        "pending storage too small for (b, D, P)"
    qc, kc, vc = (_vec(x.reshape(b, D), dt) for x in (q, k, v))
    gc = gamma.reshape(b).float().contiguous()
    out = torch.empty(b, D, device=q.device, dtype=dt)
    if workspace is None:
        workspace = _lazy_workspace(b, D, q.device)
    with torch.cuda.device(q.device):
        rc = lib().verace_decode_cham_lazy(qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), gc.data_ptr(),
                                           H_real.data_ptr(), H_imag.data_ptr(), pending.data_ptr(), P,
                                           out.data_ptr(), b, D, _DTYPE[dt], workspace.data_ptr(),
                                           workspace.numel(), torch.cuda.current_stream(q.device).cuda_stream)
    check(rc, "verace_decode_cham_lazy")
    return out


def launch_decode_cham_lazy_projected(y: torch.Tensor, H_real, H_imag, pending: torch.Tensor, P: int,
                                      workspace: Optional[torch.Tensor] = None) -> torch.Tensor:
    """:func:`launch_decode_cham_lazy` from the layer's raw projection rows y [b, ld] (or
    [b, 1, ld]; row = q | k | v | gate of ContinuousHolographicMemory's concatenated
    projection, :meth:`ContinuousHolographicMemory.projection`), the projection epilogue
    (SiLU on v, L2 normalisation, the gate) run inside the step's first kernel."""
    assert y.is_cuda, "This kernel requires CUDA tensors"
    assert y.dtype in _DTYPE, f"unsupported dtype {y.dtype}"
    b, D = H_real.shape[0], H_real.shape[-1]
    for H in (H_real, H_imag):
        assert H.dtype == torch.float32 and H.is_contiguous() and tuple(H.shape) == (b, D, D), \
            "H_real / H_imag must be contiguous fp32 [b, D, D] tensors (updated in place)"
    assert pending.dtype == torch.uint8 and pending.numel() >= lib().verace_decode_pending_bytes(b, D, P), \
        "pending storage too small for (b, D, P)"
    y2 = y.reshape(b, y.shape[-1])
    assert y2.stride(-1) == 1, "projection rows must be contiguous"
    out = torch.empty(b, D, device=y.device, dtype=y.dtype)
    if workspace is None:
        workspace = _lazy_workspace(b, D, y.device)
    with torch.cuda.device(y.device):
        rc = lib().verace_decode_cham_lazy_projected(y2.data_ptr(), y2.stride(0), H_real.data_ptr(),
                                                     H_imag.data_ptr(), pending.data_ptr(), P, out.data_ptr(), b, D,
                                                     _DTYPE[y.dtype], workspace.data_ptr(), workspace.numel(),
                                                     torch.cuda.current_stream(y.device).cuda_stream)
    check(rc, "verace_decode_cham_lazy_projected")
    return out


def flush_pending(H_real: torch.Tensor, H_imag: torch.Tensor, pending: torch.Tensor, P: int) -> None:
    """Fold the pending factors into the stored planes and empty the list."""
    b, D = H_real.shape[0], H_real.shape[-1]
    with torch.cuda.device(H_real.device):
        rc = lib().verace_decode_cham_flush(H_real.data_ptr(), H_imag.data_ptr(), pending.data_ptr(), P, b, D,
                                            torch.cuda.current_stream(H_real.device).cuda_stream)
    check(rc, "verace_decode_cham_flush")


def device_status(device=None) -> int:
    """Synchronise and return (then clear) the library's device status: 0, or
    VERACE_ERR_TIMEOUT (5) / VERACE_ERR_STATE (6)."""
    dev = torch.device("cuda" if device is None else device)
    with torch.cuda.device(dev):
        return int(lib().verace_device_status(torch.cuda.current_stream(dev).cuda_stream))


class DecodeState:
    """Resident SSSD and CHAM states of ``layers`` layers for a batch of ``batch`` items.

    psi: [layers, batch, h, d, d] fp32; H_real, H_imag: [layers, batch, D, D] fp32,
    initialised to the identity (the reference's ``None`` state).  :meth:`step` advances
    one layer in place; a whole decode step calls it once per layer.

    With ``pending_depth`` P > 0 (the default, 8) unitary-readout CHAM steps defer their
    hologram updates (module docstring); H_real / H_imag then hold the stored part, and
    :meth:`flush` (called by :meth:`layer_states`, and before any step that needs the
    planes themselves) folds the pending factors in.
    """

    def __init__(self, layers: int, batch: int, num_heads: int, head_dim: int,
                 holographic_dim: int, device="cuda", pending_depth: int = 8):
        self.layers, self.batch = layers, batch
        self.h, self.d, self.D = num_heads, head_dim, holographic_dim
        eye_d = torch.eye(head_dim, device=device, dtype=torch.float32)
        eye_D = torch.eye(holographic_dim, device=device, dtype=torch.float32)
        self.psi = eye_d.expand(layers, batch, num_heads, head_dim, head_dim).contiguous()
        self.H_real = eye_D.expand(layers, batch, holographic_dim, holographic_dim).contiguous()
        self.H_imag = torch.zeros_like(self.H_real)
        self.workspace = _workspace(batch, holographic_dim, device)
        self.P = pending_depth
        if self.P > 0:
            nb = int(lib().verace_decode_pending_bytes(batch, holographic_dim, self.P))
            self.pending = torch.zeros(layers, nb, dtype=torch.uint8, device=device)
            self.lazy_workspace = _lazy_workspace(batch, holographic_dim, device)

    def _lazy(self, q: torch.Tensor, mode: Optional[str]) -> bool:
        return self.P > 0 and _mode(mode, q.dtype if q.dtype in _DTYPE else torch.float32) == 0

    def step(self, layer: int, sssd: Sequence[torch.Tensor], cham: Sequence[torch.Tensor],
             mode: Optional[str] = None) -> Tuple[torch.Tensor, torch.Tensor]:
        """sssd: (q, k, v, delta); cham: (q, k, v, gamma) of one token per item.
        Returns (sssd_out [b, h, d], cham_out [b, D])."""
        if self._lazy(cham[0], mode):
            return self.step_sssd(layer, *sssd, mode=mode), self.step_cham(layer, *cham, mode=mode)
        self.flush(layer)
        return launch_decode_step(tuple(sssd) + (self.psi[layer],),
                                  tuple(cham) + (self.H_real[layer], self.H_imag[layer]),
                                  mode=mode, workspace=self.workspace)

    def step_sssd(self, layer: int, q, k, v, delta, mode: Optional[str] = None) -> torch.Tensor:
        """SSSD half only (the layer's CHAM input depends on its SSSD output)."""
        return launch_decode_step((q, k, v, delta, self.psi[layer]), None, mode=mode,
                                  workspace=self.workspace)[0]

    def step_cham(self, layer: int, q, k, v, gamma, mode: Optional[str] = None) -> torch.Tensor:
        """CHAM half only (deferred updates for the unitary readout when pending_depth > 0)."""
        if self._lazy(q, mode):
            return launch_decode_cham_lazy(q, k, v, gamma, self.H_real[layer], self.H_imag[layer],
                                           self.pending[layer], self.P, workspace=self.lazy_workspace)
        self.flush(layer)
        return launch_decode_step(None, (q, k, v, gamma, self.H_real[layer], self.H_imag[layer]),
                                  mode=mode, workspace=self.workspace)[1]

    def step_cham_projected(self, layer: int, y: torch.Tensor, active_mask=None) -> torch.Tensor:
        """CHAM half from the layer's raw projection rows (unitary readout): with deferred
        updates the projection epilogue runs inside the step
        (:func:`launch_decode_cham_lazy_projected`); otherwise through the mixer prologue."""
        if self.P > 0 and active_mask is None:
            return launch_decode_cham_lazy_projected(y, self.H_real[layer], self.H_imag[layer],
                                                     self.pending[layer], self.P, workspace=self.lazy_workspace)
        from .kernels import mixer_prologue
        q, k, v, g = mixer_prologue(y.reshape(self.batch, -1), 1, self.D, 1, True, active_mask)
        return self.step_cham(layer, q, k, v, g, mode="unitary")

    def flush(self, layer: Optional[int] = None) -> None:
        """Fold the pending hologram factors of one layer (or all) into H_real / H_imag."""
        if self.P <= 0:
            return
        for l in (range(self.layers) if layer is None else (layer,)):
            flush_pending(self.H_real[l], self.H_imag[l], self.pending[l], self.P)

    def load_layer(self, layer: int, psi: Optional[torch.Tensor],
                   hologram: Optional[Tuple[torch.Tensor, torch.Tensor]]) -> None:
        """Copy one layer's batched states in ([b, h, d, d] and ([b, D, D], [b, D, D]))."""
        if psi is not None:
            self.psi[layer].copy_(psi)
        if hologram is not None:
            if self.P > 0:
                self.pending[layer].zero_()   # the loaded planes are the whole state
            self.H_real[layer].copy_(hologram[0])
            self.H_imag[layer].copy_(hologram[1])

    @classmethod
    def from_layer_states(cls, layer_states: List[List[Tuple]], device="cuda") -> "DecodeState":
        """From the reference's per-layer, per-item tuples (acd_engine.py:46-60)."""
        first = layer_states[0][0]
        psi0, (hr0, _) = first
        st = cls(len(layer_states), len(layer_states[0]), psi0.shape[-3], psi0.shape[-1], hr0.shape[-1],
                 device=device)
        for l, items in enumerate(layer_states):
            st.psi[l].copy_(torch.cat([it[0].reshape(1, st.h, st.d, st.d) for it in items]))
            st.H_real[l].copy_(torch.cat([it[1][0].reshape(1, st.D, st.D) for it in items]))
            st.H_imag[l].copy_(torch.cat([it[1][1].reshape(1, st.D, st.D) for it in items]))
        return st

    def layer_states(self) -> List[List[Tuple]]:
        """The reference's per-layer, per-item tuples, as views of this container (after
        folding any pending hologram factors in)."""
        self.flush()
        return [[(self.psi[l, i:i + 1], (self.H_real[l, i:i + 1], self.H_imag[l, i:i + 1]))
                 for i in range(self.batch)] for l in range(self.layers)]
