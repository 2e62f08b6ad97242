"""ContinuousHolographicMemory with the reference's constructor, parameters and
forward signature (verace_v1/modules/cham_memory.py:99-243), running its scan and
readout retraction on the sm_100a kernels.

A reference ``state_dict`` loads unchanged (w_q, w_k, w_v, w_gamma, w_out, norm).
The forward mirrors the reference's fast path (cham_memory.py:127-168):
q, k = normalize(W x), v = normalize(silu(w_v x)), gamma = 0.1 sigmoid(w_gamma x)
masked by ``active_mask``, the scan (exact Cayley updates, raw state exported,
Newton-Schulz retraction on the readout) and ``norm(w_out(rec))``.

``newton_schulz_unitary_retraction`` is the CUDA version of the reference function
of the same name (cham_memory.py:21-51).
"""
from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from .kernels import apply_rmsnorm, cham_retract, concat_weights, launch_cham_update, mixer_prologue
from .sssd_attention import _require_inference


def newton_schulz_unitary_retraction(H_real: torch.Tensor, H_imag: torch.Tensor, steps: int = 3
                                     ) -> Tuple[torch.Tensor, torch.Tensor]:
    return cham_retract(H_real, H_imag, steps)


class ContinuousHolographicMemory(nn.Module):
    def __init__(self, hidden_dim: int = 16384, holographic_dim: int = 1024):
        super().__init__()
        self.hidden_dim = hidden_dim
        self.holographic_dim = holographic_dim
        self.w_q = nn.Linear(hidden_dim, holographic_dim, bias=False)
        self.w_k = nn.Linear(hidden_dim, holographic_dim, bias=False)
        self.w_v = nn.Linear(hidden_dim, holographic_dim, bias=False)
        self.w_gamma = nn.Linear(hidden_dim, 1, bias=False)
        self.w_out = nn.Linear(holographic_dim, hidden_dim, bias=False)
        self.norm = nn.RMSNorm(hidden_dim)

    def projection(self, x: torch.Tensor) -> torch.Tensor:
        """The concatenated projection y = x [W_q; W_k; W_v; W_gamma]ᵀ, [b, s, ld] (rows
        q | k | v | gate, zero-padded to a multiple of 8): the GEMM of :meth:`project`
        without its epilogue, as the deferred decode step consumes it."""
        W = concat_weights(self, [self.w_q.weight, self.w_k.weight, self.w_v.weight, self.w_gamma.weight])
        return F.linear(x, W)

    def project(self, x: torch.Tensor, active_mask: Optional[torch.Tensor] = None):
        """q, k, v [b, s, D] and gamma [b, s] (cham_memory.py:129-153): one GEMM with the
        concatenated projection weights, then the fused normalisation/SiLU/gate pass."""
        b, s, _ = x.shape
        D = self.holographic_dim
        if D % 8:   # widths the fused pass does not tile: the same math as torch ops on the GPU
            q = F.normalize(self.w_q(x), p=2, dim=-1)
            k = F.normalize(self.w_k(x), p=2, dim=-1)
            v = F.normalize(F.silu(self.w_v(x)), p=2, dim=-1)
            gamma = 0.1 * torch.sigmoid(self.w_gamma(x)).view(b, s)
            if active_mask is not None:
                gamma = gamma * active_mask.reshape(b, s).to(gamma.dtype)
            return q, k, v, gamma
        W = concat_weights(self, [self.w_q.weight, self.w_k.weight, self.w_v.weight, self.w_gamma.weight])
        y = F.linear(x, W).reshape(b * s, -1)
        q, k, v, gamma = mixer_prologue(y, 1, D, 1, True, active_mask)
        return q.view(b, s, D), k.view(b, s, D), v.view(b, s, D), gamma.view(b, s)

    def forward(self, x: torch.Tensor,
                initial_hologram: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
                active_mask: Optional[torch.Tensor] = None
                ) -> Tuple[torch.Tensor, Tuple[torch.Tensor, torch.Tensor]]:
        _require_inference(x, "ContinuousHolographicMemory.forward")
        q, k, v, gamma = self.project(x, active_mask)
        rec, (h_real, h_imag) = launch_cham_update(q, k, v, gamma, initial_hologram)
        return self.finish(rec), (h_real, h_imag)

    def finish(self, rec: torch.Tensor) -> torch.Tensor:
        """Module output from the scan's readout rec [b, s, D] (cham_memory.py:241)."""
        return apply_rmsnorm(self.norm, self.w_out(rec))
