"""SSSDAttention with the reference's constructor, parameters and forward signature
(verace_v1/modules/sssd_attention.py:74-182), running its scan on the sm_100a kernel.

A reference ``state_dict`` loads unchanged (same submodule names: w_q, w_k, w_v,
w_delta, head_rmsnorm, w_out).  The forward mirrors the reference's fast path
(sssd_attention.py:113-136): projections and L2-normalisation (cuBLAS through
torch), the gate delta = 0.1 sigmoid(w_delta x) masked by ``active_mask``, the scan,
head RMSNorm and ``w_out``.  The scan itself follows the eager path's recurrence
R_t = (I + delta A/2)^-1 (I - delta A/2) exactly (no small-delta skip).

Only the inference path exists: inputs must be CUDA tensors that do not require
grad (the condition under which the reference leaves its eager training path).
"""
from typing import Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from .kernels import apply_rmsnorm, concat_weights, launch_sssd_scan, mixer_prologue


def _require_inference(x: torch.Tensor, who: str):
    if not x.is_cuda or x.requires_grad:
        raise RuntimeError(
            f"{who}: this is the B200 inference path; it needs a CUDA input that does not "
            "require grad (training and CPU use the reference's eager path; there is no fallback)")


class SSSDAttention(nn.Module):
    def __init__(self, hidden_dim: int = 16384, num_heads: int = 128, head_dim: int = 128,
                 spectral_dim: int = 256):
        super().__init__()
        self.hidden_dim = hidden_dim
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.spectral_dim = spectral_dim
        self.w_q = nn.Linear(hidden_dim, num_heads * head_dim, bias=False)
        self.w_k = nn.Linear(hidden_dim, num_heads * head_dim, bias=False)
        self.w_v = nn.Linear(hidden_dim, num_heads * head_dim, bias=False)
        self.w_delta = nn.Linear(hidden_dim, num_heads, bias=False)
        self.head_rmsnorm = nn.RMSNorm(head_dim)
        self.w_out = nn.Linear(num_heads * head_dim, hidden_dim, bias=False)

    def project(self, x: torch.Tensor, active_mask: Optional[torch.Tensor] = None):
        """q, k, v [b, s, h, d] and delta [b, s, h] (sssd_attention.py:116-126): one GEMM
        with the concatenated projection weights, then the fused normalisation/gate pass."""
        b, s, _ = x.shape
        h, d = self.num_heads, self.head_dim
        if d % 8:   # head widths the fused pass does not tile: the same math as torch ops on the GPU
            q = F.normalize(self.w_q(x).view(b, s, h, d), p=2, dim=-1)
            k = F.normalize(self.w_k(x).view(b, s, h, d), p=2, dim=-1)
            v = F.normalize(self.w_v(x).view(b, s, h, d), p=2, dim=-1)
            delta = 0.1 * torch.sigmoid(self.w_delta(x)).view(b, s, h)
            if active_mask is not None:
                delta = delta * active_mask.reshape(b, s, 1).to(delta.dtype)
            return q, k, v, delta
        W = concat_weights(self, [self.w_q.weight, self.w_k.weight, self.w_v.weight, self.w_delta.weight])
        y = F.linear(x, W).reshape(b * s, -1)
        q, k, v, delta = mixer_prologue(y, h, d, h, False, active_mask)
        return q.view(b, s, h, d), k.view(b, s, h, d), v.view(b, s, h, d), delta.view(b, s, h)

    def forward(self, x: torch.Tensor, initial_state: Optional[torch.Tensor] = None,
                return_state: bool = False, active_mask: Optional[torch.Tensor] = None
                ) -> Tuple[torch.Tensor, Optional[torch.Tensor]]:
        _require_inference(x, "SSSDAttention.forward")
        b, s, _ = x.shape
        q, k, v, delta = self.project(x, active_mask)
        o, psi = launch_sssd_scan(q, k, v, delta, initial_state)
        return self.finish(o), (psi if return_state else None)

    def finish(self, o: torch.Tensor) -> torch.Tensor:
        """Module output from the scan's readout o [b, s, h, d] (sssd_attention.py:177-182)."""
        b, s = o.shape[0], o.shape[1]
        return self.w_out(apply_rmsnorm(self.head_rmsnorm, o).view(b, s, self.num_heads * self.head_dim))
