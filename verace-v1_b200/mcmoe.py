"""M-CMoE (Manifold Continuous Mixture-of-Experts) on sm_100a: drop-ins for the reference's
``ManifoldContinuousMoE`` (verace_v1/modules/mcmoe.py:20-120), ``SiTUGLU``
(verace_v1/modules/activations.py) and ``launch_mcmoe_triton_projection``
(verace_v1/serving/triton_kernels.py:688-723).

The modules keep the reference's constructor arguments, parameter names, shapes and
creation order (so ``state_dict`` and seeded initialisation match) and its forward
signature.  The forward pass runs as:

* base FFN: the gate and up projections as one GEMM (torch / cuBLAS), the SiTU-GLU
  activation in one kernel (``verace_situ_glu``), then ``base_w_down``;
* routing: router GEMM, then top-K and the softmax over the kept logits in one kernel
  (``verace_mcmoe_route``);
* manifold projection: ``verace_mcmoe_projection`` (tcgen05 GEMMs with the routing and
  the hyper-network's sigmoid folded into the epilogue for bf16; a direct fp32 kernel
  otherwise), from the hyper-network's pre-activation;
* ``base + RMSNorm(manifold)`` in one pass (``verace_add_rmsnorm``).
"""
from typing import Optional, Tuple

import torch
import torch.nn as nn

from ._lib import check, lib
from .kernels import _DTYPE, _stream, _workspace, add_rmsnorm, fused_norm_supported


def launch_mcmoe_route(logits: torch.Tensor, k: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """Top-k of each row of ``logits`` [n, C] (descending, as torch.topk) and the softmax
    over the kept logits (mcmoe.py:92-96).  Returns (indices [n, k] int64, weights [n, k]
    in the logits' dtype)."""
    assert logits.is_cuda, "This kernel requires CUDA tensors"
    lg = logits.contiguous()
    if lg.dtype not in _DTYPE:
        lg = lg.float()
    n, C = lg.shape
    idx = torch.empty(n, k, dtype=torch.int64, device=lg.device)
    w = torch.empty(n, k, dtype=lg.dtype, device=lg.device)
    with torch.cuda.device(lg.device):
        rc = lib().verace_mcmoe_route(lg.data_ptr(), n, C, k, idx.data_ptr(), w.data_ptr(), _DTYPE[lg.dtype],
                                      _stream(lg.device))
    check(rc, "verace_mcmoe_route")
    return idx, w


def launch_mcmoe_projection(x_flat: torch.Tensor, u_basis: torch.Tensor, v_basis: torch.Tensor,
                            topk_indices: torch.Tensor, topk_weights: torch.Tensor, sigma: torch.Tensor,
                            sigma_is_logits: bool = False) -> torch.Tensor:
    """The reference launcher's contract (triton_kernels.py:688-723): x_flat [n, d],
    u_basis [C, d, r], v_basis [C, r, d], topk_indices / topk_weights [n, K], sigma
    [n, C, r] (post-sigmoid; with ``sigma_is_logits`` the pre-activation, the sigmoid then
    applied inside).  Returns manifold_adapt [n, d] in x's dtype, freshly allocated."""
    assert x_flat.is_cuda, "This kernel requires CUDA tensors"
    x = x_flat.contiguous()
    if x.dtype not in _DTYPE:
        x = x.float()
    dt = x.dtype
    n, d = x.shape
    C, d_u, r = u_basis.shape
    assert d_u == d and tuple(v_basis.shape) == (C, r, d), "basis shapes must be [C, d, r] and [C, r, d]"
    K = topk_indices.shape[1]
    u = u_basis.to(dt).contiguous()
    v = v_basis.to(dt).contiguous()
    idx = topk_indices.to(torch.int64).contiguous()
    w = topk_weights.to(dt).contiguous()
    sg = sigma.reshape(n, C * r).to(dt).contiguous()
    out = torch.empty_like(x)
    ws_bytes = int(lib().verace_mcmoe_workspace(n, d, C, r, _DTYPE[dt]))
    ws = _workspace(ws_bytes, x.device)
    with torch.cuda.device(x.device):
        rc = lib().verace_mcmoe_projection(x.data_ptr(), u.data_ptr(), v.data_ptr(), idx.data_ptr(), w.data_ptr(),
                                           sg.data_ptr(), 1 if sigma_is_logits else 0, out.data_ptr(), n, d, C, r, K,
                                           _DTYPE[dt], ws.data_ptr(), ws.numel(), _stream(x.device))
    check(rc, "verace_mcmoe_projection")
    return out


launch_mcmoe_triton_projection = launch_mcmoe_projection


def situ_glu(gate_linear: torch.Tensor, up_linear: torch.Tensor, beta1: float, beta2: float) -> torch.Tensor:
    """[beta1 tanh(g/beta1) sigmoid(g)] * [beta2 tanh(u/beta2)] in one pass (g and u may be
    the two halves of one [.., 2 cols] tensor)."""
    assert gate_linear.is_cuda, "This kernel requires CUDA tensors"
    cols = gate_linear.shape[-1]
    assert up_linear.shape == gate_linear.shape and up_linear.dtype == gate_linear.dtype
    n = gate_linear.numel() // cols
    g2, u2 = gate_linear.reshape(n, cols), up_linear.reshape(n, cols)
    ld = g2.stride(0)
    if not (g2.stride(1) == 1 and u2.stride(1) == 1 and u2.stride(0) == ld):
        g2, u2 = g2.contiguous(), u2.contiguous()
        ld = cols
    out = torch.empty(gate_linear.shape, dtype=gate_linear.dtype, device=gate_linear.device)
    with torch.cuda.device(out.device):
        rc = lib().verace_situ_glu(g2.data_ptr(), u2.data_ptr(), ld, out.data_ptr(), n, cols, float(beta1),
                                   float(beta2), _DTYPE[out.dtype], _stream(out.device))
    check(rc, "verace_situ_glu")
    return out


class SiTUGLU(nn.Module):
    """SiTUGLU (verace_v1/modules/activations.py): same parameters (w_gate, w_up)."""

    def __init__(self, in_features: int, hidden_features: int, beta1: float = 4.0, beta2: float = 25.0):
        super().__init__()
        self.in_features = in_features
        self.hidden_features = hidden_features
        self.beta1 = beta1
        self.beta2 = beta2
        self.w_gate = nn.Linear(in_features, hidden_features, bias=False)
        self.w_up = nn.Linear(in_features, hidden_features, bias=False)
        self._stacked: Optional[torch.Tensor] = None
        self._stacked_key = None

    def _gate_up_weight(self) -> torch.Tensor:
        # [W_gate; W_up] for one GEMM, rebuilt when either parameter changes
        key = (self.w_gate.weight.data_ptr(), self.w_up.weight.data_ptr(), self.w_gate.weight._version,
               self.w_up.weight._version, self.w_gate.weight.dtype, self.w_gate.weight.device)
        if self._stacked is None or self._stacked_key != key:
            self._stacked = torch.cat([self.w_gate.weight, self.w_up.weight], 0).detach()
            self._stacked_key = key
        return self._stacked

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not x.is_cuda or torch.is_grad_enabled() and x.requires_grad:
            raise RuntimeError("SiTUGLU runs on CUDA inputs for inference (no autograd path)")
        gu = torch.nn.functional.linear(x, self._gate_up_weight())
        hf = self.hidden_features
        return situ_glu(gu[..., :hf], gu[..., hf:], self.beta1, self.beta2)


class ManifoldContinuousMoE(nn.Module):
    """ManifoldContinuousMoE (verace_v1/modules/mcmoe.py:20-120) on the sm_100a kernels."""

    def __init__(self, hidden_dim: int = 16384, rank: int = 32, num_components: int = 64,
                 top_k_components: int = 8, beta1: float = 4.0, beta2: float = 25.0):
        super().__init__()
        self.hidden_dim = hidden_dim
        self.rank = rank
        self.num_components = num_components
        self.top_k_components = top_k_components
        self.base_situ_glu = SiTUGLU(hidden_dim, hidden_dim * 2, beta1=beta1, beta2=beta2)
        self.base_w_down = nn.Linear(hidden_dim * 2, hidden_dim, bias=False)
        self.u_basis = nn.Parameter(torch.randn(num_components, hidden_dim, rank) * 0.02)
        self.v_basis = nn.Parameter(torch.randn(num_components, rank, hidden_dim) * 0.02)
        self.router = nn.Linear(hidden_dim, num_components, bias=False)
        self.hyper_sigma = nn.Linear(hidden_dim, num_components * rank, bias=False)
        self.norm = nn.RMSNorm(hidden_dim)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """x: [batch, seq_len, hidden_dim] -> [batch, seq_len, hidden_dim]"""
        if not x.is_cuda or torch.is_grad_enabled() and x.requires_grad:
            raise RuntimeError("ManifoldContinuousMoE runs on CUDA inputs for inference (no autograd path)")
        b, s, d = x.shape
        x_flat = x.reshape(b * s, d).contiguous()
        base_out = self.base_w_down(self.base_situ_glu(x_flat)).contiguous()
        k_val = min(self.top_k_components, self.num_components)
        idx, w = launch_mcmoe_route(self.router(x_flat), k_val)
        sig_pre = self.hyper_sigma(x_flat)
        manifold = launch_mcmoe_projection(x_flat, self.u_basis, self.v_basis, idx, w, sig_pre, sigma_is_logits=True)
        if fused_norm_supported(base_out) and self.norm.weight.dtype == base_out.dtype:
            add_rmsnorm(base_out, manifold, y_norm=self.norm)   # base_out <- base_out + norm(manifold)
            y = base_out
        else:
            y = base_out + self.norm(manifold)
        return y.view(b, s, d)
