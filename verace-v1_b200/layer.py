"""One Verace V1 decoder layer and the Adaptive Cognitive Depth Engine, batched over items.

Drop-ins for ``VeraceV1Layer`` (verace_v1/modules/backbone.py:20-101) and
``AdaptiveCognitiveDepthEngine`` (verace_v1/modules/acd_engine.py:13-167): same
constructor arguments, parameter names, creation order (so ``state_dict`` and seeded
initialisation match) and forward signatures / return values.

``VeraceV1Layer.forward``: AttnRes mixing over the block-residual candidates and the
snapshot commit every 12 layers (backbone.py:70-80), then the three sub-layers with their
pre-norms and residual adds (backbone.py:82-99), the norms and adds as fused kernels.

``AdaptiveCognitiveDepthEngine.execute_adaptive_recurrent_loop``: the reference runs each
layer once per batch item on that item's gathered active tokens (acd_engine.py:94-127,
``torch.nonzero`` and a host sync per item and layer).  Here each layer runs once on the
whole batch with the active mask: a halted token gets the identity recurrence factor
(delta = gamma = 0, the modules' own active_mask gating), so every SSSD / CHAM state
and every active token's output equals the gathered computation's, and the halted
tokens' rows are kept from the previous layer.  The halting arithmetic is the
reference's, unchanged.  There is no host sync inside the loop; the one at the end
restores the states of (layer, item) pairs the reference would not have touched (an
item with no active token at a layer, layers after every token halted).  Inside the
reference loop the block residual never gains a candidate (each item's [s, 0, d] buffer
takes the layer's [S, 1, d] snapshot by broadcasting, acd_engine.py:115-124), so the
layers are called without one, which is the same computation.
"""
from typing import List, Optional, Tuple

import torch
import torch.nn as nn

from .cham_memory import ContinuousHolographicMemory
from .kernels import add_rmsnorm, apply_rmsnorm, fused_norm_supported
from .mcmoe import ManifoldContinuousMoE
from .sssd_attention import SSSDAttention


def _residual(h: torch.Tensor, y: torch.Tensor, out_norm: Optional[nn.Module]) -> Optional[torch.Tensor]:
    """h <- h + y in place; returns out_norm(h) when given (fused where the kernel applies)."""
    w = getattr(out_norm, "weight", None) if out_norm is not None else None
    if (fused_norm_supported(h) and y.dtype == h.dtype and h.is_contiguous()
            and (w is None or (w.dtype == h.dtype and w.device == h.device))):
        return add_rmsnorm(h, y.contiguous(), out_norm=out_norm)
    h.add_(y)
    return apply_rmsnorm(out_norm, h) if out_norm is not None else None


class VeraceV1Layer(nn.Module):
    """VeraceV1Layer (backbone.py:20-101): SSSD, CHAM and M-CMoE sub-layers."""

    def __init__(self, layer_idx: int, config):
        super().__init__()
        self.layer_idx = layer_idx
        self.config = config
        self.sssd_norm = nn.RMSNorm(config.hidden_dim, eps=config.rms_norm_eps)
        self.sssd_attn = SSSDAttention(hidden_dim=config.hidden_dim, num_heads=config.num_heads,
                                       head_dim=config.head_dim, spectral_dim=config.spectral_dim)
        self.cham_norm = nn.RMSNorm(config.hidden_dim, eps=config.rms_norm_eps)
        self.cham_memory = ContinuousHolographicMemory(hidden_dim=config.hidden_dim,
                                                       holographic_dim=config.chams_holographic_dim)
        self.mcmoe_norm = nn.RMSNorm(config.hidden_dim, eps=config.rms_norm_eps)
        self.mcmoe = ManifoldContinuousMoE(hidden_dim=config.hidden_dim, rank=config.mcmoe_rank,
                                           num_components=config.mcmoe_num_components, beta1=4.0, beta2=25.0)

    def forward(self, h_in: torch.Tensor, block_residual: Optional[torch.Tensor] = None,
                sssd_state: Optional[torch.Tensor] = None,
                cham_hologram: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
                active_mask: Optional[torch.Tensor] = None):
        """h_in [b, s, hidden]; block_residual [b*s, blocks, hidden]; active_mask [b, s].
        Returns (h_out, block_residual, sssd_state, cham_hologram)."""
        b, s, h = h_in.shape
        flat_h = h_in.reshape(b * s, h)
        if block_residual is None:
            block_residual = flat_h.new_zeros(b * s, 0, h)
        if block_residual.shape[1] > 0:   # AttnRes mixing (backbone.py:70-74)
            wts = torch.softmax(torch.matmul(flat_h.unsqueeze(1), block_residual.transpose(-1, -2)).squeeze(1), dim=-1)
            h_in = (flat_h + torch.matmul(wts.unsqueeze(1), block_residual).squeeze(1)).view(b, s, h)
        if self.layer_idx % 12 == 0:      # snapshot commit (backbone.py:77-78)
            block_residual = torch.cat([block_residual, flat_h.unsqueeze(1)], dim=1)
        hcur = h_in.contiguous().clone()
        n = apply_rmsnorm(self.sssd_norm, hcur)
        sssd_out, new_sssd_state = self.sssd_attn(n, initial_state=sssd_state, return_state=True,
                                                  active_mask=active_mask)
        n = _residual(hcur, sssd_out, self.cham_norm)            # h_mid1, RMSNorm(h_mid1)
        cham_out, new_cham_hologram = self.cham_memory(n, initial_hologram=cham_hologram, active_mask=active_mask)
        n = _residual(hcur, cham_out, self.mcmoe_norm)           # h_mid2, RMSNorm(h_mid2)
        _residual(hcur, self.mcmoe(n), None)                     # h_out
        return hcur, block_residual, new_sssd_state, new_cham_hologram


def _stack_states(items: List[Optional[Tuple]], b: int, h: int, d: int, D: int, device, dtype=torch.float32):
    """Per-item (psi [1,h,d,d], (Hr [1,D,D], Hi [1,D,D])) tuples (or None) -> batched
    (psi [b,h,d,d] or None, (Hr, Hi) [b,D,D] or None); None items become the identity."""
    if all(x is None for x in items):
        return None, None
    psi = torch.eye(d, device=device, dtype=dtype).expand(b, h, d, d).clone()
    hr = torch.eye(D, device=device, dtype=dtype).expand(b, D, D).clone()
    hi = torch.zeros(b, D, D, device=device, dtype=dtype)
    for i, st in enumerate(items):
        if st is None:
            continue
        if st[0] is not None:
            psi[i] = st[0].reshape(h, d, d)
        if st[1] is not None:
            hr[i] = st[1][0].reshape(D, D)
            hi[i] = st[1][1].reshape(D, D)
    return psi, (hr, hi)


class AdaptiveCognitiveDepthEngine(nn.Module):
    """AdaptiveCognitiveDepthEngine (acd_engine.py:13-167), batched over items."""

    def __init__(self, hidden_dim: int = 16384, energy_threshold: float = 0.99):
        super().__init__()
        self.hidden_dim = hidden_dim
        self.energy_threshold = energy_threshold
        self.w_halting = nn.Linear(hidden_dim, 1)
        nn.init.constant_(self.w_halting.bias, -3.0)
        nn.init.normal_(self.w_halting.weight, std=0.01)

    def compute_halting_probability(self, h_l: torch.Tensor) -> torch.Tensor:
        return torch.sigmoid(self.w_halting(h_l)).squeeze(-1)

    def execute_adaptive_recurrent_loop(self, layers: nn.ModuleList, h_in: torch.Tensor, max_depth: int = 128,
                                        min_depth: int = 2,
                                        initial_layer_states: Optional[List[Optional[List[Optional[Tuple]]]]] = None):
        """Same contract as the reference (acd_engine.py:36-63): returns (final_hidden
        [b,s,d], depth_counts [b,s], layer_states: per layer a per-item list of
        (sssd_state [1,h,d,d], (Hr [1,D,D], Hi [1,D,D])) or None)."""
        b, s, d = h_in.shape
        device = h_in.device
        h_curr = h_in.clone()
        final_h = torch.zeros_like(h_in)
        accumulated_prob = torch.zeros(b, s, device=device, dtype=h_in.dtype)
        depth_counts = torch.zeros(b, s, device=device, dtype=h_in.dtype)
        active_mask = torch.ones(b, s, device=device, dtype=torch.bool)
        num_layers = min(len(layers), max_depth)
        init = [(list(initial_layer_states[l]) if initial_layer_states is not None and l < len(initial_layer_states)
                 and initial_layer_states[l] is not None else [None] * b) for l in range(num_layers)]
        computed = []     # per layer: (psi [b,h,d,d], (Hr, Hi) [b,D,D])
        ran = []          # per layer: [b] bool, the item had an active token
        for l_idx in range(num_layers):
            layer = layers[l_idx]
            sa = layer.sssd_attn
            psi0, holo0 = _stack_states(init[l_idx], b, sa.num_heads, sa.head_dim,
                                        layer.cham_memory.holographic_dim, device)
            ran.append(active_mask.any(dim=1))
            out, _, psi, holo = layer(h_curr, sssd_state=psi0, cham_hologram=holo0, active_mask=active_mask)
            h_next = torch.where(active_mask.unsqueeze(-1), out, h_curr)
            computed.append((psi, holo))

            p_l = self.compute_halting_probability(h_next)
            if l_idx < min_depth:
                p_l = torch.zeros_like(p_l)
            new_accum = accumulated_prob + p_l
            newly_halted = (new_accum >= self.energy_threshold) & active_mask
            still_active = active_mask & (~newly_halted)
            remainder_weight = (1.0 - accumulated_prob).clamp(min=0.0)
            weight_layer = torch.where(newly_halted, remainder_weight, p_l)
            update_mask = (active_mask | newly_halted)
            final_h = final_h + (weight_layer * update_mask.to(h_in.dtype)).unsqueeze(-1) * h_next
            depth_counts = depth_counts + active_mask.to(h_in.dtype)
            depth_counts = depth_counts + remainder_weight * newly_halted.to(h_in.dtype)
            accumulated_prob = new_accum
            active_mask = still_active
            h_curr = h_next

        remainder_weight = (1.0 - accumulated_prob).clamp(min=0.0)
        final_h = final_h + (remainder_weight * active_mask.to(h_in.dtype)).unsqueeze(-1) * h_curr
        depth_counts = depth_counts + remainder_weight * active_mask.to(h_in.dtype)

        # one host read: which (layer, item) pairs ran (the reference skips items without
        # active tokens and stops after the layer where every token has halted)
        ran_host = torch.stack(ran).cpu() if ran else torch.zeros(0, b, dtype=torch.bool)
        layer_states_out: List[List[Optional[Tuple]]] = []
        for l_idx in range(num_layers):
            psi, (hr, hi) = computed[l_idx]
            items = []
            for i in range(b):
                if bool(ran_host[l_idx, i]):
                    items.append((psi[i:i + 1], (hr[i:i + 1], hi[i:i + 1])))
                else:
                    items.append(init[l_idx][i])
            layer_states_out.append(items)
        return final_h, depth_counts, layer_states_out
