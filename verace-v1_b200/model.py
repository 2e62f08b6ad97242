"""VeraceV1Model's text path with the reference's constructor and forward signature
(verace_v1/modules/backbone.py:104-210), running its layers on the sm_100a kernels.

Drop-in for the part of ``VeraceV1Model`` this path covers: token embedding tied to the
LM head, the decoder layers (``VeraceV1Layer``: SSSD, CHAM, M-CMoE), the Adaptive
Cognitive Depth Engine loop (batched over items), the final RMSNorm and the LM head, with
the reference's ``forward(input_ids, images, use_adaptive_depth, return_hidden,
layer_states, return_layer_states)`` contract, incremental decoding through
``layer_states`` included (the convention of verace_v1/serving/hyper_generate.py:58-77).

Outside this path and not built: the vision encoder (``images`` must be None) and the
latent energy critic.  Their parameters are absent, so a reference ``state_dict`` loads
through :meth:`load_reference_state_dict`, which drops ``vision_encoder.*`` and
``energy_critic.*`` and loads the rest strictly.  Seeded construction does not reproduce
the reference's weights (the reference draws the vision encoder's between the LM head and
the layers); load the reference's state_dict instead.
"""
from typing import List, Optional

import torch
import torch.nn as nn

from .kernels import apply_rmsnorm
from .layer import AdaptiveCognitiveDepthEngine, VeraceV1Layer

OUT_OF_PATH = ("vision_encoder.", "energy_critic.")


class VeraceV1Model(nn.Module):
    def __init__(self, config):
        super().__init__()
        self.config = config
        self.embed_tokens = nn.Embedding(config.vocab_size, config.hidden_dim)
        self.lm_head = nn.Linear(config.hidden_dim, config.vocab_size, bias=False)
        self.embed_tokens.weight = self.lm_head.weight   # weight tying, as the reference
        self.layers = nn.ModuleList([VeraceV1Layer(layer_idx=i, config=config) for i in range(config.num_layers)])
        self.acd_engine = AdaptiveCognitiveDepthEngine(hidden_dim=config.hidden_dim,
                                                       energy_threshold=config.energy_halting_threshold)
        self.final_norm = nn.RMSNorm(config.hidden_dim, eps=config.rms_norm_eps)

    def load_reference_state_dict(self, state_dict):
        """Load a reference VeraceV1Model state_dict: the vision-encoder and energy-critic
        entries (outside this path) are dropped, every other entry must match."""
        sd = {k: v for k, v in state_dict.items() if not k.startswith(OUT_OF_PATH)}
        return self.load_state_dict(sd, strict=True)

    def forward(self, input_ids: torch.Tensor, images: Optional[torch.Tensor] = None,
                use_adaptive_depth: bool = True, return_hidden: bool = False,
                layer_states: Optional[List] = None, return_layer_states: bool = False):
        """input_ids [b, s] -> (logits [b, s, vocab], depth_counts [b, s]) (+ the post-norm
        hidden state when return_hidden, + the per-layer, per-item states when
        return_layer_states), as backbone.py:144-210."""
        if images is not None:
            raise ValueError("VeraceV1Model: image inputs (the vision encoder) are outside this path")
        b, s = input_ids.shape
        token_embeds = self.embed_tokens(input_ids)
        final_layer_states = None
        if use_adaptive_depth:
            final_h, depth_counts, final_layer_states = self.acd_engine.execute_adaptive_recurrent_loop(
                layers=self.layers, h_in=token_embeds, max_depth=self.config.max_cognitive_depth,
                min_depth=self.config.min_cognitive_depth, initial_layer_states=layer_states)
        else:
            h_curr = token_embeds
            for layer in self.layers:
                h_curr, _, _, _ = layer(h_curr)
            final_h = h_curr
            depth_counts = torch.full((b, s), float(len(self.layers)), device=input_ids.device,
                                      dtype=token_embeds.dtype)
        norm_final_h = apply_rmsnorm(self.final_norm, final_h.contiguous())
        logits = self.lm_head(norm_final_h)
        if return_hidden and return_layer_states:
            return logits, depth_counts, norm_final_h, final_layer_states
        if return_hidden:
            return logits, depth_counts, norm_final_h
        if return_layer_states:
            return logits, depth_counts, final_layer_states
        return logits, depth_counts
