"""The fields of the reference's ``VeraceV1Config`` (verace_v1/config.py:13-60) that the
layer, ACDE and M-CMoE modules read, with the same names and defaults.  The modules accept
any object with these attributes, the reference's config included."""
from dataclasses import dataclass


@dataclass
class VeraceV1Config:
    vocab_size: int = 163840
    hidden_dim: int = 1024
    num_layers: int = 12
    num_heads: int = 8
    head_dim: int = 128
    spectral_dim: int = 256
    sssd_phase_scale: float = 1.0
    chams_holographic_dim: int = 1024
    chams_memory_decay: float = 0.001
    mcmoe_rank: int = 32
    mcmoe_num_components: int = 64
    max_cognitive_depth: int = 12
    min_cognitive_depth: int = 2
    energy_halting_threshold: float = 0.99
    rms_norm_eps: float = 1e-6
