"""B200-native (sm_100a) implementation of Verace V1's recurrent sequence-mixing path:
the SSSD Cayley-rotation scan and the CHAM holographic-memory update with its
Newton-Schulz readout retraction.

Public surface (mirrors the reference package verace_v1 for this path):
    SSSDAttention, ContinuousHolographicMemory, newton_schulz_unitary_retraction
    launch_sssd_scan / launch_sssd_triton_scan
    launch_cham_update / launch_cham_triton_update
    rmsnorm, add_rmsnorm                             (block glue: RMSNorm, residual + RMSNorm)
    DecodeState, launch_decode_step, device_status   (batched incremental decode)
    launch_decode_cham_lazy, flush_pending, pending_storage (deferred hologram updates)
    launch_decode_cham_lazy_projected                (the same from the raw projection rows)
    ManifoldContinuousMoE, SiTUGLU, launch_mcmoe_projection / launch_mcmoe_triton_projection,
    launch_mcmoe_route, situ_glu                     (M-CMoE sub-layer)
    VeraceV1Layer, AdaptiveCognitiveDepthEngine, VeraceV1Config (a decoder layer; the
                                                     ACDE loop batched over items)
    VeraceV1Model                                    (embedding, ACDE over the layers, final
                                                     norm, LM head; incremental decode
                                                     through layer_states)
The kernels live in libverace_b200.so (C ABI: include/verace_b200.h), built by
build.py; nothing here falls back to CPU or Python arithmetic.
"""
from .kernels import (add_rmsnorm, cham_retract, launch_cham_triton_update, launch_cham_update,
                      launch_sssd_scan, launch_sssd_triton_scan, rmsnorm)
from .decode import (DecodeState, device_status, flush_pending, launch_decode_cham_lazy,
                     launch_decode_cham_lazy_projected, launch_decode_step, pending_storage)
from .sssd_attention import SSSDAttention
from .cham_memory import ContinuousHolographicMemory, newton_schulz_unitary_retraction
from .mcmoe import (ManifoldContinuousMoE, SiTUGLU, launch_mcmoe_projection, launch_mcmoe_route,
                    launch_mcmoe_triton_projection, situ_glu)
from .config import VeraceV1Config
from .layer import AdaptiveCognitiveDepthEngine, VeraceV1Layer
from .model import VeraceV1Model

__all__ = [
    "SSSDAttention", "ContinuousHolographicMemory", "newton_schulz_unitary_retraction",
    "launch_sssd_scan", "launch_sssd_triton_scan", "launch_cham_update",
    "launch_cham_triton_update", "cham_retract", "DecodeState", "launch_decode_step",
    "device_status", "rmsnorm", "add_rmsnorm", "launch_decode_cham_lazy", "flush_pending", "pending_storage",
    "launch_decode_cham_lazy_projected",
    "ManifoldContinuousMoE", "SiTUGLU", "launch_mcmoe_projection", "launch_mcmoe_triton_projection",
    "launch_mcmoe_route", "situ_glu", "VeraceV1Config", "VeraceV1Layer", "AdaptiveCognitiveDepthEngine",
    "VeraceV1Model",
]
