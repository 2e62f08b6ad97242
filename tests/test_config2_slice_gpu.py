"""A slice of benchmark config 2 on the GPU against the fp64 oracle: the bench's 12-layer
SSSD -> CHAM chain (hidden 1024, 8 heads x 128, D = 1024, weights seeded and cast to bf16,
token embeddings of uniform random ids) on 1 item x 256 tokens, bf16 activations and fp32
recurrent states through the drop-in modules.

The oracle runs the same chain in fp64 on the same bf16-rounded weights and embeddings:
the eager SSSD (dense per-token Cayley solves and prefix products) and the CHAM scan in
O(D^2) per token (``cham_scan_rank2_c``, pinned to the dense oracle and to the reference
at config 1 by tests/test_oracle_config1.py).  Bar: north_star's bf16 tolerance,
relative Frobenius error <= 2e-2, on the final hidden state and on the last layer's
exported states.  RMSNorms with eps=None take bf16's machine epsilon in both (what
torch.nn.RMSNorm uses for bf16 input).
"""
import numpy as np
import pytest
import torch

import oracle
import verace_v1_b200 as V
from gpu_util import rel_fro, to_np

pytestmark = pytest.mark.gpu

LAYERS, HID, HEADS, HD, D, VOCAB, S = 12, 1024, 8, 128, 1024, 32000, 256


def _build(dev):
    torch.manual_seed(0)
    layers = []
    for _ in range(LAYERS):
        layers.append(torch.nn.ModuleDict(dict(
            sssd_norm=torch.nn.RMSNorm(HID, eps=1e-6),
            sssd=V.SSSDAttention(HID, HEADS, HD, 256),
            cham_norm=torch.nn.RMSNorm(HID, eps=1e-6),
            cham=V.ContinuousHolographicMemory(HID, D))).to(dev, torch.bfloat16).eval())
    embed = torch.nn.Embedding(VOCAB, HID).to(dev, torch.bfloat16)
    ids = torch.randint(0, VOCAB, (1, S), generator=torch.Generator().manual_seed(0)).to(dev)
    return layers, embed, ids


def test_config2_slice_12_layers_bf16_matches_fp64_oracle():
    dev = torch.device("cuda")
    layers, embed, ids = _build(dev)
    with torch.no_grad():
        x = embed(ids)
        h = x.clone()
        for L in layers:
            o, psi = L["sssd"](L["sssd_norm"](h), return_state=True)
            h = h + o
            y, H = L["cham"](L["cham_norm"](h))
            h = h + y
    bf_eps = float(torch.finfo(torch.bfloat16).eps)
    sd = lambda m: {k: to_np(v).astype(np.float64) for k, v in m.state_dict().items()}
    hr = to_np(x).astype(np.float64)
    for L in layers:
        n = oracle.rms_norm(hr, to_np(L["sssd_norm"].weight).astype(np.float64), 1e-6)
        o_r, psi_r = oracle.sssd_forward(sd(L["sssd"]), n, HEADS, HD, return_state=True, norm_eps=bf_eps)
        hr = hr + o_r
        n = oracle.rms_norm(hr, to_np(L["cham_norm"].weight).astype(np.float64), 1e-6)
        y_r, H_r = oracle.cham_forward(sd(L["cham"]), n, norm_eps=bf_eps, rank2=True)
        hr = hr + y_r
    err_h = rel_fro(to_np(h), hr)
    err_psi = rel_fro(to_np(psi), psi_r)
    err_H = rel_fro(to_np(H[0]) + 1j * to_np(H[1]), H_r[0] + 1j * H_r[1])
    print(f"config-2 slice: hidden {err_h:.2e}, last SSSD state {err_psi:.2e}, last CHAM state {err_H:.2e}")
    assert err_h <= 2e-2
    assert err_psi <= 2e-2
    assert err_H <= 2e-2
