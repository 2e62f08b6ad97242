"""GPU parity of the decoder layer and the batched ACDE loop against the reference's own
outputs (tests/golden/layer_golden.npz, made by running VeraceV1Layer and
AdaptiveCognitiveDepthEngine on CPU).  The reference's ACDE runs each item's gathered
active tokens through the layers; the batched loop runs the whole batch under the active
mask, which must give the same outputs, ponder costs and states.  fp32: 1e-4 relative
Frobenius on outputs and state sketches; bf16 layer: 2e-2.
"""
import numpy as np
import pytest
import torch

import verace_v1_b200 as V
from conftest import GOLDEN
from gpu_util import rel_fro, to_np

pytestmark = pytest.mark.gpu

Z = np.load(f"{GOLDEN}/layer_golden.npz")
CFG = V.VeraceV1Config(vocab_size=100, hidden_dim=256, num_layers=4, num_heads=2, head_dim=128,
                       spectral_dim=64, chams_holographic_dim=256, mcmoe_rank=16, mcmoe_num_components=8)


def _layers(dtype=torch.float32):
    torch.manual_seed(0)
    layers = torch.nn.ModuleList([V.VeraceV1Layer(i, CFG) for i in range(4)])
    acde = V.AdaptiveCognitiveDepthEngine(hidden_dim=256, energy_threshold=0.99)
    with torch.no_grad():
        acde.w_halting.weight.copy_(torch.from_numpy(Z["acde/w_halting.weight"]))
        acde.w_halting.bias.copy_(torch.from_numpy(Z["acde/w_halting.bias"]))
    return layers.to("cuda", dtype).eval(), acde.to("cuda", dtype).eval()


def _sketch_err(prefix, psi, holo):
    r_d = torch.from_numpy(Z["sketch/r_d"]).cuda()
    r_D = torch.from_numpy(Z["sketch/r_D"]).cuda()
    e = [rel_fro(to_np(psi.float() @ r_d), Z[f"{prefix}/psi_r"]),
         rel_fro(to_np(holo[0].float() @ r_D), Z[f"{prefix}/hr_r"]),
         rel_fro(to_np(holo[1].float() @ r_D), Z[f"{prefix}/hi_r"])]
    return max(e)


def test_layers_match_reference_golden():
    layers, _ = _layers()
    x = torch.from_numpy(Z["L0/x"]).cuda()
    with torch.no_grad():
        h1, br1, s1, c1 = layers[0](x)
        assert rel_fro(to_np(h1), Z["L0/h"]) <= 1e-4
        assert rel_fro(to_np(br1), Z["L0/br"]) <= 1e-6       # the committed snapshot (layer 0)
        assert _sketch_err("L0", s1, c1) <= 1e-4
        mask = torch.from_numpy(Z["L1/mask"]).cuda()
        h2, br2, s2, c2 = layers[1](h1, block_residual=br1, sssd_state=s1, cham_hologram=c1, active_mask=mask)
        assert rel_fro(to_np(h2), Z["L1/h"]) <= 1e-4         # AttnRes mixing, carried states, masked tokens
        assert br2.shape == br1.shape                        # layer 1 commits nothing
        assert _sketch_err("L1", s2, c2) <= 1e-4
    assert V.device_status() == 0


def test_bf16_layer_matches_reference_golden():
    """bf16 weights and activations against the fp32 golden.  The norms built with
    eps=None (SSSD's head norm, CHAM's and M-CMoE's output norms) take fp32's machine
    epsilon, as they do for the reference's bf16 runs (fp32 weights under autocast); a
    bf16 norm's own epsilon (2^-7) would dominate the small M-CMoE mean square."""
    layers, _ = _layers(torch.bfloat16)
    for m in layers.modules():
        if isinstance(m, torch.nn.RMSNorm) and m.eps is None:
            m.eps = torch.finfo(torch.float32).eps
    x = torch.from_numpy(Z["L0/x"]).to(torch.bfloat16).cuda()
    with torch.no_grad():
        h1, _, s1, c1 = layers[0](x)
    assert h1.dtype == torch.bfloat16
    assert rel_fro(to_np(h1), Z["L0/h"]) <= 2e-2
    assert _sketch_err("L0", s1, c1) <= 2e-2


def test_batched_acde_matches_the_gathered_reference_loop():
    layers, acde = _layers()
    with torch.no_grad():
        fh, dc, st = acde.execute_adaptive_recurrent_loop(layers, torch.from_numpy(Z["A0/x"]).cuda(),
                                                          max_depth=12, min_depth=2)
        assert rel_fro(to_np(fh), Z["A0/final_h"]) <= 1e-4
        np.testing.assert_allclose(to_np(dc), Z["A0/depth"], rtol=0, atol=1e-4)
        for l in range(4):
            for i in range(2):
                assert tuple(st[l][i][0].shape) == (1, 2, 128, 128) and tuple(st[l][i][1][0].shape) == (1, 256, 256)
                assert _sketch_err(f"A0/s{l}_{i}", st[l][i][0], st[l][i][1]) <= 1e-4, (l, i)
        # continuation with four new tokens from the returned states
        fh2, dc2, st2 = acde.execute_adaptive_recurrent_loop(layers, torch.from_numpy(Z["A1/x"]).cuda(),
                                                            max_depth=12, min_depth=2, initial_layer_states=st)
        assert rel_fro(to_np(fh2), Z["A1/final_h"]) <= 1e-4
        np.testing.assert_allclose(to_np(dc2), Z["A1/depth"], rtol=0, atol=1e-4)
        for l in range(4):
            for i in range(2):
                assert _sketch_err(f"A1/s{l}_{i}", st2[l][i][0], st2[l][i][1]) <= 1e-4, (l, i)
    assert V.device_status() == 0


def test_acde_stops_where_every_token_has_halted():
    """A halting unit that fires at once (after min_depth) halts every token at layer 2;
    the reference then leaves layer 3's states as they were given (None here)."""
    layers, acde = _layers()
    with torch.no_grad():
        acde.w_halting.weight.zero_()
        acde.w_halting.bias.fill_(10.0)
        x = torch.from_numpy(Z["A0/x"]).cuda()
        fh, dc, st = acde.execute_adaptive_recurrent_loop(layers, x, max_depth=12, min_depth=2)
    assert all(st[3][i] is None for i in range(2)) and all(st[2][i] is not None for i in range(2))
    # N = 3 layers (0, 1, 2) plus R = 1 - 0 at the halting step (layers 0 and 1 add no probability)
    np.testing.assert_allclose(to_np(dc), 4.0, atol=1e-5)
