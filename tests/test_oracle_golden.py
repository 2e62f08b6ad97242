"""Pins the CPU oracle (oracle/verace_oracle.py) to golden vectors produced by the
reference implementation itself (tests/golden/make_golden.py).

CPU only.  These tests are what make the oracle trustworthy as the parity checker
for the CUDA path.  Tolerances are those the reference's own tests use for its fp32
eager path vs. independent recomputation: rtol 1e-3 / atol 1e-4
(tests/test_triton_kernels.py:31) on outputs, and the same on states.
"""
import numpy as np
import pytest

import oracle
from conftest import load_golden, mcmoe_weights

TOL = dict(rtol=1e-3, atol=1e-4)

SSSD = load_golden("sssd")
CHAM = load_golden("cham")
NS = load_golden("ns")
MCMOE = load_golden("mcmoe")


@pytest.mark.parametrize("case", [c for c in SSSD if c != "roundtrip"])
def test_oracle_sssd_matches_reference(case):
    g = SSSD[case]
    b, s, d, h, hid = (int(x) for x in g["dims"])
    out, st = oracle.sssd_forward(g["p"], g["x"], h, d, return_state=True,
                                  active_mask=g.get("mask"), dtype=np.float64)
    np.testing.assert_allclose(out, g["out"], **TOL)
    np.testing.assert_allclose(st, g["state"], **TOL)


def test_oracle_sssd_state_roundtrip_matches_reference():
    g = SSSD["roundtrip"]
    b, s, d, h, hid = (int(x) for x in g["dims"])
    out1, st1 = oracle.sssd_forward(g["p"], g["x1"], h, d, return_state=True)
    out2, st2 = oracle.sssd_forward(g["p"], g["x2"], h, d, initial_state=st1, return_state=True)
    np.testing.assert_allclose(out1, g["out1"], **TOL)
    np.testing.assert_allclose(st1, g["state1"], **TOL)
    np.testing.assert_allclose(out2, g["out2"], **TOL)
    np.testing.assert_allclose(st2, g["state2"], **TOL)


@pytest.mark.parametrize("case", [c for c in CHAM
                                  if c not in ("roundtrip", "nonunitary_h0", "D1024")])
def test_oracle_cham_matches_reference(case):
    g = CHAM[case]
    y, (Hr, Hi) = oracle.cham_forward(g["p"], g["x"], active_mask=g.get("mask"))
    np.testing.assert_allclose(y, g["out"], **TOL)
    np.testing.assert_allclose(Hr, g["Hr"], **TOL)
    np.testing.assert_allclose(Hi, g["Hi"], **TOL)


def test_oracle_cham_roundtrip_matches_reference():
    g = CHAM["roundtrip"]
    y1, H1 = oracle.cham_forward(g["p"], g["x1"])
    y2, H2 = oracle.cham_forward(g["p"], g["x2"], initial_hologram=H1)
    for a, b in [(y1, g["out1"]), (H1[0], g["Hr1"]), (H1[1], g["Hi1"]),
                 (y2, g["out2"]), (H2[0], g["Hr2"]), (H2[1], g["Hi2"])]:
        np.testing.assert_allclose(a, b, **TOL)


def test_oracle_cham_nonunitary_initial_hologram_matches_reference():
    g = CHAM["nonunitary_h0"]
    y, (Hr, Hi) = oracle.cham_forward(g["p"], g["x"], initial_hologram=(g["H0r"], g["H0i"]))
    np.testing.assert_allclose(y, g["out"], **TOL)
    np.testing.assert_allclose(Hr, g["Hr"], **TOL)
    np.testing.assert_allclose(Hi, g["Hi"], **TOL)


def test_oracle_cham_D1024_matches_reference():
    g = CHAM["D1024"]
    y, (Hr, Hi) = oracle.cham_forward(g["p"], g["x"], dtype=np.float32)
    np.testing.assert_allclose(y, g["out"], **TOL)
    np.testing.assert_allclose(Hr[:, :4], g["Hr_rows"], **TOL)
    np.testing.assert_allclose(Hi[:, :4], g["Hi_rows"], **TOL)
    np.testing.assert_allclose(np.diagonal(Hr, axis1=-2, axis2=-1), g["Hr_diag"], **TOL)
    np.testing.assert_allclose(Hr.sum(-2), g["Hr_colsum"], rtol=1e-3, atol=1e-3)
    np.testing.assert_allclose(Hi.sum(-2), g["Hi_colsum"], rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("case", list(NS))
def test_oracle_newton_schulz_matches_reference(case):
    g = NS[case]
    r, i = oracle.newton_schulz_unitary_retraction(g["Hr"].astype(np.float64), g["Hi"].astype(np.float64))
    np.testing.assert_allclose(r, g["out_r"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(i, g["out_i"], rtol=1e-5, atol=1e-5)


def test_oracle_zero_gamma_is_identity():
    """tests/test_triton_kernels.py:200-223: every token halted -> H stays exactly (I, 0)."""
    g = CHAM["zero_gamma"]
    _, (Hr, Hi) = oracle.cham_forward(g["p"], g["x"], active_mask=g["mask"])
    D = Hr.shape[-1]
    np.testing.assert_array_equal(Hr, np.broadcast_to(np.eye(D), Hr.shape))
    np.testing.assert_array_equal(Hi, 0.0)


def test_oracle_detects_a_planted_error():
    """A mistake planted in the oracle's input (one flipped k sign) must break parity,
    so the golden comparison above is not vacuous."""
    g = SSSD["sweep_b2_s8_d16_h2"]
    b, s, d, h, hid = (int(x) for x in g["dims"])
    p = dict(g["p"])
    p["w_k.weight"] = p["w_k.weight"].copy()
    p["w_k.weight"][:d] *= -1.0
    out, _ = oracle.sssd_forward(p, g["x"], h, d, return_state=True)
    assert not np.allclose(out, g["out"], **TOL)


@pytest.mark.parametrize("case", sorted(MCMOE))
def test_oracle_mcmoe_matches_reference(case):
    """ManifoldContinuousMoE.forward (mcmoe.py:58-120): routing, base FFN and output."""
    g = MCMOE[case]
    b, s, d, rank, C, K = (int(x) for x in g["dims"])
    p = mcmoe_weights(g)
    xf = g["x"].reshape(b * s, d).astype(np.float64)
    idx, w = oracle.mcmoe_route(g["logits"].astype(np.float64), min(K, C))
    assert np.array_equal(idx, g["topk_idx"])
    np.testing.assert_allclose(w, g["topk_w"], rtol=1e-5, atol=1e-7)
    pd = {k: v.astype(np.float64) for k, v in p.items()}
    base = oracle.situ_glu(pd, xf) @ pd["base_w_down.weight"].T
    np.testing.assert_allclose(base, g["base"], **TOL)
    y = oracle.mcmoe_forward(p, g["x"], rank, C, K)
    np.testing.assert_allclose(y, g["y"], **TOL)


def test_layer_and_acde_weights_match_the_reference_construction():
    """Our VeraceV1Layer (and its SSSD / CHAM / M-CMoE modules) consume the RNG in the
    reference's order, so seeded construction gives the reference's weights (the layer
    goldens rely on it)."""
    import torch
    import verace_v1_b200 as V
    from conftest import GOLDEN
    z = np.load(f"{GOLDEN}/layer_golden.npz")
    cfg = V.VeraceV1Config(vocab_size=100, hidden_dim=256, num_layers=4, num_heads=2, head_dim=128,
                           spectral_dim=64, chams_holographic_dim=256, mcmoe_rank=16, mcmoe_num_components=8)
    torch.manual_seed(0)
    layers = torch.nn.ModuleList([V.VeraceV1Layer(i, cfg) for i in range(4)])
    sd = layers.state_dict()
    fps = {k[len("layers/fp/"):]: z[k] for k in z.files if k.startswith("layers/fp/")}
    assert sorted(fps) == sorted(sd)
    for k, v in sd.items():
        f = v.detach().double().numpy().ravel()
        np.testing.assert_allclose(np.concatenate([[f.sum(), (f * f).sum()], f[:16]]), fps[k], rtol=1e-6,
                                   atol=1e-6, err_msg=k)
