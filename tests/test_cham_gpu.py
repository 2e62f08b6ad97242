"""CHAM parity on the B200: the sm_100a scan + readout retraction (through the C ABI)
against the reference's outputs (golden vectors) and the fp64 oracle, plus the
reference's invariants at production width D = 1024.

Tolerances: the reference's fp64-gold tolerance rtol 1e-4 / atol 1e-4
(tests/test_triton_kernels.py:32) on module outputs, relative Frobenius <= 1e-4 for
fp32 scans (<= 2e-2 with bf16 inputs), unitarity of the retracted state
max|HᴴH - I| <= 1e-3.
"""
import numpy as np
import pytest
import torch

import oracle
import verace_v1_b200 as V
from conftest import load_golden
from gpu_util import cham_module, random_cham_inputs, rel_fro, to_np

pytestmark = pytest.mark.gpu
TOL = dict(rtol=1e-3, atol=1e-4)
FP64_TOL = dict(rtol=1e-4, atol=1e-4)
CHAM = load_golden("cham")
NS = load_golden("ns")


@pytest.mark.parametrize("case", [c for c in CHAM if c not in ("roundtrip", "nonunitary_h0", "D1024")])
def test_cham_module_matches_reference_golden(case):
    g = CHAM[case]
    m = cham_module(g)
    x = torch.from_numpy(g["x"]).cuda()
    mask = torch.from_numpy(g["mask"]).cuda() if "mask" in g else None
    with torch.no_grad():
        y, (Hr, Hi) = m(x, active_mask=mask)
    np.testing.assert_allclose(to_np(y), g["out"], **TOL)
    np.testing.assert_allclose(to_np(Hr), g["Hr"], **TOL)
    np.testing.assert_allclose(to_np(Hi), g["Hi"], **TOL)
    # fp64 gold (the oracle in float64, = _cham_fp64_reference of the reference tests)
    gold, _ = oracle.cham_forward(g["p"], g["x"], active_mask=g.get("mask"), dtype=np.float64)
    np.testing.assert_allclose(to_np(y), gold, **FP64_TOL)


def test_cham_roundtrip_matches_reference_golden():
    g = CHAM["roundtrip"]
    m = cham_module(g)
    with torch.no_grad():
        y1, H1 = m(torch.from_numpy(g["x1"]).cuda())
        y2, H2 = m(torch.from_numpy(g["x2"]).cuda(), initial_hologram=H1)
    for a, b in [(y1, g["out1"]), (H1[0], g["Hr1"]), (H1[1], g["Hi1"]),
                 (y2, g["out2"]), (H2[0], g["Hr2"]), (H2[1], g["Hi2"])]:
        np.testing.assert_allclose(to_np(a), b, **TOL)


def test_cham_nonunitary_initial_hologram_matches_reference_golden():
    """H_0 far from unitary: the readout retraction of H_0 is what is being tested."""
    g = CHAM["nonunitary_h0"]
    m = cham_module(g)
    H0 = (torch.from_numpy(g["H0r"]).cuda(), torch.from_numpy(g["H0i"]).cuda())
    with torch.no_grad():
        y, (Hr, Hi) = m(torch.from_numpy(g["x"]).cuda(), initial_hologram=H0)
    np.testing.assert_allclose(to_np(y), g["out"], **TOL)
    np.testing.assert_allclose(to_np(Hr), g["Hr"], **TOL)
    np.testing.assert_allclose(to_np(Hi), g["Hi"], **TOL)


def test_cham_D1024_matches_reference_golden():
    g = CHAM["D1024"]
    m = cham_module(g)
    with torch.no_grad():
        y, (Hr, Hi) = m(torch.from_numpy(g["x"]).cuda())
    np.testing.assert_allclose(to_np(y), g["out"], **TOL)
    np.testing.assert_allclose(to_np(Hr[:, :4]), g["Hr_rows"], **TOL)
    np.testing.assert_allclose(to_np(Hi[:, :4]), g["Hi_rows"], **TOL)
    np.testing.assert_allclose(to_np(torch.diagonal(Hr, dim1=-2, dim2=-1)), g["Hr_diag"], **TOL)
    np.testing.assert_allclose(to_np(Hr.sum(-2)), g["Hr_colsum"], rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("case", list(NS))
def test_newton_schulz_retraction_matches_reference_golden(case):
    g = NS[case]
    r, i = V.newton_schulz_unitary_retraction(torch.from_numpy(g["Hr"]).cuda(), torch.from_numpy(g["Hi"]).cuda())
    np.testing.assert_allclose(to_np(r), g["out_r"], rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(to_np(i), g["out_i"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("b,D,scale", [(2, 1024, 0.02), (3, 256, 0.03), (1, 200, 0.03)])
def test_newton_schulz_retraction_at_width_matches_fp64_oracle(b, D, scale):
    """The dense retraction (tensor-core complex GEMMs, fp32 operands in three bf16 parts)
    against the fp64 oracle on holograms drifted off the unitary group (||HᴴH - I||_2 from
    0.35 to 0.55: inside the region where the iteration converges, sigma^2 < 3), widths that
    do and do not fill the 128 x 128 GEMM tiles."""
    gen = torch.Generator().manual_seed(D)
    Hr = torch.eye(D).expand(b, D, D) + scale * torch.randn(b, D, D, generator=gen) / (D / 16) ** 0.5
    Hi = scale * torch.randn(b, D, D, generator=gen) / (D / 16) ** 0.5
    r, i = V.newton_schulz_unitary_retraction(Hr.cuda(), Hi.cuda())
    rr, ri = oracle.newton_schulz_unitary_retraction(Hr.double().numpy(), Hi.double().numpy())
    err = rel_fro(to_np(r) + 1j * to_np(i), rr + 1j * ri)
    print(f"retraction b={b} D={D} scale={scale}: relative error {err:.2e}")
    assert err <= 1e-5
    np.testing.assert_allclose(to_np(r), rr, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(to_np(i), ri, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("b,s,D", [(2, 8, 16), (1, 1, 16), (2, 5, 20), (2, 40, 64), (1, 70, 160),
                                   (1, 33, 100), (2, 6, 1024)])
def test_cham_scan_matches_fp64_oracle(b, s, D):
    q, k, v, gamma = random_cham_inputs(b, s, D, seed=200 + s + D)
    out, (Hr, Hi) = V.launch_cham_update(q, k, v, gamma)
    r_ref, (Hr_ref, Hi_ref) = oracle.cham_scan(to_np(q), to_np(k), to_np(v), to_np(gamma))
    assert rel_fro(to_np(out), r_ref) <= 1e-4
    assert rel_fro(to_np(Hr), Hr_ref) <= 1e-4
    assert rel_fro(to_np(Hi), Hi_ref) <= 1e-4 * max(1.0, np.linalg.norm(Hr_ref) / max(np.linalg.norm(Hi_ref), 1e-30))


@pytest.mark.parametrize("b,s,D", [(2, 9, 24), (1, 40, 64), (1, 3, 1024)])
def test_cham_scan_nonunitary_h0_matches_fp64_oracle(b, s, D):
    q, k, v, gamma = random_cham_inputs(b, s, D, seed=300 + s + D)
    gen = torch.Generator().manual_seed(5)
    H0r = (torch.eye(D) + 0.05 * torch.randn(b, D, D, generator=gen) / (D / 16) ** 0.5).cuda()
    H0i = (0.05 * torch.randn(b, D, D, generator=gen) / (D / 16) ** 0.5).cuda()
    out, (Hr, Hi) = V.launch_cham_update(q, k, v, gamma, (H0r, H0i))
    r_ref, (Hr_ref, Hi_ref) = oracle.cham_scan(to_np(q), to_np(k), to_np(v), to_np(gamma), (to_np(H0r), to_np(H0i)))
    assert rel_fro(to_np(out), r_ref) <= 1e-4
    assert rel_fro(to_np(Hr), Hr_ref) <= 1e-4


def test_cham_bf16_inputs_within_bf16_tolerance():
    q, k, v, gamma = random_cham_inputs(2, 40, 256, seed=21, dtype=torch.bfloat16)
    out, (Hr, Hi) = V.launch_cham_update(q, k, v, gamma)
    assert out.dtype == torch.bfloat16 and Hr.dtype == torch.float32
    r_ref, (Hr_ref, _) = oracle.cham_scan(to_np(q), to_np(k), to_np(v), to_np(gamma))
    assert rel_fro(to_np(out), r_ref) <= 2e-2
    assert rel_fro(to_np(Hr), Hr_ref) <= 1e-4


def test_cham_zero_gamma_is_exact_noop():
    """tests/test_triton_kernels.py:200-223: every token halted -> H stays exactly (I, 0)."""
    q, k, v, gamma = random_cham_inputs(2, 45, 64, seed=22)
    out, (Hr, Hi) = V.launch_cham_update(q, k, v, torch.zeros_like(gamma))
    assert torch.equal(Hr, torch.eye(64, device="cuda").expand(2, 64, 64))
    assert torch.equal(Hi, torch.zeros_like(Hi))
    torch.testing.assert_close(out, q)    # readout of the identity hologram is q itself


def test_cham_D1024_long_sequence_invariants():
    """At production width: raw state stays unitary (tests/test_cham.py:301-349 bound
    0.05 on ||HᴴH - I||_F), its retraction is unitary to 1e-3, chunked continuation
    equals one shot, and the last readout equals Re(NS3(H_T)) q_T formed densely."""
    b, s, D = 1, 256, 1024
    q, k, v, gamma = random_cham_inputs(b, s, D, seed=23)
    out, (Hr, Hi) = V.launch_cham_update(q, k, v, gamma)
    HH_r = Hr[0].T @ Hr[0] + Hi[0].T @ Hi[0]
    eye = torch.eye(D, device="cuda")
    assert torch.linalg.matrix_norm(HH_r - eye).item() < 0.05
    Rr, Ri = V.newton_schulz_unitary_retraction(Hr, Hi)
    HHr = Rr[0].T @ Rr[0] + Ri[0].T @ Ri[0]
    HHi = Rr[0].T @ Ri[0] - Ri[0].T @ Rr[0]
    assert (HHr - eye).abs().max().item() <= 1e-3 and HHi.abs().max().item() <= 1e-3
    last = Rr[0] @ q[0, -1]
    assert rel_fro(to_np(out[0, -1]), to_np(last)) <= 1e-4
    o1, H1 = V.launch_cham_update(q[:, :100], k[:, :100], v[:, :100], gamma[:, :100])
    o2, H2 = V.launch_cham_update(q[:, 100:], k[:, 100:], v[:, 100:], gamma[:, 100:], H1)
    assert rel_fro(to_np(torch.cat([o1, o2], 1)), to_np(out)) <= 1e-4
    assert rel_fro(to_np(H2[0]), to_np(Hr)) <= 1e-4


def test_cham_nonfinite_token_is_replaced_by_identity():
    q, k, v, gamma = random_cham_inputs(1, 50, 48, seed=24)
    v_bad = v.clone()
    v_bad[0, 33, 5] = float("inf")
    out_bad, (Hr_bad, Hi_bad) = V.launch_cham_update(q, k, v_bad, gamma)
    g_id = gamma.clone()
    g_id[0, 33] = 0.0
    out_id, (Hr_id, Hi_id) = V.launch_cham_update(q, k, v, g_id)
    torch.testing.assert_close(Hr_bad, Hr_id)
    torch.testing.assert_close(out_bad, out_id)


def test_cham_empty_sequence_returns_initial_state():
    q, k, v, gamma = random_cham_inputs(2, 0, 16, seed=1)
    out, (Hr, Hi) = V.launch_cham_update(q, k, v, gamma)
    assert out.shape == (2, 0, 16)
    assert torch.equal(Hr, torch.eye(16, device="cuda").expand(2, 16, 16)) and not Hi.any()
