"""Pins the CPU oracle at benchmark config 1 (one SSSD + CHAM layer in fp32, hidden 1024,
8 heads x 128, D = 1024, b = 2, s = 512) to the reference's own output at that size
(tests/golden/config1_golden.npz, made by tests/golden/make_golden.py --only config1 from
the reference's eager modules, CHAM fed in 64-token chunks through initial_hologram).

Also pins the O(D^2)-per-token CHAM oracle (``cham_scan_rank2`` in numpy and its C twin
``cham_scan_rank2_c``) to the dense per-token oracle (``cham_scan``: dense Cayley solves,
prefix products, per-position Newton-Schulz) on small cases, so that the long-sequence
parity tests can rely on it.  CPU only.
"""
import numpy as np
import pytest

import oracle
from conftest import config1_case


def rel(a, b):
    return float(np.linalg.norm(np.asarray(a) - b) / np.linalg.norm(b))


@pytest.fixture(scope="module")
def c1():
    sssd, cham, x, g = config1_case()
    ps = {k: v.numpy().astype(np.float64) for k, v in sssd.state_dict().items()}
    pc = {k: v.numpy().astype(np.float64) for k, v in cham.state_dict().items()}
    return ps, pc, x.numpy().astype(np.float64), g


def test_oracle_sssd_at_config1_matches_reference(c1):
    ps, _, x, g = c1
    out, psi = oracle.sssd_forward(ps, x, 8, 128, return_state=True)
    # the reference is fp32 (its Blelloch products round at each level); the oracle fp64
    assert rel(out @ g["sketch/r_out"], g["sssd/out_sk"]) <= 1e-4
    assert rel(out[:, g["sketch/rows"]], g["sssd/out_rows"]) <= 1e-4
    assert rel(psi @ g["sketch/r_d"], g["sssd/psi_sk"]) <= 2e-4
    assert rel(np.diagonal(psi, axis1=-2, axis2=-1), g["sssd/psi_diag"]) <= 2e-4


def test_oracle_cham_at_config1_matches_reference(c1):
    _, pc, x, g = c1
    q, k, v, gam = oracle.cham_projections(pc, x)
    rec, (Hr, Hi) = oracle.cham_scan_rank2_c(q, k, v, gam)
    y = oracle.rms_norm(rec @ pc["w_out.weight"].T, pc["norm.weight"], np.finfo(np.float32).eps)
    assert rel(y @ g["sketch/r_out"], g["cham/out_sk"]) <= 1e-4
    assert rel(y[:, g["sketch/rows"]], g["cham/out_rows"]) <= 1e-4
    assert rel(Hr @ g["sketch/r_D"], g["cham/hr_sk"]) <= 1e-4
    assert rel(Hi @ g["sketch/r_D"], g["cham/hi_sk"]) <= 1e-4
    assert rel(np.diagonal(Hr, axis1=-2, axis2=-1), g["cham/hr_diag"]) <= 1e-4


def _inputs(rng, b, s, D):
    nz = lambda *sh: oracle.l2_normalize(rng.standard_normal(sh))
    q, k = nz(b, s, D), nz(b, s, D)
    v = oracle.l2_normalize(oracle.silu(rng.standard_normal((b, s, D))))
    return q, k, v, 0.1 * oracle.sigmoid(rng.standard_normal((b, s)))


@pytest.mark.parametrize("b,s,D,kind", [(2, 9, 16, "fresh"), (2, 7, 24, "nonunitary"), (1, 6, 64, "nonunitary"),
                                        (2, 5, 20, "masked"), (1, 4, 128, "fresh")])
def test_rank2_cham_oracle_equals_dense_oracle(b, s, D, kind):
    rng = np.random.default_rng(D + s)
    q, k, v, gam = _inputs(rng, b, s, D)
    H0 = None
    if kind == "nonunitary":
        H0 = (np.eye(D) + 0.05 * rng.standard_normal((b, D, D)), 0.05 * rng.standard_normal((b, D, D)))
    if kind == "masked":
        gam[:, 2:4] = 0.0
    r_d, (hr_d, hi_d) = oracle.cham_scan(q, k, v, gam, H0)
    r_n, (hr_n, hi_n), dense = oracle.cham_scan_rank2(q, k, v, gam, H0, dense_ns_at=range(s))
    r_c, (hr_c, hi_c) = oracle.cham_scan_rank2_c(q, k, v, gam, H0)
    for a in (r_n, r_c):
        np.testing.assert_allclose(a, r_d, rtol=0, atol=1e-12)
    for a, bb in ((hr_n, hr_d), (hi_n, hi_d), (hr_c, hr_d), (hi_c, hi_d)):
        np.testing.assert_allclose(a, bb, rtol=0, atol=1e-12)
    for t, rt in dense.items():      # the NS identity against the dense retraction of H_t
        np.testing.assert_allclose(rt, r_d[:, t], rtol=0, atol=1e-12)
