"""benchmark config 1 at its own size on the GPU: one SSSD + CHAM layer in fp32, hidden
1024, 8 heads x 128, D = 1024, x = randn(2, 512, 1024) under seed 0, weights seeded as
the reference built them (checked against the reference's fingerprints).

The drop-in modules' outputs and exported states are compared with the reference's own
output at this size (tests/golden/config1_golden.npz: sketches with fixed random matrices
plus full rows at ten positions) and with the fp64 oracle (full tensors).  Tolerances are
north_star's fp32 bar, relative Frobenius error <= 1e-4, except for the SSSD state against
the reference file: the reference's fp32 Blelloch products leave its own Psi 8e-5 from
the fp64 oracle (tests/test_oracle_config1.py), so that comparison allows 2e-4 and the
1e-4 bar is applied against the fp64 oracle instead.  Invariants: the SSSD state is
orthogonal and the retracted CHAM state unitary to max-abs 1e-3.
"""
import numpy as np
import pytest
import torch

import oracle
import verace_v1_b200 as V
from conftest import config1_case
from gpu_util import rel_fro, to_np

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def c1():
    sssd, cham, x, g = config1_case()
    ps = {k: v.numpy().astype(np.float64) for k, v in sssd.state_dict().items()}
    pc = {k: v.numpy().astype(np.float64) for k, v in cham.state_dict().items()}
    xn = x.numpy().astype(np.float64)
    o_ref, psi_ref = oracle.sssd_forward(ps, xn, 8, 128, return_state=True)
    q, k, v, gam = oracle.cham_projections(pc, xn)
    rec, H = oracle.cham_scan_rank2_c(q, k, v, gam)
    y_ref = oracle.rms_norm(rec @ pc["w_out.weight"].T, pc["norm.weight"], np.finfo(np.float32).eps)
    dev = torch.device("cuda")
    return dict(sssd=sssd.to(dev).eval(), cham=cham.to(dev).eval(), x=x.to(dev), g=g,
                o_ref=o_ref, psi_ref=psi_ref, y_ref=y_ref, H_ref=H)


def test_sssd_config1_matches_reference_and_oracle(c1):
    g = c1["g"]
    with torch.no_grad():
        out, psi = c1["sssd"](c1["x"], return_state=True)
    out, psi = to_np(out), to_np(psi)
    assert rel_fro(out @ g["sketch/r_out"], g["sssd/out_sk"]) <= 1e-4
    assert rel_fro(out[:, g["sketch/rows"]], g["sssd/out_rows"]) <= 1e-4
    assert rel_fro(psi @ g["sketch/r_d"], g["sssd/psi_sk"]) <= 2e-4
    assert rel_fro(out, c1["o_ref"]) <= 1e-4
    assert rel_fro(psi, c1["psi_ref"]) <= 1e-4
    eye = np.eye(128)
    assert np.abs(np.swapaxes(psi, -1, -2).astype(np.float64) @ psi - eye).max() <= 1e-3


@pytest.mark.parametrize("chunked", [False, True], ids=["one_call", "64_token_calls"])
def test_cham_config1_matches_reference_and_oracle(c1, chunked):
    g, x = c1["g"], c1["x"]
    with torch.no_grad():
        if chunked:    # the survey's chunked drive: 8 calls through initial_hologram
            H, ys = None, []
            for c0 in range(0, 512, 64):
                y, H = c1["cham"](x[:, c0:c0 + 64], initial_hologram=H)
                ys.append(y)
            y = torch.cat(ys, dim=1)
        else:
            y, H = c1["cham"](x)
        Hq = V.newton_schulz_unitary_retraction(H[0], H[1], 3)
    y, hr, hi = to_np(y), to_np(H[0]), to_np(H[1])
    assert rel_fro(y @ g["sketch/r_out"], g["cham/out_sk"]) <= 1e-4
    assert rel_fro(y[:, g["sketch/rows"]], g["cham/out_rows"]) <= 1e-4
    assert rel_fro(hr @ g["sketch/r_D"], g["cham/hr_sk"]) <= 1e-4
    assert rel_fro(hi @ g["sketch/r_D"], g["cham/hi_sk"]) <= 1e-4
    assert rel_fro(y, c1["y_ref"]) <= 1e-4
    assert rel_fro(hr + 1j * hi, c1["H_ref"][0] + 1j * c1["H_ref"][1]) <= 1e-4
    Q = to_np(Hq[0]).astype(np.float64) + 1j * to_np(Hq[1])
    QhQ = np.conj(np.swapaxes(Q, -1, -2)) @ Q
    assert np.abs(QhQ - np.eye(1024)).max() <= 1e-3
    Hc = hr.astype(np.float64) + 1j * hi
    assert np.abs(np.conj(np.swapaxes(Hc, -1, -2)) @ Hc - np.eye(1024)).max() <= 1e-3
