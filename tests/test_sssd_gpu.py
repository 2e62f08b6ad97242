"""SSSD parity on the B200: the sm_100a scan (through the C ABI) against the reference's
own outputs (golden vectors) and against the fp64 oracle.

Tolerances: the reference's kernel-vs-eager tolerance rtol 1e-3 / atol 1e-4
(tests/test_triton_kernels.py:31) elementwise, and the north-star bound
relative Frobenius error <= 1e-4 for fp32 (<= 2e-2 for bf16 inputs), on outputs and
exported states.  Orthogonality of the state from Psi_0 = I: max|PsiᵀPsi - I| <= 1e-3.
"""
import numpy as np
import pytest
import torch

import oracle
import verace_v1_b200 as V
from conftest import load_golden
from gpu_util import random_sssd_inputs, rel_fro, sssd_module, to_np

pytestmark = pytest.mark.gpu
TOL = dict(rtol=1e-3, atol=1e-4)
SSSD = load_golden("sssd")


@pytest.mark.parametrize("case", [c for c in SSSD if c != "roundtrip"])
def test_sssd_module_matches_reference_golden(case):
    g = SSSD[case]
    b, s, d, h, hid = (int(x) for x in g["dims"])
    m = sssd_module(g)
    x = torch.from_numpy(g["x"]).cuda()
    mask = torch.from_numpy(g["mask"]).cuda() if "mask" in g else None
    with torch.no_grad():
        out, st = m(x, return_state=True, active_mask=mask)
    np.testing.assert_allclose(to_np(out), g["out"], **TOL)
    np.testing.assert_allclose(to_np(st), g["state"], **TOL)
    assert rel_fro(to_np(out), g["out"]) <= 1e-4
    assert rel_fro(to_np(st), g["state"]) <= 1e-4


def test_sssd_initial_state_roundtrip_matches_reference_golden():
    g = SSSD["roundtrip"]
    m = sssd_module(g)
    with torch.no_grad():
        out1, st1 = m(torch.from_numpy(g["x1"]).cuda(), return_state=True)
        out2, st2 = m(torch.from_numpy(g["x2"]).cuda(), initial_state=st1, return_state=True)
    for a, b in [(out1, g["out1"]), (st1, g["state1"]), (out2, g["out2"]), (st2, g["state2"])]:
        np.testing.assert_allclose(to_np(a), b, **TOL)


@pytest.mark.parametrize("b,s,h,d", [(2, 8, 2, 16), (1, 1, 1, 16), (2, 13, 2, 16), (2, 8, 2, 24),
                                     (1, 33, 2, 128), (2, 100, 3, 64), (1, 129, 1, 128), (1, 64, 2, 5)])
def test_sssd_scan_matches_fp64_oracle(b, s, h, d):
    q, k, v, delta = random_sssd_inputs(b, s, h, d, seed=100 + s + d)
    out, st = V.launch_sssd_scan(q, k, v, delta)
    o_ref, st_ref = oracle.sssd_scan(to_np(q), to_np(k), to_np(v), to_np(delta))
    assert rel_fro(to_np(out), o_ref) <= 1e-4
    assert rel_fro(to_np(st), st_ref) <= 1e-4
    np.testing.assert_allclose(to_np(out), o_ref, **TOL)


def test_sssd_scan_with_initial_state_and_mask_matches_oracle():
    b, s, h, d = 2, 70, 2, 128
    q, k, v, delta = random_sssd_inputs(b, s, h, d, seed=7)
    delta[:, 20:35] = 0.0          # halted tokens: exact identity factors
    gen = torch.Generator().manual_seed(8)
    psi0 = torch.linalg.qr(torch.randn(b, h, d, d, generator=gen))[0].cuda()
    out, st = V.launch_sssd_scan(q, k, v, delta, psi0)
    o_ref, st_ref = oracle.sssd_scan(to_np(q), to_np(k), to_np(v), to_np(delta), to_np(psi0))
    assert rel_fro(to_np(out), o_ref) <= 1e-4
    assert rel_fro(to_np(st), st_ref) <= 1e-4


def test_sssd_bf16_inputs_within_bf16_tolerance():
    b, s, h, d = 2, 96, 4, 128
    q, k, v, delta = random_sssd_inputs(b, s, h, d, seed=9, dtype=torch.bfloat16)
    out, st = V.launch_sssd_scan(q, k, v, delta)
    assert out.dtype == torch.bfloat16 and st.dtype == torch.float32
    o_ref, st_ref = oracle.sssd_scan(to_np(q), to_np(k), to_np(v), to_np(delta))
    assert rel_fro(to_np(out), o_ref) <= 2e-2
    assert rel_fro(to_np(st), st_ref) <= 1e-4   # the state is fp32 from bf16-exact inputs


def test_sssd_state_stays_orthogonal_over_long_sequence():
    """tests/test_sssd.py:10-26 (norm conservation), at 2048 tokens and d=128."""
    b, s, h, d = 1, 2048, 2, 128
    q, k, v, delta = random_sssd_inputs(b, s, h, d, seed=11)
    _, st = V.launch_sssd_scan(q, k, v, delta)
    eye = torch.eye(d, device="cuda")
    dev = (st.transpose(-1, -2) @ st - eye).abs().max().item()
    assert dev <= 1e-3
    norm = torch.linalg.matrix_norm(st[0, 0]).item()
    assert abs(norm - d ** 0.5) < 1e-3


def test_sssd_chunked_continuation_equals_one_shot():
    b, s, h, d = 2, 300, 2, 128
    q, k, v, delta = random_sssd_inputs(b, s, h, d, seed=12)
    out, st = V.launch_sssd_scan(q, k, v, delta)
    o1, s1 = V.launch_sssd_scan(q[:, :77], k[:, :77], v[:, :77], delta[:, :77])
    o2, s2 = V.launch_sssd_scan(q[:, 77:], k[:, 77:], v[:, 77:], delta[:, 77:], s1)
    torch.testing.assert_close(torch.cat([o1, o2], 1), out, rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(s2, st, rtol=1e-4, atol=1e-5)


def test_sssd_nonfinite_token_is_replaced_by_identity():
    """A token whose factor is non-finite acts as the identity, as the reference's
    _solve_cayley substitution makes it (sssd_attention.py:52-71)."""
    b, s, h, d = 1, 40, 1, 32
    q, k, v, delta = random_sssd_inputs(b, s, h, d, seed=13)
    k_bad = k.clone()
    k_bad[0, 17, 0, 3] = float("nan")
    out_bad, st_bad = V.launch_sssd_scan(q, k_bad, v, delta)
    delta_id = delta.clone()
    delta_id[0, 17, 0] = 0.0
    out_id, st_id = V.launch_sssd_scan(q, k, v, delta_id)
    torch.testing.assert_close(st_bad, st_id)
    torch.testing.assert_close(out_bad, out_id)


def test_sssd_empty_sequence_returns_initial_state():
    q, k, v, delta = random_sssd_inputs(2, 0, 2, 16, seed=1)
    out, st = V.launch_sssd_scan(q, k, v, delta)
    assert out.shape == (2, 0, 2, 16)
    torch.testing.assert_close(st, torch.eye(16, device="cuda").expand(2, 2, 16, 16))


def test_sssd_rejects_cpu_and_grad_inputs():
    m = V.SSSDAttention(32, 2, 16)
    with pytest.raises(RuntimeError, match="inference path"):
        m(torch.randn(1, 4, 32))
    with pytest.raises(AssertionError, match="CUDA"):
        V.launch_sssd_scan(*[torch.randn(1, 2, 1, 4) for _ in range(3)], torch.rand(1, 2, 1))
