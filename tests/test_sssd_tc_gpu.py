"""The tcgen05 SSSD scan (head_dim 128, state resident in tensor memory) against the
fp64 oracle and against the fp32 SIMT kernels, across 64-token chunk boundaries,
carried states, halted and non-finite tokens, fp32 and bf16 inputs.

Tolerances: relative Frobenius <= 1e-4 vs the fp64 oracle for fp32 inputs (outputs and
states), <= 2e-2 on bf16 outputs, orthogonality of the state <= 1e-3.
"""
import os

import numpy as np
import pytest
import torch

import oracle
import verace_v1_b200 as V
from gpu_util import random_sssd_inputs, rel_fro, to_np
from verace_v1_b200 import _lib

pytestmark = pytest.mark.gpu


def _status_ok():
    _lib.check(_lib.lib().verace_device_status(torch.cuda.current_stream().cuda_stream), "device status")


def _simt(*args):
    os.environ["VERACE_SSSD_SIMT"] = "1"
    try:
        return V.launch_sssd_scan(*args)
    finally:
        del os.environ["VERACE_SSSD_SIMT"]


@pytest.mark.parametrize("b,s,h", [(1, 1, 1), (2, 63, 2), (1, 64, 1), (2, 65, 3), (1, 200, 2)])
def test_tc_sssd_fp32_matches_fp64_oracle(b, s, h):
    q, k, v, delta = random_sssd_inputs(b, s, h, 128, seed=800 + s + h)
    out, st = V.launch_sssd_scan(q, k, v, delta)
    _status_ok()
    o_ref, st_ref = oracle.sssd_scan(to_np(q), to_np(k), to_np(v), to_np(delta))
    assert rel_fro(to_np(out), o_ref) <= 1e-4
    assert rel_fro(to_np(st), st_ref) <= 1e-4


def test_tc_sssd_bf16_with_state_and_halted_tokens():
    b, s, h = 2, 150, 4
    q, k, v, delta = random_sssd_inputs(b, s, h, 128, seed=901, dtype=torch.bfloat16)
    delta[:, 40:70] = 0.0
    gen = torch.Generator().manual_seed(902)
    psi0 = torch.linalg.qr(torch.randn(b, h, 128, 128, generator=gen))[0].cuda()
    out, st = V.launch_sssd_scan(q, k, v, delta, psi0)
    _status_ok()
    o_ref, st_ref = oracle.sssd_scan(to_np(q), to_np(k), to_np(v), to_np(delta), to_np(psi0))
    assert rel_fro(to_np(out), o_ref) <= 2e-2
    assert rel_fro(to_np(st), st_ref) <= 1e-4


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_tc_sssd_matches_simt_kernels_long_sequence(dtype):
    q, k, v, delta = random_sssd_inputs(2, 1000, 4, 128, seed=903, dtype=dtype)
    out, st = V.launch_sssd_scan(q, k, v, delta)
    _status_ok()
    out_s, st_s = _simt(q, k, v, delta)
    assert rel_fro(to_np(out), to_np(out_s)) <= (1e-4 if dtype == torch.float32 else 1e-2)
    assert rel_fro(to_np(st), to_np(st_s)) <= 1e-4
    eye = torch.eye(128, device="cuda")
    assert (st.transpose(-1, -2) @ st - eye).abs().max().item() <= 1e-3


def test_tc_sssd_nonfinite_token_is_identity():
    q, k, v, delta = random_sssd_inputs(1, 130, 2, 128, seed=904)
    v_bad = v.clone()
    v_bad[0, 100, 1, 7] = float("inf")
    out_b, st_b = V.launch_sssd_scan(q, k, v_bad, delta)
    d_id = delta.clone()
    d_id[0, 100, 1] = 0.0
    out_i, st_i = V.launch_sssd_scan(q, k, v, d_id)
    _status_ok()
    torch.testing.assert_close(st_b, st_i)
    torch.testing.assert_close(out_b, out_i)


def test_tc_sssd_bf16_split_launch_chunk_ranges():
    """bf16 with few chains and many chunks takes the split launch (the prep of chunk range
    p + 1 beside the scan of range p, the state passed on through psi_out): 10 chunks in
    uneven ranges, a partial last chunk, a carried state, halted tokens across a range
    boundary and a non-finite token; then the same call again (shared side-stream
    resources)."""
    b, s, h = 1, 613, 8
    q, k, v, delta = random_sssd_inputs(b, s, h, 128, seed=905, dtype=torch.bfloat16)
    delta[:, 120:200] = 0.0
    k[0, 333, 5, 11] = float("nan")
    gen = torch.Generator().manual_seed(906)
    psi0 = torch.linalg.qr(torch.randn(b, h, 128, 128, generator=gen))[0].cuda()
    out, st = V.launch_sssd_scan(q, k, v, delta, psi0)
    _status_ok()
    d_ref = to_np(delta).copy()
    d_ref[0, 333, 5] = 0.0
    k_ref = to_np(k).copy()
    k_ref[0, 333, 5, 11] = 0.0
    o_ref, st_ref = oracle.sssd_scan(to_np(q), k_ref, to_np(v), d_ref, to_np(psi0))
    assert np.isfinite(to_np(out)).all()
    assert rel_fro(to_np(out), o_ref) <= 2e-2
    assert rel_fro(to_np(st), st_ref) <= 1e-4
    out2, st2 = V.launch_sssd_scan(q, k, v, delta, psi0)
    torch.testing.assert_close(out2, out, rtol=0, atol=0)
    torch.testing.assert_close(st2, st, rtol=0, atol=0)
