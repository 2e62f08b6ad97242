"""The tcgen05 CHAM scan (holographic width a multiple of 128, fresh hologram) against
the fp64 oracle and against the fp32 SIMT kernels, across chunk boundaries (64-token
chunks), batch sizes, input dtypes and edge cases.

Tolerances: relative Frobenius <= 1e-4 vs the fp64 oracle for fp32 inputs (the
north-star fp32 bound), <= 2e-2 on bf16 outputs, <= 1e-4 on fp32 states.
"""
import os

import numpy as np
import pytest
import torch

import oracle
import verace_v1_b200 as V
from gpu_util import random_cham_inputs, rel_fro, to_np
from verace_v1_b200 import _lib

pytestmark = pytest.mark.gpu


def _status_ok():
    _lib.check(_lib.lib().verace_device_status(torch.cuda.current_stream().cuda_stream), "device status")


def _simt(q, k, v, g):
    os.environ["VERACE_CHAM_SIMT"] = "1"
    try:
        return V.launch_cham_update(q, k, v, g)
    finally:
        del os.environ["VERACE_CHAM_SIMT"]


@pytest.mark.parametrize("b,s,D", [(1, 1, 128), (2, 63, 128), (1, 64, 128), (2, 65, 256),
                                   (1, 130, 128), (3, 7, 256)])
def test_tc_scan_fp32_matches_fp64_oracle(b, s, D):
    q, k, v, g = random_cham_inputs(b, s, D, seed=400 + s + D)
    out, (Hr, Hi) = V.launch_cham_update(q, k, v, g)
    _status_ok()
    r_ref, (Hr_ref, Hi_ref) = oracle.cham_scan(to_np(q), to_np(k), to_np(v), to_np(g))
    assert rel_fro(to_np(out), r_ref) <= 1e-4
    assert rel_fro(to_np(Hr), Hr_ref) <= 1e-4
    assert np.abs(to_np(Hi) - Hi_ref).max() <= 1e-4


@pytest.mark.parametrize("b,s,D", [(2, 100, 256), (1, 64, 1024)])
def test_tc_scan_bf16_matches_fp64_oracle(b, s, D):
    q, k, v, g = random_cham_inputs(b, s, D, seed=500 + s, dtype=torch.bfloat16)
    out, (Hr, Hi) = V.launch_cham_update(q, k, v, g)
    _status_ok()
    assert out.dtype == torch.bfloat16
    r_ref, (Hr_ref, Hi_ref) = oracle.cham_scan(to_np(q), to_np(k), to_np(v), to_np(g))
    assert rel_fro(to_np(out), r_ref) <= 2e-2
    assert rel_fro(to_np(Hr), Hr_ref) <= 1e-4
    assert np.abs(to_np(Hi) - Hi_ref).max() <= 1e-4


@pytest.mark.parametrize("sched", ["batched", "fused"])
@pytest.mark.parametrize("b,s,D", [(2, 700, 256), (1, 64, 128), (3, 65, 128), (2, 1733, 128)])
def test_tc_scan_bf16_schedules_match_fp64_oracle(sched, b, s, D):
    """The column-pass schedules chosen at larger batches (state in place with TMA
    reductions and ring copies for the readout; one fused pass per chunk), forced at sizes
    the oracle runs in seconds.  s = 700 is 11 chunks, one group of the batched schedule;
    s = 1733 is 28 chunks: groups of 12, 12 and 4, the second and third group launches
    running the previous group's readouts from the pre-split ring, whose 24 slots are
    reused by chunks 24-26."""
    q, k, v, g = random_cham_inputs(b, s, D, seed=550 + s, dtype=torch.bfloat16)
    os.environ["VERACE_CHAM_SCHEDULE"] = sched
    try:
        out, (Hr, Hi) = V.launch_cham_update(q, k, v, g)
    finally:
        del os.environ["VERACE_CHAM_SCHEDULE"]
    _status_ok()
    r_ref, (Hr_ref, Hi_ref) = oracle.cham_scan(to_np(q), to_np(k), to_np(v), to_np(g))
    assert rel_fro(to_np(out), r_ref) <= 2e-2
    assert rel_fro(to_np(Hr), Hr_ref) <= 1e-4
    assert np.abs(to_np(Hi) - Hi_ref).max() <= 1e-4


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_tc_scan_matches_simt_kernels_at_production_width(dtype):
    q, k, v, g = random_cham_inputs(2, 200, 1024, seed=600, dtype=dtype)
    out, (Hr, Hi) = V.launch_cham_update(q, k, v, g)
    _status_ok()
    out_s, (Hr_s, Hi_s) = _simt(q, k, v, g)
    assert rel_fro(to_np(out), to_np(out_s)) <= (1e-4 if dtype == torch.float32 else 1e-2)
    assert rel_fro(to_np(Hr), to_np(Hr_s)) <= 1e-5
    assert rel_fro(to_np(Hi), to_np(Hi_s)) <= 1e-4


def test_tc_scan_zero_gamma_and_nonfinite_tokens():
    q, k, v, g = random_cham_inputs(2, 70, 128, seed=700)
    out, (Hr, Hi) = V.launch_cham_update(q, k, v, torch.zeros_like(g))
    _status_ok()
    torch.testing.assert_close(Hr, torch.eye(128, device="cuda").expand(2, 128, 128), rtol=0, atol=1e-6)
    assert Hi.abs().max().item() <= 1e-6
    torch.testing.assert_close(out, q, rtol=1e-5, atol=1e-5)
    k_bad = k.clone()
    k_bad[1, 66, 3] = float("nan")
    out_b, (Hr_b, _) = V.launch_cham_update(q, k_bad, v, g)
    g_id = g.clone()
    g_id[1, 66] = 0.0
    out_i, (Hr_i, _) = V.launch_cham_update(q, k, v, g_id)
    _status_ok()
    torch.testing.assert_close(Hr_b, Hr_i)
    torch.testing.assert_close(out_b, out_i)


@pytest.mark.parametrize("b,s,D", [(3, 600, 256), (2, 130, 1024), (1, 64, 128), (2, 10, 128), (2, 1733, 128),
                                   (1, 900, 1024)])
def test_schedules_agree(b, s, D):
    """The three bf16 schedules (merged per-chunk launches; column passes two CTAs per SM
    with batched readouts; one fused pass per chunk) run the same arithmetic, so the
    results agree to fp32 accumulation order (the E partials are summed atomically)."""
    q, k, v, g = random_cham_inputs(b, s, D, seed=800 + s, dtype=torch.bfloat16)
    k[0, min(5, s - 1), 3] = float("nan")
    res = {}
    try:
        for sched in ("merged", "batched", "fused"):
            os.environ["VERACE_CHAM_SCHEDULE"] = sched
            res[sched] = V.launch_cham_update(q, k, v, g)
    finally:
        del os.environ["VERACE_CHAM_SCHEDULE"]
    _status_ok()
    out_m, (Hr_m, Hi_m) = res["merged"]
    for sched in ("batched", "fused"):
        out, (Hr, Hi) = res[sched]
        # the complex state against its own norm (its imaginary part is ~50x smaller, and the
        # schedules sum the hi- and lo-operand products in different orders)
        H, H_m = to_np(Hr) + 1j * to_np(Hi), to_np(Hr_m) + 1j * to_np(Hi_m)
        assert rel_fro(H, H_m) <= 1e-6, sched
        assert rel_fro(to_np(out), to_np(out_m)) <= 1e-2, sched   # bf16 outputs: one rounding step apart
        assert torch.isfinite(out.float()).all()
