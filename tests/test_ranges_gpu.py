"""Sequence-parallel scans (ranges.py) for long sequences on few chains (benchmark
config 4's shape, shortened): the sequence is cut into ranges scanned side by side from
the identity, the range products are chained in fp32, and the ranges are scanned again
from the carried states.  Checked against the fp64 oracle and against the one-chain scan
(_ranges=False), including a length that needs padding and a non-unitary initial
hologram.  Tolerances: bf16 2e-2, fp32 1e-4 relative Frobenius error.
"""
import numpy as np
import pytest
import torch

import oracle
import verace_v1_b200 as V
from verace_v1_b200 import kernels as K
from verace_v1_b200.ranges import pick_ranges
from gpu_util import random_cham_inputs, random_sssd_inputs, rel_fro, to_np

pytestmark = pytest.mark.gpu
f64 = lambda t: t.double().cpu().numpy()


def test_config4_shape_picks_ranges_that_fill_the_gpu():
    dev = torch.device("cuda")
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    R_sssd = pick_ranges(16, 65536, dev, per_sm=1)
    R_cham = pick_ranges(32, 65536, dev, per_sm=2)
    assert 16 * R_sssd <= sms < 32 * R_sssd and 32 * R_cham <= 2 * sms < 64 * R_cham
    assert pick_ranges(8 * 32, 2048, dev, per_sm=2) == 1       # config 2 stays one pass
    assert pick_ranges(8 * 8, 2048, dev, per_sm=1) == 1


def test_cham_ranges_bf16_match_oracle_and_one_chain():
    b, s, D = 1, 8192, 1024
    q, k, v, g = random_cham_inputs(b, s, D, seed=51, dtype=torch.bfloat16)
    assert pick_ranges(b * D // 32, s, q.device, per_sm=2) > 1
    with torch.no_grad():
        out, H = V.launch_cham_update(q, k, v, g)
        out1, H1 = V.launch_cham_update(q, k, v, g, _ranges=False)
    rec, Hr = oracle.cham_scan_rank2_c(f64(q), f64(k), f64(v), f64(g))
    assert rel_fro(to_np(out), rec) <= 2e-2
    assert rel_fro(to_np(H[0]) + 1j * to_np(H[1]), Hr[0] + 1j * Hr[1]) <= 2e-2
    assert rel_fro(to_np(out), to_np(out1)) <= 2e-2
    Hc = to_np(H[0]).astype(np.float64) + 1j * to_np(H[1])
    assert np.abs(np.conj(np.swapaxes(Hc, -1, -2)) @ Hc - np.eye(D)).max() <= 1e-3


def test_sssd_ranges_bf16_with_padding_match_oracle():
    b, s, h, d = 1, 4196, 16, 128           # not a multiple of the range length: padded
    q, k, v, dl = random_sssd_inputs(b, s, h, d, seed=52, dtype=torch.bfloat16)
    assert pick_ranges(b * h, s, q.device, per_sm=1) == 2
    gen = torch.Generator().manual_seed(53)
    psi0 = torch.linalg.qr(torch.randn(b, h, d, d, generator=gen))[0].cuda()   # an orthogonal start
    with torch.no_grad():
        out, psi = V.launch_sssd_scan(q, k, v, dl, psi0)
    o_ref, psi_ref = oracle.sssd_scan(f64(q), f64(k), f64(v), f64(dl), f64(psi0))
    assert tuple(out.shape) == (b, s, h, d)
    assert rel_fro(to_np(out), o_ref) <= 2e-2
    assert rel_fro(to_np(psi), psi_ref) <= 2e-2


def test_cham_ranges_fp32_non_unitary_start_match_oracle():
    b, s, D = 1, 4196, 256
    q, k, v, g = random_cham_inputs(b, s, D, seed=54)
    gen = torch.Generator().manual_seed(55)
    H0r = torch.eye(D).expand(b, D, D) + 0.02 * torch.randn(b, D, D, generator=gen)
    H0i = 0.02 * torch.randn(b, D, D, generator=gen)
    assert pick_ranges(b * D // 32, s, q.device, per_sm=2) == 2
    with torch.no_grad():
        out, H = V.launch_cham_update(q, k, v, g, initial_hologram=(H0r.cuda(), H0i.cuda()))
    assert K.last_carried_path == "exact"      # the carried starts keep H0's drift
    rec, Hr = oracle.cham_scan_rank2_c(f64(q), f64(k), f64(v), f64(g), initial_hologram=(f64(H0r), f64(H0i)))
    assert rel_fro(to_np(out), rec) <= 1e-4
    assert rel_fro(to_np(H[0]) + 1j * to_np(H[1]), Hr[0] + 1j * Hr[1]) <= 1e-4
