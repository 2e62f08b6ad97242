"""CHAM continuing from a carried hologram (initial_hologram, cham_memory.py:117-122 and
:229-239): the launcher probes the hologram's unitarity and continues a unitary one on
the tensor-core scan (one token: the decode kernel's first-order readout), any other on
the exact readout polynomial.  Each case is checked against the fp64 oracle and against
the path it must take.  Tolerances: fp32 1e-4, bf16 2e-2 relative Frobenius error.
"""
import numpy as np
import pytest
import torch

import oracle
import verace_v1_b200 as V
from verace_v1_b200 import kernels as K
from gpu_util import random_cham_inputs, rel_fro, to_np

pytestmark = pytest.mark.gpu


def _probe_signs(D, probes=4):
    c = np.arange(D, dtype=np.uint64)
    out = []
    for j in range(probes):
        h = ((c * np.uint64(2654435761)) & np.uint64(0xFFFFFFFF)) ^ np.uint64(((j + 1) * 0x9E3779B9) & 0xFFFFFFFF)
        out.append(np.where((h >> np.uint64(15)) & np.uint64(1), 1.0, -1.0))
    return np.stack(out)


def test_unitarity_probe_matches_its_definition():
    g = torch.Generator().manual_seed(4)
    b, D = 3, 256
    Hr = torch.eye(D).expand(b, D, D).clone()
    Hi = torch.zeros(b, D, D)
    Hr[1] += 1e-3 * torch.randn(D, D, generator=g)
    Hi[2] += 0.05 * torch.randn(D, D, generator=g)
    eps = to_np(K.hologram_unitarity(Hr.cuda(), Hi.cuda()))
    H = Hr.double().numpy() + 1j * Hi.double().numpy()
    E = np.conj(np.swapaxes(H, -1, -2)) @ H - np.eye(D)
    R = _probe_signs(D)
    want = np.sqrt(np.max(np.sum(np.abs(E @ R.T) ** 2, axis=1), axis=-1) / D)
    assert eps[0] == 0.0
    np.testing.assert_allclose(eps, want, rtol=1e-5, atol=1e-12)


@pytest.mark.parametrize("dtype,D,tol", [(torch.bfloat16, 1024, 2e-2), (torch.bfloat16, 256, 2e-2),
                                         (torch.float32, 256, 1e-4)])
def test_continuation_from_grown_hologram_takes_tensor_cores(dtype, D, tol):
    b, s1, s2 = 2, 130, 200
    q, k, v, g = random_cham_inputs(b, s1 + s2, D, seed=41, dtype=dtype)
    with torch.no_grad():
        out1, H1 = V.launch_cham_update(q[:, :s1], k[:, :s1], v[:, :s1], g[:, :s1])
        out2, H2 = V.launch_cham_update(q[:, s1:], k[:, s1:], v[:, s1:], g[:, s1:], initial_hologram=H1)
    eps = float(K.hologram_unitarity(*H1).max())
    print(f"{dtype} D={D}: unitarity probe of the grown hologram {eps:.2e}")
    f64 = lambda t: t.double().cpu().numpy()
    rec, Hr = oracle.cham_scan_rank2_c(f64(q), f64(k), f64(v), f64(g))
    if dtype == torch.float32 and eps > K.UNITARY_TOL[dtype]:
        assert K.last_carried_path == "exact"
    else:
        assert K.last_carried_path == "unitary"
    assert rel_fro(to_np(out2), rec[:, s1:]) <= tol
    assert rel_fro(to_np(H2[0]) + 1j * to_np(H2[1]), Hr[0] + 1j * Hr[1]) <= tol


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-4), (torch.bfloat16, 2e-2)])
def test_non_unitary_hologram_takes_the_exact_readout(dtype, tol):
    b, s, D = 2, 70, 256
    q, k, v, g = random_cham_inputs(b, s, D, seed=43, dtype=dtype)
    gen = torch.Generator().manual_seed(44)
    H0r = torch.eye(D).expand(b, D, D) + 0.02 * torch.randn(b, D, D, generator=gen)
    H0i = 0.02 * torch.randn(b, D, D, generator=gen)
    with torch.no_grad():
        out, H = V.launch_cham_update(q, k, v, g, initial_hologram=(H0r.cuda(), H0i.cuda()))
    assert K.last_carried_path == "exact"
    f64 = lambda t: t.double().cpu().numpy()
    rec, Hr = oracle.cham_scan_rank2_c(f64(q), f64(k), f64(v), f64(g), initial_hologram=(f64(H0r), f64(H0i)))
    assert rel_fro(to_np(out), rec) <= tol
    assert rel_fro(to_np(H[0]) + 1j * to_np(H[1]), Hr[0] + 1j * Hr[1]) <= tol


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-4), (torch.bfloat16, 2e-2)])
def test_one_token_continuation_takes_the_decode_kernel(dtype, tol):
    b, s1, D = 3, 96, 1024
    q, k, v, g = random_cham_inputs(b, s1 + 1, D, seed=45, dtype=dtype)
    with torch.no_grad():
        _, H1 = V.launch_cham_update(q[:, :s1], k[:, :s1], v[:, :s1], g[:, :s1])
        out, H2 = V.launch_cham_update(q[:, s1:], k[:, s1:], v[:, s1:], g[:, s1:], initial_hologram=H1)
    assert K.last_carried_path == "first_order"
    f64 = lambda t: t.double().cpu().numpy()
    # the reference's formula at the last token: the dense Newton-Schulz retraction of H_t
    rec, Hr = oracle.cham_scan_rank2_c(f64(q), f64(k), f64(v), f64(g))
    Qr, _ = oracle.newton_schulz_unitary_retraction(Hr[0], Hr[1], 3)
    dense = (Qr @ f64(q)[:, -1, :, None])[..., 0]
    assert rel_fro(to_np(out)[:, 0], dense) <= tol
    assert rel_fro(to_np(H2[0]) + 1j * to_np(H2[1]), Hr[0] + 1j * Hr[1]) <= tol


def test_capture_takes_the_exact_path_without_a_host_read():
    b, s, D = 1, 5, 128
    q, k, v, g = random_cham_inputs(b, s, D, seed=46)
    eye = (torch.eye(D, device="cuda").expand(b, D, D).contiguous(), torch.zeros(b, D, D, device="cuda"))
    with torch.no_grad():
        V.launch_cham_update(q, k, v, g, initial_hologram=eye)    # warm-up (workspaces, module load)
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            with torch.cuda.graph(graph, stream=side):
                out, _ = V.launch_cham_update(q, k, v, g, initial_hologram=eye)
        assert K.last_carried_path == "exact"
        graph.replay()
        torch.cuda.synchronize()
    f64 = lambda t: t.double().cpu().numpy()
    rec, _ = oracle.cham_scan_rank2_c(f64(q), f64(k), f64(v), f64(g))
    assert rel_fro(to_np(out), rec) <= 1e-4
    del graph
