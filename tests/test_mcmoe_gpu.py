"""GPU parity of the M-CMoE kernels (routing, manifold projection, SiTU-GLU, module) against
the oracle (oracle/verace_oracle.py, pinned to the reference in test_oracle_golden.py)
and the reference's golden outputs.  Tolerances: fp32 1e-4 relative Frobenius (the
direct kernel), bf16 2e-2 (the tensor-core GEMMs: bf16 operands, fp32 accumulation).
"""
import numpy as np
import pytest
import torch

import oracle
import verace_v1_b200 as V
from conftest import load_golden, mcmoe_weights
from gpu_util import rel_fro, to_np

pytestmark = pytest.mark.gpu

MCMOE = load_golden("mcmoe")


def _module(g, dtype):
    b, s, d, rank, C, K = (int(x) for x in g["dims"])
    m = V.ManifoldContinuousMoE(hidden_dim=d, rank=rank, num_components=C, top_k_components=K)
    m.load_state_dict({k: torch.from_numpy(v) for k, v in mcmoe_weights(g).items()})
    return m.to("cuda", dtype).eval()


def _round(x, dtype):
    return torch.as_tensor(np.asarray(x, dtype=np.float32)).to(dtype).float().numpy().astype(np.float64)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("n,C,K", [(1000, 64, 8), (333, 8, 8), (257, 200, 16), (64, 16, 1)])
def test_route_matches_oracle(dtype, n, C, K):
    gen = torch.Generator().manual_seed(900 + C + K)
    logits = torch.randn(n, C, generator=gen).to(dtype)
    idx, w = V.launch_mcmoe_route(logits.cuda(), K)
    assert idx.dtype == torch.int64 and w.dtype == dtype and tuple(idx.shape) == (n, K)
    ref_i, ref_w = oracle.mcmoe_route(logits.float().numpy().astype(np.float64), K)
    assert np.array_equal(to_np(idx).astype(np.int64), ref_i)   # ties (bf16) go to the lower index on both
    tol = 1e-6 if dtype == torch.float32 else 8e-3
    np.testing.assert_allclose(to_np(w), ref_w, rtol=tol, atol=tol)


def test_route_matches_the_reference_golden():
    for case, g in MCMOE.items():
        K = int(g["dims"][5])
        idx, w = V.launch_mcmoe_route(torch.from_numpy(g["logits"]).cuda(), K)
        assert np.array_equal(to_np(idx).astype(np.int64), g["topk_idx"]), case
        np.testing.assert_allclose(to_np(w), g["topk_w"], rtol=1e-6, atol=1e-7)


def _projection_case(g, dtype):
    b, s, d, rank, C, K = (int(x) for x in g["dims"])
    p = mcmoe_weights(g)
    xf = g["x"].reshape(b * s, d)
    pre = xf.astype(np.float64) @ p["hyper_sigma.weight"].astype(np.float64).T
    sig = oracle.sigmoid(pre).reshape(b * s, C, rank)
    t = lambda a: torch.from_numpy(np.asarray(a, dtype=np.float32)).to(dtype).cuda()
    args = (t(xf), t(p["u_basis"]), t(p["v_basis"]), torch.from_numpy(g["topk_idx"]).cuda(), t(g["topk_w"]))
    return args, sig, pre, (b * s, d, C, rank, K)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("case", sorted(MCMOE))
def test_projection_matches_oracle(dtype, case):
    """launch_mcmoe_projection (the launcher contract of triton_kernels.py:688-723) with
    the reference's routing; the oracle sees the same dtype-rounded operands."""
    args, sig, pre, (n, d, C, r, K) = _projection_case(MCMOE[case], dtype)
    x, u, v, idx, w = args
    out = V.launch_mcmoe_projection(x, u, v, idx, w, torch.from_numpy(sig.astype(np.float32)).to(dtype).cuda())
    assert out.dtype == dtype and tuple(out.shape) == (n, d)
    rd = lambda a: _round(a, dtype)
    ref = oracle.mcmoe_projection(rd(to_np(x)), rd(to_np(u)), rd(to_np(v)), to_np(idx).astype(np.int64),
                                  rd(to_np(w)), rd(sig))
    assert rel_fro(to_np(out), ref) <= (1e-5 if dtype == torch.float32 else 2e-2)
    # the hyper-network's pre-activation, sigmoid applied inside (rounded to the dtype)
    out2 = V.launch_mcmoe_projection(x, u, v, idx, w, torch.from_numpy(pre.astype(np.float32)).to(dtype).cuda(),
                                     sigma_is_logits=True)
    assert rel_fro(to_np(out2), ref) <= (1e-5 if dtype == torch.float32 else 2e-2)
    assert V.device_status() == 0


@pytest.mark.parametrize("n,d,C,r,K", [(300, 256, 64, 32, 8), (129, 384, 16, 16, 4), (40, 96, 12, 8, 3)])
def test_projection_partial_tiles_and_shapes(n, d, C, r, K):
    """Row counts that leave a partial 128-row tile, other widths / ranks (tensor-core
    path when d % 128 == 0 and C*r % 128 == 0, else the direct kernel), bf16."""
    gen = torch.Generator().manual_seed(n + d)
    x = torch.randn(n, d, generator=gen)
    u = torch.randn(C, d, r, generator=gen) * 0.05
    v = torch.randn(C, r, d, generator=gen) * 0.05
    logits = torch.randn(n, C, generator=gen)
    idx = torch.topk(logits, K, dim=-1).indices
    w = torch.softmax(torch.gather(logits, -1, idx), -1)
    sig = torch.sigmoid(torch.randn(n, C, r, generator=gen))
    bf = lambda a: a.to(torch.bfloat16).cuda()
    out = V.launch_mcmoe_projection(bf(x), bf(u), bf(v), idx.cuda(), bf(w), bf(sig))
    rd = lambda a: a.to(torch.bfloat16).double().numpy()
    ref = oracle.mcmoe_projection(rd(x), rd(u), rd(v), idx.numpy(), rd(w), rd(sig))
    assert rel_fro(to_np(out), ref) <= 2e-2


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_situ_glu_matches_the_reference_formula(dtype):
    gen = torch.Generator().manual_seed(77)
    gu = (torch.randn(37, 2 * 160, generator=gen) * 6).to(dtype).cuda()
    g, u = gu[:, :160], gu[:, 160:]
    out = V.situ_glu(g, u, 4.0, 25.0)
    # SiTUGLU.forward's op sequence (activations.py), in the same dtype
    ref = (4.0 * torch.tanh(g / 4.0) * torch.sigmoid(g)) * (25.0 * torch.tanh(u / 25.0))
    tol = 1e-6 if dtype == torch.float32 else 1.6e-2
    torch.testing.assert_close(out.float(), ref.float(), rtol=tol, atol=tol)


@pytest.mark.parametrize("case", sorted(MCMOE))
def test_module_fp32_matches_reference_golden(case):
    g = MCMOE[case]
    b, s, d = (int(x) for x in g["dims"][:3])
    m = _module(g, torch.float32)
    with torch.no_grad():
        y = m(torch.from_numpy(g["x"]).cuda())
    assert tuple(y.shape) == (b, s, d)
    assert rel_fro(to_np(y), g["y"]) <= 1e-4
    assert V.device_status() == 0


@pytest.mark.parametrize("case", sorted(MCMOE))
def test_module_bf16_matches_oracle(case):
    """bf16 weights and activations (tensor-core projection where the shape allows); the
    oracle runs in fp64 on the same bf16 weights and input, with the routing the kernel
    chose from the bf16 router logits (a near-tie can flip between precisions)."""
    g = MCMOE[case]
    b, s, d, rank, C, K = (int(x) for x in g["dims"])
    m = _module(g, torch.bfloat16)
    x = torch.from_numpy(g["x"]).to(torch.bfloat16).cuda()
    with torch.no_grad():
        y = m(x)
        idx, w = V.launch_mcmoe_route(m.router(x.reshape(b * s, d)), K)
    p = {k: v.detach().double().cpu().numpy() for k, v in m.state_dict().items()}
    xf = to_np(x).astype(np.float64).reshape(b * s, d)
    base = oracle.situ_glu(p, xf) @ p["base_w_down.weight"].T
    sig = oracle.sigmoid(xf @ p["hyper_sigma.weight"].T).reshape(b * s, C, rank)
    man = oracle.mcmoe_projection(xf, p["u_basis"], p["v_basis"], to_np(idx).astype(np.int64),
                                  to_np(w).astype(np.float64), sig)
    # RMSNorm(eps=None) on bf16 activations uses bf16's machine epsilon, as torch does
    ref = base + oracle.rms_norm(man, p["norm.weight"], float(torch.finfo(torch.bfloat16).eps))
    assert rel_fro(to_np(y).reshape(b * s, d), ref) <= 2e-2
    assert V.device_status() == 0
