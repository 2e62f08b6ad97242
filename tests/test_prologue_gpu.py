"""The fused projection epilogue (verace_mixer_prologue) against the reference's
elementwise code on the same projection outputs (sssd_attention.py:116-126,
cham_memory.py:129-153): per-head L2 normalisation, SiLU on CHAM's v, gates
0.1 sigmoid(.) * mask.  And the module-level project() (one concatenated GEMM + the
fused pass) against the reference formula with separate projections.
"""
import pytest
import torch
import torch.nn.functional as F

import verace_v1_b200 as V
from verace_v1_b200.kernels import concat_weights, mixer_prologue

pytestmark = pytest.mark.gpu


def _reference(y, h, d, g, silu_v, mask):
    n = y.shape[0]
    yf = y.float()
    hd = h * d
    q = F.normalize(yf[:, :hd].view(n, h, d), p=2, dim=-1).view(n, hd)
    k = F.normalize(yf[:, hd:2 * hd].view(n, h, d), p=2, dim=-1).view(n, hd)
    vv = yf[:, 2 * hd:3 * hd]
    if silu_v:
        vv = F.silu(vv)
    v = F.normalize(vv.view(n, h, d), p=2, dim=-1).view(n, hd)
    gate = 0.1 * torch.sigmoid(yf[:, 3 * hd:3 * hd + g])
    if mask is not None:
        gate = gate * mask.view(n, 1).float()
    return q, k, v, gate


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("h,d,g,silu_v", [(8, 128, 8, False), (1, 1024, 1, True), (3, 64, 3, False), (1, 160, 1, True),
                                          (16, 128, 16, False), (2, 1024, 2, True), (4, 512, 4, True)])
def test_prologue_matches_reference_elementwise(dtype, h, d, g, silu_v):
    """16-bit activations at 4133 rows with h d a multiple of 256 take the row-per-warp kernel
    (one segment of 12 rounds at h d = 1024, two at 2048; head vectors of half a round, two
    rounds or four rounds); the other cases the general split (as does a decode step's
    handful of rows, test_decode_gpu)."""
    n = 4133 if dtype != torch.float32 else 333   # 16-bit rows from 4096 take the row-per-warp kernel
    ld = 3 * h * d + g + ((-(3 * h * d + g)) % 8)
    gen = torch.Generator().manual_seed(900 + d)
    y = torch.randn(n, ld, generator=gen).to("cuda", dtype)
    mask = torch.rand(n, generator=gen) > 0.2
    q, k, v, gate = mixer_prologue(y, h, d, g, silu_v, mask.cuda())
    rq, rk, rv, rg = _reference(y, h, d, g, silu_v, mask.cuda())
    tol = 1e-6 if dtype == torch.float32 else 8e-3
    for a, r in ((q, rq), (k, rk), (v, rv)):
        assert a.dtype == dtype
        assert (a.float() - r).abs().max().item() <= tol
    assert gate.dtype == torch.float32
    assert (gate - rg).abs().max().item() <= 1e-6
    assert torch.all(gate[~mask.cuda()] == 0)


def test_zero_vector_normalises_to_zero_and_no_mask():
    y = torch.zeros(4, 8 * 128 * 3 + 8, device="cuda", dtype=torch.bfloat16)
    q, k, v, gate = mixer_prologue(y, 8, 128, 8, False, None)
    assert torch.all(q == 0) and torch.all(k == 0) and torch.all(v == 0)
    assert torch.allclose(gate, torch.full_like(gate, 0.05))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_module_project_matches_separate_projections(dtype):
    torch.manual_seed(0)
    s_mod = V.SSSDAttention(256, 4, 64).cuda().to(dtype)
    c_mod = V.ContinuousHolographicMemory(256, 128).cuda().to(dtype)
    x = torch.randn(2, 37, 256, device="cuda", dtype=dtype)
    mask = torch.rand(2, 37, device="cuda") > 0.1
    with torch.no_grad():
        q, k, v, dl = s_mod.project(x, mask)
        rq = F.normalize(s_mod.w_q(x).view(2, 37, 4, 64).float(), dim=-1)
        rd = 0.1 * torch.sigmoid(s_mod.w_delta(x).float()) * mask[..., None]
        cq, ck, cv, cg = c_mod.project(x, mask)
        rcv = F.normalize(F.silu(c_mod.w_v(x).float()), dim=-1)
        rcg = 0.1 * torch.sigmoid(c_mod.w_gamma(x).float()).view(2, 37) * mask
    tol = 2e-5 if dtype == torch.float32 else 2e-2
    assert (q.float() - rq).abs().max().item() <= tol
    assert (dl - rd).abs().max().item() <= (1e-6 if dtype == torch.float32 else 2e-3)
    assert (cv.float() - rcv).abs().max().item() <= tol
    assert (cg - rcg).abs().max().item() <= (1e-6 if dtype == torch.float32 else 2e-3)
    # the concatenated weight follows in-place weight updates
    with torch.no_grad():
        s_mod.w_q.weight.mul_(2.0)
    W = concat_weights(s_mod, [s_mod.w_q.weight, s_mod.w_k.weight, s_mod.w_v.weight, s_mod.w_delta.weight])
    assert torch.equal(W[:256], s_mod.w_q.weight)
