"""The block glue kernels (verace_rmsnorm, verace_add_rmsnorm) against an fp32 PyTorch
reference of torch.nn.RMSNorm (x * rsqrt(mean(x^2) + eps) * weight) and of the residual
steps around the mixers (verace_v1/modules/backbone.py; sssd_attention.py:177-182;
cham_memory.py:241).  fp32 to 1e-5; bf16 to 2 bf16 roundings (8e-3 relative to the row
scale); fp16 to 2e-3.
"""
import pytest
import torch

import verace_v1_b200 as V
from verace_v1_b200.kernels import apply_rmsnorm

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-5, torch.bfloat16: 1.6e-2, torch.float16: 2e-3}


def _ref_norm(x, w, eps):
    xf = x.float()
    r = xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)
    return r * w.float() if w is not None else r


def _norm(cols, dtype, eps=1e-6, affine=True, seed=0):
    m = torch.nn.RMSNorm(cols, eps=eps, elementwise_affine=affine).to("cuda", dtype)
    if affine:
        gen = torch.Generator().manual_seed(seed)
        with torch.no_grad():
            m.weight.copy_((1 + 0.5 * torch.randn(cols, generator=gen)).to(dtype))
    return m


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows,cols", [(1, 8), (37, 24), (1000, 128), (333, 1024), (70, 2048), (5, 1000)])
@pytest.mark.parametrize("affine", [True, False])
def test_rmsnorm_matches_reference(dtype, rows, cols, affine):
    gen = torch.Generator().manual_seed(rows + cols)
    x = (3 * torch.randn(rows, cols, generator=gen)).to("cuda", dtype)
    m = _norm(cols, dtype, affine=affine)
    y = V.rmsnorm(x, m)
    r = _ref_norm(x, m.weight if affine else None, 1e-6)
    assert y.dtype == dtype and y.shape == x.shape
    assert (y.float() - r).abs().max().item() <= TOL[dtype] * max(1.0, r.abs().max().item())
    # and against torch's own module
    assert (y.float() - m(x).float()).abs().max().item() <= TOL[dtype] * max(1.0, r.abs().max().item())


def test_rmsnorm_eps_default_is_the_dtype_epsilon():
    x = torch.full((4, 64), 0.01, device="cuda", dtype=torch.bfloat16)   # mean(x^2) ~ eps scale
    m = torch.nn.RMSNorm(64).to("cuda", torch.bfloat16)                 # eps=None
    y = V.rmsnorm(x, m)
    r = _ref_norm(x, m.weight, torch.finfo(torch.bfloat16).eps)
    assert (y.float() - r).abs().max().item() <= 1e-2 * r.abs().max().item()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("norm_y,norm_out", [(False, True), (True, True), (True, False), (False, False)])
@pytest.mark.parametrize("rows,cols", [(513, 1024), (64, 128), (9, 40)])
def test_add_rmsnorm_matches_reference(dtype, norm_y, norm_out, rows, cols):
    gen = torch.Generator().manual_seed(7 * rows + cols)
    h = torch.randn(rows, cols, generator=gen).to("cuda", dtype)
    y = (2 * torch.randn(rows, cols, generator=gen)).to("cuda", dtype)
    my = _norm(cols, dtype, eps=1e-5, seed=1) if norm_y else None
    mo = _norm(cols, dtype, eps=1e-6, seed=2) if norm_out else None
    h0 = h.clone()
    n = V.add_rmsnorm(h, y, y_norm=my, out_norm=mo)
    hr = h0.float() + (_ref_norm(y, my.weight, 1e-5) if norm_y else y.float())
    tol = TOL[dtype]
    assert (h.float() - hr).abs().max().item() <= tol * max(1.0, hr.abs().max().item())
    if norm_out:
        nr = _ref_norm(h, mo.weight, 1e-6)   # from the stored (rounded) h, as the kernel does
        assert n.dtype == dtype
        assert (n.float() - nr).abs().max().item() <= tol * max(1.0, nr.abs().max().item())
    else:
        assert n is None


def test_block_residual_chain_matches_unfused_glue():
    """Two layers of the block's residual steps through the fused glue against the same
    steps written with torch modules (fp32)."""
    gen = torch.Generator().manual_seed(11)
    dt, rows, cols = torch.float32, 256, 1024
    h = torch.randn(rows, cols, generator=gen).to("cuda", dt)
    pre = [_norm(cols, dt, seed=3 + i) for i in range(2)]
    mid = [_norm(cols, dt, seed=5 + i) for i in range(2)]
    out = [_norm(cols, dt, eps=None, seed=7 + i) for i in range(2)]
    mix = [torch.randn(cols, cols, generator=gen).to("cuda", dt) / 32 for _ in range(4)]
    ref = h.clone()
    for i in range(2):
        ref = ref + pre[i](ref) @ mix[2 * i]
        ref = ref + out[i](mid[i](ref) @ mix[2 * i + 1])
    n = V.rmsnorm(h, pre[0])
    for i in range(2):
        n = V.add_rmsnorm(h, n @ mix[2 * i], out_norm=mid[i])
        n = V.add_rmsnorm(h, n @ mix[2 * i + 1], y_norm=out[i], out_norm=pre[1] if i == 0 else None)
    assert (h - ref).abs().max().item() <= 1e-4 * ref.abs().max().item()


def test_unsupported_width_raises_and_module_path_falls_back():
    x = torch.randn(4, 12, device="cuda")
    m = torch.nn.RMSNorm(12).cuda()
    with pytest.raises(RuntimeError, match="cols 12 unsupported"):
        V.rmsnorm(x, m)
    assert torch.allclose(apply_rmsnorm(m, x), m(x))
