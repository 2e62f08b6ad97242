"""pytest configuration: the ``gpu`` marker, the package loader and shared fixtures.

The product package lives in the directory ``verace-v1_b200/`` (not an importable
identifier), so it is registered here under the module name ``verace_v1_b200``.
"""
import importlib.util
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def _load_package():
    if "verace_v1_b200" in sys.modules:
        return sys.modules["verace_v1_b200"]
    pkg_dir = os.path.join(ROOT, "verace-v1_b200")
    spec = importlib.util.spec_from_file_location(
        "verace_v1_b200", os.path.join(pkg_dir, "__init__.py"),
        submodule_search_locations=[pkg_dir])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["verace_v1_b200"] = mod
    spec.loader.exec_module(mod)
    return mod


_load_package()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


GOLDEN = os.path.join(ROOT, "tests", "golden")


def load_golden(name):
    """Return {case: {key: array}} for tests/golden/<name>_golden.npz."""
    z = np.load(os.path.join(GOLDEN, f"{name}_golden.npz"))
    out = {}
    for key in z.files:
        case, rest = key.split("/", 1)
        d = out.setdefault(case, {"p": {}})
        if rest.startswith("p/"):
            d["p"][rest[2:]] = z[key]
        else:
            d[rest] = z[key]
    return out


def mcmoe_weights(g):
    """The fp32 weights of an M-CMoE golden case, re-created with the module's constructor
    under seed 0 (as tests/golden/make_golden.py built the reference's) and checked
    against the fingerprints the reference's weights left in the golden file."""
    import torch
    import verace_v1_b200 as V
    b, s, d, rank, C, K = (int(x) for x in g["dims"])
    torch.manual_seed(0)
    m = V.ManifoldContinuousMoE(hidden_dim=d, rank=rank, num_components=C, top_k_components=K)
    sd = {k: v.detach().numpy().astype(np.float32) for k, v in m.state_dict().items()}
    fps = {k[3:]: v for k, v in g.items() if k.startswith("fp/")}
    assert sorted(fps) == sorted(sd), "parameter names differ from the reference's"
    for k, v in sd.items():
        f = v.astype(np.float64).ravel()
        mine = np.concatenate([[f.sum(), (f * f).sum()], f[:16]])
        np.testing.assert_allclose(mine, fps[k], rtol=1e-6, atol=1e-6, err_msg=f"weights of {k} differ")
    return sd


def config1_case():
    """benchmark config 1 (one SSSD + CHAM layer, fp32, hidden 1024, 8 heads x 128, D = 1024,
    x = randn(2, 512, 1024) under seed 0, weights default-initialised under seed 0, SSSD
    first): (sssd module, cham module, x, golden dict) on the CPU.  The modules and x are
    re-created from the seeds, as tests/golden/make_golden.py built the reference's, and
    checked against the fingerprints the reference left in config1_golden.npz."""
    import torch
    import verace_v1_b200 as V
    z = np.load(os.path.join(GOLDEN, "config1_golden.npz"))
    g = {k: z[k] for k in z.files}
    torch.manual_seed(0)
    sssd = V.SSSDAttention(1024, 8, 128, 256)
    cham = V.ContinuousHolographicMemory(1024, 1024)
    torch.manual_seed(0)
    x = torch.randn(2, 512, 1024)

    def fp(t):
        f = t.detach().double().reshape(-1)
        return torch.cat([torch.stack([f.sum(), (f * f).sum()]), f[:16]]).numpy()

    np.testing.assert_allclose(fp(x), g["x/fp"], rtol=1e-9, atol=1e-9, err_msg="config-1 input differs")
    for prefix, m in (("sssd", sssd), ("cham", cham)):
        sd = m.state_dict()
        names = sorted(k[len(prefix) + 4:] for k in g if k.startswith(prefix + "/fp/"))
        assert names == sorted(sd), f"{prefix} parameter names differ from the reference's"
        for k, v in sd.items():
            np.testing.assert_allclose(fp(v), g[f"{prefix}/fp/{k}"], rtol=1e-9, atol=1e-9,
                                       err_msg=f"{prefix} weights of {k} differ")
    return sssd, cham, x, g


MODEL_OUT_OF_PATH = ("vision_encoder.", "energy_critic.")


def model_reinit(model, seed=0):
    """Deterministic re-initialisation of a VeraceV1Model's in-path parameters (the
    reference's or the drop-in's: same names), so that a reference model and the drop-in
    hold the same weights without storing them: parameters in sorted-name order from one
    generator; RMSNorm weights 1 + 0.1 N(0,1), the M-CMoE bases 0.02 N(0,1), the ACDE
    halting unit N(0, 0.2^2) with bias 3 (tokens halt at different layers), every other
    matrix N(0,1)/sqrt(fan_in)."""
    import torch
    g = torch.Generator().manual_seed(seed)
    params = dict(model.named_parameters())
    with torch.no_grad():
        for name in sorted(params):
            if name.startswith(MODEL_OUT_OF_PATH):
                continue
            p = params[name]
            if name.endswith("norm.weight"):
                p.copy_(1.0 + 0.1 * torch.randn(p.shape, generator=g))
            elif name.endswith(("u_basis", "v_basis")):
                p.copy_(0.02 * torch.randn(p.shape, generator=g))
            elif name == "acd_engine.w_halting.weight":
                p.copy_(0.2 * torch.randn(p.shape, generator=g))
            elif name == "acd_engine.w_halting.bias":
                p.fill_(3.0)
            else:
                p.copy_(torch.randn(p.shape, generator=g) / p.shape[-1] ** 0.5)


def model_fingerprints(model):
    """{name: [sum, sum of squares, first 16 values]} of the in-path parameters."""
    out = {}
    for k, v in model.state_dict().items():
        if k.startswith(MODEL_OUT_OF_PATH):
            continue
        f = v.detach().double().reshape(-1).cpu().numpy()
        out[k] = np.concatenate([[f.sum(), (f * f).sum()], f[:16]])
    return out
