"""Helpers shared by the GPU parity tests (imported only by tests)."""
import numpy as np
import torch

import verace_v1_b200 as V


def rel_fro(a, b):
    """Relative Frobenius error; complex inputs are compared as complex."""
    cplx = np.iscomplexobj(a) or np.iscomplexobj(b)
    a = np.asarray(a, dtype=np.complex128 if cplx else np.float64)
    b = np.asarray(b, dtype=np.complex128 if cplx else np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def to_np(t):
    return t.detach().float().cpu().numpy()


def sssd_module(g, device="cuda"):
    b, s, d, h, hid = (int(x) for x in g["dims"])
    m = V.SSSDAttention(hidden_dim=hid, num_heads=h, head_dim=d)
    m.load_state_dict({k: torch.from_numpy(v) for k, v in g["p"].items()})
    return m.to(device).eval()


def cham_module(g, device="cuda"):
    b, s, D, hid = (int(x) for x in g["dims"])
    m = V.ContinuousHolographicMemory(hidden_dim=hid, holographic_dim=D)
    m.load_state_dict({k: torch.from_numpy(v) for k, v in g["p"].items()})
    return m.to(device).eval()


def random_sssd_inputs(b, s, h, d, seed, dtype=torch.float32, device="cuda"):
    gen = torch.Generator().manual_seed(seed)
    q = torch.nn.functional.normalize(torch.randn(b, s, h, d, generator=gen), dim=-1)
    k = torch.nn.functional.normalize(torch.randn(b, s, h, d, generator=gen), dim=-1)
    v = torch.nn.functional.normalize(torch.randn(b, s, h, d, generator=gen), dim=-1)
    delta = 0.1 * torch.sigmoid(torch.randn(b, s, h, generator=gen))
    q, k, v = (x.to(dtype) for x in (q, k, v))
    return q.to(device), k.to(device), v.to(device), delta.to(device)


def random_cham_inputs(b, s, D, seed, dtype=torch.float32, device="cuda"):
    gen = torch.Generator().manual_seed(seed)
    q = torch.nn.functional.normalize(torch.randn(b, s, D, generator=gen), dim=-1)
    k = torch.nn.functional.normalize(torch.randn(b, s, D, generator=gen), dim=-1)
    v = torch.nn.functional.normalize(torch.nn.functional.silu(torch.randn(b, s, D, generator=gen)), dim=-1)
    gamma = 0.1 * torch.sigmoid(torch.randn(b, s, generator=gen))
    q, k, v = (x.to(dtype) for x in (q, k, v))
    return q.to(device), k.to(device), v.to(device), gamma.to(device)
