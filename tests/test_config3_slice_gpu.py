"""A slice of benchmark config 3 on the GPU against the fp64 oracle: one layer's SSSD
(8 heads x 128) and CHAM (D = 1024) states for 2 items, a 1024-token prompt prefilled by
the scans, then 256 single-token decode steps through DecodeState with the bench's
settings (bf16 inputs, the "unitary" CHAM readout Re(H q), hologram updates deferred and
folded every P = 8 steps).

The oracle runs the reference's algorithm over all 1280 tokens in fp64: the eager SSSD
and the CHAM scan in O(D^2) per token (``cham_scan_rank2_c``), whose readout is
Re(NS3(H_t) q_t) through the Newton-Schulz identity; at four of the decode steps the
readout is also formed by the dense per-position retraction of H_t
(``newton_schulz_unitary_retraction``), the reference's own formula, and the GPU's
readout is compared with that too.  Bar: north_star's bf16 tolerance, relative Frobenius
error <= 2e-2, on every step's outputs and on the flushed states after the last step;
the final hologram's drift from unitarity max|HᴴH - I| is reported and bounded by 1e-3.
"""
import numpy as np
import pytest
import torch

import oracle
import verace_v1_b200 as V
from gpu_util import rel_fro, to_np

pytestmark = pytest.mark.gpu

B, H, HD, D, PROMPT, STEPS = 2, 8, 128, 1024, 1024, 256
CHECK = (0, 85, 170, 255)


def _inputs():
    g = torch.Generator().manual_seed(3)
    nrm = torch.nn.functional.normalize
    n = PROMPT + STEPS
    sq, sk, sv = (nrm(torch.randn(B, n, H, HD, generator=g), dim=-1) for _ in range(3))
    dl = 0.1 * torch.sigmoid(torch.randn(B, n, H, generator=g))
    cq, ck = (nrm(torch.randn(B, n, D, generator=g), dim=-1) for _ in range(2))
    cv = nrm(torch.nn.functional.silu(torch.randn(B, n, D, generator=g)), dim=-1)
    gm = 0.1 * torch.sigmoid(torch.randn(B, n, generator=g))
    bf = lambda t: t.to(torch.bfloat16)
    return bf(sq), bf(sk), bf(sv), dl, bf(cq), bf(ck), bf(cv), gm


def test_config3_slice_decode_matches_fp64_oracle():
    sq, sk, sv, dl, cq, ck, cv, gm = _inputs()
    dev = torch.device("cuda")
    P = PROMPT
    with torch.no_grad():
        _, psi = V.launch_sssd_scan(sq[:, :P].to(dev), sk[:, :P].to(dev), sv[:, :P].to(dev), dl[:, :P].to(dev))
        _, holo = V.launch_cham_update(cq[:, :P].to(dev), ck[:, :P].to(dev), cv[:, :P].to(dev), gm[:, :P].to(dev))
        st = V.DecodeState(1, B, H, HD, D, device=dev, pending_depth=8)
        st.load_layer(0, psi, holo)
        s_out, c_out = [], []
        for t in range(P, P + STEPS):
            s_out.append(to_np(st.step_sssd(0, sq[:, t].to(dev), sk[:, t].to(dev), sv[:, t].to(dev), dl[:, t].to(dev))))
            c_out.append(to_np(st.step_cham(0, cq[:, t].to(dev), ck[:, t].to(dev), cv[:, t].to(dev), gm[:, t].to(dev))))
        st.flush()
        assert V.device_status(dev) == 0
        psi_g, hr_g, hi_g = to_np(st.psi[0]), to_np(st.H_real[0]), to_np(st.H_imag[0])
    s_out = np.stack(s_out, 1)           # [B, STEPS, H, HD]
    c_out = np.stack(c_out, 1)           # [B, STEPS, D]

    f64 = lambda t: t.double().numpy()
    o_ref, psi_ref = oracle.sssd_scan(f64(sq), f64(sk), f64(sv), f64(dl))
    assert rel_fro(s_out, o_ref[:, P:]) <= 2e-2
    assert rel_fro(psi_g, psi_ref) <= 2e-2

    q, k, v, g = f64(cq), f64(ck), f64(cv), f64(gm)
    _, Hc = oracle.cham_scan_rank2_c(q[:, :P], k[:, :P], v[:, :P], g[:, :P])
    rec = np.zeros((B, STEPS, D))
    t0 = 0
    for tc in CHECK:     # decode tokens [t0, tc] from the state after token P + t0 - 1
        a, b = P + t0, P + tc + 1
        r, Hc = oracle.cham_scan_rank2_c(q[:, a:b], k[:, a:b], v[:, a:b], g[:, a:b], initial_hologram=Hc)
        rec[:, t0:tc + 1] = r
        Qr, _ = oracle.newton_schulz_unitary_retraction(Hc[0], Hc[1], 3)
        dense = (Qr @ q[:, b - 1, :, None])[..., 0]       # the reference's per-position readout
        assert rel_fro(c_out[:, tc], dense) <= 2e-2, f"decode step {tc} vs dense NS3 readout"
        t0 = tc + 1
    assert rel_fro(c_out, rec) <= 2e-2
    Hg = hr_g.astype(np.float64) + 1j * hi_g
    assert rel_fro(Hg, Hc[0] + 1j * Hc[1]) <= 2e-2
    drift = np.abs(np.conj(np.swapaxes(Hg, -1, -2)) @ Hg - np.eye(D)).max()
    print(f"config-3 slice: SSSD out {rel_fro(s_out, o_ref[:, P:]):.2e}, CHAM out {rel_fro(c_out, rec):.2e}, "
          f"max|H^H H - I| after {PROMPT}+{STEPS} tokens {drift:.2e}")
    assert drift <= 1e-3
