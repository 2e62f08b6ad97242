"""The fused single-token decode step (verace_decode_step) against the fp64 oracle.

One decode step of the reference is SSSDAttention / ContinuousHolographicMemory forward
with s = 1 and the previous state (verace_v1/serving/hyper_generate.py:58-77); the oracle
for it is the launcher-level scan over that one token from the given state, including
the CHAM readout's Newton-Schulz retraction.  Also: several steps in a row, incremental
decode against a full-sequence scan (the reference's
tests/test_incremental_generation.py:27-57 property), the first-order readout on a
hologram that is not unitary, the drift status, non-finite tokens, and shape limits.
And the deferred-update CHAM step (verace_decode_cham_lazy) against the eager unitary
step, across folds of the pending list.

Tolerances: relative Frobenius <= 1e-4 for fp32 outputs and for every fp32 state,
<= 2e-2 for bf16 outputs.
"""
import numpy as np
import pytest
import torch

import oracle
import verace_v1_b200 as V
from gpu_util import random_cham_inputs, random_sssd_inputs, rel_fro, to_np

pytestmark = pytest.mark.gpu

VERACE_ERR_STATE = 6


def _unitary(b, D, seed):
    """Random unitary matrices (QR of a complex Gaussian, phases fixed), complex128."""
    rng = np.random.default_rng(seed)
    Z = rng.standard_normal((b, D, D)) + 1j * rng.standard_normal((b, D, D))
    Q, R = np.linalg.qr(Z)
    ph = np.diagonal(R, axis1=-2, axis2=-1)
    return Q * (ph / np.abs(ph))[..., None, :]


def _holo(H):
    return (torch.from_numpy(H.real.astype(np.float32)).cuda().contiguous(),
            torch.from_numpy(H.imag.astype(np.float32)).cuda().contiguous())


def _psi0(b, h, d, seed):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(b, h, d, d, generator=g) / d ** 0.5).cuda().contiguous()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("b,h,d", [(3, 8, 128), (2, 3, 64), (1, 2, 12)])
def test_sssd_decode_matches_oracle(dtype, b, h, d):
    q, k, v, dl = random_sssd_inputs(b, 1, h, d, seed=700 + d, dtype=dtype)
    psi0 = _psi0(b, h, d, 701)
    psi = psi0.clone()
    out, none = V.launch_decode_step((q[:, 0], k[:, 0], v[:, 0], dl[:, 0], psi), None)
    assert none is None and out.dtype == dtype and tuple(out.shape) == (b, h, d)
    assert V.device_status() == 0
    o_ref, psi_ref = oracle.sssd_scan(to_np(q), to_np(k), to_np(v), to_np(dl), initial_state=to_np(psi0))
    assert rel_fro(to_np(out), o_ref[:, 0]) <= (1e-4 if dtype == torch.float32 else 2e-2)
    assert rel_fro(to_np(psi), psi_ref) <= 1e-5


@pytest.mark.parametrize("dtype,mode", [(torch.float32, "first_order"), (torch.float32, "unitary"),
                                        (torch.bfloat16, "unitary"), (torch.bfloat16, "first_order")])
@pytest.mark.parametrize("b,D", [(3, 128), (2, 160), (2, 256), (2, 1024)])
def test_cham_decode_matches_oracle(dtype, mode, b, D):
    q, k, v, g = random_cham_inputs(b, 1, D, seed=710 + D, dtype=dtype)
    H0 = _unitary(b, D, 711 + D)
    hr, hi = _holo(H0)
    h0r, h0i = hr.clone(), hi.clone()
    none, out = V.launch_decode_step(None, (q[:, 0], k[:, 0], v[:, 0], g[:, 0], hr, hi), mode=mode)
    assert none is None and out.dtype == dtype and tuple(out.shape) == (b, D)
    assert V.device_status() == 0
    r_ref, (Hr_ref, Hi_ref) = oracle.cham_scan(to_np(q), to_np(k), to_np(v), to_np(g),
                                               initial_hologram=(to_np(h0r), to_np(h0i)))
    assert rel_fro(to_np(out), r_ref[:, 0]) <= (1e-4 if dtype == torch.float32 else 2e-2)
    H_ref = Hr_ref + 1j * Hi_ref
    assert rel_fro(to_np(hr) + 1j * to_np(hi), H_ref) <= 1e-5


@pytest.mark.parametrize("mode", ["first_order", "unitary"])
def test_fused_layer_steps_match_oracle(mode):
    """SSSD and CHAM in the same launch, 6 tokens in a row (fp32)."""
    b, h, d, D, s = 3, 4, 128, 256, 6
    sq, sk, sv, dl = random_sssd_inputs(b, s, h, d, seed=720)
    cq, ck, cv, g = random_cham_inputs(b, s, D, seed=721)
    psi0 = _psi0(b, h, d, 722)
    H0 = _unitary(b, D, 723)
    psi = psi0.clone()
    hr, hi = _holo(H0)
    h0r, h0i = hr.clone(), hi.clone()
    so, co = [], []
    for t in range(s):
        o1, o2 = V.launch_decode_step((sq[:, t], sk[:, t], sv[:, t], dl[:, t], psi),
                                      (cq[:, t], ck[:, t], cv[:, t], g[:, t], hr, hi), mode=mode)
        so.append(o1)
        co.append(o2)
    assert V.device_status() == 0
    so = torch.stack(so, 1)
    co = torch.stack(co, 1)
    o_ref, psi_ref = oracle.sssd_scan(to_np(sq), to_np(sk), to_np(sv), to_np(dl), initial_state=to_np(psi0))
    r_ref, (Hr_ref, Hi_ref) = oracle.cham_scan(to_np(cq), to_np(ck), to_np(cv), to_np(g),
                                               initial_hologram=(to_np(h0r), to_np(h0i)))
    assert rel_fro(to_np(so), o_ref) <= 1e-4
    assert rel_fro(to_np(psi), psi_ref) <= 1e-5
    assert rel_fro(to_np(co), r_ref) <= 1e-4
    assert rel_fro(to_np(hr) + 1j * to_np(hi), Hr_ref + 1j * Hi_ref) <= 1e-5


def test_first_order_readout_on_a_non_unitary_hologram():
    """H0 = Q (I + eps S): the unitary readout is off by about |E q| / 2, the first-order
    readout by O(eps²); neither trips the drift status (|E q| < 1e-2 |q|)."""
    b, D, eps = 2, 256, 1.5e-3
    rng = np.random.default_rng(730)
    S = rng.standard_normal((b, D, D)) + 1j * rng.standard_normal((b, D, D))
    S = 0.5 * (S + np.conj(np.swapaxes(S, -1, -2)))
    S /= np.linalg.norm(S, ord=2, axis=(-2, -1))[:, None, None]
    H0 = _unitary(b, D, 731) @ (np.eye(D) + eps * S)
    q, k, v, g = random_cham_inputs(b, 1, D, seed=732)
    r_ref, _ = oracle.cham_scan(to_np(q), to_np(k), to_np(v), to_np(g),
                                initial_hologram=(H0.real, H0.imag))
    errs = {}
    for mode in ("unitary", "first_order"):
        hr, hi = _holo(H0)
        _, out = V.launch_decode_step(None, (q[:, 0], k[:, 0], v[:, 0], g[:, 0], hr, hi), mode=mode)
        assert V.device_status() == 0
        errs[mode] = rel_fro(to_np(out), r_ref[:, 0])
    assert errs["first_order"] <= 1e-4
    assert errs["unitary"] >= 5 * errs["first_order"]


def test_first_order_mode_flags_a_hologram_far_from_unitary():
    b, D = 2, 128
    q, k, v, g = random_cham_inputs(b, 1, D, seed=740)
    H0 = 1.2 * _unitary(b, D, 741)      # E = 0.44 I
    hr, hi = _holo(H0)
    V.launch_decode_step(None, (q[:, 0], k[:, 0], v[:, 0], g[:, 0], hr, hi), mode="first_order")
    assert V.device_status() == VERACE_ERR_STATE
    assert V.device_status() == 0      # reading clears it
    hr, hi = _holo(_unitary(b, D, 742))
    V.launch_decode_step(None, (q[:, 0], k[:, 0], v[:, 0], g[:, 0], hr, hi), mode="first_order")
    assert V.device_status() == 0


def test_nonfinite_tokens_take_the_identity_factor():
    b, h, d, D = 3, 2, 128, 128
    sq, sk, sv, dl = random_sssd_inputs(b, 1, h, d, seed=750)
    cq, ck, cv, g = random_cham_inputs(b, 1, D, seed=751)
    dl[2, 0, 0] = float("inf")
    sk[1, 0, 1, 5] = float("nan")
    ck[1, 0, 7] = float("nan")
    g[2, 0] = float("nan")
    psi0 = _psi0(b, h, d, 752)
    H0 = _unitary(b, D, 753)
    psi = psi0.clone()
    hr, hi = _holo(H0)
    h0r, h0i = hr.clone(), hi.clone()
    so, co = V.launch_decode_step((sq[:, 0], sk[:, 0], sv[:, 0], dl[:, 0], psi),
                                  (cq[:, 0], ck[:, 0], cv[:, 0], g[:, 0], hr, hi), mode="first_order")
    assert V.device_status() == 0
    # untouched states where the factor is the identity
    assert torch.equal(psi[2, 0], psi0[2, 0]) and torch.equal(psi[1, 1], psi0[1, 1])
    assert torch.equal(hr[1], h0r[1]) and torch.equal(hi[2], h0i[2])
    # the oracle sees the same tokens made identity by a zero gate instead
    dl_id, sk_id, ck_id, g_id = (to_np(x).copy() for x in (dl, sk, ck, g))
    dl_id[2, 0, 0] = 0.0
    dl_id[1, 0, 1] = 0.0
    sk_id[1, 0, 1, 5] = 0.0
    ck_id[1, 0, 7] = 0.0
    g_id[1, 0] = 0.0
    g_id[2, 0] = 0.0
    o_ref, psi_ref = oracle.sssd_scan(to_np(sq), sk_id, to_np(sv), dl_id, initial_state=to_np(psi0))
    r_ref, (Hr_ref, Hi_ref) = oracle.cham_scan(to_np(cq), ck_id, to_np(cv), g_id,
                                               initial_hologram=(to_np(h0r), to_np(h0i)))
    assert np.isfinite(to_np(so)).all() and np.isfinite(to_np(co)).all()
    assert rel_fro(to_np(so), o_ref[:, 0]) <= 1e-4
    assert rel_fro(to_np(psi), psi_ref) <= 1e-5
    assert rel_fro(to_np(co), r_ref[:, 0]) <= 1e-4
    assert rel_fro(to_np(hr) + 1j * to_np(hi), Hr_ref + 1j * Hi_ref) <= 1e-5


def test_either_half_alone_matches_the_fused_call():
    b, h, d, D = 2, 4, 128, 256
    sq, sk, sv, dl = random_sssd_inputs(b, 1, h, d, seed=760, dtype=torch.bfloat16)
    cq, ck, cv, g = random_cham_inputs(b, 1, D, seed=761, dtype=torch.bfloat16)
    psi0 = _psi0(b, h, d, 762)
    H0 = _holo(_unitary(b, D, 763))
    p1, p2 = psi0.clone(), psi0.clone()
    h1 = [x.clone() for x in H0]
    h2 = [x.clone() for x in H0]
    so1, co1 = V.launch_decode_step((sq[:, 0], sk[:, 0], sv[:, 0], dl[:, 0], p1),
                                    (cq[:, 0], ck[:, 0], cv[:, 0], g[:, 0], h1[0], h1[1]))
    so2, _ = V.launch_decode_step((sq[:, 0], sk[:, 0], sv[:, 0], dl[:, 0], p2), None)
    _, co2 = V.launch_decode_step(None, (cq[:, 0], ck[:, 0], cv[:, 0], g[:, 0], h2[0], h2[1]))
    assert torch.equal(so1, so2) and torch.equal(p1, p2)
    assert torch.equal(co1, co2) and torch.equal(h1[0], h2[0]) and torch.equal(h1[1], h2[1])


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_incremental_decode_matches_full_scan(dtype):
    """Prefill s0 tokens with the scans, decode n more with DecodeState: the decode
    outputs and final states equal one scan over all s0 + n tokens."""
    b, h, d, D, s0, n = 2, 8, 128, 1024, 70, 5
    sq, sk, sv, dl = random_sssd_inputs(b, s0 + n, h, d, seed=770, dtype=dtype)
    cq, ck, cv, g = random_cham_inputs(b, s0 + n, D, seed=771, dtype=dtype)
    so_full, psi_full = V.launch_sssd_scan(sq, sk, sv, dl)
    co_full, (hr_full, hi_full) = V.launch_cham_update(cq, ck, cv, g)
    _, psi_p = V.launch_sssd_scan(sq[:, :s0], sk[:, :s0], sv[:, :s0], dl[:, :s0])
    _, holo_p = V.launch_cham_update(cq[:, :s0], ck[:, :s0], cv[:, :s0], g[:, :s0])
    st = V.DecodeState(1, b, h, d, D)
    st.load_layer(0, psi_p, holo_p)
    so, co = [], []
    for t in range(s0, s0 + n):
        o1, o2 = st.step(0, (sq[:, t], sk[:, t], sv[:, t], dl[:, t]), (cq[:, t], ck[:, t], cv[:, t], g[:, t]))
        so.append(o1)
        co.append(o2)
    assert V.device_status() == 0
    st.flush()   # bf16 takes the unitary readout with deferred hologram updates
    tol = 1e-4 if dtype == torch.float32 else 2e-2
    assert rel_fro(to_np(torch.stack(so, 1)), to_np(so_full[:, s0:])) <= tol
    assert rel_fro(to_np(torch.stack(co, 1)), to_np(co_full[:, s0:])) <= tol
    assert rel_fro(to_np(st.psi[0]), to_np(psi_full)) <= 1e-4
    assert rel_fro(to_np(st.H_real[0]), to_np(hr_full)) <= 1e-4
    assert rel_fro(to_np(st.H_imag[0]), to_np(hi_full)) <= 1e-4


def test_decode_state_layer_states_round_trip():
    st = V.DecodeState(2, 3, 2, 64, 128)
    st.psi.copy_(torch.randn_like(st.psi))
    st.H_real.copy_(torch.randn_like(st.H_real))
    st.H_imag.copy_(torch.randn_like(st.H_imag))
    ls = st.layer_states()
    assert len(ls) == 2 and len(ls[0]) == 3
    psi, (hr, hi) = ls[1][2]
    assert tuple(psi.shape) == (1, 2, 64, 64) and tuple(hr.shape) == (1, 128, 128)
    st2 = V.DecodeState.from_layer_states(ls)
    assert torch.equal(st2.psi, st.psi) and torch.equal(st2.H_real, st.H_real)
    assert torch.equal(st2.H_imag, st.H_imag)


def test_unsupported_shapes_are_refused():
    q, k, v, g = random_cham_inputs(1, 1, 80, seed=780)
    hr, hi = _holo(_unitary(1, 80, 781))
    with pytest.raises(RuntimeError, match="unsupported"):
        V.launch_decode_step(None, (q[:, 0], k[:, 0], v[:, 0], g[:, 0], hr, hi))
    sq, sk, sv, dl = random_sssd_inputs(1, 1, 1, 130, seed=782)
    psi = _psi0(1, 1, 130, 783)
    with pytest.raises(RuntimeError, match="unsupported"):
        V.launch_decode_step((sq[:, 0], sk[:, 0], sv[:, 0], dl[:, 0], psi), None)
    with pytest.raises(ValueError):
        V.launch_decode_step((sq[:, 0], sk[:, 0], sv[:, 0], dl[:, 0], psi), None, mode="exact")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("b,D,P", [(3, 256, 4), (2, 1024, 8), (1, 128, 1), (1, 256, 16)])
def test_lazy_cham_decode_matches_eager_unitary_steps(dtype, b, D, P):
    """21 steps from a unitary hologram (folds every P steps; one non-finite token):
    the deferred-update step's outputs and, after a flush, its planes equal the eager
    unitary step's to fp32 rounding order.  P <= 8 folds with double-buffered factor
    rows, P = 16 with one buffer; bf16 with P <= 8 folds on the tensor cores."""
    n = 21
    q, k, v, g = random_cham_inputs(b, n, D, seed=790 + D + P, dtype=dtype)
    k[0, 5, 3] = float("nan")
    hr0, hi0 = _holo(_unitary(b, D, 791))
    er, ei = hr0.clone(), hi0.clone()
    lr, li = hr0.clone(), hi0.clone()
    pend = V.pending_storage(b, D, P)
    for t in range(n):
        _, ye = V.launch_decode_step(None, (q[:, t], k[:, t], v[:, t], g[:, t], er, ei), mode="unitary")
        yl = V.launch_decode_cham_lazy(q[:, t], k[:, t], v[:, t], g[:, t], lr, li, pend, P)
        assert yl.dtype == dtype and tuple(yl.shape) == (b, D)
        assert rel_fro(to_np(yl), to_np(ye)) <= (2e-6 if dtype == torch.float32 else 1e-2), t
    assert V.device_status() == 0
    V.flush_pending(lr, li, pend, P)
    assert rel_fro(to_np(lr) + 1j * to_np(li), to_np(er) + 1j * to_np(ei)) <= 2e-6
    V.flush_pending(lr, li, pend, P)   # an empty list: no change
    assert rel_fro(to_np(lr) + 1j * to_np(li), to_np(er) + 1j * to_np(ei)) <= 2e-6


def test_decode_state_defers_unitary_steps_and_flushes_for_layer_states():
    b, h, d, D, n = 2, 2, 64, 256, 11
    sq, sk, sv, dl = random_sssd_inputs(b, n, h, d, seed=795, dtype=torch.bfloat16)
    cq, ck, cv, g = random_cham_inputs(b, n, D, seed=796, dtype=torch.bfloat16)
    lazy = V.DecodeState(2, b, h, d, D, pending_depth=4)
    eager = V.DecodeState(2, b, h, d, D, pending_depth=0)
    for t in range(n):
        for l in range(2):
            a = lazy.step(l, (sq[:, t], sk[:, t], sv[:, t], dl[:, t]), (cq[:, t], ck[:, t], cv[:, t], g[:, t]))
            e = eager.step(l, (sq[:, t], sk[:, t], sv[:, t], dl[:, t]), (cq[:, t], ck[:, t], cv[:, t], g[:, t]))
            assert rel_fro(to_np(a[0]), to_np(e[0])) <= 1e-6 and rel_fro(to_np(a[1]), to_np(e[1])) <= 1e-2
    ls = lazy.layer_states()           # folds the pending factors in
    for l in range(2):
        H = to_np(lazy.H_real[l]) + 1j * to_np(lazy.H_imag[l])
        He = to_np(eager.H_real[l]) + 1j * to_np(eager.H_imag[l])
        assert rel_fro(H, He) <= 2e-6
    assert torch.equal(ls[1][0][1][0], lazy.H_real[1, 0:1])
    # an eager (first-order) step after deferred ones folds the list first
    o_l = lazy.step_cham(0, cq[:, 0].float(), ck[:, 0].float(), cv[:, 0].float(), g[:, 0], mode="first_order")
    o_e = eager.step_cham(0, cq[:, 0].float(), ck[:, 0].float(), cv[:, 0].float(), g[:, 0], mode="first_order")
    assert rel_fro(to_np(o_l), to_np(o_e)) <= 1e-5


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("b,D,P", [(3, 256, 4), (2, 1024, 8)])
def test_projected_lazy_step_matches_prologue_then_lazy_step(dtype, b, D, P):
    """verace_decode_cham_lazy_projected (the projection epilogue inside the step's first
    kernel) against the mixer prologue followed by verace_decode_cham_lazy, over 19 steps
    from a unitary hologram (folds included; one token's k non-finite): outputs, and the
    planes after a flush."""
    n = 19
    ld = 3 * D + 1 + 7                         # q | k | v | gate, padded to a multiple of 8
    g = torch.Generator().manual_seed(830 + D + P)
    ys = (torch.randn(n, b, ld, generator=g) * 0.3).to("cuda", dtype)
    ys[6, b - 1, D + 11] = float("nan")        # a k element of the last item at step 6
    hr0, hi0 = _holo(_unitary(b, D, 831))
    fr, fi = hr0.clone(), hi0.clone()
    rr, ri = hr0.clone(), hi0.clone()
    pf, pr = V.pending_storage(b, D, P), V.pending_storage(b, D, P)
    tol_y = 1e-5 if dtype == torch.float32 else 1e-2
    for t in range(n):
        yf = V.launch_decode_cham_lazy_projected(ys[t], fr, fi, pf, P)
        q, k, v, gm = V.kernels.mixer_prologue(ys[t], 1, D, 1, True)
        yr = V.launch_decode_cham_lazy(q, k, v, gm, rr, ri, pr, P)
        assert yf.dtype == dtype and tuple(yf.shape) == (b, D)
        assert rel_fro(to_np(yf), to_np(yr)) <= tol_y, t
    assert V.device_status() == 0
    V.flush_pending(fr, fi, pf, P)
    V.flush_pending(rr, ri, pr, P)
    tol_h = 1e-6 if dtype == torch.float32 else 1e-3
    assert rel_fro(to_np(fr) + 1j * to_np(fi), to_np(rr) + 1j * to_np(ri)) <= tol_h


@pytest.mark.parametrize("P", [3, 5])   # folds at steps P, 2P, ...: the odd ones are bf16 steps
def test_lazy_tensor_core_fold_of_fp32_factors(P):
    """Alternating fp32 and bf16 deferred steps on one pending list: the bf16 steps' kernel
    folds on the tensor cores factors whose k, v came from fp32 steps (not exact in bf16;
    they enter as hi + mid + lo pieces).  Outputs and, after a flush, the planes against
    eager unitary steps of the same dtypes."""
    b, D, n = 2, 256, 17
    q, k, v, g = random_cham_inputs(b, n, D, seed=840 + P)
    hr0, hi0 = _holo(_unitary(b, D, 841))
    er, ei = hr0.clone(), hi0.clone()
    lr, li = hr0.clone(), hi0.clone()
    pend = V.pending_storage(b, D, P)
    for t in range(n):
        dt = torch.float32 if t % 2 == 0 else torch.bfloat16
        args = (q[:, t].to(dt), k[:, t].to(dt), v[:, t].to(dt), g[:, t])
        _, ye = V.launch_decode_step(None, args + (er, ei), mode="unitary")
        yl = V.launch_decode_cham_lazy(*args, lr, li, pend, P)
        assert rel_fro(to_np(yl), to_np(ye)) <= (2e-6 if dt == torch.float32 else 1e-2), t
    assert V.device_status() == 0
    V.flush_pending(lr, li, pend, P)
    assert rel_fro(to_np(lr) + 1j * to_np(li), to_np(er) + 1j * to_np(ei)) <= 2e-6
