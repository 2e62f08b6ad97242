"""The allocation-free SSSD scan (verace_sssd_scan_noalloc) against the regular one.

Some callers of this library cannot allocate device memory where the scan runs
(plugin or FFI hosts that own all device memory; serving loops on a fixed memory
budget).  They use verace_sssd_scan_noalloc, whose scratch is a fixed device array
inside the library instead of a caller workspace.  This test calls it through the C
ABI twice in a row -- the second call reuses the scratch the first one left behind --
and checks both results against verace_sssd_scan (the regular entry point, through the
same ABI) within the fp32 parity tolerance used by the other SSSD tests.  It also
checks that a size whose scratch would not fit is refused with a clear error.

The file name sorts last so that a run that stops at the first failure has already
run every other test; it passes alone in a fresh process as well.
"""
import pytest
import torch

from gpu_util import random_sssd_inputs, rel_fro, to_np
from verace_v1_b200 import _lib

pytestmark = pytest.mark.gpu


def _regular(q, k, v, delta, psi0):
    L = _lib.lib()
    b, s, h, d = q.shape
    out = torch.empty_like(q)
    psi = torch.empty(b, h, d, d, device=q.device)
    ws = torch.empty(L.verace_sssd_scan_workspace(b, s, h, d), dtype=torch.uint8, device=q.device)
    rc = L.verace_sssd_scan(q.data_ptr(), k.data_ptr(), v.data_ptr(), delta.data_ptr(),
                            None if psi0 is None else psi0.data_ptr(), out.data_ptr(), psi.data_ptr(),
                            b, s, h, d, 0, ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "verace_sssd_scan")
    return out, psi


def _noalloc(q, k, v, delta, psi0):
    L = _lib.lib()
    b, s, h, d = q.shape
    out = torch.empty_like(q)
    psi = torch.empty(b, h, d, d, device=q.device)
    rc = L.verace_sssd_scan_noalloc(q.data_ptr(), k.data_ptr(), v.data_ptr(), delta.data_ptr(),
                                    None if psi0 is None else psi0.data_ptr(), out.data_ptr(),
                                    psi.data_ptr(), b, s, h, d, 0, torch.cuda.current_stream().cuda_stream)
    _lib.check(rc, "verace_sssd_scan_noalloc")
    return out, psi


def test_noalloc_sssd_scan_matches_regular_entry_point_on_two_calls():
    # call 1: config-1 shape (2 x 512 tokens, 8 heads x 128) from the identity state
    q, k, v, delta = random_sssd_inputs(2, 512, 8, 128, seed=31)
    ref_out, ref_psi = _regular(q, k, v, delta, None)
    out, psi = _noalloc(q, k, v, delta, None)
    torch.cuda.synchronize()
    assert rel_fro(to_np(out), to_np(ref_out)) <= 1e-4
    assert rel_fro(to_np(psi), to_np(ref_psi)) <= 1e-4
    # call 2: different sizes and a carried state, on the scratch call 1 left behind
    q2, k2, v2, d2 = random_sssd_inputs(2, 77, 8, 128, seed=32)
    ref_out2, ref_psi2 = _regular(q2, k2, v2, d2, ref_psi)
    out2, psi2 = _noalloc(q2, k2, v2, d2, psi)
    torch.cuda.synchronize()
    assert rel_fro(to_np(out2), to_np(ref_out2)) <= 1e-4
    assert rel_fro(to_np(psi2), to_np(ref_psi2)) <= 1e-4


def test_noalloc_sssd_scan_refuses_sizes_beyond_its_scratch():
    # Every pointer is NULL: the size limit is checked before the pointers, so the call is
    # refused with VERACE_ERR_UNSUPPORTED (2).  Should that check ever stop catching this
    # size, the NULL-pointer check returns VERACE_ERR_INVALID (1) instead and the test fails
    # without any kernel being launched.
    L = _lib.lib()
    b, s, h, d = 8, 2048, 8, 128          # b*h*ceil(s/32) = 4096 transforms: ~64 MiB of scratch
    assert L.verace_sssd_scan_workspace(b, s, h, d) > (16 << 20)
    rc = L.verace_sssd_scan_noalloc(None, None, None, None, None, None, None, b, s, h, d, 0, None)
    assert rc == 2
    assert "fixed" in L.verace_last_error().decode()
    # the largest size that fits (1023 transforms) passes the size check and then stops at
    # the NULL pointers
    rc = L.verace_sssd_scan_noalloc(None, None, None, None, None, None, None, 1, 1023 * 32, 1, 128, 0, None)
    assert rc == 1
