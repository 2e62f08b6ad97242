"""CPU checks of the C ABI: the library loads without a GPU, exports every function
include/verace_b200.h declares, sizes its workspaces, and rejects bad arguments with
a status code and message before touching the device."""
import ctypes

import pytest

from verace_v1_b200 import _lib


def test_library_loads_and_exports_every_header_symbol():
    L = _lib.lib()
    declared = _lib.header_symbols()
    assert len(declared) >= 8
    for name in declared:
        assert hasattr(L, name), f"{name} declared in include/verace_b200.h but not exported"
    assert set(declared) == set(_lib._SIGNATURES), "ctypes signatures out of sync with the header"
    assert L.verace_version() >= 10000


def test_workspace_queries_grow_with_problem_size():
    L = _lib.lib()
    a = L.verace_sssd_scan_workspace(2, 512, 8, 128)
    b = L.verace_sssd_scan_workspace(2, 1024, 8, 128)
    assert 0 < a < b
    for has_h0 in (0, 1):
        c0 = L.verace_cham_scan_workspace(2, 512, 1024, has_h0)
        c1 = L.verace_cham_scan_workspace(2, 1024, 1024, has_h0)
        assert 0 < c0 < c1
    assert L.verace_cham_retract_workspace(2, 1024) >= 4 * 2 * 1024 * 1024 * 4


def _err():
    return _lib.lib().verace_last_error().decode()


def _no_device():
    """The rejection tests below pass a placeholder pointer that no call may dereference;
    they run where no GPU is visible, so a regressed argument check can never reach one."""
    import torch
    return not torch.cuda.is_available()


host_only = pytest.mark.skipif(not _no_device(), reason="placeholder pointers: run without a GPU only")


@host_only
def test_sssd_rejects_bad_arguments_without_a_device():
    L = _lib.lib()
    fake = ctypes.c_void_p(256)
    rc = L.verace_sssd_scan(fake, fake, fake, fake, None, fake, fake, 1, 4, 2, 256, 0, fake, 1 << 20, None)
    assert rc == 2 and "head_dim" in _err()
    rc = L.verace_sssd_scan(fake, fake, fake, fake, None, fake, fake, 1, 4, 2, 64, 7, fake, 1 << 20, None)
    assert rc == 1 and "dtype" in _err()
    rc = L.verace_sssd_scan(fake, fake, fake, fake, None, fake, fake, 1, 4, 2, 64, 0, None, 0, None)
    assert rc == 4 and "workspace" in _err()
    rc = L.verace_sssd_scan(fake, fake, fake, fake, None, fake, fake, -1, 4, 2, 64, 0, fake, 1 << 20, None)
    assert rc == 1


@host_only
def test_cham_rejects_bad_arguments_without_a_device():
    L = _lib.lib()
    fake = ctypes.c_void_p(256)
    rc = L.verace_cham_scan(fake, fake, fake, fake, fake, None, fake, fake, fake, 1, 4, 16, 0, fake, 1 << 20, None)
    assert rc == 1 and "both" in _err()
    rc = L.verace_cham_scan(fake, fake, fake, fake, None, None, fake, fake, fake, 1, 4, 16, 0, None, 0, None)
    assert rc == 4
    rc = L.verace_cham_retract(fake, fake, fake, fake, 1, 16, -1, fake, 1 << 20, None)
    assert rc == 1


def test_status_error_raises_runtime_error():
    with pytest.raises(RuntimeError, match="status 2"):
        _lib.check(2, "probe")


@host_only
def test_decode_step_rejects_bad_arguments_without_a_device():
    L = _lib.lib()
    fake = ctypes.c_void_p(256)
    f = [fake] * 13
    ws = L.verace_decode_workspace(4, 1024)
    assert ws >= 4 * 32 * 1024 * 4 and L.verace_decode_workspace(4, 512) < ws
    rc = L.verace_decode_step(*f, 2, 8, 128, 1024, 0, 7, fake, ws, None)
    assert rc == 1 and "mode" in _err()
    rc = L.verace_decode_step(*f, 2, 8, 128, 1024, 5, 0, fake, ws, None)
    assert rc == 1 and "dtype" in _err()
    rc = L.verace_decode_step(*f, 2, 8, 128, 80, 0, 0, fake, ws, None)
    assert rc == 2 and "holographic" in _err()
    rc = L.verace_decode_step(*f, 2, 8, 130, 0, 0, 0, fake, ws, None)
    assert rc == 2 and "head_dim" in _err()
    rc = L.verace_decode_step(*f, 2, 8, 128, 1024, 0, 0, None, 0, None)
    assert rc == 4 and "workspace" in _err()
    rc = L.verace_decode_step(*([None] * 6), *f[:7], 2, 8, 128, 1024, 0, 0, fake, ws, None)
    assert rc == 1 and "SSSD" in _err()
    # nothing to do: returns before touching the device
    assert L.verace_decode_step(*f, 0, 8, 128, 1024, 0, 0, None, 0, None) == 0
    assert L.verace_decode_step(*f, 2, 0, 0, 0, 0, 0, None, 0, None) == 0


def test_decode_python_api_requires_cuda_tensors():
    import torch
    from verace_v1_b200 import decode
    x = torch.zeros(1, 2, 4)
    with pytest.raises(AssertionError, match="CUDA"):
        decode.launch_decode_step((x, x, x, torch.zeros(1, 2), torch.zeros(1, 2, 4, 4)), None)


@host_only
def test_norm_glue_rejects_bad_arguments_without_a_device():
    L = _lib.lib()
    fake = ctypes.c_void_p(256)
    assert L.verace_rmsnorm(fake, None, fake, 4, 12, 1e-6, 1, None) == 2 and "cols 12" in _err()
    assert L.verace_rmsnorm(fake, None, fake, 4, 64, 1e-6, 9, None) == 1 and "dtype" in _err()
    assert L.verace_rmsnorm(fake, None, fake, -1, 64, 1e-6, 1, None) == 1 and "rows" in _err()
    assert L.verace_rmsnorm(None, None, None, 0, 64, 1e-6, 1, None) == 0     # nothing to do
    assert L.verace_add_rmsnorm(fake, fake, 0, None, 0.0, None, 0.0, None, 4, 4096, 1, None) == 2
    assert L.verace_add_rmsnorm(None, fake, 0, None, 0.0, None, 0.0, None, 4, 64, 1, None) == 1
    assert "NULL" in _err()


@host_only
def test_lazy_decode_rejects_bad_arguments_without_a_device():
    L = _lib.lib()
    fake = ctypes.c_void_p(256)
    ws = L.verace_decode_lazy_workspace(4, 1024)
    assert ws > L.verace_decode_lazy_workspace(4, 512) > 0
    assert L.verace_decode_pending_bytes(4, 1024, 8) == 256 + 4 * 8 * 6 * 1024 * 4
    f = [fake] * 7
    assert L.verace_decode_cham_lazy(*f, 0, fake, 4, 1024, 1, fake, ws, None) == 1 and "pending depth" in _err()
    assert L.verace_decode_cham_lazy(*f, 17, fake, 4, 1024, 1, fake, ws, None) == 1
    assert L.verace_decode_cham_lazy(*f, 8, fake, 4, 80, 1, fake, ws, None) == 2 and "holographic" in _err()
    assert L.verace_decode_cham_lazy(*f, 8, fake, 4, 1024, 1, fake, 16, None) == 4 and "workspace" in _err()
    assert L.verace_decode_cham_lazy(*f, 8, fake, 4, 1024, 7, fake, ws, None) == 1 and "dtype" in _err()
    assert L.verace_decode_cham_lazy(*f, 8, fake, 0, 1024, 1, None, 0, None) == 0    # nothing to do
    assert L.verace_decode_cham_flush(fake, fake, fake, 0, 4, 1024, None) == 1
    assert L.verace_decode_cham_flush(fake, fake, fake, 8, 0, 1024, None) == 0


@host_only
def test_mcmoe_rejects_bad_arguments_without_a_device():
    L = _lib.lib()
    fake = ctypes.c_void_p(256)
    assert L.verace_mcmoe_route(fake, 4, 300, 8, fake, fake, 1, None) == 2 and "C=300" in _err()
    assert L.verace_mcmoe_route(fake, 4, 64, 17, fake, fake, 1, None) == 2
    assert L.verace_mcmoe_route(fake, 4, 64, 8, fake, fake, 7, None) == 1 and "dtype" in _err()
    assert L.verace_mcmoe_route(None, 0, 64, 8, None, None, 1, None) == 0   # nothing to do
    assert L.verace_mcmoe_projection(fake, fake, fake, fake, fake, None, 0, fake, 4, 256, 64, 32, 8, 1, None, 0,
                                     None) == 1 and "NULL" in _err()
    # bf16 tensor-core path without its workspace
    assert L.verace_mcmoe_projection(fake, fake, fake, fake, fake, fake, 0, fake, 4, 256, 64, 32, 8, 1, None, 0,
                                     None) == 4 and "workspace" in _err()
    assert L.verace_mcmoe_workspace(4, 256, 64, 32, 1) > L.verace_mcmoe_workspace(1, 256, 64, 32, 1)
    assert L.verace_mcmoe_workspace(4, 100, 64, 32, 1) == 256            # direct path: none
    assert L.verace_situ_glu(fake, fake, 4, fake, 2, 8, 4.0, 25.0, 1, None) == 1 and "ld" in _err()
    assert L.verace_situ_glu(fake, fake, 8, fake, 2, 8, 4.0, 25.0, 5, None) == 1 and "dtype" in _err()


@host_only
def test_projected_lazy_decode_rejects_bad_arguments_without_a_device():
    L = _lib.lib()
    fake = ctypes.c_void_p(256)
    ws = L.verace_decode_lazy_workspace(4, 1024)
    f = [fake, fake, fake]
    assert L.verace_decode_cham_lazy_projected(fake, 3080, *f, 0, fake, 4, 1024, 1, fake, ws, None) == 1
    assert "pending depth" in _err()
    assert L.verace_decode_cham_lazy_projected(fake, 3072, *f, 8, fake, 4, 1024, 1, fake, ws, None) == 1
    assert "row stride" in _err()
    assert L.verace_decode_cham_lazy_projected(None, 3080, *f, 8, fake, 4, 1024, 1, fake, ws, None) == 1
    assert L.verace_decode_cham_lazy_projected(fake, 3080, *f, 8, fake, 4, 1024, 7, fake, ws, None) == 1
    assert "dtype" in _err()
    assert L.verace_decode_cham_lazy_projected(fake, 3080, *f, 8, fake, 4, 80, 1, fake, ws, None) == 2
    assert "holographic" in _err()
    assert L.verace_decode_cham_lazy_projected(fake, 3080, *f, 8, fake, 4, 1024, 1, fake, 16, None) == 4
    assert "workspace" in _err()
    assert L.verace_decode_cham_lazy_projected(None, 0, None, None, None, 8, None, 0, 1024, 1, None, 0, None) == 0
