"""CPU checks of the C-ABI library: it loads, exports every symbol include/ssm_b200.h declares,
answers workspace queries and rejects bad arguments with the reference's error meaning.
None of these calls launches a kernel."""

import ctypes
import os
import re

import pytest

from conftest import ROOT
from mamba_ssm_benchmark_b200 import _native as nat

HEADER = os.path.join(ROOT, "include", "ssm_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"SSM_API\s+[\w\s\*]+?\b((?:ssm|selective)_\w+)\s*\(", text)))


def test_header_declares_every_binding():
    assert declared_symbols() == sorted(nat.EXPORTED)


def test_library_exports_every_declared_symbol():
    lib = nat.lib()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    assert lib.ssm_abi_version() == nat.ABI_VERSION


def test_library_is_not_a_cpu_fallback():
    """The .so carries sm_100a device code (an ELF cubin section) and links no torch."""
    blob = open(nat.LIB_PATH, "rb").read()
    assert b".nv_fatbin" in blob or b"__nv_relfatbin" in blob
    assert b"libtorch" not in blob


@pytest.mark.parametrize("B,L,D,N", [(1, 4096, 512, 16), (16, 512, 512, 16), (8, 8192, 5120, 16), (2, 37, 50, 8)])
def test_workspace_sizes(B, L, D, N):
    bwd = nat.bwd_workspace_bytes(B, L, D, N)
    ndt = -(-D // 32)
    assert bwd >= 4 * (B * ndt * L * 2 * N + B * D * N + B * D)
    fwd = nat.fwd_workspace_bytes(B, L, D, N)
    assert fwd >= 0


def test_bad_arguments_raise_value_error():
    with pytest.raises(ValueError, match="d_state"):
        nat.fwd_workspace_bytes(1, 16, 32, 12)
    with pytest.raises(ValueError, match="positive"):
        nat.bwd_workspace_bytes(1, 0, 32, 16)
    lib = nat.lib()
    v = nat.NULL_VIEW
    rc = lib.ssm_scan_fwd(1, 16, 32, 16, 7, v, v, None, v, v, None, v, None, v, v, None, None, None, 0, None)
    assert rc == nat.SSM_ERR_INVALID
    assert b"method" in lib.ssm_last_error_message()
    rc = lib.ssm_scan_fwd(1, 16, 32, 16, 0, v, v, None, v, v, None, v, None, v, v, None, None, None, 0, None)
    assert rc == nat.SSM_ERR_INVALID and b"u is required" in lib.ssm_last_error_message()


def test_mixed_dtypes_are_rejected_by_the_abi():
    lib = nat.lib()
    u = nat.SsmView(ctypes.c_void_p(256), nat.SSM_F32, 0, 16 * 32, 32)
    d = nat.SsmView(ctypes.c_void_p(256), nat.SSM_BF16, 0, 16 * 32, 32)
    rc = lib.ssm_scan_fwd(1, 16, 32, 16, 0, u, d, ctypes.c_void_p(256), u, u, None, nat.NULL_VIEW, None, u,
                          nat.NULL_VIEW, None, None, None, 0, None)
    assert rc == nat.SSM_ERR_DTYPE


def test_python_api_rejects_like_the_reference():
    import torch
    from mamba_ssm_benchmark_b200 import selective_scan, selective_scan_triton
    x = torch.zeros(1, 4, 8)
    A = -torch.ones(8, 16)
    Bm = torch.zeros(1, 4, 16)
    with pytest.raises(ValueError, match="discretization"):
        selective_scan_triton(x, x, A, Bm, Bm, method="rk4")
    with pytest.raises(ValueError, match="power of two"):
        selective_scan_triton(x, x, -torch.ones(8, 12), torch.zeros(1, 4, 12), torch.zeros(1, 4, 12))
    with pytest.raises(ValueError, match="unknown scan"):
        selective_scan(x, x, A, Bm, Bm, scan="fft")
    for name in ("chunked", "reference", "blelloch"):     # the reference's names: no CPU path here
        with pytest.raises(RuntimeError, match="CUDA"):
            selective_scan(x, x, A, Bm, Bm, scan=name)
    with pytest.raises(RuntimeError, match="CUDA"):
        selective_scan_triton(x, x, A, Bm, Bm)
    for shape in ((1, 0, 8), (0, 4, 8)):
        e = torch.zeros(*shape)
        with pytest.raises(ValueError, match="positive"):
            selective_scan_triton(e, e, A, torch.zeros(shape[0], shape[1], 16), torch.zeros(shape[0], shape[1], 16))
