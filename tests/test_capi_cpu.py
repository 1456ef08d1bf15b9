"""The C-ABI library without a GPU: it loads, exports every entry point that
include/mhc_b200.h declares, and rejects bad arguments before touching the
device."""
import ctypes
import os
import re

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "mhc_b200.h")


def _declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(mhc_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    from FlagOS_mhc import _C
    lib = ctypes.CDLL(_C.lib_path())
    names = _declared_functions()
    assert "mhc_post_fwd" in names and "mhc_pre_bwd" in names
    for n in names:
        assert hasattr(lib, n), n
    # the Python binding declares a signature for each of them
    for n in names:
        assert n in _C._SIGS, n


def test_status_strings_and_version():
    from FlagOS_mhc import _C
    L = _C.lib()
    assert L.mhc_version() >= 100
    for code in range(9):
        assert len(L.mhc_status_string(code)) > 0


def test_argument_checks_precede_device_use():
    from FlagOS_mhc import _C
    L = _C.lib()
    nul = None
    # N out of range
    assert L.mhc_post_fwd(nul, nul, nul, nul, nul, 4, 9, 64, 2, nul) == _C.MHC_ERR_UNSUPPORTED_N
    assert L.mhc_post_fwd(nul, nul, nul, nul, nul, 4, 0, 64, 2, nul) == _C.MHC_ERR_UNSUPPORTED_N
    # dtype out of range
    assert L.mhc_post_bwd(nul, nul, nul, nul, nul, nul, nul, nul, nul, 4, 4, 64, 7, nul) == \
        _C.MHC_ERR_UNSUPPORTED_DTYPE
    # bad sizes
    assert L.mhc_post_fwd(nul, nul, nul, nul, nul, -1, 4, 64, 2, nul) == \
        _C.MHC_ERR_INVALID_ARGUMENT
    assert L.mhc_post_fwd(nul, nul, nul, nul, nul, 4, 4, 0, 2, nul) == \
        _C.MHC_ERR_INVALID_ARGUMENT
    # empty token range is a no-op
    assert L.mhc_post_fwd(nul, nul, nul, nul, nul, 0, 4, 64, 2, nul) == _C.MHC_OK
    # null tensors
    assert L.mhc_post_fwd(nul, nul, nul, nul, nul, 4, 4, 64, 2, nul) == \
        _C.MHC_ERR_INVALID_ARGUMENT
    # pre forward: missing workspace
    args = [ctypes.c_void_p(16)] * 4 + [8, 4, 64, 2, 1e-6, 1e-6, 0.0, 0.0, 20] + \
        [ctypes.c_void_p(16)] * 3 + [ctypes.c_void_p(16), None, ctypes.c_void_p(16), None,
                                     ctypes.c_void_p(16), None, 0, None]
    assert L.mhc_pre_fwd(*args) == _C.MHC_ERR_WORKSPACE
    # negative iteration count
    args[12] = -1
    assert L.mhc_pre_fwd(*args) == _C.MHC_ERR_INVALID_ARGUMENT


def test_workspace_sizes():
    from FlagOS_mhc import _C
    L = _C.lib()
    a = L.mhc_pre_fwd_workspace_bytes(32768, 4, 7168, 2)
    b = L.mhc_pre_bwd_workspace_bytes(32768, 4, 7168, 2, 20)
    assert a > 0 and b > 0
    assert L.mhc_pre_bwd_workspace_bytes(32768, 4, 7168, 2, 40) > b   # Sinkhorn history grows
    assert L.mhc_pre_fwd_workspace_bytes(32768, 11, 7168, 2) == 0      # unsupported N
    # the tensor-core regions: fp32 x adds its own (tf32 phi rows, bwd32 operand rows),
    # larger than the 16-bit ones
    assert L.mhc_pre_fwd_workspace_bytes(4096, 4, 4096, 0) > \
        L.mhc_pre_fwd_workspace_bytes(4096, 4, 4096, 2)
    assert L.mhc_pre_bwd_workspace_bytes(4096, 8, 4096, 0, 20) > \
        L.mhc_pre_bwd_workspace_bytes(4096, 8, 4096, 2, 20)


def test_peer_region_layout():
    """[stage | result | flags 2 x 8 ranks x 256 CTAs | control block]: the stage and result
    areas are n rounded up to 64 floats; the control block (device-kept epoch) is 256 B."""
    from FlagOS_mhc import _C
    L = _C.lib()
    for n in (1, 64, 65, 24 * 28672 + 27):
        cap = (n + 63) // 64 * 64
        assert L.mhc_peer_region_bytes(n) == 4 * (2 * cap + 2 * 8 * 256) + 256
    assert L.mhc_peer_region_bytes(0) == 0
    assert L.mhc_peer_handle_bytes() == 64


def test_cpu_tensors_raise_no_fallback():
    import FlagOS_mhc as M
    x = torch.randn(4, 4, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        M.mhc_post(x, torch.randn(4, 4, 4), torch.randn(4, 64, dtype=torch.bfloat16),
                   torch.randn(4, 4))
    phi = torch.randn(24, 256)
    with pytest.raises(RuntimeError, match="CUDA"):
        M.mhc_pre_clamp_sinkhorn(x, phi, torch.ones(3), torch.zeros(24))


def test_shape_errors_match_reference():
    import FlagOS_mhc as M
    with pytest.raises(ValueError):
        M.mhc_post(torch.randn(4, 64), torch.randn(4, 4), torch.randn(64), torch.randn(4))
    x = torch.randn(2, 4, 16)
    with pytest.raises(AssertionError):
        M.mhc_pre_clamp_sinkhorn(x, torch.randn(24, 63), torch.ones(3), torch.zeros(24))
    with pytest.raises(NotImplementedError):
        M.mhc_pre_clamp_sinkhorn(torch.randn(2, 9, 16), torch.randn(99, 144), torch.ones(3),
                                 torch.zeros(99))
