"""The fused cross-GPU gradient sum (mhc_grad_sum_peers / PeerGradReducer).

- 2+ GPUs: a torchrun child job checks it bitwise against the rank-order sum and
  against NCCL over several calls and sizes (skipped with fewer than 2 GPUs).
- 1 GPU: a one-rank call returns its input; and a two-rank call whose second
  "rank" is a second region on the same GPU that nobody ever signals runs into
  the kernel's bounded wait, returns early and reports MHC_ERR_TIMEOUT through
  mhc_device_status -- the failure path, with no GPU fault and a usable context
  afterwards."""
import ctypes
import os
import socket
import subprocess
import sys

import pytest
import torch

from FlagOS_mhc import _C

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _region(n):
    r = ctypes.c_void_p()
    assert _C.lib().mhc_peer_region_alloc(n, ctypes.byref(r)) == 0
    return r


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_grad_sum_two_ranks():
    n = min(torch.cuda.device_count(), 4)
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
           "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(ROOT, "tests", "_peer_worker.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0 and "PEER_OK" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]


def test_peer_grad_sum_one_rank_is_identity():
    L = _C.lib()
    n = 1001
    reg = _region(n)
    ptrs = (ctypes.c_void_p * 8)(reg.value)
    x = torch.randn(n, device="cuda")
    y = torch.empty_like(x)
    for epoch in (1, 2):
        st = L.mhc_grad_sum_peers(_C.ptr(x), _C.ptr(y), n, ptrs, 0, 1, epoch, 10 ** 9,
                                  _C.stream_of(x))
        assert st == 0
        torch.cuda.synchronize()
        assert torch.equal(x, y)
    assert L.mhc_device_status() == 0
    assert L.mhc_peer_region_free(reg) == 0
    # the device-kept epoch (epoch argument 0), several calls in a row on a fresh region
    reg = _region(n)
    ptrs = (ctypes.c_void_p * 8)(reg.value)
    for call in range(3):
        x = torch.randn(n, device="cuda")
        st = L.mhc_grad_sum_peers(_C.ptr(x), _C.ptr(y), n, ptrs, 0, 1, 0, 10 ** 9,
                                  _C.stream_of(x))
        assert st == 0
        torch.cuda.synchronize()
        assert torch.equal(x, y)
    assert L.mhc_device_status() == 0
    assert L.mhc_peer_region_free(reg) == 0


def test_peer_wait_times_out_and_reports():
    L = _C.lib()
    n = 4096
    mine, ghost = _region(n), _region(n)   # "rank 1" never runs a kernel
    ptrs = (ctypes.c_void_p * 8)(mine.value, ghost.value)
    x = torch.randn(n, device="cuda")
    y = torch.zeros_like(x)
    st = L.mhc_grad_sum_peers(_C.ptr(x), _C.ptr(y), n, ptrs, 0, 2, 1, 50 * 10 ** 6,
                              _C.stream_of(x))
    assert st == 0                       # launched; the failure shows on the device
    assert L.mhc_device_status() == _C.MHC_ERR_TIMEOUT
    assert L.mhc_device_status() == 0    # read and cleared
    assert float(y.abs().sum()) == 0.0   # nothing written to dst
    # the context is still usable: a one-rank sum on a fresh region works
    L.mhc_peer_region_free(mine)
    L.mhc_peer_region_free(ghost)
    reg = _region(n)
    ptrs = (ctypes.c_void_p * 8)(reg.value)
    st = L.mhc_grad_sum_peers(_C.ptr(x), _C.ptr(y), n, ptrs, 0, 1, 1, 10 ** 9, _C.stream_of(x))
    assert st == 0
    torch.cuda.synchronize()
    assert torch.equal(x, y)
    L.mhc_peer_region_free(reg)


def test_peer_argument_checks():
    L = _C.lib()
    ptrs = (ctypes.c_void_p * 8)()
    x = torch.zeros(8, device="cuda")
    s = _C.stream_of(x)
    assert L.mhc_grad_sum_peers(_C.ptr(x), _C.ptr(x), 8, ptrs, 0, 9, 1, 1, s) == 1   # world > 8
    assert L.mhc_grad_sum_peers(_C.ptr(x), _C.ptr(x), 8, ptrs, 2, 2, 1, 1, s) == 1   # rank
    assert L.mhc_grad_sum_peers(_C.ptr(x), _C.ptr(x), 8, ptrs, 0, 1, 1, 0, s) == 1   # timeout 0
    assert L.mhc_grad_sum_peers(_C.ptr(x), _C.ptr(x), 8, ptrs, 0, 1, 1, 1, s) == 1   # null region
