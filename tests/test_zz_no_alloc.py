"""mhc_pre_fwd_noalloc: the pre forward for callers that cannot allocate device
memory where they run the operator (an arena allocator that owns the device
budget, or a cgo/JNI/C binding without a device allocator).  Its scratch is a
static device array of the library; this test calls it through the C ABI and
checks every output against mhc_pre_fwd (caller workspace) on two calls in a
row, the second with other inputs, so stale scratch contents would show.

The file name sorts last so a run that stops at the first failure has already
run every other test."""
import ctypes

import pytest
import torch

from tests._util import TOL_FP32

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _inputs(T, N, D, seed):
    g = torch.Generator().manual_seed(seed)
    hm, hc = N * (N + 2), N * D
    x = torch.randn(T, N, D, generator=g).to(torch.bfloat16).to(DEV)
    phi = (torch.randn(hm, hc, generator=g) / hc ** 0.5).to(DEV)
    alpha = (torch.rand(3, generator=g) + 0.5).to(DEV)
    base = (torch.randn(hm, generator=g) * 0.1).to(DEV)
    return x, phi, alpha, base


def _outputs(T, N, D):
    f = dict(dtype=torch.float32, device=DEV)
    return dict(y=torch.empty(T, D, dtype=torch.bfloat16, device=DEV),
                post_out=torch.empty(T, N, **f), comb_frag=torch.empty(T, N, N, **f),
                inv_rms=torch.empty(T, **f), x_scaled=torch.empty(T, N * D, **f),
                mixes=torch.empty(T, N * (N + 2), **f), h_res_logits=torch.empty(T, N, N, **f),
                pre=torch.empty(T, N, **f))


ORDER = ("y", "post_out", "comb_frag", "inv_rms", "x_scaled", "mixes", "h_res_logits", "pre")


def _call(L, fn, x, phi, alpha, base, o, T, N, D, ws=None):
    from FlagOS_mhc import _C
    p = _C.ptr
    head = [p(x), p(phi), p(alpha), p(base), T, N, D, _C.MHC_BF16, 1e-6, 1e-6, -10.0, 10.0, 20]
    outs = [p(o[k]) for k in ORDER]
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    if fn == "mhc_pre_fwd":
        return L.mhc_pre_fwd(*head, *outs, p(ws), ws.numel(), stream)
    return L.mhc_pre_fwd_noalloc(*head, *outs, stream)


def test_noalloc_matches_workspace_entry_point_twice():
    from FlagOS_mhc import _C
    L = _C.lib()
    torch.cuda.set_device(0)
    for call, (T, N, D, seed) in enumerate([(3000, 4, 1024, 1), (1234, 4, 512, 2)]):
        x, phi, alpha, base = _inputs(T, N, D, seed)
        want, got = _outputs(T, N, D), _outputs(T, N, D)
        ws = torch.empty(L.mhc_pre_fwd_workspace_bytes(T, N, D, _C.MHC_BF16), dtype=torch.uint8,
                         device=DEV)
        assert _call(L, "mhc_pre_fwd", x, phi, alpha, base, want, T, N, D, ws) == _C.MHC_OK
        assert _call(L, "mhc_pre_fwd_noalloc", x, phi, alpha, base, got, T, N, D) == _C.MHC_OK
        torch.cuda.synchronize()
        for k in ORDER:
            a, b = got[k].double(), want[k].double()
            err = ((a - b).abs().max() / b.abs().max().clamp_min(1e-30)).item()
            assert err <= TOL_FP32, (call, k, err)


def test_noalloc_rejects_problems_beyond_its_scratch():
    from FlagOS_mhc import _C
    L = _C.lib()
    limit = 16 << 20
    T = 1
    while L.mhc_pre_fwd_workspace_bytes(T, 4, 7168, _C.MHC_BF16) <= limit:
        T *= 2
    x, phi, alpha, base = _inputs(1, 4, 64, 3)  # pointers are never touched
    o = _outputs(1, 4, 64)
    st = _call(L, "mhc_pre_fwd_noalloc", x, phi, alpha, base, o, T, 4, 7168)
    assert st == _C.MHC_ERR_SCRATCH_LIMIT
    assert b"scratch" in L.mhc_status_string(st)
    # N=8 at D=7168: the bf16 hi/lo split of phi alone (160 x 57344 bf16) is over
    # the limit, so even one token is rejected
    assert L.mhc_pre_fwd_workspace_bytes(1, 8, 7168, _C.MHC_BF16) > limit
    st = _call(L, "mhc_pre_fwd_noalloc", x, phi, alpha, base, o, 1, 8, 7168)
    assert st == _C.MHC_ERR_SCRATCH_LIMIT
    # the documented limits: N=4, D=7168 up to T=167,770; N=8, D=4096 up to T=51,780
    assert L.mhc_pre_fwd_workspace_bytes(167770, 4, 7168, _C.MHC_BF16) <= limit
    assert L.mhc_pre_fwd_workspace_bytes(167771, 4, 7168, _C.MHC_BF16) > limit
    assert L.mhc_pre_fwd_workspace_bytes(51780, 8, 4096, _C.MHC_BF16) <= limit
    assert L.mhc_pre_fwd_workspace_bytes(51781, 8, 4096, _C.MHC_BF16) > limit
    # fp32 x: the tf32 phi rows are fp32, so N=8 fits only up to D=2048
    assert L.mhc_pre_fwd_workspace_bytes(1, 8, 4096, _C.MHC_F32) > limit
    assert L.mhc_pre_fwd_workspace_bytes(51780, 8, 2048, _C.MHC_F32) <= limit
    assert L.mhc_pre_fwd_workspace_bytes(167770, 4, 7168, _C.MHC_F32) <= limit
