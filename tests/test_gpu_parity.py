"""CUDA kernels vs the CPU oracle (and the reference goldens) on the same seeded
inputs.  Tolerances: fp32 outputs <= 1e-5 normwise relative; bf16/fp16 outputs
<= 2e-2 normwise relative; Sinkhorn matrices <= 1e-4 absolute."""
import pytest
import torch

import FlagOS_mhc as M
from oracle import mhc_oracle as O
from tests._util import (TOL_BF16, TOL_FP32, TOL_SINKHORN_ABS, abs_err, golden_cases,
                         load_golden, rel_err)
from tests.gen import post_inputs, pre_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda"
F64 = torch.float64


def _tol(dt):
    return TOL_FP32 if dt == torch.float32 else TOL_BF16


# ---------------------------------------------------------------- goldens
@pytest.mark.parametrize("path", golden_cases("post"), ids=lambda p: p.split("/")[-1])
def test_post_golden(path):
    t, dt, _ = load_golden(path)
    x, ho, gy = (t[k].to(dt).to(DEV) for k in ("x", "h_out", "grad_y"))
    hr, hp = t["h_res"].to(DEV), t["h_post"].to(DEV)
    y = M.mhc_post(x, hr, ho, hp)
    assert y.dtype == dt and y.shape == x.shape
    assert rel_err(y, t["y"]) <= _tol(dt)
    gx, ghr, gho, ghp = M.mhc_post_backward(gy, x, hr, ho, hp)
    assert rel_err(gx, t["grad_x"]) <= _tol(dt)
    assert rel_err(gho, t["grad_h_out"]) <= _tol(dt)
    assert rel_err(ghr, t["grad_h_res"]) <= TOL_FP32
    assert rel_err(ghp, t["grad_h_post"]) <= TOL_FP32


@pytest.mark.parametrize("path", golden_cases("pre"), ids=lambda p: p.split("/")[-1])
def test_pre_golden(path):
    t, dt, sc = load_golden(path)
    kw = dict(norm_eps=sc["norm_eps"], hc_eps=sc["hc_eps"], clamp_min=sc["clamp_min"],
              clamp_max=sc["clamp_max"], iter_times=int(sc["iter_times"]))
    x, gy = t["x"].to(dt).to(DEV), t["grad_y"].to(dt).to(DEV)
    phi, alpha, base = (t[k].to(DEV) for k in ("phi", "alpha", "base"))
    out = M.mhc_pre_clamp_sinkhorn(x, phi, alpha, base, need_backward=True, **kw)
    assert rel_err(out["y"], t["y"]) <= _tol(dt)
    for k in ("post_out", "inv_rms", "mixes", "h_res_logits", "pre"):
        assert rel_err(out[k], t[k]) <= TOL_FP32, k
    assert abs_err(out["comb_frag"], t["comb_frag"]) <= TOL_SINKHORN_ABS
    gx, gphi, ga, gb = M.mhc_pre_clamp_sinkhorn_backward(
        x, phi, alpha, base, out["inv_rms"], out["x_scaled"], out["mixes"],
        out["h_res_logits"], out["pre"], gy, t["grad_post_out"].to(DEV),
        t["grad_comb_frag"].to(DEV), **kw)
    assert rel_err(gx, t["grad_x"]) <= _tol(dt)
    # the bar (1e-5) is against exact arithmetic: the fp64 oracle on the same saved
    # forward tensors the kernels start from
    xc, gyc = x.cpu(), gy.cpu()
    want = O.pre_bwd_from_saved(xc, t["phi"], t["alpha"], t["base"], out["inv_rms"].cpu(),
                                out["mixes"].cpu(), out["pre"].cpu(), gyc, t["grad_post_out"],
                                t["grad_comb_frag"], hc_eps=kw["hc_eps"],
                                clamp_min=kw["clamp_min"], clamp_max=kw["clamp_max"],
                                iter_times=kw["iter_times"], dtype=F64)
    exact = O.pre_bwd(xc, t["phi"], t["alpha"], t["base"], gyc, t["grad_post_out"],
                      t["grad_comb_frag"], dtype=F64, **kw)
    for got, w, e, key in zip((gphi, ga, gb), want[1:], exact[1:],
                              ("grad_phi", "grad_alpha", "grad_base")):
        assert rel_err(got, w) <= TOL_FP32, key
        # against the reference's own fp32 result: 1e-5 plus that result's measured
        # distance from exact arithmetic (the reference rounds in fp32 too) plus the
        # part of our forward's rounding that the backward carries (saved vs exact)
        slack = rel_err(t[key], e) + rel_err(w, e)
        assert rel_err(got, t[key]) <= TOL_FP32 + slack, (key, slack)


# ---------------------------------------------------------------- oracle sweeps
POST_SHAPES = [(1, 4, 64), (3, 4, 7168), (63, 4, 200), (65, 4, 1000), (37, 8, 256), (300, 8, 4096), (29, 8, 96), (21, 8, 192),
               (17, 1, 48), (9, 2, 24), (11, 3, 40), (7, 5, 72), (6, 6, 96), (5, 7, 80),
               (40, 4, 1), (13, 4, 7)]


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("T,N,D", POST_SHAPES)
def test_post_vs_oracle(T, N, D, dt):
    x, hr, ho, hp, gy = post_inputs(T, N, D, dt, seed=T * 31 + N * 7 + D)
    y = M.mhc_post(x.to(DEV), hr.to(DEV), ho.to(DEV), hp.to(DEV))
    ref = O.post_fwd(x, hr, ho, hp, dtype=F64)
    assert rel_err(y, ref) <= _tol(dt)
    got = M.mhc_post_backward(gy.to(DEV), x.to(DEV), hr.to(DEV), ho.to(DEV), hp.to(DEV))
    want = O.post_bwd(gy, x, hr, ho, hp, dtype=F64)
    for a, b, tol in zip(got, want, (_tol(dt), TOL_FP32, _tol(dt), TOL_FP32)):
        assert a.shape == b.shape
        assert rel_err(a, b) <= tol


def test_post_4d_and_unaligned_views():
    B, S, N, D = 2, 5, 4, 136
    x, hr, ho, hp, gy = post_inputs(B * S, N, D, torch.bfloat16, seed=11)
    x4, hr4, ho4, hp4, gy4 = (x.reshape(B, S, N, D), hr.reshape(B, S, N, N),
                              ho.reshape(B, S, D), hp.reshape(B, S, N), gy.reshape(B, S, N, D))
    y = M.mhc_post(x4.to(DEV), hr4.to(DEV), ho4.to(DEV), hp4.to(DEV))
    assert y.shape == (B, S, N, D)
    assert rel_err(y, O.post_fwd(x4, hr4, ho4, hp4, dtype=F64)) <= TOL_BF16
    # a non-contiguous x (every other token) goes through the flatten path
    xs = torch.randn(2 * B * S, N, D).to(torch.bfloat16)[::2]
    y2 = M.mhc_post(xs.to(DEV), hr.to(DEV), ho.to(DEV), hp.to(DEV))
    assert rel_err(y2, O.post_fwd(xs.contiguous(), hr, ho, hp, dtype=F64)) <= TOL_BF16
    g = M.mhc_post_backward(gy4.to(DEV), x4.to(DEV), hr4.to(DEV), ho4.to(DEV), hp4.to(DEV))
    assert g[0].shape == (B, S, N, D) and g[2].shape == (B, S, D)


PRE_SHAPES = [(1, 4, 64), (5, 4, 7168), (63, 4, 256), (130, 4, 64), (9, 8, 64), (7, 1, 32),
              (11, 2, 40), (6, 3, 24), (5, 5, 16), (4, 6, 32), (3, 7, 24), (33, 4, 36)]


@pytest.mark.parametrize("clamp", [(0.0, 0.0), (-1.0, 1.0)])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("T,N,D", PRE_SHAPES)
def test_pre_vs_oracle(T, N, D, dt, clamp):
    x, phi, alpha, base, gy, gpost, gcomb = pre_inputs(T, N, D, dt, seed=T * 13 + N * 5 + D,
                                                       phi_std=2.0 / (N * D) ** 0.5)
    kw = dict(norm_eps=1e-6, hc_eps=1e-6, clamp_min=clamp[0], clamp_max=clamp[1], iter_times=20)
    out = M.mhc_pre_clamp_sinkhorn(x.to(DEV), phi.to(DEV), alpha.to(DEV), base.to(DEV),
                                   need_backward=True, **kw)
    ref = O.pre_fwd(x, phi, alpha, base, dtype=F64, **kw)
    assert rel_err(out["y"], ref["y"]) <= _tol(dt)
    for k in ("post_out", "inv_rms", "mixes", "h_res_logits", "pre", "x_scaled"):
        assert rel_err(out[k], ref[k]) <= TOL_FP32, k
    assert abs_err(out["comb_frag"], ref["comb_frag"]) <= TOL_SINKHORN_ABS
    got = M.mhc_pre_clamp_sinkhorn_backward(
        x.to(DEV), phi.to(DEV), alpha.to(DEV), base.to(DEV), out["inv_rms"], out["x_scaled"],
        out["mixes"], out["h_res_logits"], out["pre"], gy.to(DEV), gpost.to(DEV),
        gcomb.to(DEV), **kw)
    # the backward mirrors the reference's: it starts from the saved forward tensors
    want = O.pre_bwd_from_saved(x, phi, alpha, base, out["inv_rms"].cpu(), out["mixes"].cpu(),
                                out["pre"].cpu(), gy, gpost, gcomb, hc_eps=1e-6,
                                clamp_min=clamp[0], clamp_max=clamp[1], iter_times=20,
                                dtype=F64)
    assert rel_err(got[0], want[0]) <= _tol(dt)
    for a, b, name in zip(got[1:], want[1:], ("grad_phi", "grad_alpha", "grad_base")):
        assert rel_err(a, b) <= TOL_FP32, name


@pytest.mark.parametrize("iters", [0, 1, 2, 7, 33])
def test_pre_iteration_counts(iters):
    x, phi, alpha, base, gy, gpost, gcomb = pre_inputs(40, 4, 64, torch.bfloat16, seed=iters)
    kw = dict(norm_eps=1e-6, hc_eps=1e-6, clamp_min=-3.0, clamp_max=3.0, iter_times=iters)
    out = M.mhc_pre_clamp_sinkhorn(x.to(DEV), phi.to(DEV), alpha.to(DEV), base.to(DEV),
                                   need_backward=True, **kw)
    ref = O.pre_fwd(x, phi, alpha, base, dtype=F64, **kw)
    assert abs_err(out["comb_frag"], ref["comb_frag"]) <= TOL_SINKHORN_ABS
    got = M.mhc_pre_clamp_sinkhorn_backward(
        x.to(DEV), phi.to(DEV), alpha.to(DEV), base.to(DEV), out["inv_rms"], out["x_scaled"],
        out["mixes"], out["h_res_logits"], out["pre"], gy.to(DEV), gpost.to(DEV),
        gcomb.to(DEV), **kw)
    want = O.pre_bwd_from_saved(x, phi, alpha, base, out["inv_rms"].cpu(), out["mixes"].cpu(),
                                out["pre"].cpu(), gy, gpost, gcomb, hc_eps=1e-6,
                                clamp_min=-3.0, clamp_max=3.0, iter_times=iters, dtype=F64)
    assert rel_err(got[0], want[0]) <= TOL_BF16
    for a, b, name in zip(got[1:], want[1:], ("grad_phi", "grad_alpha", "grad_base")):
        assert rel_err(a, b) <= TOL_FP32, name


def test_pre_need_backward_false_matches_ref_semantics():
    """Unlike the reference fast path (which always clamps and runs 20 iterations
    when need_backward=False), the result follows the _ref semantics."""
    x, phi, alpha, base, *_ = pre_inputs(70, 4, 64, torch.bfloat16, seed=5, phi_std=0.3)
    kw = dict(norm_eps=1e-6, hc_eps=1e-6, clamp_min=0.0, clamp_max=0.0, iter_times=3)
    out = M.mhc_pre_clamp_sinkhorn(x.to(DEV), phi.to(DEV), alpha.to(DEV), base.to(DEV), **kw)
    assert set(out) == {"y", "post_out", "comb_frag"}
    ref = O.pre_fwd(x, phi, alpha, base, dtype=F64, **kw)
    assert abs_err(out["comb_frag"], ref["comb_frag"]) <= TOL_SINKHORN_ABS


def test_pre_empty_token_range():
    x = torch.empty(0, 4, 64, dtype=torch.bfloat16, device=DEV)
    phi = torch.randn(24, 256, device=DEV)
    out = M.mhc_pre_clamp_sinkhorn(x, phi, torch.ones(3, device=DEV), torch.zeros(24, device=DEV),
                                   need_backward=True)
    assert out["y"].shape == (0, 64)
    g = M.mhc_pre_clamp_sinkhorn_backward(
        x, phi, torch.ones(3, device=DEV), torch.zeros(24, device=DEV), out["inv_rms"],
        out["x_scaled"], out["mixes"], out["h_res_logits"], out["pre"],
        torch.empty(0, 64, dtype=torch.bfloat16, device=DEV), torch.empty(0, 4, device=DEV),
        torch.empty(0, 4, 4, device=DEV))
    assert g[0].shape == (0, 4, 64) and float(g[1].abs().sum()) == 0.0


# ---------------------------------------------------------------- autograd
def test_autograd_wrappers_match_oracle():
    T, N, D = 24, 4, 128
    x, phi, alpha, base, gy, gpost, gcomb = pre_inputs(T, N, D, torch.bfloat16, seed=9)
    xd = x.to(DEV).requires_grad_(True)
    phid, ad, bd = (t.to(DEV).requires_grad_(True) for t in (phi, alpha, base))
    y, post, comb = M.mhc_pre_clamp_sinkhorn_fn(xd, phid, ad, bd, clamp_min=-5.0, clamp_max=5.0)
    loss = (y.float() * gy.to(DEV).float()).sum() + (post * gpost.to(DEV)).sum() + \
        (comb * gcomb.to(DEV)).sum()
    loss.backward()
    # the forward is deterministic: the same call gives the tensors the wrapper saved
    sv = M.mhc_pre_clamp_sinkhorn(xd.detach(), phid.detach(), ad.detach(), bd.detach(),
                                  clamp_min=-5.0, clamp_max=5.0, need_backward=True)
    want = O.pre_bwd_from_saved(x, phi, alpha, base, sv["inv_rms"].cpu(), sv["mixes"].cpu(),
                                sv["pre"].cpu(), gy, gpost, gcomb, hc_eps=1e-6, clamp_min=-5.0,
                                clamp_max=5.0, iter_times=20, dtype=F64)
    assert rel_err(xd.grad, want[0]) <= TOL_BF16
    for g_, w, name in zip((phid.grad, ad.grad, bd.grad), want[1:],
                           ("grad_phi", "grad_alpha", "grad_base")):
        assert rel_err(g_, w) <= TOL_FP32, name
    # mhc_post through autograd
    x2, hr, ho, hp, gy2 = post_inputs(T, N, D, torch.bfloat16, seed=10)
    leaves = [t.to(DEV).requires_grad_(True) for t in (x2, hr, ho, hp)]
    out = M.mhc_post_fn(*leaves)
    out.backward(gy2.to(DEV))
    want = O.post_bwd(gy2, x2, hr, ho, hp, dtype=F64)
    for leaf, w in zip(leaves, want):
        assert rel_err(leaf.grad, w) <= TOL_BF16


# ---------------------------------------------------------------- full-size properties
def test_post_full_size_token_sample():
    """Config C2 (T=32768, N=4, D=7168 bf16): tokens are independent, so a
    random sample of tokens checked against the oracle covers the full launch."""
    T, N, D = 32768, 4, 7168
    x, hr, ho, hp, gy = post_inputs(T, N, D, torch.bfloat16, seed=2, device=DEV)
    y = M.mhc_post(x, hr, ho, hp)
    g = M.mhc_post_backward(gy, x, hr, ho, hp)
    idx = torch.randperm(T, generator=torch.Generator().manual_seed(0))[:48]
    s = lambda t: t[idx.to(t.device)].cpu()  # noqa: E731
    assert rel_err(s(y), O.post_fwd(s(x), s(hr), s(ho), s(hp), dtype=F64)) <= TOL_BF16
    want = O.post_bwd(s(gy), s(x), s(hr), s(ho), s(hp), dtype=F64)
    for a, b, tol in zip(g, want, (TOL_BF16, TOL_FP32, TOL_BF16, TOL_FP32)):
        assert rel_err(s(a), b) <= tol


def test_pre_full_size_sample_and_linearity():
    """Config C3 shapes (N=4, D=7168).  Per-token outputs: a token sample against
    the oracle.  grad_phi/alpha/base are sums over tokens: the full-range result
    equals the sum of the results over two halves (linearity)."""
    T, N, D = 8192, 4, 7168
    x, phi, alpha, base, gy, gpost, gcomb = pre_inputs(T, N, D, torch.bfloat16, seed=3,
                                                       device=DEV)
    kw = dict(norm_eps=1e-6, hc_eps=1e-6, clamp_min=-10.0, clamp_max=10.0, iter_times=20)
    out = M.mhc_pre_clamp_sinkhorn(x, phi, alpha, base, need_backward=True, **kw)
    idx = torch.randperm(T, generator=torch.Generator().manual_seed(1))[:24].to(DEV)
    ref = O.pre_fwd(x[idx].cpu(), phi.cpu(), alpha.cpu(), base.cpu(), dtype=F64, **kw)
    for k in ("post_out", "mixes", "pre", "inv_rms"):
        assert rel_err(out[k][idx], ref[k]) <= TOL_FP32, k
    assert abs_err(out["comb_frag"][idx], ref["comb_frag"]) <= TOL_SINKHORN_ABS
    assert rel_err(out["y"][idx], ref["y"]) <= TOL_BF16

    def bwd(sl):
        return M.mhc_pre_clamp_sinkhorn_backward(
            x[sl], phi, alpha, base, out["inv_rms"][sl], out["x_scaled"][sl], out["mixes"][sl],
            out["h_res_logits"][sl], out["pre"][sl], gy[sl], gpost[sl], gcomb[sl], **kw)
    full = bwd(slice(0, T))
    h1, h2 = bwd(slice(0, T // 2)), bwd(slice(T // 2, T))
    for i in (1, 2, 3):
        assert rel_err(full[i], h1[i].double() + h2[i].double()) <= 2e-5
    assert torch.equal(full[0][: T // 2], h1[0])
    want = O.pre_bwd_from_saved(x[idx].cpu(), phi.cpu(), alpha.cpu(), base.cpu(),
                                out["inv_rms"][idx].cpu(), out["mixes"][idx].cpu(),
                                out["pre"][idx].cpu(), gy[idx].cpu(), gpost[idx].cpu(),
                                gcomb[idx].cpu(), hc_eps=1e-6, clamp_min=-10.0, clamp_max=10.0,
                                iter_times=20, dtype=F64)
    assert rel_err(full[0][idx], want[0]) <= TOL_BF16


def test_deterministic_backward():
    T, N, D = 4096, 4, 1024
    x, phi, alpha, base, gy, gpost, gcomb = pre_inputs(T, N, D, torch.bfloat16, seed=12,
                                                       device=DEV)
    out = M.mhc_pre_clamp_sinkhorn(x, phi, alpha, base, need_backward=True)
    args = (x, phi, alpha, base, out["inv_rms"], out["x_scaled"], out["mixes"],
            out["h_res_logits"], out["pre"], gy, gpost, gcomb)
    a = M.mhc_pre_clamp_sinkhorn_backward(*args)
    b = M.mhc_pre_clamp_sinkhorn_backward(*args)
    for u, v in zip(a, b):
        assert torch.equal(u, v)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("N", [4, 8])
def test_pre_many_tiles_ragged(N, dt):
    """More 128-token tiles than SMs (each persistent CTA runs several tiles,
    alternating TMEM buffers) and a ragged last tile; fp32 x runs the kind::tf32 mix
    (x_hi and x_lo against phi_hi and phi_lo)."""
    T, D = 148 * 128 * 2 + 77, 64 if dt == torch.bfloat16 else 72
    x, phi, alpha, base, gy, gpost, gcomb = pre_inputs(T, N, D, dt, seed=N,
                                                       phi_std=2.0 / (N * D) ** 0.5)
    kw = dict(norm_eps=1e-6, hc_eps=1e-6, clamp_min=-4.0, clamp_max=4.0, iter_times=20)
    out = M.mhc_pre_clamp_sinkhorn(x.to(DEV), phi.to(DEV), alpha.to(DEV), base.to(DEV),
                                   need_backward=True, **kw)
    ref = O.pre_fwd(x, phi, alpha, base, dtype=F64, **kw)
    for k in ("post_out", "inv_rms", "mixes", "h_res_logits", "pre"):
        assert rel_err(out[k], ref[k]) <= TOL_FP32, k
    assert abs_err(out["comb_frag"], ref["comb_frag"]) <= TOL_SINKHORN_ABS
    assert rel_err(out["y"], ref["y"]) <= _tol(dt)
    from FlagOS_mhc import _C
    assert _C.lib().mhc_device_status() == 0


@pytest.mark.parametrize("T,D,dt,xs", [(148 * 64 + 5, 48, torch.bfloat16, True),
                                        (148 * 64 * 3 + 41, 400, torch.bfloat16, True),
                                        (148 * 64 * 2 + 7, 400, torch.float16, True),
                                        (148 * 64 * 2 + 7, 400, torch.bfloat16, False)])
def test_pre_forward_large_ragged(T, D, dt, xs):
    """N=4 forward over more tiles than SMs: ragged last tile, a K row (N*D) that is not a
    multiple of the 128-column mix stage, d not a multiple of 32-byte apply groups of a
    warp, with and without x_scaled; repeated calls are bitwise equal."""
    N = 4
    x, phi, alpha, base, gy, gpost, gcomb = pre_inputs(T, N, D, dt, seed=T + D,
                                                       phi_std=2.0 / (N * D) ** 0.5)
    kw = dict(norm_eps=1e-6, hc_eps=1e-6, clamp_min=-4.0, clamp_max=4.0, iter_times=20)
    d = [t.to(DEV) for t in (x, phi, alpha, base)]
    out = M.mhc_pre_clamp_sinkhorn(*d, need_backward=True, materialize_x_scaled=xs, **kw)
    again = M.mhc_pre_clamp_sinkhorn(*d, need_backward=True, materialize_x_scaled=xs, **kw)
    for k in ("y", "post_out", "comb_frag", "inv_rms", "mixes", "pre"):
        assert torch.equal(out[k], again[k]), k
    ref = O.pre_fwd(x, phi, alpha, base, dtype=F64, **kw)
    for k in ("post_out", "inv_rms", "mixes", "h_res_logits", "pre"):
        assert rel_err(out[k], ref[k]) <= TOL_FP32, k
    assert abs_err(out["comb_frag"], ref["comb_frag"]) <= TOL_SINKHORN_ABS
    assert rel_err(out["y"], ref["y"]) <= _tol(dt)
    if xs:
        assert rel_err(out["x_scaled"], ref["x_scaled"]) <= TOL_FP32
    from FlagOS_mhc import _C
    assert _C.lib().mhc_device_status() == 0


def test_pre_bwd_full_grad_phi_vs_oracle():
    """Config-3 widths (N=4, D=7168) at T=8192: grad_phi / grad_alpha / grad_base
    (sums over every token) against the fp64 oracle run on the same saved tensors."""
    T, N, D = 8192, 4, 7168
    x, phi, alpha, base, gy, gpost, gcomb = pre_inputs(T, N, D, torch.bfloat16, seed=33)
    kw = dict(norm_eps=1e-6, hc_eps=1e-6, clamp_min=-10.0, clamp_max=10.0, iter_times=20)
    d = [t.to(DEV) for t in (x, phi, alpha, base, gy, gpost, gcomb)]
    out = M.mhc_pre_clamp_sinkhorn(d[0], d[1], d[2], d[3], need_backward=True, **kw)
    got = M.mhc_pre_clamp_sinkhorn_backward(
        d[0], d[1], d[2], d[3], out["inv_rms"], out["x_scaled"], out["mixes"],
        out["h_res_logits"], out["pre"], d[4], d[5], d[6], **kw)
    want = O.pre_bwd_from_saved(x, phi, alpha, base, out["inv_rms"].cpu(), out["mixes"].cpu(),
                                out["pre"].cpu(), gy, gpost, gcomb, hc_eps=1e-6,
                                clamp_min=-10.0, clamp_max=10.0, iter_times=20, dtype=F64)
    for a, b, name in zip(got[1:], want[1:], ("grad_phi", "grad_alpha", "grad_base")):
        assert rel_err(a, b) <= TOL_FP32, name
    assert rel_err(got[0], want[0]) <= TOL_BF16


def test_pre_skip_x_scaled_opt_in():
    """materialize_x_scaled=False: same outputs and gradients, no fp32 copy of x."""
    T, N, D = 300, 4, 256
    x, phi, alpha, base, gy, gpost, gcomb = pre_inputs(T, N, D, torch.bfloat16, seed=21)
    d = [t.to(DEV) for t in (x, phi, alpha, base, gy, gpost, gcomb)]
    a = M.mhc_pre_clamp_sinkhorn(d[0], d[1], d[2], d[3], need_backward=True)
    b = M.mhc_pre_clamp_sinkhorn(d[0], d[1], d[2], d[3], need_backward=True,
                                 materialize_x_scaled=False)
    assert b["x_scaled"].numel() == 0
    for k in ("y", "post_out", "comb_frag", "mixes", "pre", "inv_rms", "h_res_logits"):
        assert torch.equal(a[k], b[k]), k
    ga = M.mhc_pre_clamp_sinkhorn_backward(d[0], d[1], d[2], d[3], a["inv_rms"], a["x_scaled"],
                                           a["mixes"], a["h_res_logits"], a["pre"], d[4], d[5],
                                           d[6])
    gb = M.mhc_pre_clamp_sinkhorn_backward(d[0], d[1], d[2], d[3], b["inv_rms"], b["x_scaled"],
                                           b["mixes"], b["h_res_logits"], b["pre"], d[4], d[5],
                                           d[6])
    for u, v in zip(ga, gb):
        assert torch.equal(u, v)
    xd = d[0].clone().requires_grad_(True)
    y, post, comb = M.mhc_pre_clamp_sinkhorn_fn(xd, d[1], d[2], d[3], materialize_x_scaled=False)
    (y.float().sum() + comb.sum()).backward()
    assert xd.grad is not None and torch.isfinite(xd.grad.float()).all()


@pytest.mark.parametrize("T,D", [(148 * 128 + 77, 256), (1000, 4096)])
def test_pre_bwd_n8_tensor_core(T, D):
    """N=8 (hcMix=80) tensor-core backward: grad_x tiles over many 64-column steps with
    CTA ranges that start mid-tile, and grad_phi column tiles shared by several CTAs
    (partials summed in a fixed order), against the fp64 oracle on the same saved
    tensors; repeated calls are bitwise equal."""
    N = 8
    x, phi, alpha, base, gy, gpost, gcomb = pre_inputs(T, N, D, torch.bfloat16, seed=T + D,
                                                       phi_std=1.0 / (N * D) ** 0.5)
    kw = dict(norm_eps=1e-6, hc_eps=1e-6, clamp_min=-10.0, clamp_max=10.0, iter_times=20)
    d = [t.to(DEV) for t in (x, phi, alpha, base, gy, gpost, gcomb)]
    out = M.mhc_pre_clamp_sinkhorn(d[0], d[1], d[2], d[3], need_backward=True, **kw)
    args = (d[0], d[1], d[2], d[3], out["inv_rms"], out["x_scaled"], out["mixes"],
            out["h_res_logits"], out["pre"], d[4], d[5], d[6])
    got = M.mhc_pre_clamp_sinkhorn_backward(*args, **kw)
    again = M.mhc_pre_clamp_sinkhorn_backward(*args, **kw)
    for u, v in zip(got, again):
        assert torch.equal(u, v)
    want = O.pre_bwd_from_saved(x, phi, alpha, base, out["inv_rms"].cpu(), out["mixes"].cpu(),
                                out["pre"].cpu(), gy, gpost, gcomb, hc_eps=1e-6,
                                clamp_min=-10.0, clamp_max=10.0, iter_times=20, dtype=F64)
    assert rel_err(got[0], want[0]) <= TOL_BF16
    for a, b, name in zip(got[1:], want[1:], ("grad_phi", "grad_alpha", "grad_base")):
        assert rel_err(a, b) <= TOL_FP32, name
    from FlagOS_mhc import _C
    assert _C.lib().mhc_device_status() == 0


@pytest.mark.parametrize("T,N,D,dt", [(300, 4, 256, torch.bfloat16), (300, 4, 256, torch.float16),
                                      (300, 8, 128, torch.bfloat16), (300, 8, 128, torch.float16),
                                      (37, 4, 100, torch.bfloat16), (130, 4, 64, torch.float32)])
def test_pre_bwd_grad_x_accumulate(T, N, D, dt):
    """grad_x_accumulate (layer fusion: the post backward's grad_x added inside the pre
    backward): grad_x = own contribution + accumulator, rounded once; the parameter
    gradients are bitwise those of the plain call; the C entry point may run in place."""
    x, phi, alpha, base, gy, gpost, gcomb = pre_inputs(T, N, D, dt, seed=T + N + D,
                                                       phi_std=1.0 / (N * D) ** 0.5)
    kw = dict(norm_eps=1e-6, hc_eps=1e-6, clamp_min=-10.0, clamp_max=10.0, iter_times=20)
    d = [t.to(DEV) for t in (x, phi, alpha, base, gy, gpost, gcomb)]
    out = M.mhc_pre_clamp_sinkhorn(d[0], d[1], d[2], d[3], need_backward=True, **kw)
    args = (d[0], d[1], d[2], d[3], out["inv_rms"], out["x_scaled"], out["mixes"],
            out["h_res_logits"], out["pre"], d[4], d[5], d[6])
    g = torch.Generator().manual_seed(7)
    acc = torch.randn(T, N, D, generator=g).to(dt).to(DEV)
    plain = M.mhc_pre_clamp_sinkhorn_backward(*args, **kw)
    fused = M.mhc_pre_clamp_sinkhorn_backward(*args, grad_x_accumulate=acc, **kw)
    for u, v in zip(plain[1:], fused[1:]):
        assert torch.equal(u, v)
    want = O.pre_bwd_from_saved(x, phi, alpha, base, out["inv_rms"].cpu(), out["mixes"].cpu(),
                                out["pre"].cpu(), gy, gpost, gcomb, hc_eps=1e-6,
                                clamp_min=-10.0, clamp_max=10.0, iter_times=20, dtype=F64)
    ref = want[0].to(F64) + acc.cpu().to(F64)
    assert rel_err(fused[0], ref) <= _tol(dt)
    # in place through the C ABI: grad_x and the accumulator are one buffer
    from FlagOS_mhc import _C
    L = _C.lib()
    code = _C.dtype_code(dt)
    f32 = lambda t: t.float().contiguous()  # noqa: E731
    buf = acc.clone()
    ws_bytes = L.mhc_pre_bwd_workspace_bytes(T, N, D, code, 20)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=DEV)
    gphi = torch.empty_like(plain[1]); ga = torch.empty(3, device=DEV); gb = torch.empty_like(plain[3])
    st = L.mhc_pre_bwd_accumulate(
        _C.ptr(d[0]), _C.ptr(f32(d[1])), _C.ptr(f32(d[2])), _C.ptr(f32(d[3])),
        _C.ptr(out["inv_rms"]), _C.ptr(out["mixes"]), _C.ptr(out["pre"]), _C.ptr(d[4]),
        _C.ptr(d[5]), _C.ptr(d[6]), T, N, D, code, 1e-6, 1e-6, -10.0, 10.0, 20,
        _C.ptr(buf), _C.ptr(buf), _C.ptr(gphi), _C.ptr(ga), _C.ptr(gb), _C.ptr(ws), ws_bytes,
        _C.stream_of(d[0]))
    assert st == 0
    torch.cuda.synchronize()
    assert torch.equal(buf, fused[0])
    assert L.mhc_device_status() == 0


@pytest.mark.parametrize("iters", [0, 1, 2, 5, 20, 33, 70])
def test_pre_bwd_n8_iteration_counts(iters):
    """N=8 backward (hcMix=80 small-stage VJP, tensor-core main pass) at iteration counts
    from 0 to 70 against the fp64 oracle on the same saved tensors."""
    T, N, D = 300, 8, 256
    x, phi, alpha, base, gy, gpost, gcomb = pre_inputs(T, N, D, torch.bfloat16, seed=iters + 3,
                                                       phi_std=2.0 / (N * D) ** 0.5)
    kw = dict(norm_eps=1e-6, hc_eps=1e-6, clamp_min=-3.0, clamp_max=3.0, iter_times=iters)
    d = [t.to(DEV) for t in (x, phi, alpha, base, gy, gpost, gcomb)]
    out = M.mhc_pre_clamp_sinkhorn(d[0], d[1], d[2], d[3], need_backward=True, **kw)
    got = M.mhc_pre_clamp_sinkhorn_backward(
        d[0], d[1], d[2], d[3], out["inv_rms"], out["x_scaled"], out["mixes"],
        out["h_res_logits"], out["pre"], d[4], d[5], d[6], **kw)
    want = O.pre_bwd_from_saved(x, phi, alpha, base, out["inv_rms"].cpu(), out["mixes"].cpu(),
                                out["pre"].cpu(), gy, gpost, gcomb, hc_eps=1e-6,
                                clamp_min=-3.0, clamp_max=3.0, iter_times=iters, dtype=F64)
    assert rel_err(got[0], want[0]) <= TOL_BF16
    for a, b, name in zip(got[1:], want[1:], ("grad_phi", "grad_alpha", "grad_base")):
        assert rel_err(a, b) <= TOL_FP32, name


@pytest.mark.parametrize("N,D", [(4, 96), (8, 64)])
def test_pre_bwd_fp32_tensor_core_many_tiles(N, D):
    """fp32 x on the tensor-core backward: grad_x from the bf16 operand rows (gxs) with an
    fp32 epilogue, grad_phi on kind::tf32 (x as stored plus x_lo written in shared memory,
    against the tf32 hi / lo parts of inv*grad_mixes): many tiles, a ragged last tile, fp32
    tolerances against the fp64 oracle on the same saved tensors."""
    T = 148 * 64 * 3 + 41
    x, phi, alpha, base, gy, gpost, gcomb = pre_inputs(T, N, D, torch.float32, seed=7 + N,
                                                       phi_std=2.0 / (N * D) ** 0.5)
    kw = dict(norm_eps=1e-6, hc_eps=1e-6, clamp_min=-4.0, clamp_max=4.0, iter_times=20)
    d = [t.to(DEV) for t in (x, phi, alpha, base, gy, gpost, gcomb)]
    out = M.mhc_pre_clamp_sinkhorn(d[0], d[1], d[2], d[3], need_backward=True, **kw)
    got = M.mhc_pre_clamp_sinkhorn_backward(
        d[0], d[1], d[2], d[3], out["inv_rms"], out["x_scaled"], out["mixes"],
        out["h_res_logits"], out["pre"], d[4], d[5], d[6], **kw)
    want = O.pre_bwd_from_saved(x, phi, alpha, base, out["inv_rms"].cpu(), out["mixes"].cpu(),
                                out["pre"].cpu(), gy, gpost, gcomb, hc_eps=1e-6,
                                clamp_min=-4.0, clamp_max=4.0, iter_times=20, dtype=F64)
    for a, b, name in zip(got, want, ("grad_x", "grad_phi", "grad_alpha", "grad_base")):
        assert rel_err(a, b) <= TOL_FP32, name
    from FlagOS_mhc import _C
    assert _C.lib().mhc_device_status() == 0


@pytest.mark.parametrize("N,D", [(4, 256), (8, 192)])
def test_pre_bwd_fp16_tensor_core_many_tiles(N, D):
    """fp16 x on the tensor-core backward (fp16 operand rows scaled by powers of two from
    the maxima of phi, grad_mixes and inv*grad_mixes; N=4 single pass, N=8 gx + grad_phi
    kernels): many tiles, a ragged last tile, against the fp64 oracle on the same saved
    tensors."""
    T = 148 * 128 + 77
    x, phi, alpha, base, gy, gpost, gcomb = pre_inputs(T, N, D, torch.float16, seed=5,
                                                       phi_std=2.0 / (N * D) ** 0.5)
    kw = dict(norm_eps=1e-6, hc_eps=1e-6, clamp_min=-4.0, clamp_max=4.0, iter_times=20)
    d = [t.to(DEV) for t in (x, phi, alpha, base, gy, gpost, gcomb)]
    out = M.mhc_pre_clamp_sinkhorn(d[0], d[1], d[2], d[3], need_backward=True, **kw)
    got = M.mhc_pre_clamp_sinkhorn_backward(
        d[0], d[1], d[2], d[3], out["inv_rms"], out["x_scaled"], out["mixes"],
        out["h_res_logits"], out["pre"], d[4], d[5], d[6], **kw)
    want = O.pre_bwd_from_saved(x, phi, alpha, base, out["inv_rms"].cpu(), out["mixes"].cpu(),
                                out["pre"].cpu(), gy, gpost, gcomb, hc_eps=1e-6,
                                clamp_min=-4.0, clamp_max=4.0, iter_times=20, dtype=F64)
    assert rel_err(got[0], want[0]) <= TOL_BF16
    for a, b, name in zip(got[1:], want[1:], ("grad_phi", "grad_alpha", "grad_base")):
        assert rel_err(a, b) <= TOL_FP32, name
    from FlagOS_mhc import _C
    assert _C.lib().mhc_device_status() == 0


# ---------------------------------------------------------------- named configs
def _oracle_fwd_chunked(x, phi, alpha, base, kw, chunk=4096):
    """The fp64 oracle over every token, run on the GPU in token chunks (it is plain
    tensor arithmetic; the GPU only makes the full-size check fast)."""
    outs = []
    for a in range(0, x.shape[0], chunk):
        outs.append(O.pre_fwd(x[a:a + chunk], phi, alpha, base, dtype=F64, **kw))
    return {k: torch.cat([o[k] for o in outs]) for k in outs[0]}


def test_config_c1_pre_forward_full():
    """Config C1: T=16384, N=4, D=4096 bf16, phi ~ N(0, 1/128^2), clamp +-10, 20
    iterations, need_backward=True, seed 1 -- every token of every output against
    the fp64 oracle."""
    T, N, D = 16384, 4, 4096
    g = torch.Generator(device=DEV).manual_seed(1)
    x = torch.randn(T, N, D, generator=g, device=DEV).to(torch.bfloat16)
    phi = torch.randn(24, N * D, generator=g, device=DEV) / 128.0
    alpha = torch.rand(3, generator=g, device=DEV) + 0.5
    base = torch.randn(24, generator=g, device=DEV) * 0.1
    kw = dict(norm_eps=1e-6, hc_eps=1e-6, clamp_min=-10.0, clamp_max=10.0, iter_times=20)
    out = M.mhc_pre_clamp_sinkhorn(x, phi, alpha, base, need_backward=True, **kw)
    ref = _oracle_fwd_chunked(x, phi, alpha, base, kw)
    for k in ("post_out", "inv_rms", "mixes", "h_res_logits", "pre", "x_scaled"):
        assert rel_err(out[k], ref[k]) <= TOL_FP32, k
    assert abs_err(out["comb_frag"], ref["comb_frag"]) <= TOL_SINKHORN_ABS
    assert rel_err(out["y"], ref["y"]) <= TOL_BF16


def test_config_c4_layer_chain_autograd():
    """Config C4: the N=8 layer step pre -> h_out = y.W -> post, forward and backward
    through mhc_pre_clamp_sinkhorn_fn / mhc_post_fn at T=65536, D=4096 (seed 4).
    Per-token results on a token sample against the fp64 oracle, stage by stage (each
    stage fed the GPU's own inputs to it); grad_phi / grad_alpha / grad_base, sums over
    all 65536 tokens, against the fp64 oracle over every token."""
    T, N, D = 65536, 8, 4096
    HM = N * (N + 2)
    g = torch.Generator(device=DEV).manual_seed(4)
    x = torch.randn(T, N, D, generator=g, device=DEV).to(torch.bfloat16)
    phi = torch.randn(HM, N * D, generator=g, device=DEV) / 181.0
    alpha = torch.rand(3, generator=g, device=DEV) + 0.5
    base = torch.randn(HM, generator=g, device=DEV) * 0.1
    W = (torch.randn(D, D, generator=g, device=DEV) / 64.0).to(torch.bfloat16)
    gz = torch.randn(T, N, D, generator=g, device=DEV).to(torch.bfloat16)
    kw = dict(norm_eps=1e-6, hc_eps=1e-6, clamp_min=-10.0, clamp_max=10.0, iter_times=20)
    xl = x.clone().requires_grad_(True)
    pl, al, bl = (t.clone().requires_grad_(True) for t in (phi, alpha, base))
    y, post, comb = M.mhc_pre_clamp_sinkhorn_fn(xl, pl, al, bl, **kw)
    for t in (y, post, comb):
        t.retain_grad()
    h_out = y @ W
    h_out.retain_grad()
    z = M.mhc_post_fn(xl, comb, h_out, post)
    z.backward(gz)
    sv = M.mhc_pre_clamp_sinkhorn(x, phi, alpha, base, need_backward=True,
                                  materialize_x_scaled=False, **kw)
    idx = torch.randperm(T, generator=torch.Generator().manual_seed(4))[:32].to(DEV)
    # forward
    ref = O.pre_fwd(x[idx], phi, alpha, base, dtype=F64, **kw)
    assert rel_err(post[idx], ref["post_out"]) <= TOL_FP32
    assert abs_err(comb[idx], ref["comb_frag"]) <= TOL_SINKHORN_ABS
    assert rel_err(y[idx], ref["y"]) <= TOL_BF16
    zr = O.post_fwd(x[idx], comb[idx].detach(), h_out[idx].detach(), post[idx].detach(),
                    dtype=F64)
    assert rel_err(z[idx], zr) <= TOL_BF16
    # post backward
    pw = O.post_bwd(gz[idx], x[idx], comb[idx].detach(), h_out[idx].detach(),
                    post[idx].detach(), dtype=F64)
    assert rel_err(comb.grad[idx], pw[1]) <= TOL_FP32
    assert rel_err(h_out.grad[idx], pw[2]) <= TOL_BF16
    assert rel_err(post.grad[idx], pw[3]) <= TOL_FP32
    # pre backward (from the saved forward tensors, as the kernels are) + x's two grads
    qw = O.pre_bwd_from_saved(x[idx], phi, alpha, base, sv["inv_rms"][idx], sv["mixes"][idx],
                              sv["pre"][idx], y.grad[idx], post.grad[idx], comb.grad[idx],
                              hc_eps=1e-6, clamp_min=-10.0, clamp_max=10.0, iter_times=20,
                              dtype=F64)
    gx_want = pw[0].double() + qw[0].double()
    assert rel_err(xl.grad[idx], gx_want) <= TOL_BF16
    # parameter gradients over every token (fp64 oracle, token chunks)
    acc = None
    for a in range(0, T, 2048):
        s = slice(a, a + 2048)
        r = O.pre_bwd_from_saved(x[s], phi, alpha, base, sv["inv_rms"][s], sv["mixes"][s],
                                 sv["pre"][s], y.grad[s], post.grad[s], comb.grad[s],
                                 hc_eps=1e-6, clamp_min=-10.0, clamp_max=10.0, iter_times=20,
                                 dtype=F64)[1:]
        acc = list(r) if acc is None else [u + v for u, v in zip(acc, r)]
    for got, want, name in zip((pl.grad, al.grad, bl.grad), acc,
                               ("grad_phi", "grad_alpha", "grad_base")):
        assert rel_err(got, want) <= TOL_FP32, name


# ---------------------------------------------------------------- token-strided views
def _kernels_launched(fn):
    """Names of the CUDA kernels fn() launches (torch profiler)."""
    from torch.profiler import ProfilerActivity, profile
    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        out = fn()
        torch.cuda.synchronize()
    names = [e.name for e in prof.events() if e.device_type.name == "CUDA"]
    return out, names


def _ours(names):
    return all(n.startswith(("void mhc::", "mhc::")) or "mhc::" in n for n in names)


@pytest.mark.parametrize("pad", [64, 3])   # 16-byte aligned token rows / misaligned rows
def test_strided_views_in_place(pad):
    """Token-strided x / h_out / grad_y (slices of larger buffers) run in place -- every
    kernel launched is one of this library's.  With 16-byte aligned token rows the same
    kernels run as for packed tensors (bitwise equal results); misaligned rows take the
    general kernels (checked against the oracle)."""
    T, N, D = 300, 4, 256
    dt = torch.bfloat16
    same = pad % 8 == 0

    def close(a, b, tol):
        return torch.equal(a, b) if same else rel_err(a, b) <= tol

    x, hr, ho, hp, gy = (t.to(DEV) for t in post_inputs(T, N, D, dt, seed=pad))

    def strided(t, inner):
        big = torch.zeros(t.shape[0], inner + pad, dtype=t.dtype, device=DEV)
        big[:, :inner] = t.reshape(t.shape[0], inner)
        return big[:, :inner].view(t.shape)

    xv, hv, gv = strided(x, N * D), strided(ho, D), strided(gy, N * D)
    assert not xv.is_contiguous() and xv.stride(0) == N * D + pad
    y_ref = M.mhc_post(x, hr, ho, hp)
    y, names = _kernels_launched(lambda: M.mhc_post(xv, hr, hv, hp))
    assert _ours(names), names
    assert close(y, y_ref, TOL_BF16)
    g_ref = M.mhc_post_backward(gy, x, hr, ho, hp)
    g, names = _kernels_launched(lambda: M.mhc_post_backward(gv, xv, hr, hv, hp))
    assert _ours(names), names
    for a, b, tol in zip(g, g_ref, (TOL_BF16, TOL_FP32, TOL_BF16, TOL_FP32)):
        assert close(a, b, tol)
    # pre forward / backward
    xp, phi, alpha, base, gyp, gpost, gcomb = (t.to(DEV) for t in pre_inputs(T, N, D, dt, seed=7))
    xpv, gyv = strided(xp, N * D), strided(gyp, D)
    kw = dict(clamp_min=-5.0, clamp_max=5.0)
    o_ref = M.mhc_pre_clamp_sinkhorn(xp, phi, alpha, base, need_backward=True, **kw)
    o, names = _kernels_launched(
        lambda: M.mhc_pre_clamp_sinkhorn(xpv, phi, alpha, base, need_backward=True, **kw))
    assert _ours(names), names
    for k in o_ref:
        tol = TOL_BF16 if k == "y" else TOL_FP32
        if k == "comb_frag" and not same:
            assert abs_err(o[k], o_ref[k]) <= TOL_SINKHORN_ABS
        else:
            assert close(o[k], o_ref[k], tol), k
    sv = [o_ref[k] for k in ("inv_rms", "x_scaled", "mixes", "h_res_logits", "pre")]
    b_ref = M.mhc_pre_clamp_sinkhorn_backward(xp, phi, alpha, base, *sv, gyp, gpost, gcomb, **kw)
    b, names = _kernels_launched(
        lambda: M.mhc_pre_clamp_sinkhorn_backward(xpv, phi, alpha, base, *sv, gyv, gpost, gcomb,
                                                  **kw))
    assert _ours(names), names
    for u, v, tol in zip(b, b_ref, (TOL_BF16, TOL_FP32, TOL_FP32, TOL_FP32)):
        assert close(u, v, tol)


def test_strided_bsnd_view_and_irregular_fallback():
    """(B,S,N,D) views: every other token of a packed buffer (regular B/S strides) is
    read in place; a view whose B stride is not S times its S stride is packed first
    (as the reference's x.stride(1) assumption cannot hold there); both match the
    oracle."""
    B, S, N, D = 3, 40, 4, 128
    dt = torch.bfloat16
    big = torch.randn(B * S * 2, N, D, generator=torch.Generator().manual_seed(3)).to(dt).to(DEV)
    xv = big[::2].view(B, S, N, D)                     # stride_B == S * stride_S
    assert xv.stride(0) == S * xv.stride(1) and not xv.is_contiguous()
    x2 = torch.randn(B, S + 2, N, D, generator=torch.Generator().manual_seed(4)).to(dt)
    x2 = x2.to(DEV)[:, 1:S + 1]                        # stride_B != S * stride_S
    assert x2.stride(0) != S * x2.stride(1)
    _, phi, alpha, base, _, _, _ = pre_inputs(B * S, N, D, dt, seed=9)
    phi, alpha, base = phi.to(DEV), alpha.to(DEV), base.to(DEV)
    for xx in (xv, x2):
        out = M.mhc_pre_clamp_sinkhorn(xx, phi, alpha, base, need_backward=True)
        ref = O.pre_fwd(xx.cpu(), phi.cpu(), alpha.cpu(), base.cpu(), dtype=F64)
        assert out["y"].shape == (B, S, D)
        assert rel_err(out["y"], ref["y"]) <= TOL_BF16
        for k in ("mixes", "inv_rms", "pre", "post_out"):
            assert rel_err(out[k], ref[k]) <= TOL_FP32, k
