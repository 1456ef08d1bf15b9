"""The CPU oracle against golden vectors produced by the reference's own *_ref
functions (tests/golden/make_golden.py).  Pins the oracle before it is used as
the checker of the CUDA kernels."""
import pytest
import torch

from oracle import mhc_oracle as O
from tests._util import golden_cases, load_golden, rel_err, abs_err

# oracle (fp32) vs reference (fp32): same math, different summation order
TOL = 2e-5


@pytest.mark.parametrize("path", golden_cases("post"), ids=lambda p: p.split("/")[-1])
def test_post_oracle_vs_reference(path):
    t, dt, _ = load_golden(path)
    x, ho, gy = t["x"].to(dt), t["h_out"].to(dt), t["grad_y"].to(dt)
    y = O.post_fwd(x, t["h_res"], ho, t["h_post"])
    assert y.dtype == dt and y.shape == x.shape
    assert rel_err(y, t["y"]) <= (TOL if dt == torch.float32 else 8e-3)
    gx, ghr, gho, ghp = O.post_bwd(gy, x, t["h_res"], ho, t["h_post"])
    tol16 = TOL if dt == torch.float32 else 8e-3
    assert rel_err(gx, t["grad_x"]) <= tol16
    assert rel_err(gho, t["grad_h_out"]) <= tol16
    assert rel_err(ghr, t["grad_h_res"]) <= TOL
    assert rel_err(ghp, t["grad_h_post"]) <= TOL


@pytest.mark.parametrize("path", golden_cases("pre"), ids=lambda p: p.split("/")[-1])
def test_pre_oracle_vs_reference(path):
    t, dt, sc = load_golden(path)
    kw = dict(norm_eps=sc["norm_eps"], hc_eps=sc["hc_eps"], clamp_min=sc["clamp_min"],
              clamp_max=sc["clamp_max"], iter_times=int(sc["iter_times"]))
    x = t["x"].to(dt)
    gy = t["grad_y"].to(dt)
    f = O.pre_fwd(x, t["phi"], t["alpha"], t["base"], **kw)
    for k in ("post_out", "inv_rms", "mixes", "h_res_logits", "pre"):
        assert rel_err(f[k], t[k]) <= TOL, k
    assert abs_err(f["comb_frag"], t["comb_frag"]) <= 1e-5
    assert rel_err(f["y"], t["y"]) <= (TOL if dt == torch.float32 else 8e-3)
    gx, gphi, ga, gb = O.pre_bwd(x, t["phi"], t["alpha"], t["base"], gy,
                                 t["grad_post_out"], t["grad_comb_frag"], **kw)
    assert rel_err(gx, t["grad_x"]) <= (1e-4 if dt == torch.float32 else 8e-3)
    assert rel_err(gphi, t["grad_phi"]) <= 1e-4
    assert rel_err(ga, t["grad_alpha"]) <= 1e-4
    assert rel_err(gb, t["grad_base"]) <= 1e-4
    # the from-saved-tensors form the kernels mirror gives the same grads
    gx2, gphi2, ga2, gb2 = O.pre_bwd_from_saved(
        x, t["phi"], t["alpha"], t["base"], f["inv_rms"], f["mixes"], f["pre"], gy,
        t["grad_post_out"], t["grad_comb_frag"], hc_eps=kw["hc_eps"],
        clamp_min=kw["clamp_min"], clamp_max=kw["clamp_max"], iter_times=kw["iter_times"])
    assert rel_err(gphi2, t["grad_phi"]) <= 1e-4
    assert rel_err(ga2, t["grad_alpha"]) <= 1e-4
    assert rel_err(gb2, t["grad_base"]) <= 1e-4
    assert rel_err(gx2, t["grad_x"]) <= (1e-4 if dt == torch.float32 else 8e-3)


def test_sinkhorn_invariants_fp64():
    """Properties independent of torch's kernels: Sinkhorn output rows/cols sum
    to ~1, post in (0,2), pre in (eps, 1+eps)."""
    g = torch.Generator().manual_seed(7)
    T, N = 64, 4
    mixes = torch.randn(T, N * (N + 2), generator=g, dtype=torch.float64) * 3
    s = O.small_fwd(mixes, torch.tensor([1.0, 1.0, 1.0], dtype=torch.float64),
                    torch.zeros(N * (N + 2), dtype=torch.float64), N, 1e-6, -10.0, 10.0, 20)
    M = s["comb"]
    assert (M.sum(-2) - 1).abs().max() < 1e-5
    assert (M.sum(-1) - 1).abs().max() < 0.1   # rows converge more slowly
    assert (s["post_out"] > 0).all() and (s["post_out"] < 2).all()
    assert (s["pre"] > 1e-6).all() and (s["pre"] < 1 + 1e-6 + 1e-12).all()


def test_small_bwd_gradcheck_fp64():
    """The explicit small-stage VJP equals autograd's in fp64."""
    g = torch.Generator().manual_seed(3)
    T, N = 5, 4
    hm = N * (N + 2)
    mixes = (torch.randn(T, hm, generator=g, dtype=torch.float64) * 2).requires_grad_(True)
    alpha = (torch.rand(3, generator=g, dtype=torch.float64) + 0.5).requires_grad_(True)
    base = (torch.randn(hm, generator=g, dtype=torch.float64) * 0.1).requires_grad_(True)
    gp, gq, gc = (torch.randn(T, N, generator=g, dtype=torch.float64),
                  torch.randn(T, N, generator=g, dtype=torch.float64),
                  torch.randn(T, N, N, generator=g, dtype=torch.float64))
    s = O.small_fwd(mixes, alpha, base, N, 1e-6, -2.0, 2.0, 7)
    loss = (s["pre"] * gp).sum() + (s["post_out"] * gq).sum() + (s["comb"] * gc).sum()
    ref = torch.autograd.grad(loss, (mixes, alpha, base))
    with torch.no_grad():
        got = O.small_bwd(mixes, alpha, base, N, 1e-6, -2.0, 2.0, 7, gp, gq, gc)
    for a, b in zip(got, ref):
        assert rel_err(a, b) < 1e-10
