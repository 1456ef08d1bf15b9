"""Layer-level fusion of the forward pass: mhc_post(..., next_phi=phi) writes x_{l+1}
and, in the same pass, the mix partials of the next layer's pre operator, which
mhc_pre_clamp_sinkhorn(..., premix=...) then uses instead of re-reading x_{l+1}.
Checked against the two-op chain and the fp64 oracle."""
import pytest
import torch

import FlagOS_mhc as M
from oracle import mhc_oracle as O
from tests._util import TOL_BF16, TOL_FP32, TOL_SINKHORN_ABS, abs_err, rel_err
from tests.gen import post_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda"
F64 = torch.float64
KW = dict(norm_eps=1e-6, hc_eps=1e-6, clamp_min=-10.0, clamp_max=10.0, iter_times=20)


def _phi(N, D, seed, dev=DEV):
    g = torch.Generator().manual_seed(seed)
    hm = N * (N + 2)
    phi = torch.randn(hm, N * D, generator=g) / (N * D) ** 0.5
    alpha = torch.rand(3, generator=g) + 0.5
    base = torch.randn(hm, generator=g) * 0.1
    return phi.to(dev), alpha.to(dev), base.to(dev)


# (T, D): one K range per tile; several K ranges (few tiles); ragged last tile
@pytest.mark.parametrize("T,D", [(20000, 512), (300, 7168), (1000, 256), (77, 64)])
@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float16])
def test_fused_forward_matches_two_op_chain(T, D, dt):
    N = 4
    x, hr, ho, hp, _ = (t.to(DEV) for t in post_inputs(T, N, D, dt, seed=T + D))
    phi, alpha, base = _phi(N, D, seed=D)
    out_ref = M.mhc_post(x, hr, ho, hp)
    out, pm = M.mhc_post(x, hr, ho, hp, next_phi=phi)
    assert pm is not None and pm.layers >= 1
    assert torch.equal(out, out_ref)                   # same expression, same rounding
    want = M.mhc_pre_clamp_sinkhorn(out_ref, phi, alpha, base, need_backward=True, **KW)
    got = M.mhc_pre_clamp_sinkhorn(out, phi, alpha, base, need_backward=True, premix=pm, **KW)
    for k in ("post_out", "inv_rms", "mixes", "h_res_logits", "pre", "x_scaled"):
        assert rel_err(got[k], want[k]) <= TOL_FP32, k
    assert abs_err(got["comb_frag"], want["comb_frag"]) <= TOL_SINKHORN_ABS
    assert rel_err(got["y"], want["y"]) <= TOL_BF16
    # and against exact arithmetic on a token sample
    idx = torch.randperm(T, generator=torch.Generator().manual_seed(0))[:32].to(DEV)
    ref = O.pre_fwd(out[idx], phi, alpha, base, dtype=F64, **KW)
    for k in ("post_out", "inv_rms", "mixes", "pre"):
        assert rel_err(got[k][idx], ref[k]) <= TOL_FP32, k
    assert abs_err(got["comb_frag"][idx], ref["comb_frag"]) <= TOL_SINKHORN_ABS


def test_premix_is_ignored_for_other_tensors():
    """A premix made for (out, phi) is not applied to a modified out or another phi."""
    T, N, D = 512, 4, 256
    x, hr, ho, hp, _ = (t.to(DEV) for t in post_inputs(T, N, D, torch.bfloat16, seed=5))
    phi, alpha, base = _phi(N, D, seed=6)
    phi2 = phi * 1.5
    out, pm = M.mhc_post(x, hr, ho, hp, next_phi=phi)
    a = M.mhc_pre_clamp_sinkhorn(out, phi2, alpha, base, premix=pm, **KW)
    b = M.mhc_pre_clamp_sinkhorn(out, phi2, alpha, base, **KW)
    assert torch.equal(a["post_out"], b["post_out"])
    out.mul_(2)                                        # bumps out's version
    a = M.mhc_pre_clamp_sinkhorn(out, phi, alpha, base, premix=pm, **KW)
    b = M.mhc_pre_clamp_sinkhorn(out, phi, alpha, base, **KW)
    assert torch.equal(a["post_out"], b["post_out"])


def test_not_eligible_returns_none():
    x, hr, ho, hp, _ = (t.to(DEV) for t in post_inputs(64, 8, 128, torch.bfloat16, seed=1))
    phi, _, _ = _phi(8, 128, seed=2)
    out, pm = M.mhc_post(x, hr, ho, hp, next_phi=phi)
    assert pm is None and torch.equal(out, M.mhc_post(x, hr, ho, hp))


def test_two_layer_autograd_chain():
    """pre(l) -> y.W -> post(l, next_phi) -> pre(l+1, premix) through the autograd
    wrappers: outputs and every gradient match the unfused chain."""
    T, N, D = 2048, 4, 256
    dt = torch.bfloat16
    g = torch.Generator().manual_seed(11)
    x0 = torch.randn(T, N, D, generator=g).to(dt).to(DEV)
    W = (torch.randn(D, D, generator=g) / D ** 0.5).to(dt).to(DEV)
    p1, a1, b1 = _phi(N, D, seed=21)
    p2, a2, b2 = _phi(N, D, seed=22)
    gy = torch.randn(T, D, generator=g).to(dt).to(DEV)

    def run(fused):
        leaves = [t.clone().requires_grad_(True) for t in (x0, p1, a1, b1, p2, a2, b2)]
        x, q1, c1, d1, q2, c2, d2 = leaves
        y, post, comb = M.mhc_pre_clamp_sinkhorn_fn(x, q1, c1, d1, **KW)
        h = y @ W
        if fused:
            x1, pm = M.mhc_post_fn(x, comb, h, post, next_phi=q2)
            assert pm is not None
        else:
            x1, pm = M.mhc_post_fn(x, comb, h, post), None
        y2, post2, comb2 = M.mhc_pre_clamp_sinkhorn_fn(x1, q2, c2, d2, premix=pm, **KW)
        loss = (y2.float() * gy.float()).sum() + post2.sum() + (comb2 * comb2).sum()
        loss.backward()
        return [y2, post2, comb2] + [t.grad for t in leaves]

    a, b = run(True), run(False)
    # layer 2's parameter grads see the fused mix directly (1e-4); layer 1's arrive
    # through bf16-stored activation gradients, where a rounding flip is 2^-8 (bf16 bar)
    tols = [TOL_BF16, TOL_FP32, None, TOL_BF16, TOL_BF16, TOL_BF16, TOL_BF16, 1e-4, 1e-4, 1e-4]
    for u, v, tol in zip(a, b, tols):
        if tol is None:
            assert abs_err(u, v) <= TOL_SINKHORN_ABS
        else:
            assert rel_err(u, v) <= tol
