"""The package's pure-PyTorch *_ref functions (part of the reference API) agree
with the oracle and with the reference goldens, on CPU."""
import pytest
import torch

import FlagOS_mhc as M
from oracle import mhc_oracle as O
from tests._util import golden_cases, load_golden, rel_err


@pytest.mark.parametrize("path", golden_cases("pre"), ids=lambda p: p.split("/")[-1])
def test_pre_ref_functions_vs_golden(path):
    t, dt, sc = load_golden(path)
    kw = dict(norm_eps=sc["norm_eps"], hc_eps=sc["hc_eps"], clamp_min=sc["clamp_min"],
              clamp_max=sc["clamp_max"], iter_times=int(sc["iter_times"]))
    x, gy = t["x"].to(dt), t["grad_y"].to(dt)
    out = M.mhc_pre_clamp_sinkhorn_ref(x, t["phi"], t["alpha"], t["base"], **kw)
    for k in ("post_out", "comb_frag", "mixes", "pre", "inv_rms"):
        assert rel_err(out[k], t[k]) < 1e-6, k
    g = M.mhc_pre_clamp_sinkhorn_backward_ref(x, t["phi"], t["alpha"], t["base"], gy,
                                              t["grad_post_out"], t["grad_comb_frag"], **kw)
    for got, k in zip(g, ("grad_x", "grad_phi", "grad_alpha", "grad_base")):
        assert rel_err(got, t[k]) < 1e-5, k


@pytest.mark.parametrize("path", golden_cases("post"), ids=lambda p: p.split("/")[-1])
def test_post_ref_functions_vs_golden(path):
    t, dt, _ = load_golden(path)
    x, ho, gy = t["x"].to(dt), t["h_out"].to(dt), t["grad_y"].to(dt)
    assert rel_err(M.mhc_post_ref(x, t["h_res"], ho, t["h_post"]), t["y"]) < 1e-6
    g = M.mhc_post_backward_ref(gy, x, t["h_res"], ho, t["h_post"])
    for got, k in zip(g, ("grad_x", "grad_h_res", "grad_h_out", "grad_h_post")):
        assert rel_err(got, t[k]) < 1e-6, k
