"""The operators under CUDA-graph capture: one step (pre forward + post forward + post
backward + pre backward) captured once and replayed on new inputs copied into the
captured tensors gives bitwise the results of eager calls on the same inputs."""
import pytest
import torch

import FlagOS_mhc as M
from tests.gen import post_inputs, pre_inputs

pytestmark = pytest.mark.gpu
DEV = "cuda"
KW = dict(norm_eps=1e-6, hc_eps=1e-6, clamp_min=-10.0, clamp_max=10.0, iter_times=20)


def _step(d):
    o = M.mhc_pre_clamp_sinkhorn(d["x"], d["phi"], d["alpha"], d["base"], need_backward=True,
                                 **KW)
    y = M.mhc_post(d["xp"], d["hr"], d["ho"], d["hp"])
    pg = M.mhc_post_backward(d["gyp"], d["xp"], d["hr"], d["ho"], d["hp"])
    g = M.mhc_pre_clamp_sinkhorn_backward(d["x"], d["phi"], d["alpha"], d["base"],
                                          o["inv_rms"], o["x_scaled"], o["mixes"],
                                          o["h_res_logits"], o["pre"], d["gy"], d["gpost"],
                                          d["gcomb"], **KW)
    return [o["y"], o["post_out"], o["comb_frag"], o["x_scaled"], y, *pg, *g]


def _inputs(T, N, D, seed):
    x, phi, alpha, base, gy, gpost, gcomb = pre_inputs(T, N, D, torch.bfloat16, seed=seed,
                                                       phi_std=1.0 / (N * D) ** 0.5)
    xp, hr, ho, hp, gyp = post_inputs(T, N, D, torch.bfloat16, seed=seed + 1)
    d = dict(x=x, phi=phi, alpha=alpha, base=base, gy=gy, gpost=gpost, gcomb=gcomb, xp=xp,
             hr=hr, ho=ho, hp=hp, gyp=gyp)
    return {k: v.to(DEV) for k, v in d.items()}


@pytest.mark.parametrize("T,N,D", [(300, 4, 256), (5000, 4, 512), (700, 8, 128)])
def test_step_graph_replay_matches_eager(T, N, D):
    d = _inputs(T, N, D, seed=T + N)
    _step(d)                                  # warm-up: attributes, tensor maps
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            outs = _step(d)
    torch.cuda.synchronize()
    for rep in range(2):
        new = _inputs(T, N, D, seed=100 * rep + 7)
        for k, v in new.items():
            d[k].copy_(v)
        graph.replay()
        torch.cuda.synchronize()
        want = _step(new)
        torch.cuda.synchronize()
        for i, (a, b) in enumerate(zip(outs, want)):
            assert torch.equal(a, b), (rep, i)
    from FlagOS_mhc import _C
    assert _C.lib().mhc_device_status() == 0
