"""Generate the golden fixtures in this directory from the REFERENCE itself.

Runs the reference's own pure-PyTorch functions (``mhc_post_ref``,
``mhc_post_backward_ref``, ``mhc_pre_clamp_sinkhorn_ref``,
``mhc_pre_clamp_sinkhorn_backward_ref``; liuhycs/FlagOS-mhc ``src/``) on small
seeded inputs and stores inputs and outputs as ``.npz``.  Tensors of dtype
bf16/fp16 are stored widened to float32 (exact) with their dtype recorded.

Usage (only where the reference checkout exists):
    python tests/golden/make_golden.py --ref <path to FlagOS-mhc checkout>
"""
import argparse
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

POST_CASES = [
    # name, shape (B,S) or (T,), N, D, dtype
    ("post_bsnd_n4_bf16", (2, 8), 4, 64, torch.bfloat16),
    ("post_tnd_n8_fp32", (16,), 8, 48, torch.float32),
    ("post_tnd_n4_fp16", (5,), 4, 40, torch.float16),
    ("post_tnd_n2_bf16", (3,), 2, 24, torch.bfloat16),
]

PRE_CASES = [
    # name, lead shape, N, D, dtype, clamp (min,max), iters, style
    ("pre_bsnd_n4_bf16_c3", (2, 8), 4, 64, torch.bfloat16, (-3.0, 3.0), 20, "reftest"),
    ("pre_tnd_n4_bf16_noclamp", (16,), 4, 64, torch.bfloat16, (0.0, 0.0), 20, "config"),
    ("pre_tnd_n8_bf16_c10", (8,), 8, 32, torch.bfloat16, (-10.0, 10.0), 20, "config"),
    ("pre_tnd_n4_fp32_c1_it5", (6,), 4, 32, torch.float32, (-1.0, 1.0), 5, "hot"),
    ("pre_tnd_n2_bf16_it1", (4,), 2, 16, torch.bfloat16, (0.0, 0.0), 1, "config"),
]


def _np(t):
    return t.detach().to(torch.float32).cpu().numpy()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("MHC_REFERENCE"),
                    help="checkout of liuhycs/FlagOS-mhc (or set MHC_REFERENCE)")
    args = ap.parse_args()
    if not args.ref:
        ap.error("give --ref <reference checkout> or set MHC_REFERENCE")
    sys.path.insert(0, args.ref)
    from src import (mhc_post_ref, mhc_post_backward_ref, mhc_pre_clamp_sinkhorn_ref,
                     mhc_pre_clamp_sinkhorn_backward_ref)

    for i, (name, lead, N, D, dt) in enumerate(POST_CASES):
        g = torch.Generator().manual_seed(100 + i)
        x = torch.randn(*lead, N, D, generator=g).to(dt)
        h_res = torch.randn(*lead, N, N, generator=g)
        h_out = torch.randn(*lead, D, generator=g).to(dt)
        h_post = torch.randn(*lead, N, generator=g)
        gy = torch.randn(*lead, N, D, generator=g).to(dt)
        y = mhc_post_ref(x, h_res, h_out, h_post)
        gx, ghr, gho, ghp = mhc_post_backward_ref(gy, x, h_res, h_out, h_post)
        np.savez_compressed(
            os.path.join(HERE, name + ".npz"), kind="post", dtype=str(dt).split(".")[-1],
            x=_np(x), h_res=_np(h_res), h_out=_np(h_out), h_post=_np(h_post), grad_y=_np(gy),
            y=_np(y), grad_x=_np(gx), grad_h_res=_np(ghr), grad_h_out=_np(gho),
            grad_h_post=_np(ghp))

    for i, (name, lead, N, D, dt, (cmin, cmax), iters, style) in enumerate(PRE_CASES):
        g = torch.Generator().manual_seed(200 + i)
        hc_mix = N * (N + 2)
        if style == "reftest":
            x = (torch.randn(*lead, N, D, generator=g) * 0.1).to(dt)
            phi = torch.randn(hc_mix, N * D, generator=g) * 0.1
            alpha = torch.tensor([0.5, 0.5, 0.5])
            base = torch.randn(hc_mix, generator=g) * 0.01
        elif style == "hot":
            # large logits so the clamp is active on many entries
            x = torch.randn(*lead, N, D, generator=g).to(dt)
            phi = torch.randn(hc_mix, N * D, generator=g) * (3.0 / (N * D) ** 0.5)
            alpha = torch.rand(3, generator=g) + 0.5
            base = torch.randn(hc_mix, generator=g) * 0.1
        else:
            x = torch.randn(*lead, N, D, generator=g).to(dt)
            phi = torch.randn(hc_mix, N * D, generator=g) / (N * D) ** 0.5
            alpha = torch.rand(3, generator=g) + 0.5
            base = torch.randn(hc_mix, generator=g) * 0.1
        T = int(np.prod(lead))
        gy = torch.randn(*lead, D, generator=g).to(dt)
        gpost = torch.randn(T, N, generator=g)
        gcomb = torch.randn(T, N, N, generator=g)
        kw = dict(norm_eps=1e-6, hc_eps=1e-6, clamp_min=cmin, clamp_max=cmax, iter_times=iters)
        out = mhc_pre_clamp_sinkhorn_ref(x, phi, alpha, base, **kw)
        gx, gphi, ga, gb = mhc_pre_clamp_sinkhorn_backward_ref(x, phi, alpha, base, gy, gpost,
                                                               gcomb, **kw)
        np.savez_compressed(
            os.path.join(HERE, name + ".npz"), kind="pre", dtype=str(dt).split(".")[-1],
            clamp_min=cmin, clamp_max=cmax, iter_times=iters, norm_eps=1e-6, hc_eps=1e-6,
            x=_np(x), phi=_np(phi), alpha=_np(alpha), base=_np(base), grad_y=_np(gy),
            grad_post_out=_np(gpost), grad_comb_frag=_np(gcomb),
            y=_np(out["y"]), post_out=_np(out["post_out"]), comb_frag=_np(out["comb_frag"]),
            inv_rms=_np(out["inv_rms"]), mixes=_np(out["mixes"]),
            h_res_logits=_np(out["h_res_logits"]), pre=_np(out["pre"]),
            grad_x=_np(gx), grad_phi=_np(gphi), grad_alpha=_np(ga), grad_base=_np(gb))
    print("wrote", len(POST_CASES) + len(PRE_CASES), "fixtures to", HERE)


if __name__ == "__main__":
    main()
