"""torch.autograd.Function wrappers pairing each forward with its backward.

Drop-in for ``src/autograd.py`` of liuhycs/FlagOS-mhc (same classes, same
saved tensors, same defaults).
"""
from __future__ import annotations

import torch

from .mhc_post import mhc_post
from .mhc_post_backward import mhc_post_backward
from .mhc_pre_clamp_sinkhorn import mhc_pre_clamp_sinkhorn
from .mhc_pre_clamp_sinkhorn_backward import mhc_pre_clamp_sinkhorn_backward


class MhcPostFn(torch.autograd.Function):
    """src/autograd.py:14-27.  With ``next_phi`` (optional) the forward also computes the
    next layer's mix partials and appends them to ``premix_sink`` (they carry no
    gradient)."""

    @staticmethod
    def forward(ctx, x, h_res, h_out, h_post, next_phi=None, premix_sink=None):
        if next_phi is not None:
            y, pm = mhc_post(x, h_res, h_out, h_post, next_phi=next_phi.detach())
            if premix_sink is not None:
                premix_sink.append(pm)
        else:
            y = mhc_post(x, h_res, h_out, h_post)
        ctx.save_for_backward(x, h_res, h_out, h_post)
        return y

    @staticmethod
    def backward(ctx, grad_y):
        x, h_res, h_out, h_post = ctx.saved_tensors
        return mhc_post_backward(grad_y.contiguous(), x, h_res, h_out, h_post) + (None, None)


def mhc_post_fn(x, h_res, h_out, h_post, next_phi=None):
    """Autograd-aware mhc_post.

    ``next_phi`` (optional, not in the reference API): the next layer's phi; the call
    then returns ``(out, premix)`` for ``mhc_pre_clamp_sinkhorn_fn(out, next_phi, ...,
    premix=premix)`` (see :func:`FlagOS_mhc.mhc_post`).  premix carries no gradient."""
    if next_phi is None:
        return MhcPostFn.apply(x, h_res, h_out, h_post)
    sink = []
    y = MhcPostFn.apply(x, h_res, h_out, h_post, next_phi, sink)
    pm = sink[0] if sink else None
    if pm is not None:  # key it to the tensor autograd hands back
        pm._key = (y.data_ptr(), y._version, tuple(y.shape)) + pm._key[3:]
    return y, pm


class MhcPreClampSinkhornFn(torch.autograd.Function):
    """src/autograd.py:35-74: the forward runs with need_backward=True and saves
    (x, phi, alpha, base, inv_rms, x_scaled, mixes, h_res_logits, pre)."""

    @staticmethod
    def forward(ctx, x, phi, alpha, base, norm_eps, hc_eps, clamp_min, clamp_max, iter_times,
                materialize_x_scaled=True, premix=None):
        out = mhc_pre_clamp_sinkhorn(x, phi, alpha, base, norm_eps=norm_eps, hc_eps=hc_eps,
                                     clamp_min=clamp_min, clamp_max=clamp_max,
                                     iter_times=iter_times, need_backward=True,
                                     materialize_x_scaled=materialize_x_scaled, premix=premix)
        ctx.save_for_backward(x, phi, alpha, base, out["inv_rms"], out["x_scaled"],
                              out["mixes"], out["h_res_logits"], out["pre"])
        ctx.norm_eps = norm_eps
        ctx.hc_eps = hc_eps
        ctx.clamp_min = clamp_min
        ctx.clamp_max = clamp_max
        ctx.iter_times = iter_times
        return out["y"], out["post_out"], out["comb_frag"]

    @staticmethod
    def backward(ctx, grad_y, grad_post_out, grad_comb_frag):
        (x, phi, alpha, base, inv_rms, x_scaled, mixes, h_res_logits, pre) = ctx.saved_tensors
        # autograd passes None for an output that did not reach the loss
        if grad_y is None:
            grad_y = torch.zeros(x.shape[:-2] + x.shape[-1:], dtype=x.dtype, device=x.device)
        if grad_post_out is None:
            grad_post_out = torch.zeros_like(pre)
        if grad_comb_frag is None:
            grad_comb_frag = torch.zeros_like(h_res_logits)
        gx, gphi, galpha, gbase = mhc_pre_clamp_sinkhorn_backward(
            x, phi, alpha, base, inv_rms, x_scaled, mixes, h_res_logits, pre,
            grad_y.contiguous(), grad_post_out.contiguous(), grad_comb_frag.contiguous(),
            norm_eps=ctx.norm_eps, hc_eps=ctx.hc_eps, clamp_min=ctx.clamp_min,
            clamp_max=ctx.clamp_max, iter_times=ctx.iter_times)
        return (gx, gphi.to(phi.dtype), galpha.to(alpha.dtype), gbase.to(base.dtype),
                None, None, None, None, None, None, None)


def mhc_pre_clamp_sinkhorn_fn(x, phi, alpha, base, norm_eps=1e-6, hc_eps=1e-6, clamp_min=0.0,
                              clamp_max=0.0, iter_times=20, materialize_x_scaled=True,
                              premix=None):
    """Autograd-aware mhc_pre_clamp_sinkhorn. Returns (y, post_out, comb_frag).

    ``materialize_x_scaled=False`` (opt-in, not in the reference API) saves an empty
    x_scaled instead of the fp32 copy of x; the backward does not need it.
    ``premix`` (optional, not in the reference API): the mix partials that
    ``mhc_post_fn(..., next_phi=phi)`` returned with x."""
    return MhcPreClampSinkhornFn.apply(x, phi, alpha, base, norm_eps, hc_eps, clamp_min,
                                       clamp_max, iter_times, materialize_x_scaled, premix)
