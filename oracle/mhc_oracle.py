"""CPU oracle for the mHC operators -- TEST INFRASTRUCTURE ONLY.

This module restates, on the CPU and in plain tensor arithmetic, the algorithm
of the four mHC operators of liuhycs/FlagOS-mhc.  It is the parity checker for
the CUDA kernels of this repository and the CPU baseline timed by
``bench.py --impl reference``.  Only ``tests/``, ``__graft_entry__.smoke()``
and ``bench.py``'s CPU-baseline leg may import it; the shipped package never
does.

Every function names the reference lines it follows.  The backward of the
pre operator is written out as explicit vector-Jacobian products (the
reference computes it with ``torch.autograd`` through a re-run of its forward,
``src/mhc_pre_clamp_sinkhorn_backward.py:1397-1453``); the explicit chain
follows the order of the reference's small-stage kernel
(``src/mhc_pre_clamp_sinkhorn_backward.py:1144-1209``) and the RMS/GEMM
backward (``:1371-1384``, ``:161-207``).

Parity pin: ``tests/golden/*.npz`` hold outputs of the reference's own
``*_ref`` functions run on the same seeded inputs (generator:
``tests/golden/make_golden.py``); ``tests/test_oracle_golden.py`` checks this
module against them.

All arithmetic runs in ``dtype`` (float32 by default, float64 for tight
checks).  Inputs of lower precision (bf16/fp16) are widened exactly first,
as the reference does with ``.float()``.
"""

from __future__ import annotations

import torch


def _widen(t, dtype):
    return t.detach().to(dtype)


def _flat_post(x, h_res, h_out, h_post):
    """Token flattening of ``src/mhc_post.py:274-292``: (B,S,N,D) or (T,N,D)."""
    if x.dim() == 4:
        B, S, N, D = x.shape
        T = B * S
    elif x.dim() == 3:
        T, N, D = x.shape
    else:
        raise ValueError(f"unsupported x.dim()={x.dim()}, expect 3 or 4")
    return (x.reshape(T, N, D), h_res.reshape(T, N, N), h_out.reshape(T, D),
            h_post.reshape(T, N), T, N, D)


# --------------------------------------------------------------------------
# mhc_post
# --------------------------------------------------------------------------
def post_fwd(x, h_res, h_out, h_post, dtype=torch.float32):
    """out[t,i,:] = sum_j h_res[t,j,i] x[t,j,:] + h_post[t,i] h_out[t,:].

    Follows ``mhc_post_ref`` (``src/mhc_post.py:344-352``): widen, mix with the
    transposed h_res, add the rank-1 term, cast back to x.dtype.
    """
    xf, hr, ho, hp, T, N, D = _flat_post(x, h_res, h_out, h_post)
    xw, hrw, how, hpw = (_widen(a, dtype) for a in (xf, hr, ho, hp))
    mix = torch.einsum("tji,tjd->tid", hrw, xw)
    out = mix + hpw.unsqueeze(-1) * how.unsqueeze(1)
    return out.to(x.dtype).reshape(x.shape)


def post_bwd(grad_y, x, h_res, h_out, h_post, dtype=torch.float32):
    """The four VJPs of mhc_post (``src/mhc_post_backward.py:624-643``).

    grad_x[j]      = sum_i h_res[j,i] gy[i]        (cast to x.dtype)
    grad_h_res[j,i]= sum_d x[j,d] gy[i,d]          (fp32)
    grad_h_out     = sum_i h_post[i] gy[i]         (cast to x.dtype, :635)
    grad_h_post[i] = sum_d h_out[d] gy[i,d]        (fp32)
    """
    gyf, _, _, _, T, N, D = _flat_post(grad_y, h_res, h_out, h_post)
    xf, hr, ho, hp, _, _, _ = _flat_post(x, h_res, h_out, h_post)
    gyw, xw, hrw, how, hpw = (_widen(a, dtype) for a in (gyf, xf, hr, ho, hp))
    gx = torch.einsum("tji,tid->tjd", hrw, gyw).to(x.dtype)
    ghres = torch.einsum("tjd,tid->tji", xw, gyw)
    ghout = torch.einsum("ti,tid->td", hpw, gyw).to(x.dtype)
    ghpost = torch.einsum("td,tid->ti", how, gyw)
    out_shape = x.shape[:-2] + (D,)
    return (gx.reshape(x.shape), ghres.reshape(h_res.shape),
            ghout.reshape(out_shape), ghpost.reshape(h_post.shape))


# --------------------------------------------------------------------------
# mhc_pre_clamp_sinkhorn: small stage (heads, clamp, softmax, Sinkhorn)
# --------------------------------------------------------------------------
def _clamp_on(clamp_min, clamp_max):
    # src/mhc_pre_clamp_sinkhorn.py:923 and :1000 -- enabled iff either bound != 0
    return clamp_min != 0.0 or clamp_max != 0.0


def small_fwd(mixes, alpha, base, N, hc_eps, clamp_min, clamp_max, iter_times,
              keep_history=False):
    """Heads + clamp + row softmax + Sinkhorn, ``src/mhc_pre_clamp_sinkhorn.py:995-1010``.

    Order: P = softmax_row(clamp(logits)); M = P + eps; M /= colsum + eps;
    then (iter_times - 1) x { M /= rowsum + eps; M /= colsum + eps }.
    Returns pre, post_out, logits (pre-clamp), comb and, if asked, the list of
    intermediates the backward needs.
    """
    T = mixes.shape[0]
    a, b = alpha, base
    z_pre = mixes[:, :N] * a[0] + b[:N]
    z_post = mixes[:, N:2 * N] * a[1] + b[N:2 * N]
    s_pre = torch.sigmoid(z_pre)
    s_post = torch.sigmoid(z_post)
    pre = s_pre + hc_eps
    post_out = 2.0 * s_post
    logits = (mixes[:, 2 * N:] * a[2] + b[2 * N:]).reshape(T, N, N)
    lc = torch.clamp(logits, clamp_min, clamp_max) if _clamp_on(clamp_min, clamp_max) else logits
    e = (lc - lc.max(dim=-1, keepdim=True).values).exp()
    P = e / e.sum(dim=-1, keepdim=True)
    M0 = P + hc_eps
    cs0 = M0.sum(dim=-2, keepdim=True) + hc_eps
    M = M0 / cs0
    hist = [(M0, cs0)]          # (matrix before the col-norm, col divisor)
    for _ in range(iter_times - 1):
        rs = M.sum(dim=-1, keepdim=True) + hc_eps
        Q = M / rs
        cs = Q.sum(dim=-2, keepdim=True) + hc_eps
        if keep_history:
            hist.append((M, rs, Q, cs))
        M = Q / cs
    out = dict(pre=pre, post_out=post_out, logits=logits, comb=M)
    if keep_history:
        out.update(hist=hist, P=P, s_pre=s_pre, s_post=s_post, lc=lc)
    return out


def small_bwd(mixes, alpha, base, N, hc_eps, clamp_min, clamp_max, iter_times,
              grad_pre, grad_post, grad_comb):
    """VJP of :func:`small_fwd` -> (grad_mixes, grad_alpha, grad_base).

    Column-norm VJP ``dp = (du - sum_i du*u) / c`` and row-norm VJP
    ``dp = (dq - sum_j dq*q) / r`` as in
    ``src/mhc_pre_clamp_sinkhorn_backward.py:1144-1163``; iteration 0 and the
    softmax VJP as in ``:1165-1184``; heads as in ``:1193-1209``.  The clamp
    mask is the one ``torch.clamp`` autograd applies in the reference's
    autograd oracle (``:1437-1440``): the gradient passes where
    ``clamp_min <= l <= clamp_max``.
    """
    f = small_fwd(mixes, alpha, base, N, hc_eps, clamp_min, clamp_max,
                  iter_times, keep_history=True)
    g = grad_comb.reshape(-1, N, N).to(mixes.dtype)
    hist = f["hist"]
    # iterations iter_times-1 .. 1 : M_out = Q / cs, Q = M_in / rs
    for (M_in, rs, Q, cs) in reversed(hist[1:]):
        U = Q / cs
        dQ = (g - (g * U).sum(dim=-2, keepdim=True)) / cs
        g = (dQ - (dQ * Q).sum(dim=-1, keepdim=True)) / rs
    # iteration 0 : M_out = M0 / cs0, M0 = P + eps
    M0, cs0 = hist[0]
    U0 = M0 / cs0
    dP = (g - (g * U0).sum(dim=-2, keepdim=True)) / cs0
    P = f["P"]
    dlc = P * (dP - (dP * P).sum(dim=-1, keepdim=True))
    logits = f["logits"]
    if _clamp_on(clamp_min, clamp_max):
        mask = (logits >= clamp_min) & (logits <= clamp_max)
        dlog = torch.where(mask, dlc, torch.zeros_like(dlc))
    else:
        dlog = dlc
    dlog = dlog.reshape(-1, N * N)
    s_pre, s_post = f["s_pre"], f["s_post"]
    dz_pre = grad_pre.to(mixes.dtype) * s_pre * (1.0 - s_pre)
    dz_post = grad_post.to(mixes.dtype) * 2.0 * s_post * (1.0 - s_post)
    a = alpha
    grad_mixes = torch.cat([dz_pre * a[0], dz_post * a[1], dlog * a[2]], dim=1)
    grad_alpha = torch.stack([
        (dz_pre * mixes[:, :N]).sum(),
        (dz_post * mixes[:, N:2 * N]).sum(),
        (dlog * mixes[:, 2 * N:]).sum(),
    ])
    grad_base = torch.cat([dz_pre.sum(0), dz_post.sum(0), dlog.sum(0)])
    return grad_mixes, grad_alpha, grad_base


# --------------------------------------------------------------------------
# mhc_pre_clamp_sinkhorn forward / backward
# --------------------------------------------------------------------------
def _flat_pre(x):
    """``src/mhc_pre_clamp_sinkhorn.py:844-854``."""
    if x.dim() == 4:
        B, S, N, D = x.shape
        return x.reshape(B * S, N, D), (B, S, D)
    if x.dim() == 3:
        T, N, D = x.shape
        return x, (T, D)
    raise ValueError(f"unsupported x.dim()={x.dim()}")


def pre_fwd(x, phi, alpha, base, norm_eps=1e-6, hc_eps=1e-6, clamp_min=0.0,
            clamp_max=0.0, iter_times=20, dtype=torch.float32):
    """``mhc_pre_clamp_sinkhorn_ref`` (``src/mhc_pre_clamp_sinkhorn.py:974-1022``)
    plus the ``x_scaled`` tensor its fast path saves (``:896-903``)."""
    xf, y_shape = _flat_pre(x)
    T, N, D = xf.shape
    xw = _widen(xf, dtype).reshape(T, N * D)
    ms = xw.pow(2).mean(dim=-1, keepdim=True)
    inv = torch.rsqrt(ms + norm_eps)
    x_scaled = xw * inv
    mixes = x_scaled @ _widen(phi, dtype).t()
    s = small_fwd(mixes, _widen(alpha, dtype), _widen(base, dtype), N, hc_eps,
                  clamp_min, clamp_max, iter_times)
    y = (xw.reshape(T, N, D) * s["pre"].unsqueeze(-1)).sum(dim=-2)
    return dict(y=y.to(x.dtype).reshape(y_shape), post_out=s["post_out"],
                comb_frag=s["comb"], inv_rms=inv.squeeze(-1), x_scaled=x_scaled,
                mixes=mixes, h_res_logits=s["logits"], pre=s["pre"])


def pre_bwd(x, phi, alpha, base, grad_y, grad_post_out, grad_comb_frag,
            norm_eps=1e-6, hc_eps=1e-6, clamp_min=0.0, clamp_max=0.0,
            iter_times=20, dtype=torch.float32):
    """Gradient of ``sum(y*gy) + sum(post*gpost) + sum(comb*gcomb)`` with
    respect to (x, phi, alpha, base); the loss of
    ``mhc_pre_clamp_sinkhorn_backward_ref``
    (``src/mhc_pre_clamp_sinkhorn_backward.py:1447-1453``).

    Stages (explicit): y-backward grad_pre = sum_d gy*x[n] (``:68-155``);
    small-stage VJP (:func:`small_bwd`); gxs = grad_mixes @ phi and
    grad_phi = grad_mixes^T @ x_scaled (``:1371-1373``); RMS backward
    grad_x = gy*pre[n] + inv*gxs - (inv^3/HC_D) * dot(x, gxs) * x (``:185-206``).
    Returns (grad_x in x.dtype, grad_phi, grad_alpha, grad_base) in ``dtype``.
    """
    f = pre_fwd(x, phi, alpha, base, norm_eps, hc_eps, clamp_min, clamp_max,
                iter_times, dtype)
    xf, _ = _flat_pre(x)
    T, N, D = xf.shape
    HC_D = N * D
    xw = _widen(xf, dtype)
    gy = _widen(grad_y, dtype).reshape(T, D)
    grad_pre = torch.einsum("td,tnd->tn", gy, xw)
    gm, ga, gb = small_bwd(f["mixes"], _widen(alpha, dtype), _widen(base, dtype),
                           N, hc_eps, clamp_min, clamp_max, iter_times, grad_pre,
                           _widen(grad_post_out, dtype).reshape(T, N),
                           _widen(grad_comb_frag, dtype).reshape(T, N, N))
    phiw = _widen(phi, dtype)
    gxs = gm @ phiw
    grad_phi = gm.t() @ f["x_scaled"]
    inv = f["inv_rms"].unsqueeze(-1)
    xflat = xw.reshape(T, HC_D)
    dot = (xflat * gxs).sum(dim=-1, keepdim=True)
    gx_rms = inv * gxs - (inv ** 3 / HC_D) * dot * xflat
    gx = gx_rms.reshape(T, N, D) + gy.unsqueeze(1) * f["pre"].unsqueeze(-1)
    return (gx.to(x.dtype).reshape(x.shape), grad_phi.reshape(phi.shape), ga, gb)


# --------------------------------------------------------------------------
# Backward of the pre operator from the tensors its forward saved: the same
# inputs the reference fast path's backward takes
# (``src/mhc_pre_clamp_sinkhorn_backward.py:1292-1313``).
# --------------------------------------------------------------------------
def pre_bwd_from_saved(x, phi, alpha, base, inv_rms, mixes, pre, grad_y,
                       grad_post_out, grad_comb_frag, hc_eps=1e-6,
                       clamp_min=0.0, clamp_max=0.0, iter_times=20,
                       dtype=torch.float32):
    xf, _ = _flat_pre(x)
    T, N, D = xf.shape
    HC_D = N * D
    xw = _widen(xf, dtype)
    gy = _widen(grad_y, dtype).reshape(T, D)
    mixes = _widen(mixes, dtype)
    grad_pre = torch.einsum("td,tnd->tn", gy, xw)
    gm, ga, gb = small_bwd(mixes, _widen(alpha, dtype), _widen(base, dtype), N,
                           hc_eps, clamp_min, clamp_max, iter_times, grad_pre,
                           _widen(grad_post_out, dtype).reshape(T, N),
                           _widen(grad_comb_frag, dtype).reshape(T, N, N))
    inv = _widen(inv_rms, dtype).reshape(T, 1)
    xflat = xw.reshape(T, HC_D)
    gxs = gm @ _widen(phi, dtype)
    grad_phi = gm.t() @ (xflat * inv)
    dot = (xflat * gxs).sum(dim=-1, keepdim=True)
    gx_rms = inv * gxs - (inv ** 3 / HC_D) * dot * xflat
    gx = gx_rms.reshape(T, N, D) + gy.unsqueeze(1) * _widen(pre, dtype).reshape(T, N, 1)
    return (gx.to(x.dtype).reshape(x.shape), grad_phi.reshape(phi.shape), ga, gb)
