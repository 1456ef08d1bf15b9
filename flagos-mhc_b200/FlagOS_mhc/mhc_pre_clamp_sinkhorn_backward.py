"""mhc_pre_clamp_sinkhorn backward on B200, and its autograd definition
``mhc_pre_clamp_sinkhorn_backward_ref``.

Drop-in for ``src/mhc_pre_clamp_sinkhorn_backward.py``: same 17 arguments, same
4-tuple.  The device work runs behind ``mhc_pre_bwd`` of the C ABI.
``grad_phi``, ``grad_alpha`` and ``grad_base`` are returned as views of ONE
contiguous fp32 buffer, so a data-parallel job sums all three with a single
collective (see :mod:`FlagOS_mhc.distributed`).
"""
from __future__ import annotations

import torch

from . import _C
from .mhc_pre_clamp_sinkhorn import _check_params


def mhc_pre_clamp_sinkhorn_backward(x, phi, alpha, base, inv_rms, x_scaled, mixes, h_res_logits,
                                    pre, grad_y, grad_post_out, grad_comb_frag, norm_eps=1e-6,
                                    hc_eps=1e-6, clamp_min=0.0, clamp_max=0.0, iter_times=20,
                                    grad_x_accumulate=None):
    """Returns (grad_x, grad_phi, grad_alpha, grad_base).

    Reference: ``mhc_pre_clamp_sinkhorn_backward``
    (src/mhc_pre_clamp_sinkhorn_backward.py:1292-1391).  ``x_scaled`` and
    ``h_res_logits`` are accepted for signature compatibility and not read
    (the reference does not read ``h_res_logits`` either, :1301): the kernels
    use ``grad_phi = (inv_rms*grad_mixes)^T x``, which needs no fp32 copy of x.

    ``grad_x_accumulate`` (an addition to the reference API, optional): a tensor of x's
    shape whose values are added to grad_x inside the kernel (fp32 sum, rounded once).
    A layer whose x also feeds ``mhc_post`` passes the post backward's grad_x here
    instead of letting autograd add the two gradients in a separate pass.
    """
    if x.dim() == 4:
        B, S, N, D = x.shape
        T = B * S
    elif x.dim() == 3:
        T, N, D = x.shape
    else:
        raise ValueError(f"unsupported x.dim()={x.dim()}")
    if grad_y.dim() == 3:
        assert grad_y.shape[0] * grad_y.shape[1] == T and grad_y.shape[2] == D
    elif grad_y.dim() == 2:
        assert tuple(grad_y.shape) == (T, D)
    else:
        raise ValueError(f"unsupported grad_y.dim()={grad_y.dim()}")
    hc_mix, hc_d = _check_params(N, D, phi, alpha, base)
    # token-strided x / grad_y (slices of larger buffers, regular (B,S) views) are read in
    # place, as the reference's kernels read them through x.stride(1) / grad_y.stride(1)
    xts = _C.token_view(x, 2, N * D) if x.is_cuda else None
    gts = _C.token_view(grad_y, 1, D) if grad_y.is_cuda else None
    if xts is not None and gts is not None and grad_y.dtype == x.dtype:
        xf, gy = x, grad_y
    else:
        xf = x.reshape(T, N, D).contiguous()
        gy = grad_y.reshape(T, D).contiguous()
        xts, gts = N * D, D
    _C.require_cuda(xf, gy, phi, alpha, base, inv_rms, mixes, pre, grad_post_out, grad_comb_frag)
    dev = xf.device
    gx_dtype = x.dtype
    if gy.dtype != xf.dtype:
        xf, gy = xf.reshape(T, N, D).float(), gy.reshape(T, D).float()
        xts, gts = N * D, D
    f = lambda t: t.to(torch.float32).contiguous()  # noqa: E731
    phi_f, alpha_f, base_f = f(phi), f(alpha), f(base)
    inv_f, mixes_f, pre_f = f(inv_rms.reshape(T)), f(mixes.reshape(T, hc_mix)), f(pre.reshape(T, N))
    gpost_f, gcomb_f = f(grad_post_out.reshape(T, N)), f(grad_comb_frag.reshape(T, N, N))
    grad_x = torch.empty(T, N, D, dtype=xf.dtype, device=dev)
    acc = None
    if grad_x_accumulate is not None:
        assert grad_x_accumulate.numel() == T * N * D, "grad_x_accumulate must have x's shape"
        acc = grad_x_accumulate.reshape(T, N, D).to(xf.dtype).contiguous()
        _C.require_cuda(acc)
    n_phi = hc_mix * hc_d
    packed = torch.empty(n_phi + 3 + hc_mix, dtype=torch.float32, device=dev)
    grad_phi = packed[:n_phi].view(hc_mix, hc_d)
    grad_alpha = packed[n_phi:n_phi + 3]
    grad_base = packed[n_phi + 3:]
    L = _C.lib()
    code = _C.dtype_code(xf.dtype)
    with torch.cuda.device(dev):
        ws_bytes = L.mhc_pre_bwd_workspace_bytes(T, N, D, code, int(iter_times))
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
        st = L.mhc_pre_bwd_strided(
            _C.ptr(xf), xts, _C.ptr(phi_f), _C.ptr(alpha_f), _C.ptr(base_f), _C.ptr(inv_f),
            _C.ptr(mixes_f), _C.ptr(pre_f), _C.ptr(gy), gts, _C.ptr(gpost_f), _C.ptr(gcomb_f),
            T, N, D, code, float(norm_eps), float(hc_eps), float(clamp_min), float(clamp_max),
            int(iter_times), _C.ptr(acc), _C.ptr(grad_x), _C.ptr(grad_phi), _C.ptr(grad_alpha),
            _C.ptr(grad_base), _C.ptr(ws), ws_bytes, _C.stream_of(xf))
    _C.check(st, "mhc_pre_clamp_sinkhorn_backward")
    return (grad_x.to(gx_dtype).view(x.shape), grad_phi.view(phi.shape), grad_alpha, grad_base)


def mhc_pre_clamp_sinkhorn_backward_ref(x, phi, alpha, base, grad_y, grad_post_out,
                                        grad_comb_frag, norm_eps=1e-6, hc_eps=1e-6,
                                        clamp_min=0.0, clamp_max=0.0, iter_times=20):
    """Autograd through the fp32 forward (the reference's
    ``mhc_pre_clamp_sinkhorn_backward_ref``,
    src/mhc_pre_clamp_sinkhorn_backward.py:1397-1453); any device."""
    from .mhc_pre_clamp_sinkhorn import mhc_pre_clamp_sinkhorn_ref
    orig_dtype = x.dtype
    with torch.enable_grad():
        x_ = x.detach().to(torch.float32).requires_grad_(True)
        phi_ = phi.detach().to(torch.float32).requires_grad_(True)
        alpha_ = alpha.detach().to(torch.float32).requires_grad_(True)
        base_ = base.detach().to(torch.float32).requires_grad_(True)
        out = mhc_pre_clamp_sinkhorn_ref(x_, phi_, alpha_, base_, norm_eps, hc_eps, clamp_min,
                                         clamp_max, iter_times)
        T = out["post_out"].shape[0]
        D = x.shape[-1]
        # y is recomputed in fp32 (the _ref forward rounds it to x.dtype)
        xf = x_.reshape(T, -1, D)
        y = (xf * out["pre"].unsqueeze(-1)).sum(dim=-2)
        loss = (y * grad_y.to(torch.float32).reshape(T, D)).sum() \
            + (out["post_out"] * grad_post_out).sum() + (out["comb_frag"] * grad_comb_frag).sum()
        dx, dphi, da, db = torch.autograd.grad(loss, (x_, phi_, alpha_, base_))
    return dx.to(orig_dtype), dphi, da, db
