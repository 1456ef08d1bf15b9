"""mhc_post backward on B200, and ``mhc_post_backward_ref``.

Drop-in for ``src/mhc_post_backward.py``: one fused CUDA kernel
(``mhc_post_bwd`` of the C ABI) computes all four VJPs in one pass over grad_y.
"""
from __future__ import annotations

import torch

from . import _C


def _flatten(grad_y, x, h_res, h_out, h_post):
    """src/mhc_post_backward.py:564-590."""
    if grad_y.dim() == 4:
        B, S, N, D = grad_y.shape
        T = B * S
        shape4, shape_out = (B, S, N, D), (B, S, D)
    elif grad_y.dim() == 3:
        T, N, D = grad_y.shape
        shape4, shape_out = (T, N, D), (T, D)
    else:
        raise ValueError(f"unsupported grad_y.dim()={grad_y.dim()}")
    return (grad_y.reshape(T, N, D).contiguous(), x.reshape(T, N, D).contiguous(),
            h_res.reshape(T, N, N).contiguous(), h_out.reshape(T, D).contiguous(),
            h_post.reshape(T, N).contiguous(), shape4, shape_out, T, N, D)


def mhc_post_backward(grad_y, x, h_res, h_out, h_post):
    """Returns (grad_x, grad_h_res, grad_h_out, grad_h_post).

    Reference: ``mhc_post_backward`` (src/mhc_post_backward.py:593-621).
    grad_x has x's shape and dtype; grad_h_res / grad_h_out / grad_h_post have
    the shapes and dtypes of h_res / h_out / h_post (``torch.empty_like`` in
    the reference, :599-602).
    """
    if grad_y.dim() in (3, 4) and grad_y.is_cuda and x.is_cuda and h_out.is_cuda:
        N, D = grad_y.shape[-2], grad_y.shape[-1]
        gs = _C.token_view(grad_y, 2, N * D)
        xs = _C.token_view(x, 2, N * D)
        hs = _C.token_view(h_out, 1, D)
        if (gs is not None and xs is not None and hs is not None and 1 <= N <= 8
                and grad_y.dtype == x.dtype == h_out.dtype and x.shape == grad_y.shape):
            T = grad_y.numel() // (N * D)
            hr32 = h_res.reshape(T, N, N).float().contiguous()
            hp32 = h_post.reshape(T, N).float().contiguous()
            _C.require_cuda(hr32, hp32)
            lead = grad_y.shape[:-2]
            grad_x = torch.empty(grad_y.shape, dtype=x.dtype, device=x.device)
            grad_hout = torch.empty(lead + (D,), dtype=h_out.dtype, device=x.device)
            grad_hres = torch.empty(T, N, N, dtype=torch.float32, device=x.device)
            grad_hpost = torch.empty(T, N, dtype=torch.float32, device=x.device)
            with torch.cuda.device(x.device):
                st = _C.lib().mhc_post_bwd_strided(
                    _C.ptr(grad_y), gs, _C.ptr(x), xs, _C.ptr(hr32), _C.ptr(h_out), hs,
                    _C.ptr(hp32), _C.ptr(grad_x), _C.ptr(grad_hres), _C.ptr(grad_hout),
                    _C.ptr(grad_hpost), T, N, D, _C.dtype_code(x.dtype), _C.stream_of(x))
            _C.check(st, "mhc_post_backward")
            return (grad_x, grad_hres.to(h_res.dtype).reshape(h_res.shape), grad_hout,
                    grad_hpost.to(h_post.dtype).reshape(h_post.shape))
    gy, xf, hr, ho, hp, shape4, shape_out, T, N, D = _flatten(grad_y, x, h_res, h_out, h_post)
    _C.require_cuda(gy, xf, hr, ho, hp)
    if not 1 <= N <= 8:
        raise NotImplementedError(f"mhc_post_backward: hcMult N={N} not supported (1..8)")
    gx_dtype, gho_dtype = x.dtype, h_out.dtype
    if not (gy.dtype == xf.dtype == ho.dtype):
        gy, xf, ho = gy.float(), xf.float(), ho.float()
    hr32, hp32 = hr.float(), hp.float()
    grad_x = torch.empty_like(xf)
    grad_hout = torch.empty_like(ho)
    grad_hres = torch.empty(T, N, N, dtype=torch.float32, device=xf.device)
    grad_hpost = torch.empty(T, N, dtype=torch.float32, device=xf.device)
    with torch.cuda.device(xf.device):
        st = _C.lib().mhc_post_bwd(_C.ptr(gy), _C.ptr(xf), _C.ptr(hr32), _C.ptr(ho),
                                   _C.ptr(hp32), _C.ptr(grad_x), _C.ptr(grad_hres),
                                   _C.ptr(grad_hout), _C.ptr(grad_hpost), T, N, D,
                                   _C.dtype_code(xf.dtype), _C.stream_of(xf))
    _C.check(st, "mhc_post_backward")
    return (grad_x.to(gx_dtype).reshape(shape4),
            grad_hres.to(h_res.dtype).reshape(h_res.shape),
            grad_hout.to(gho_dtype).reshape(shape_out),
            grad_hpost.to(h_post.dtype).reshape(h_post.shape))


def mhc_post_backward_ref(grad_y, x, h_res, h_out, h_post):
    """Pure-PyTorch VJPs (the reference's ``mhc_post_backward_ref``,
    src/mhc_post_backward.py:624-643); any device."""
    orig_dtype = x.dtype
    gy, xf, hr, ho, hp, shape4, shape_out, T, N, D = _flatten(grad_y, x, h_res, h_out, h_post)
    gy_f, x_f, ho_f = gy.float(), xf.float(), ho.float()
    grad_x = torch.einsum("tji,tid->tjd", hr, gy_f).to(orig_dtype)
    grad_hres = torch.einsum("tjd,tid->tji", x_f, gy_f)
    grad_hout = torch.einsum("ti,tid->td", hp, gy_f).to(orig_dtype)
    grad_hpost = torch.einsum("td,tid->ti", ho_f, gy_f)
    return (grad_x.reshape(shape4), grad_hres.reshape(h_res.shape),
            grad_hout.reshape(shape_out), grad_hpost.reshape(h_post.shape))
