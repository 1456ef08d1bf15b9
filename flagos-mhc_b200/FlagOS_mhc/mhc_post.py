"""mhc_post forward on B200, and its pure-PyTorch definition ``mhc_post_ref``.

Drop-in for ``src/mhc_post.py`` of liuhycs/FlagOS-mhc: same signature, same
shape handling ((B,S,N,D) or (T,N,D)), same output dtype.  The device work is
one CUDA kernel behind ``mhc_post_fwd`` of the C ABI.
"""
from __future__ import annotations

import torch

from . import _C


def _flatten_bsn(x, h_res, h_out, h_post):
    """(B,S,N,D)/(T,N,D) -> contiguous (T,N,D) views; src/mhc_post.py:274-292."""
    if x.dim() == 4:
        B, S, N, D = x.shape
        T = B * S
    elif x.dim() == 3:
        T, N, D = x.shape
    else:
        raise ValueError(f"unsupported x.dim()={x.dim()}, expect 3 or 4")
    return (x.reshape(T, N, D).contiguous(), h_res.reshape(T, N, N).contiguous(),
            h_out.reshape(T, D).contiguous(), h_post.reshape(T, N).contiguous(), T, N, D)


def mhc_post(x, h_res, h_out, h_post):
    """out[t,i,:] = sum_j h_res[t,j,i] x[t,j,:] + h_post[t,i] h_out[t,:].

    Reference: ``mhc_post`` (src/mhc_post.py:296-341).  Accumulates in fp32,
    rounds once to x.dtype.  Supports N = 1..8 (the reference raises
    NotImplementedError for N != 4; here N > 8 does).
    """
    xf, hr, ho, hp, T, N, D = _flatten_bsn(x, h_res, h_out, h_post)
    _C.require_cuda(xf, hr, ho, hp)
    if not 1 <= N <= 8:
        raise NotImplementedError(f"mhc_post: hcMult N={N} not supported (1..8)")
    out_dtype = x.dtype
    # mixed storage dtypes: widen to fp32 so no input is rounded before the math
    if ho.dtype != xf.dtype:
        xf, ho = xf.float(), ho.float()
    hr, hp = hr.float(), hp.float()
    out = torch.empty_like(xf)
    with torch.cuda.device(xf.device):
        st = _C.lib().mhc_post_fwd(_C.ptr(xf), _C.ptr(hr), _C.ptr(ho), _C.ptr(hp), _C.ptr(out),
                                   T, N, D, _C.dtype_code(xf.dtype), _C.stream_of(xf))
    _C.check(st, "mhc_post")
    return out.to(out_dtype).reshape(x.shape)


def mhc_post_ref(x, h_res, h_out, h_post):
    """Pure-PyTorch definition of mhc_post (the reference's ``mhc_post_ref``,
    src/mhc_post.py:344-352), kept for API compatibility; any device."""
    orig_dtype = x.dtype
    xf, hr, ho, hp, T, N, D = _flatten_bsn(x, h_res, h_out, h_post)
    mix = torch.einsum("tji,tjd->tid", hr, xf.float())
    y = (mix + hp.unsqueeze(-1) * ho.float().unsqueeze(1)).to(orig_dtype)
    return y.reshape(x.shape)
