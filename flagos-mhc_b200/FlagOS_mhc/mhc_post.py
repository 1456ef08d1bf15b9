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


class PreMix:
    """Mix partials of the NEXT layer's pre operator, produced by ``mhc_post(...,
    next_phi=phi)`` in the same pass that wrote ``out``: per token and K range, the raw
    x.phi^T and sum(x^2) of out.  ``mhc_pre_clamp_sinkhorn(out, phi, ..., premix=pm)``
    then skips its own read of out for the mix.  It carries no gradient (the pre
    backward recomputes everything from x and phi); it is used only if x and phi are
    the same, unmodified tensors it was made from, and ignored otherwise."""

    def __init__(self, part, layers, out, phi):
        self.part, self.layers = part, int(layers)
        self._key = (out.data_ptr(), out._version, tuple(out.shape), phi.data_ptr(),
                     phi._version, tuple(phi.shape))

    def matches(self, x, phi):
        return self._key == (x.data_ptr(), x._version, tuple(x.shape), phi.data_ptr(),
                             phi._version, tuple(phi.shape))


def _post_mix(x, h_res, h_out, h_post, next_phi):
    """The layer-fused forward (N=4, bf16/fp16, packed tensors) or None if not eligible."""
    if x.dim() not in (3, 4) or not (x.is_cuda and h_out.is_cuda and next_phi.is_cuda):
        return None
    N, D = x.shape[-2], x.shape[-1]
    T = x.numel() // (N * D) if N * D else 0
    L = _C.lib()
    if (T == 0 or x.dtype not in (torch.bfloat16, torch.float16) or h_out.dtype != x.dtype
            or not x.is_contiguous() or not h_out.is_contiguous()
            or tuple(next_phi.shape) != (N * (N + 2), N * D)
            or not L.mhc_post_fwd_mix_supported(T, N, D, _C.dtype_code(x.dtype))):
        return None
    code = _C.dtype_code(x.dtype)
    hr = h_res.reshape(T, N, N).float().contiguous()
    hp = h_post.reshape(T, N).float().contiguous()
    phi = next_phi.float().contiguous()
    layers = L.mhc_post_fwd_mix_layers(T, N, D, code)
    out = torch.empty_like(x)
    part = torch.empty(layers, T, N * (N + 2) + 1, dtype=torch.float32, device=x.device)
    with torch.cuda.device(x.device):
        ws_bytes = L.mhc_post_fwd_mix_workspace_bytes(T, N, D, code)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
        st = L.mhc_post_fwd_mix(_C.ptr(x), _C.ptr(hr), _C.ptr(h_out), _C.ptr(hp), _C.ptr(out),
                                T, N, D, code, _C.ptr(phi), _C.ptr(part), _C.ptr(ws), ws_bytes,
                                _C.stream_of(x))
    _C.check(st, "mhc_post")
    return out, PreMix(part, layers, out, next_phi)


def mhc_post(x, h_res, h_out, h_post, next_phi=None):
    """out[t,i,:] = sum_j h_res[t,j,i] x[t,j,:] + h_post[t,i] h_out[t,:].

    Reference: ``mhc_post`` (src/mhc_post.py:296-341).  Accumulates in fp32,
    rounds once to x.dtype.  Supports N = 1..8 (the reference raises
    NotImplementedError for N != 4; here N > 8 does).

    ``next_phi`` (an addition to the reference API, optional): the phi of the next
    layer's pre operator, which will read ``out``.  Then the call returns
    ``(out, premix)``: the same ``out``, plus a :class:`PreMix` holding that layer's mix
    partials, computed from ``out`` while it was being written (one pass instead of two
    over the layer boundary).  ``premix`` is None where the fused kernel does not apply
    (N != 4, fp32, D % 64 != 0, non-packed tensors).
    """
    if next_phi is not None:
        fused = _post_mix(x, h_res, h_out, h_post, next_phi)
        if fused is not None:
            return fused
        return mhc_post(x, h_res, h_out, h_post), None
    if x.dim() not in (3, 4):
        raise ValueError(f"unsupported x.dim()={x.dim()}, expect 3 or 4")
    N, D = x.shape[-2], x.shape[-1]
    # token-strided x / h_out (a slice of a larger buffer, a regular (B,S) view) go to the
    # kernels as they are; anything else is packed first
    xs = _C.token_view(x, 2, N * D) if x.is_cuda else None
    hs = _C.token_view(h_out, 1, D) if h_out.is_cuda else None
    if xs is not None and hs is not None and h_out.dtype == x.dtype and 1 <= N <= 8:
        T = x.numel() // (N * D)
        hr = h_res.reshape(T, N, N).float().contiguous()
        hp = h_post.reshape(T, N).float().contiguous()
        _C.require_cuda(hr, hp)
        out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
        with torch.cuda.device(x.device):
            st = _C.lib().mhc_post_fwd_strided(_C.ptr(x), xs, _C.ptr(hr), _C.ptr(h_out), hs,
                                               _C.ptr(hp), _C.ptr(out), T, N, D,
                                               _C.dtype_code(x.dtype), _C.stream_of(x))
        _C.check(st, "mhc_post")
        return out
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
