"""mhc_pre_clamp_sinkhorn forward on B200, and ``mhc_pre_clamp_sinkhorn_ref``.

Drop-in for ``src/mhc_pre_clamp_sinkhorn.py``: same arguments, same dict of
outputs (plus the saved tensors when ``need_backward=True``).  The device work
runs behind ``mhc_pre_fwd`` of the C ABI.
"""
from __future__ import annotations

import torch

from . import _C


def _flatten(x):
    """(xf (T,N,D) contiguous, y shape); src/mhc_pre_clamp_sinkhorn.py:844-854."""
    if x.dim() == 4:
        B, S, N, D = x.shape
        return x.reshape(B * S, N, D).contiguous(), (B, S, D)
    if x.dim() == 3:
        T, N, D = x.shape
        return x.contiguous(), (T, D)
    raise ValueError(f"unsupported x.dim()={x.dim()}")


def _check_params(N, D, phi, alpha, base):
    hc_mix, hc_d = N * (N + 2), N * D
    # same checks as src/mhc_pre_clamp_sinkhorn.py:884-889 (N range widened to 1..8)
    if not 1 <= N <= 8:
        raise NotImplementedError(f"hcMult N={N} not supported (1..8)")
    assert tuple(phi.shape) == (hc_mix, hc_d), f"phi shape {tuple(phi.shape)} != {(hc_mix, hc_d)}"
    assert alpha.numel() == 3
    assert base.numel() == hc_mix
    return hc_mix, hc_d


def mhc_pre_clamp_sinkhorn(x, phi, alpha, base, norm_eps=1e-6, hc_eps=1e-6, clamp_min=0.0,
                           clamp_max=0.0, iter_times=20, need_backward=False,
                           materialize_x_scaled=True, premix=None):
    """Fused RMSNorm + x.phi^T + heads + clamp + softmax + Sinkhorn + y.

    Reference: ``mhc_pre_clamp_sinkhorn`` (src/mhc_pre_clamp_sinkhorn.py:857-971).
    Returns a dict with ``y`` ((B,S,D) or (T,D), x.dtype), ``post_out`` (T,N)
    and ``comb_frag`` (T,N,N); with ``need_backward=True`` also ``inv_rms``
    (T,), ``x_scaled`` (T,N*D), ``mixes`` (T,hcMix), ``h_res_logits`` (T,N,N,
    pre-clamp) and ``pre`` (T,N), all fp32.  The clamp is applied iff
    ``clamp_min != 0 or clamp_max != 0`` and the Sinkhorn runs ``iter_times``
    iterations in both modes.

    ``materialize_x_scaled=False`` (an addition to the reference API, opt-in) skips
    writing the fp32 ``x_scaled`` (4*N*D bytes per token, the largest output) and
    returns an empty tensor in its place; the backward of this package never reads it.

    ``premix`` (an addition to the reference API, optional): the :class:`PreMix` that
    ``mhc_post(..., next_phi=phi)`` returned along with this ``x``; the mix is then not
    recomputed from x.  Ignored unless it was made from this very x and phi.
    """
    if x.dim() not in (3, 4):
        raise ValueError(f"unsupported x.dim()={x.dim()}")
    # a token-strided x (slice of a larger buffer, regular (B,S) view) is read in place
    xts = _C.token_view(x, 2, x.shape[-2] * x.shape[-1]) if x.is_cuda else None
    if xts is not None:
        N, D = x.shape[-2], x.shape[-1]
        T = x.numel() // (N * D)
        xf = x
        y_shape = tuple(x.shape[:-2]) + (D,)
    else:
        xf, y_shape = _flatten(x)
        T, N, D = xf.shape
        xts = N * D
    hc_mix, hc_d = _check_params(N, D, phi, alpha, base)
    _C.require_cuda(xf, phi, alpha, base)
    dev = xf.device
    f32 = dict(dtype=torch.float32, device=dev)
    phi_f = phi.to(torch.float32).contiguous()
    alpha_f = alpha.to(torch.float32).contiguous()
    base_f = base.to(torch.float32).contiguous()
    y = torch.empty(T, D, dtype=xf.dtype, device=dev)
    post_out = torch.empty(T, N, **f32)
    comb_frag = torch.empty(T, N, N, **f32)
    inv_rms = torch.empty(T, **f32)
    mixes = torch.empty(T, hc_mix, **f32)
    pre = torch.empty(T, N, **f32)
    x_scaled = torch.empty(T, hc_d, **f32) if (need_backward and materialize_x_scaled) else None
    h_res_logits = torch.empty(T, N, N, **f32) if need_backward else None
    L = _C.lib()
    code = _C.dtype_code(xf.dtype)
    use_premix = (premix is not None and premix.matches(x, phi) and xts == N * D
                  and premix.part.shape[1] == T)
    with torch.cuda.device(dev):
        if use_premix:
            st = L.mhc_pre_fwd_premixed(
                _C.ptr(xf), _C.ptr(premix.part), premix.layers, _C.ptr(alpha_f), _C.ptr(base_f),
                T, N, D, code, float(norm_eps), float(hc_eps), float(clamp_min),
                float(clamp_max), int(iter_times), _C.ptr(y), _C.ptr(post_out),
                _C.ptr(comb_frag), _C.ptr(inv_rms), _C.ptr(x_scaled), _C.ptr(mixes),
                _C.ptr(h_res_logits), _C.ptr(pre), _C.stream_of(xf))
        else:
            ws_bytes = L.mhc_pre_fwd_workspace_bytes(T, N, D, code)
            ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
            st = L.mhc_pre_fwd_strided(
                _C.ptr(xf), xts, _C.ptr(phi_f), _C.ptr(alpha_f), _C.ptr(base_f), T, N, D, code,
                float(norm_eps), float(hc_eps), float(clamp_min), float(clamp_max),
                int(iter_times), _C.ptr(y), _C.ptr(post_out), _C.ptr(comb_frag),
                _C.ptr(inv_rms), _C.ptr(x_scaled), _C.ptr(mixes), _C.ptr(h_res_logits),
                _C.ptr(pre), _C.ptr(ws), ws_bytes, _C.stream_of(xf))
    _C.check(st, "mhc_pre_clamp_sinkhorn")
    result = {"y": y.reshape(y_shape), "post_out": post_out, "comb_frag": comb_frag}
    if need_backward:
        if x_scaled is None:
            x_scaled = torch.empty(0, hc_d, **f32)
        result.update(inv_rms=inv_rms, x_scaled=x_scaled, mixes=mixes,
                      h_res_logits=h_res_logits, pre=pre)
    return result


def mhc_pre_clamp_sinkhorn_ref(x, phi, alpha, base, norm_eps=1e-6, hc_eps=1e-6, clamp_min=0.0,
                               clamp_max=0.0, iter_times=20):
    """Pure-PyTorch definition (the reference's ``mhc_pre_clamp_sinkhorn_ref``,
    src/mhc_pre_clamp_sinkhorn.py:974-1022); any device."""
    orig_dtype = x.dtype
    xf, shape = _flatten(x)
    T, N, D = xf.shape
    x_flat = xf.reshape(T, N * D).float()
    inv = torch.rsqrt(x_flat.pow(2).mean(dim=-1, keepdim=True) + norm_eps)
    mixes = (x_flat * inv) @ phi.float().t()
    a, b = alpha.float(), base.float()
    pre = torch.sigmoid(mixes[:, :N] * a[0] + b[:N]) + hc_eps
    post_out = 2.0 * torch.sigmoid(mixes[:, N:2 * N] * a[1] + b[N:2 * N])
    logits = (mixes[:, 2 * N:] * a[2] + b[2 * N:]).reshape(T, N, N)
    lc = torch.clamp(logits, clamp_min, clamp_max) if (clamp_min != 0.0 or clamp_max != 0.0) \
        else logits
    M = (lc - lc.max(dim=-1, keepdim=True).values).exp()
    M = M / M.sum(dim=-1, keepdim=True) + hc_eps
    M = M / (M.sum(dim=-2, keepdim=True) + hc_eps)
    for _ in range(iter_times - 1):
        M = M / (M.sum(dim=-1, keepdim=True) + hc_eps)
        M = M / (M.sum(dim=-2, keepdim=True) + hc_eps)
    y = (xf.float() * pre.unsqueeze(-1)).sum(dim=-2).to(orig_dtype)
    return {"y": y.reshape(shape), "post_out": post_out, "comb_frag": M,
            "inv_rms": inv.squeeze(-1), "mixes": mixes, "h_res_logits": logits, "pre": pre}
