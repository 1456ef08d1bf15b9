"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations (generated on the CPU, then moved)."""
import torch


def post_inputs(T, N, D, dtype, seed, device="cpu", sinkhorn_hres=True):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, N, D, generator=g).to(dtype)
    h_out = torch.randn(T, D, generator=g).to(dtype)
    if sinkhorn_hres:
        m = torch.randn(T, N, N, generator=g).exp()
        for _ in range(20):
            m = m / m.sum(-1, keepdim=True)
            m = m / m.sum(-2, keepdim=True)
        h_res = m
    else:
        h_res = torch.randn(T, N, N, generator=g)
    h_post = 2 * torch.sigmoid(torch.randn(T, N, generator=g))
    gy = torch.randn(T, N, D, generator=g).to(dtype)
    return [t.to(device) for t in (x, h_res, h_out, h_post, gy)]


def pre_inputs(T, N, D, dtype, seed, device="cpu", phi_std=None):
    g = torch.Generator().manual_seed(seed)
    hm, hc = N * (N + 2), N * D
    x = torch.randn(T, N, D, generator=g).to(dtype)
    phi = torch.randn(hm, hc, generator=g) * (phi_std if phi_std is not None else hc ** -0.5)
    alpha = torch.rand(3, generator=g) + 0.5
    base = torch.randn(hm, generator=g) * 0.1
    gy = torch.randn(T, D, generator=g).to(dtype)
    gpost = torch.randn(T, N, generator=g)
    gcomb = torch.randn(T, N, N, generator=g)
    return [t.to(device) for t in (x, phi, alpha, base, gy, gpost, gcomb)]
