"""Token-sharded data parallelism for the mHC operators.

Every operator is independent per token, so a job splits the T tokens into
contiguous ranges, one per rank, and runs the operators locally with a
replicated (phi, alpha, base).  The only exchange is the sum of the parameter
gradients of the pre operator: ``mhc_pre_clamp_sinkhorn_backward`` returns
grad_phi, grad_alpha and grad_base as views of one contiguous fp32 buffer, so
one all-reduce (NCCL over NVLink on B200) covers all three.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def token_range(T: int, rank: int, world: int):
    """[start, stop) of the tokens rank `rank` owns (contiguous, sizes differ by <= 1)."""
    base, rem = divmod(T, world)
    start = rank * base + min(rank, rem)
    return start, start + base + (1 if rank < rem else 0)


def shard_tokens(t: torch.Tensor, rank: int, world: int, token_dims: int = 1):
    """Slice this rank's tokens out of a (T, ...) tensor (or (B, S, ...) with token_dims=2)."""
    if token_dims == 2:
        t = t.reshape(t.shape[0] * t.shape[1], *t.shape[2:])
    a, b = token_range(t.shape[0], rank, world)
    return t[a:b]


def packed_buffer(grad_phi, grad_alpha, grad_base):
    """The single 1-D fp32 buffer under the three gradients, or None if they are
    not adjacent views of one storage."""
    n = grad_phi.numel() + grad_alpha.numel() + grad_base.numel()
    ok = (grad_phi.is_contiguous() and grad_alpha.is_contiguous() and grad_base.is_contiguous()
          and grad_phi.dtype == grad_alpha.dtype == grad_base.dtype == torch.float32
          and grad_phi.untyped_storage().data_ptr() == grad_base.untyped_storage().data_ptr()
          and grad_alpha.data_ptr() == grad_phi.data_ptr() + 4 * grad_phi.numel()
          and grad_base.data_ptr() == grad_alpha.data_ptr() + 4 * grad_alpha.numel())
    if not ok:
        return None
    return torch.as_strided(grad_phi, (n,), (1,))


def allreduce_pre_grads(grad_phi, grad_alpha, grad_base, group=None, average=False):
    """Sum (or average) the three parameter gradients over `group` with one
    collective, in place.  Falls back to pack / all-reduce / unpack when the
    tensors do not share one buffer."""
    buf = packed_buffer(grad_phi, grad_alpha, grad_base)
    copy_back = buf is None
    if copy_back:
        buf = torch.cat([grad_phi.reshape(-1), grad_alpha.reshape(-1), grad_base.reshape(-1)])
    dist.all_reduce(buf, op=dist.ReduceOp.SUM, group=group)
    if average:
        buf.div_(dist.get_world_size(group))
    if copy_back:
        n0, n1 = grad_phi.numel(), grad_alpha.numel()
        grad_phi.copy_(buf[:n0].view_as(grad_phi))
        grad_alpha.copy_(buf[n0:n0 + n1].view_as(grad_alpha))
        grad_base.copy_(buf[n0 + n1:].view_as(grad_base))
    return grad_phi, grad_alpha, grad_base
