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


class PeerGradReducer:
    """Sum of the packed parameter gradients over the ranks of a one-node job in ONE
    kernel over NVLink peer memory (``mhc_grad_sum_peers`` of the C ABI), in place of
    the NCCL all-reduce of :func:`allreduce_pre_grads`.

    Construction is collective: every rank of `group` allocates its peer region,
    the CUDA IPC handles are exchanged with ``all_gather_object`` and each rank maps
    the others' regions.  Calls must then be made by every rank in the same order
    (each rank's epoch counter, kept in device memory, advances once per call, so a
    call can be captured in a CUDA graph and replayed).  A wait that runs
    past `timeout_s` makes the kernel return early with MHC_ERR_TIMEOUT recorded
    (``_C.lib().mhc_device_status()``); the reducer is then unusable.  The result
    is bitwise identical on every rank (rank-order sum)."""

    def __init__(self, n: int, device, group=None, timeout_s: float = 2.0):
        import ctypes

        from . import _C
        self.L = _C.lib()
        self.n = int(n)
        self.device = torch.device(device)
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if self.world > 8:
            raise ValueError("PeerGradReducer: at most 8 ranks (one node)")
        self.timeout_ns = int(timeout_s * 1e9)
        self._opened = []
        with torch.cuda.device(self.device):
            reg = ctypes.c_void_p()
            _C.check(self.L.mhc_peer_region_alloc(self.n, ctypes.byref(reg)), "PeerGradReducer")
            self.region = reg
            hb = self.L.mhc_peer_handle_bytes()
            buf = ctypes.create_string_buffer(hb)
            _C.check(self.L.mhc_peer_handle(reg, buf), "PeerGradReducer")
            handles = [None] * self.world
            dist.all_gather_object(handles, buf.raw, group=group)
            ptrs = (ctypes.c_void_p * 8)()
            for p, h in enumerate(handles):
                if p == self.rank:
                    ptrs[p] = reg.value
                    continue
                q = ctypes.c_void_p()
                _C.check(self.L.mhc_peer_open(ctypes.create_string_buffer(h, hb), ctypes.byref(q)),
                         "PeerGradReducer")
                self._opened.append(q)
                ptrs[p] = q.value
            self.ptrs = ptrs
        dist.barrier(group=group)

    def reduce_(self, buf: torch.Tensor):
        """In-place sum over the ranks of a contiguous fp32 CUDA vector of n floats."""
        from . import _C
        assert buf.dtype == torch.float32 and buf.is_contiguous() and buf.numel() == self.n
        # epoch 0: the kernel takes the call's epoch from the region's device counter
        st = self.L.mhc_grad_sum_peers(_C.ptr(buf), _C.ptr(buf), self.n, self.ptrs, self.rank,
                                       self.world, 0, self.timeout_ns, _C.stream_of(buf))
        _C.check(st, "PeerGradReducer")
        return buf

    def __call__(self, grad_phi, grad_alpha, grad_base):
        buf = packed_buffer(grad_phi, grad_alpha, grad_base)
        if buf is not None:
            self.reduce_(buf)
            return grad_phi, grad_alpha, grad_base
        buf = torch.cat([grad_phi.reshape(-1), grad_alpha.reshape(-1), grad_base.reshape(-1)])
        self.reduce_(buf)
        n0, n1 = grad_phi.numel(), grad_alpha.numel()
        grad_phi.copy_(buf[:n0].view_as(grad_phi))
        grad_alpha.copy_(buf[n0:n0 + n1].view_as(grad_alpha))
        grad_base.copy_(buf[n0 + n1:].view_as(grad_base))
        return grad_phi, grad_alpha, grad_base

    def close(self):
        """Collective: unmap the peers' regions, wait for every rank, free ours."""
        torch.cuda.synchronize(self.device)
        with torch.cuda.device(self.device):
            for q in self._opened:
                self.L.mhc_peer_close(q)
            self._opened = []
            dist.barrier(group=self.group)
            if self.region is not None:
                self.L.mhc_peer_region_free(self.region)
                self.region = None
