"""Child process of tests/test_gpu_peer.py: one rank of a torchrun job on its own GPU.

Checks PeerGradReducer (the fused NVLink gradient sum) against the same sum formed
in rank order on the device from all ranks' vectors (bitwise), against NCCL's
all-reduce (within fp32 rounding), over several calls in a row and several sizes,
and through replays of a CUDA graph that captured one call, and prints PEER_OK on rank 0 when every check passed."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [ROOT, os.path.join(ROOT, "flagos-mhc_b200")]

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from FlagOS_mhc import _C  # noqa: E402
from FlagOS_mhc.distributed import PeerGradReducer  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", device_id=dev)
    for n in (1, 5, 4099, 24 * 28672 + 27):
        red = PeerGradReducer(n, dev)
        for call in range(4):
            g = torch.Generator(device=dev).manual_seed(1000 * call + 17 * n)
            allv = torch.randn(world, n, generator=g, device=dev) * (1 + call)
            mine = allv[rank].clone()
            want = allv[0].clone()
            for p in range(1, world):
                want += allv[p]
            got = red.reduce_(mine)
            nccl = allv[rank].clone()
            dist.all_reduce(nccl)
            torch.cuda.synchronize()
            assert torch.equal(got, want), (n, call, (got - want).abs().max().item())
            err = (got - nccl).abs().max().item() / nccl.abs().max().item()
            assert err < 1e-6, (n, call, err)
        st = _C.lib().mhc_device_status()
        assert st == 0, st
        red.close()
    # the packed (grad_phi, grad_alpha, grad_base) views go through in place
    phi = torch.empty(24 * 64 + 27, device=dev)
    phi.copy_(torch.arange(phi.numel(), device=dev, dtype=torch.float32) * (rank + 1))
    views = (phi[:24 * 64].view(24, 64), phi[24 * 64:24 * 64 + 3], phi[24 * 64 + 3:])
    red = PeerGradReducer(phi.numel(), dev)
    red(*views)
    torch.cuda.synchronize()
    k = world * (world + 1) / 2
    assert torch.equal(phi, torch.arange(phi.numel(), device=dev, dtype=torch.float32) * k)
    red.close()
    # captured once in a CUDA graph, replayed with new inputs: the device-kept epoch
    # advances on every replay, so each one is a fresh, correct sum
    n = 4099
    red = PeerGradReducer(n, dev)
    buf = torch.zeros(n, device=dev)
    red.reduce_(buf)                          # one eager call first (epoch 1)
    torch.cuda.synchronize()
    s = torch.cuda.Stream(dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph, stream=s):
            red.reduce_(buf)
    torch.cuda.synchronize()
    for rep in range(3):
        g = torch.Generator(device=dev).manual_seed(77 + rep)
        allv = torch.randn(world, n, generator=g, device=dev)
        buf.copy_(allv[rank])
        want = allv[0].clone()
        for p in range(1, world):
            want += allv[p]
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(buf, want), (rep, (buf - want).abs().max().item())
    assert _C.lib().mhc_device_status() == 0
    del graph
    red.close()
    dist.barrier()
    if rank == 0:
        print("PEER_OK", flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
