"""Token-sharded data parallelism on CPU ranks (gloo, world size 2 and 3):
shard the tokens, run the pre backward per rank (the CPU oracle stands in for
the device kernels), sum the parameter gradients with the package's one-shot
all-reduce, and compare with the single-process full-batch result."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, result_q):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "flagos-mhc_b200")]
    from FlagOS_mhc.distributed import allreduce_pre_grads, shard_tokens, packed_buffer
    from oracle import mhc_oracle as O
    from tests.gen import pre_inputs
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        T, N, D = 23, 4, 16
        x, phi, alpha, base, gy, gpost, gcomb = pre_inputs(T, N, D, torch.float32, seed=5)
        kw = dict(norm_eps=1e-6, hc_eps=1e-6, clamp_min=-2.0, clamp_max=2.0, iter_times=7)
        xs, gys, gps, gcs = (shard_tokens(t, rank, world) for t in (x, gy, gpost, gcomb))
        gx, gphi, ga, gb = O.pre_bwd(xs, phi, alpha, base, gys, gps, gcs, dtype=torch.float64,
                                     **kw)
        # pack the three like mhc_pre_clamp_sinkhorn_backward returns them
        n0 = gphi.numel()
        buf = torch.cat([gphi.reshape(-1), ga, gb])
        gphi_v, ga_v, gb_v = buf[:n0].view_as(gphi), buf[n0:n0 + 3], buf[n0 + 3:]
        assert packed_buffer(gphi_v, ga_v, gb_v) is not None or gphi_v.dtype != torch.float32
        allreduce_pre_grads(gphi_v, ga_v, gb_v)
        gxs = [torch.empty(0)] * world
        gathered = [None] * world
        dist.all_gather_object(gathered, gx)
        if rank == 0:
            # numpy arrays: pickled by value (torch tensors would travel as shared-memory
            # handles that vanish when this process exits)
            result_q.put(tuple(t.numpy().copy() for t in (torch.cat(gathered), gphi_v, ga_v, gb_v)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_token_sharded_backward_matches_full_batch(world):
    from oracle import mhc_oracle as O
    from tests.gen import pre_inputs
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = [torch.from_numpy(a) for a in q.get(timeout=120)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    T, N, D = 23, 4, 16
    x, phi, alpha, base, gy, gpost, gcomb = pre_inputs(T, N, D, torch.float32, seed=5)
    kw = dict(norm_eps=1e-6, hc_eps=1e-6, clamp_min=-2.0, clamp_max=2.0, iter_times=7)
    want = O.pre_bwd(x, phi, alpha, base, gy, gpost, gcomb, dtype=torch.float64, **kw)
    for a, b in zip(got, want):
        assert torch.allclose(a.double(), b.double(), rtol=1e-10, atol=1e-12)


def test_token_range_covers_all_tokens():
    from FlagOS_mhc.distributed import token_range
    for T in (0, 1, 7, 32768):
        for w in (1, 2, 3, 8):
            spans = [token_range(T, r, w) for r in range(w)]
            assert spans[0][0] == 0 and spans[-1][1] == T
            assert all(spans[i][1] == spans[i + 1][0] for i in range(w - 1))
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1


def test_packed_buffer_detects_views():
    from FlagOS_mhc.distributed import packed_buffer
    buf = torch.arange(10 + 3 + 4, dtype=torch.float32)
    v = (buf[:10].view(2, 5), buf[10:13], buf[13:])
    pb = packed_buffer(*v)
    assert pb is not None and pb.data_ptr() == buf.data_ptr() and pb.numel() == 17
    assert packed_buffer(torch.zeros(2, 5), torch.zeros(3), torch.zeros(4)) is None


def _failing_worker(rank, world, port, mode, result_q):
    """Rank 1 fails before the gradient sum (raises, or stalls past the process-group
    timeout); rank 0 must get an error from its collective, not hang."""
    import datetime
    import sys
    import time
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "flagos-mhc_b200")]
    from FlagOS_mhc.distributed import allreduce_pre_grads
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    # the group timeout also bounds the rendezvous, so it leaves room for a slow spawn
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=15))
    buf = torch.ones(24 * 16 + 27)
    views = (buf[:24 * 16].view(24, 16), buf[24 * 16:24 * 16 + 3], buf[24 * 16 + 3:])
    if rank == 1:
        if mode == "raise":
            os._exit(3)          # the rank dies between steps, with nothing in flight
        time.sleep(8)            # "never joins": stalls past the group timeout
        os._exit(0)
    t0 = time.time()
    try:
        allreduce_pre_grads(*views)
        result_q.put(("no error", time.time() - t0))
    except Exception as e:  # noqa: BLE001 -- any error from the collective is the point
        result_q.put((type(e).__name__, time.time() - t0))
    # flush the queue's feeder thread before the hard exit (os._exit skips it)
    result_q.close()
    result_q.join_thread()
    os._exit(0)


@pytest.mark.parametrize("mode", ["raise", "stall"])
def test_failed_rank_gives_error_not_hang(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_failing_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in procs:
        p.start()
    what, dt = q.get(timeout=60)
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert what != "no error"
    assert dt < 30
