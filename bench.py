"""mHC fwd+bwd throughput on B200 (the north-star workload).

One step = the four mHC operators over one batch of T=32768 tokens, N=4,
D=7168, bf16 storage:
    mhc_pre_clamp_sinkhorn (need_backward=True)   config-3 inputs
    mhc_post                                       config-2 inputs
    mhc_post_backward
    mhc_pre_clamp_sinkhorn_backward
and, with N>1 GPUs, one NCCL all-reduce of the packed [grad_phi|grad_alpha|grad_base].
Each rank owns its own 32768 tokens (weak scaling: the per-GPU work is fixed).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line (rank 0).  `value` is whole-job tokens/s with the inputs
resident in HBM; `e2e` is the same metric through the public API with the
inputs copied from pinned host memory every step.  `--impl reference` times
the CPU oracle (the reference's pure-PyTorch algorithm restated) on this host.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "flagos-mhc_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

T_TOK, N_HC, D_HID = 32768, 4, 7168
METRIC = "mHC fwd+bwd tokens/s (T=32768,N=4,D=7168 bf16)"
WORKLOAD = "pre_clamp_sinkhorn fwd(need_backward)+bwd and post fwd+bwd, T=32768 N=4 D=7168 bf16"


# ----------------------------------------------------------------------------- helpers
def algorithmic_bytes(T, N, D, e=2, x_scaled=True):
    """Compulsory HBM bytes per op (each input read once, each output written once)."""
    HM, HC = N * (N + 2), N * D
    xs = HC * 4 if x_scaled else 0
    post_fwd = T * (2 * N * D * e + D * e + N * N * 4 + N * 4)
    post_bwd = T * (3 * N * D * e + 2 * D * e + 2 * (N * N * 4 + N * 4))
    pre_fwd = T * (N * D * e + D * e + N * 4 + N * N * 4 + 4 + xs + HM * 4 + N * N * 4
                   + N * 4) + HM * HC * 4
    pre_bwd = T * (2 * N * D * e + D * e + N * 4 + N * N * 4 + 4 + HM * 4 + N * 4) \
        + 2 * HM * HC * 4 + (3 + HM) * 4
    return {"pre_fwd": pre_fwd, "post_fwd": post_fwd, "post_bwd": post_bwd, "pre_bwd": pre_bwd}


def hbm_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def ncu_traffic():
    p = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(p) as f:
            return json.load(f)
    except Exception:
        return {}


class ClockSampler:
    """SM clocks and throttle reasons of this process's GPU, read through NVML by a
    thread every `period_s` (in-process, so every sample carries the host time at
    which it was taken).  `stop()` summarises the samples taken between
    mark_start() and mark_stop(); `load_window` also reports the samples since
    mark_load() (the untimed soak steps right before the timed region plus the
    region itself).  Reads only; changes no GPU setting."""
    # NVML clocks-event reason bits (nvml.h: nvmlClocksEventReason*)
    BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
            "hw_thermal_slowdown": 0x40}

    def __init__(self, dev_index, period_s=0.002):
        self.period = period_s
        self.rows = []           # (host time, sm MHz, max sm MHz, reasons bitmask)
        self.t_load = self.t0 = self.t1 = None
        self._stop = False
        self._th = None
        self.err = None
        try:
            import pynvml
            pynvml.nvmlInit()
            uuid = None
            try:
                uuid = str(torch.cuda.get_device_properties(dev_index).uuid)
            except Exception:
                pass
            h = None
            if uuid:
                for i in range(pynvml.nvmlDeviceGetCount()):
                    hi = pynvml.nvmlDeviceGetHandleByIndex(i)
                    u = pynvml.nvmlDeviceGetUUID(hi)
                    u = u.decode() if isinstance(u, bytes) else u
                    if uuid.lower() in u.lower():
                        h = hi
                        break
            self.h = h if h is not None else pynvml.nvmlDeviceGetHandleByIndex(dev_index)
            self.nv = pynvml
        except Exception as e:  # no NVML: the line says so
            self.nv = None
            self.err = repr(e)

    def _loop(self):
        nv, h = self.nv, self.h
        mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        while not self._stop:
            try:
                sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
                try:
                    rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
                except Exception:
                    rs = nv.nvmlDeviceGetCurrentClocksThrottleReasons(h)
                self.rows.append((time.perf_counter(), sm, mx, rs))
            except Exception as e:
                self.err = repr(e)
                return
            time.sleep(self.period)

    def start(self):
        import threading
        if self.nv is None:
            return
        self._th = threading.Thread(target=self._loop, daemon=True)
        self._th.start()

    def mark_load(self):
        self.t_load = time.perf_counter()

    def mark_start(self):
        self.t0 = time.perf_counter()

    def mark_stop(self):
        self.t1 = time.perf_counter()

    def _summ(self, rows):
        if not rows:
            return None
        reasons = sorted({n for r in rows for n, b in self.BITS.items() if r[3] & b})
        return {"sm_mhz": statistics.median(r[1] for r in rows),
                "sm_max_mhz": max(r[2] for r in rows), "reasons": reasons,
                "samples": len(rows)}

    def stop(self):
        if self.nv is None:
            return {"error": "NVML unavailable: " + str(self.err)}
        self._stop = True
        if self._th is not None:
            self._th.join(timeout=2)
        timed = [r for r in self.rows if self.t0 <= r[0] <= self.t1]
        load = [r for r in self.rows if (self.t_load or self.t0) <= r[0] <= self.t1]
        out = self._summ(timed) or self._summ(load) or {}
        out["window"] = "timed region" if timed else "soak + timed region"
        out["load_window"] = self._summ(load)
        out["period_ms"] = self.period * 1e3
        out["source"] = "NVML in-process sampler"
        return out


def make_inputs(T, N, D, seed, dev, param_seed=3):
    """Config-2 (post) and config-3 (pre) inputs, generated on the device from a seed.
    The per-token tensors use `seed` (each rank draws its own token shard); phi,
    alpha and base use `param_seed` on every rank (they are replicated parameters)."""
    bf = torch.bfloat16
    HM, HC = N * (N + 2), N * D
    inp = {}
    gp = torch.Generator(device=dev).manual_seed(param_seed)
    inp["phi"] = torch.randn(HM, HC, generator=gp, device=dev) / HC ** 0.5
    inp["alpha"] = torch.rand(3, generator=gp, device=dev) + 0.5
    inp["base"] = torch.randn(HM, generator=gp, device=dev) * 0.1
    g = torch.Generator(device=dev).manual_seed(seed)
    inp["x_pre"] = torch.randn(T, N, D, generator=g, device=dev).to(bf)
    inp["gy_pre"] = torch.randn(T, D, generator=g, device=dev).to(bf)
    inp["gpost"] = torch.randn(T, N, generator=g, device=dev)
    inp["gcomb"] = torch.randn(T, N, N, generator=g, device=dev)
    inp["x_post"] = torch.randn(T, N, D, generator=g, device=dev).to(bf)
    inp["h_out"] = torch.randn(T, D, generator=g, device=dev).to(bf)
    m = torch.randn(T, N, N, generator=g, device=dev).exp()
    for _ in range(20):
        m = m / m.sum(-1, keepdim=True)
        m = m / m.sum(-2, keepdim=True)
    inp["h_res"] = m
    inp["h_post"] = 2 * torch.sigmoid(torch.randn(T, N, generator=g, device=dev))
    inp["gy_post"] = torch.randn(T, N, D, generator=g, device=dev).to(bf)
    return inp


KW = dict(norm_eps=1e-6, hc_eps=1e-6, clamp_min=-10.0, clamp_max=10.0, iter_times=20)
# per-step inputs that come from the host in the end-to-end measurement
HOST_INPUTS = ["x_pre", "gy_pre", "gpost", "gcomb", "x_post", "h_out", "h_res", "h_post",
               "gy_post"]


def run_step(M, inp, world, ev=None, x_scaled=True, reducer=None):
    """The four operators (+ the cross-GPU gradient sum). Returns their results."""
    if ev is not None:
        ev[0].record()
    out = M.mhc_pre_clamp_sinkhorn(inp["x_pre"], inp["phi"], inp["alpha"], inp["base"],
                                   need_backward=True, materialize_x_scaled=x_scaled, **KW)
    if ev is not None:
        ev[1].record()
    y = M.mhc_post(inp["x_post"], inp["h_res"], inp["h_out"], inp["h_post"])
    if ev is not None:
        ev[2].record()
    pg = M.mhc_post_backward(inp["gy_post"], inp["x_post"], inp["h_res"], inp["h_out"],
                             inp["h_post"])
    if ev is not None:
        ev[3].record()
    grads = M.mhc_pre_clamp_sinkhorn_backward(
        inp["x_pre"], inp["phi"], inp["alpha"], inp["base"], out["inv_rms"], out["x_scaled"],
        out["mixes"], out["h_res_logits"], out["pre"], inp["gy_pre"], inp["gpost"],
        inp["gcomb"], **KW)
    if ev is not None:
        ev[4].record()
    if world > 1:
        if reducer is not None:
            reducer(grads[1], grads[2], grads[3])
        else:
            from FlagOS_mhc.distributed import allreduce_pre_grads
            allreduce_pre_grads(grads[1], grads[2], grads[3])
    if ev is not None:
        ev[5].record()
    return out, y, pg, grads


# ----------------------------------------------------------------------------- CPU legs
def _ref_inputs(T, N, D, seed=0):
    """CPU tensors of the benchmark workload's shapes and distributions (bf16 storage,
    fp32 parameters), for the `*_ref` timing."""
    g = torch.Generator().manual_seed(seed)
    HM, HC = N * (N + 2), N * D
    bf = torch.bfloat16
    d = {"x_pre": torch.randn(T, N, D, generator=g).to(bf),
         "phi": torch.randn(HM, HC, generator=g) / HC ** 0.5,
         "alpha": torch.rand(3, generator=g) + 0.5,
         "base": torch.randn(HM, generator=g) * 0.1,
         "gy_pre": torch.randn(T, D, generator=g).to(bf),
         "gpost": torch.randn(T, N, generator=g), "gcomb": torch.randn(T, N, N, generator=g),
         "x_post": torch.randn(T, N, D, generator=g).to(bf),
         "h_out": torch.randn(T, D, generator=g).to(bf),
         "h_res": torch.softmax(torch.randn(T, N, N, generator=g), -1),
         "h_post": 2 * torch.sigmoid(torch.randn(T, N, generator=g)),
         "gy_post": torch.randn(T, N, D, generator=g).to(bf)}
    return d


def _ref_step(M, d):
    """One step of the workload through the `*_ref` functions (the reference's
    pure-PyTorch path: src/mhc_pre_clamp_sinkhorn.py:974-1022,
    src/mhc_pre_clamp_sinkhorn_backward.py:1397-1453, src/mhc_post.py:344-352,
    src/mhc_post_backward.py:624-643, restated op for op in FlagOS_mhc)."""
    M.mhc_pre_clamp_sinkhorn_ref(d["x_pre"], d["phi"], d["alpha"], d["base"], **KW)
    M.mhc_post_ref(d["x_post"], d["h_res"], d["h_out"], d["h_post"])
    M.mhc_post_backward_ref(d["gy_post"], d["x_post"], d["h_res"], d["h_out"], d["h_post"])
    M.mhc_pre_clamp_sinkhorn_backward_ref(d["x_pre"], d["phi"], d["alpha"], d["base"],
                                          d["gy_pre"], d["gpost"], d["gcomb"], **KW)


def cpu_ref_rate(T_sample, steps=None, budget_s=None, warmup=0):
    """Tokens/s of the `*_ref` path on T_sample-token slices of the benchmark shapes,
    all host threads.  Runs `steps` steps, or repeats until `budget_s` has passed."""
    import FlagOS_mhc as M
    torch.set_num_threads(os.cpu_count())
    d = _ref_inputs(T_sample, N_HC, D_HID)
    with torch.no_grad():
        for _ in range(warmup):
            _ref_step(M, d)
        times = []
        t_all = time.perf_counter()
        while True:
            t0 = time.perf_counter()
            _ref_step(M, d)
            times.append(time.perf_counter() - t0)
            if steps is not None and len(times) >= steps:
                break
            if steps is None and time.perf_counter() - t_all >= budget_s:
                break
    return T_sample * len(times) / sum(times), times


def cpu_c0(steps=20, warmup=3):
    """Config C0 at its full shape: mhc_post_ref forward plus its backward by autograd,
    fp32 on the host, T=256 (B=2, S=128), N=4, D=1024, torch seed 0."""
    import FlagOS_mhc as M
    torch.set_num_threads(os.cpu_count())
    torch.manual_seed(0)
    B, S, N, D = 2, 128, 4, 1024
    x = torch.randn(B, S, N, D, requires_grad=True)
    h_out = torch.randn(B, S, D, requires_grad=True)
    h_res = torch.softmax(torch.randn(B, S, N, N), -1).requires_grad_(True)
    h_post = (2 * torch.sigmoid(torch.randn(B, S, N))).requires_grad_(True)
    gy = torch.randn(B, S, N, D)
    times = []
    for k in range(warmup + steps):
        t0 = time.perf_counter()
        y = M.mhc_post_ref(x, h_res, h_out, h_post)
        torch.autograd.grad(y, (x, h_res, h_out, h_post), gy)
        if k >= warmup:
            times.append(time.perf_counter() - t0)
    ms = 1e3 * statistics.median(times)
    return {"config": "C0: mhc_post_ref fwd + autograd bwd, fp32 CPU, B=2 S=128 N=4 D=1024",
            "ms_per_step": ms, "tokens_per_s": B * S / (ms / 1e3), "steps": steps,
            "cores": torch.get_num_threads()}


REF_SAMPLE_NOTE = ("tokens/s is per-token independent work, so the rate of a T-token slice "
                   "is the rate of the full T=32768 step; the `*_ref` path is the "
                   "reference's pure-PyTorch algorithm (fp32 math on bf16 storage), op for op")


def reference_arm(args, rank, world):
    """The reference's CPU implementation of the path (its `*_ref` functions) on this
    host's cores: each step is one T_s-token slice of the benchmark workload."""
    if rank != 0:
        return 0
    # calibrate the slice so the whole --steps K --warmup W run is ~2 minutes of CPU work
    # (at most 3 s per step), whatever K is
    rate0, _ = cpu_ref_rate(128, steps=1, warmup=1)
    per_step_s = min(3.0, 120.0 / max(1, args.steps + args.warmup))
    T_s = int(max(64, min(4096, rate0 * per_step_s)) // 64 * 64)
    rate, times = cpu_ref_rate(T_s, steps=args.steps, warmup=args.warmup)
    cores = torch.get_num_threads()
    ms = 1e3 * sum(times) / len(times)
    sample = (f"{args.steps} steps of a {T_s}-token slice of the T=32768,N=4,D=7168 workload "
              f"(pre fwd+bwd and post fwd+bwd through the *_ref path); " + REF_SAMPLE_NOTE)
    line = {
        "metric": METRIC, "value": rate, "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
        "config": {"workload": WORKLOAD, "T": T_TOK, "N": N_HC, "D": D_HID,
                   "parallelism": "rank 0 only (CPU)", "sample_tokens": T_s,
                   "ms_per_step_is": f"one {T_s}-token slice"},
        "cpu_baseline": {"value": rate, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": rate, "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "c0": cpu_c0(),
    }
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------- other configs
def _timed(fn, steps, warmup, nev):
    """Mean ms between consecutive events that fn(ev) records, over `steps` runs."""
    for _ in range(warmup):
        fn(None)
    torch.cuda.synchronize()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(nev)] for _ in range(steps)]
    for k in range(steps):
        fn(evs[k])
    torch.cuda.synchronize()
    return [statistics.mean(evs[k][i].elapsed_time(evs[k][i + 1]) for k in range(steps))
            for i in range(nev - 1)]


def other_configs(M, dev, peak, steps=5, warmup=2, only=None):
    """`only`: a set of group names (C1, pre_dtypes, C3_boundary, C4) to run, or None for
    all.  Config C1 (pre forward, need_backward) and config C4 (the N=8 layer step:
    pre -> h_out = y.W (cuBLAS) -> post, then the backward of the same chain), synthetic
    inputs with the configs' distributions.  Reported beside the headline number."""
    res = {}
    bf = torch.bfloat16
    if only is None or "C1" in only:
        # ---- C1: T=16384, N=4, D=4096, pre forward with need_backward=True
        T, N, D = 16384, 4, 4096
        g = torch.Generator(device=dev).manual_seed(1)
        x = torch.randn(T, N, D, generator=g, device=dev).to(bf)
        phi = torch.randn(24, N * D, generator=g, device=dev) / 128.0
        alpha = torch.rand(3, generator=g, device=dev) + 0.5
        base = torch.randn(24, generator=g, device=dev) * 0.1

        def c1(ev):
            if ev is not None:
                ev[0].record()
            M.mhc_pre_clamp_sinkhorn(x, phi, alpha, base, need_backward=True, **KW)
            if ev is not None:
                ev[1].record()
        ms = _timed(c1, steps, warmup, 2)[0]
        nbytes = T * 106756
        res["C1_pre_fwd"] = {"shape": [T, N, D], "ms": ms, "tokens_per_s": T / (ms / 1e3),
                             "GB/s": nbytes / (ms / 1e3) / 1e9,
                             "frac_of_peak": nbytes / (ms / 1e3) / 1e9 / peak}
        del x, phi
        torch.cuda.empty_cache()
    if only is None or "pre_dtypes" in only:
        # ---- dtype breadth at the C1 shape (fp32 / fp16 x, N=4 and N=8) and fp32 x at the C3
        # shape: pre forward + backward, each on its tensor-core path
        dt_res = {}
        for (N, dt, T, D) in [(4, torch.float32, 16384, 4096), (4, torch.float16, 16384, 4096),
                              (8, torch.float32, 16384, 4096), (8, torch.float16, 16384, 4096),
                              (8, bf, 16384, 4096), (4, torch.float32, 32768, 7168)]:
            HM = N * (N + 2)
            g = torch.Generator(device=dev).manual_seed(1)
            x = torch.randn(T, N, D, generator=g, device=dev).to(dt)
            phi = torch.randn(HM, N * D, generator=g, device=dev) / (N * D) ** 0.5
            alpha = torch.rand(3, generator=g, device=dev) + 0.5
            base = torch.randn(HM, generator=g, device=dev) * 0.1
            gy = torch.randn(T, D, generator=g, device=dev).to(dt)
            gpost = torch.randn(T, N, generator=g, device=dev)
            gcomb = torch.randn(T, N, N, generator=g, device=dev)
            saved = {}

            def fwd_bwd(ev):
                ev[0].record() if ev is not None else None
                o = M.mhc_pre_clamp_sinkhorn(x, phi, alpha, base, need_backward=True, **KW)
                ev[1].record() if ev is not None else None
                M.mhc_pre_clamp_sinkhorn_backward(x, phi, alpha, base, o["inv_rms"],
                                                  o["x_scaled"], o["mixes"], o["h_res_logits"],
                                                  o["pre"], gy, gpost, gcomb, **KW)
                ev[2].record() if ev is not None else None
                saved["o"] = o
            t = _timed(fwd_bwd, steps, warmup, 3)
            name = {torch.float32: "f32", torch.float16: "f16", bf: "bf16"}[dt]
            key = f"N{N}_{name}" + ("_C3" if (T, D) == (32768, 7168) else "")
            dt_res[key] = {"shape": [T, N, D], "pre_fwd_ms": t[0], "pre_bwd_ms": t[1]}
            del x, gy, saved
            torch.cuda.empty_cache()
        res["pre_dtypes"] = dt_res
    if only is None or "C3_boundary" in only:
        # ---- layer boundary at C3 shapes: post forward of layer l, then the pre forward of
        # layer l+1 on its output; unfused (two passes over x_{l+1}) against the fused pair
        # (post forward writing the next layer's mix partials, pre forward from them)
        T, N, D = 32768, 4, 7168
        g = torch.Generator(device=dev).manual_seed(3)
        xl = torch.randn(T, N, D, generator=g, device=dev).to(bf)
        ho = torch.randn(T, D, generator=g, device=dev).to(bf)
        hr = torch.softmax(torch.randn(T, N, N, generator=g, device=dev), -1)
        hp = 2 * torch.sigmoid(torch.randn(T, N, generator=g, device=dev))
        phi = torch.randn(24, N * D, generator=g, device=dev) / (N * D) ** 0.5
        alpha = torch.rand(3, generator=g, device=dev) + 0.5
        base = torch.randn(24, generator=g, device=dev) * 0.1

        def boundary(ev, fused):
            ev[0].record() if ev is not None else None
            if fused:
                x1, pm = M.mhc_post(xl, hr, ho, hp, next_phi=phi)
            else:
                x1, pm = M.mhc_post(xl, hr, ho, hp), None
            ev[1].record() if ev is not None else None
            M.mhc_pre_clamp_sinkhorn(x1, phi, alpha, base, need_backward=True, premix=pm, **KW)
            ev[2].record() if ev is not None else None
        tu = _timed(lambda ev: boundary(ev, False), steps, warmup, 3)
        tf = _timed(lambda ev: boundary(ev, True), steps, warmup, 3)
        res["C3_layer_boundary_fwd"] = {
            "shape": [T, N, D],
            "unfused_ms": {"post_fwd": tu[0], "pre_fwd": tu[1], "total": tu[0] + tu[1]},
            "fused_ms": {"post_fwd_with_next_mix": tf[0], "pre_fwd_from_premix": tf[1],
                         "total": tf[0] + tf[1]},
            "saves_ms": (tu[0] + tu[1]) - (tf[0] + tf[1]),
            "note": "x_{l+1} is read once instead of twice across the layer boundary"}
        del xl, ho, hr, hp, phi
        torch.cuda.empty_cache()
    if only is None or "C4" in only:
        # ---- C4: T=65536, N=8, D=4096 layer step
        T, N, D = 65536, 8, 4096
        HM = N * (N + 2)
        g = torch.Generator(device=dev).manual_seed(4)
        x = torch.randn(T, N, D, generator=g, device=dev).to(bf)
        phi = torch.randn(HM, N * D, generator=g, device=dev) / 181.0
        alpha = torch.rand(3, generator=g, device=dev) + 0.5
        base = torch.randn(HM, generator=g, device=dev) * 0.1
        W = (torch.randn(D, D, generator=g, device=dev) / 64.0).to(bf)
        gz = torch.randn(T, N, D, generator=g, device=dev).to(bf)

        def c4(ev, fused=False):
            rec = (lambda i: ev[i].record()) if ev is not None else (lambda i: None)
            rec(0)
            out = M.mhc_pre_clamp_sinkhorn(x, phi, alpha, base, need_backward=True, **KW)
            rec(1)
            h_out = out["y"] @ W
            rec(2)
            M.mhc_post(x, out["comb_frag"], h_out, out["post_out"])
            rec(3)
            gxp, ghres, ghout, ghpost = M.mhc_post_backward(gz, x, out["comb_frag"], h_out,
                                                            out["post_out"])
            rec(4)
            gy = ghout @ W.t()
            gW = out["y"].t() @ ghout
            rec(5)
            if fused:
                # x feeds both ops: the post backward's grad_x is added inside the pre backward
                M.mhc_pre_clamp_sinkhorn_backward(
                    x, phi, alpha, base, out["inv_rms"], out["x_scaled"], out["mixes"],
                    out["h_res_logits"], out["pre"], gy, ghpost, ghres, grad_x_accumulate=gxp,
                    **KW)
                rec(6)
            else:
                gxq = M.mhc_pre_clamp_sinkhorn_backward(
                    x, phi, alpha, base, out["inv_rms"], out["x_scaled"], out["mixes"],
                    out["h_res_logits"], out["pre"], gy, ghpost, ghres, **KW)[0]
                rec(6)
                gxp.add_(gxq)
            rec(7)
            return gW
        t = _timed(c4, steps, warmup, 8)
        tf = _timed(lambda ev: c4(ev, fused=True), steps, warmup, 8)
        mhc_ms = t[0] + t[2] + t[3] + t[5]
        nbytes = T * 698728
        res["C4_layer_step"] = {
            "shape": [T, N, D],
            "ms": {"pre_fwd": t[0], "gemm_fwd": t[1], "post_fwd": t[2], "post_bwd": t[3],
                   "gemm_bwd": t[4], "pre_bwd": t[5], "grad_x_sum": t[6]},
            "fused_grad_x_sum": {"pre_bwd_with_grad_x_accumulate": tf[5],
                                 "saves_ms": t[5] + t[6] - tf[5]},
            "mhc_ms": mhc_ms, "mhc_tokens_per_s": T / (mhc_ms / 1e3),
            "mhc_GB/s": nbytes / (mhc_ms / 1e3) / 1e9,
            "mhc_frac_of_peak": nbytes / (mhc_ms / 1e3) / 1e9 / peak,
            "note": "mhc_* = the four mHC ops (698,728 algorithmic B/token); the y.W GEMMs "
                    "(cuBLAS) and the torch grad_x sum are timed separately; fused_grad_x_sum "
                    "runs the same step with the post backward's grad_x added inside the pre "
                    "backward (grad_x_accumulate) instead of the torch sum",
        }
    return res


# ----------------------------------------------------------------------------- end to end
# outputs of one step that go back to the host in the end-to-end measurement
def _step_outputs(out, y, pg, grads):
    d = {"y": out["y"], "post_out": out["post_out"], "comb_frag": out["comb_frag"],
         "inv_rms": out["inv_rms"], "mixes": out["mixes"], "h_res_logits": out["h_res_logits"],
         "pre": out["pre"], "post_out_x": y, "post_grad_x": pg[0], "grad_h_res": pg[1],
         "grad_h_out": pg[2], "grad_h_post": pg[3], "pre_grad_x": grads[0]}
    if out["x_scaled"].numel():
        d["x_scaled"] = out["x_scaled"]
    return d


def e2e_measure(M, inp, world, steps, x_scaled, reducer, dist, dev):
    """The step through the public API with host buffers: every step copies each
    per-token input from pinned host memory and every output back to pinned host
    memory.  Tokens are processed in chunks on three streams (H2D, compute, D2H), so
    the copies of one chunk overlap the kernels of its neighbours; the per-chunk
    parameter gradients are summed on the device and copied back once per step."""
    T = inp["x_pre"].shape[0]
    C = max(256, min(4096, T // 4)) if T >= 1024 else T
    chunks = [(a, min(T, a + C)) for a in range(0, T, C)]
    host_in = {k: torch.empty(inp[k].shape, dtype=inp[k].dtype, pin_memory=True)
               for k in HOST_INPUTS}
    for k in HOST_INPUTS:
        host_in[k].copy_(inp[k])
    # output shapes from one chunk-sized call
    probe = {k: inp[k][:chunks[0][1]] for k in HOST_INPUTS}
    probe.update(phi=inp["phi"], alpha=inp["alpha"], base=inp["base"])
    o = _step_outputs(*run_step(M, probe, 1, x_scaled=x_scaled))
    host_out = {k: torch.empty((T,) + tuple(v.shape[1:]), dtype=v.dtype, pin_memory=True)
                for k, v in o.items()}
    n_param = inp["phi"].numel() + 3 + inp["base"].numel()
    host_grad = torch.empty(n_param, dtype=torch.float32, pin_memory=True)
    del o, probe
    h2d = sum(t.numel() * t.element_size() for t in host_in.values())
    d2h = sum(t.numel() * t.element_size() for t in host_out.values()) + host_grad.numel() * 4
    bufs = [{k: torch.empty((C,) + tuple(inp[k].shape[1:]), dtype=inp[k].dtype, device=dev)
             for k in HOST_INPUTS} for _ in range(2)]
    s_in, s_c, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_free = [torch.cuda.Event() for _ in range(2)]
    gacc = torch.empty(n_param, dtype=torch.float32, device=dev)
    main = torch.cuda.current_stream(dev)

    def one_step():
        for i, (a, b) in enumerate(chunks):
            j, n = i % 2, b - a
            if i >= 2:
                s_in.wait_event(ev_free[j])
            with torch.cuda.stream(s_in):
                for k in HOST_INPUTS:
                    bufs[j][k][:n].copy_(host_in[k][a:b], non_blocking=True)
                ev_in[j].record(s_in)
            s_c.wait_event(ev_in[j])
            with torch.cuda.stream(s_c):
                chunk = {k: bufs[j][k][:n] for k in HOST_INPUTS}
                chunk.update(phi=inp["phi"], alpha=inp["alpha"], base=inp["base"])
                out, y, pg, grads = run_step(M, chunk, 1, x_scaled=x_scaled)
                ev_free[j].record(s_c)
                g = grads[1].reshape(-1)
                flat = torch.as_strided(g, (n_param,), (1,))  # packed [phi|alpha|base]
                if i == 0:
                    gacc.copy_(flat)
                else:
                    gacc.add_(flat)
                outs = _step_outputs(out, y, pg, grads)
                done = torch.cuda.Event()
                done.record(s_c)
            s_out.wait_event(done)
            with torch.cuda.stream(s_out):
                for k, v in outs.items():
                    host_out[k][a:b].copy_(v.reshape(host_out[k][a:b].shape), non_blocking=True)
                    v.record_stream(s_out)
        with torch.cuda.stream(s_c):
            if world > 1:
                nph = inp["phi"].numel()
                reducer(gacc[:nph].view_as(inp["phi"]), gacc[nph:nph + 3], gacc[nph + 3:])
            done = torch.cuda.Event()
            done.record(s_c)
        s_out.wait_event(done)
        with torch.cuda.stream(s_out):
            host_grad.copy_(gacc, non_blocking=True)
            gacc.record_stream(s_out)

    def fence_all(ev_start=None):
        for s in (s_in, s_c, s_out):
            if ev_start is not None:
                s.wait_event(ev_start)
            else:
                e = torch.cuda.Event()
                e.record(s)
                main.wait_event(e)

    one_step()      # warm-up (allocator, pinned pages)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(main)
    fence_all(e0)
    for _ in range(steps):
        one_step()
    fence_all()
    e1.record(main)
    torch.cuda.synchronize()
    e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e_ms = float(t.item())
    return {"value": world * T * steps / (e_ms / 1e3), "unit": "tokens/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": steps,
            "ms_per_step": e_ms / steps, "chunk_tokens": C,
            "outputs_copied_back": sorted(host_out) + ["grad_phi|grad_alpha|grad_base"],
            "note": "public API per token chunk; H2D of every per-token input from pinned "
                    "memory and D2H of every output to pinned memory, each step, inside the "
                    "CUDA-event-timed region (three streams, PCIe-bound)"}


# ----------------------------------------------------------------------------- GPU arm
def capture_step(M, inp, world, x_scaled, reducer, dev):
    """One step (the same public-API calls as run_step, the cross-GPU sum included)
    captured in a CUDA graph.  Returns (graph, library kernel launches per step) or
    (None, reason) if the capture failed."""
    from FlagOS_mhc import _C
    try:
        torch.cuda.synchronize()
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        g = torch.cuda.CUDAGraph()
        n0 = _C.lib().mhc_kernel_launches()
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                run_step(M, inp, world, x_scaled=x_scaled, reducer=reducer)
        torch.cuda.synchronize()
        return g, _C.lib().mhc_kernel_launches() - n0
    except Exception as e:  # noqa: BLE001 -- reported in the JSON line, eager timing used
        torch.cuda.synchronize()
        return None, f"{type(e).__name__}: {e}"[:200]


def timed_steps(M, inp, world, K, x_scaled, reducer, dist, dev, soak_s, clocks=None,
                graph=None, graph_launches=0):
    """K steps between two events (after a barrier and a synchronize), preceded by
    untimed soak steps for about soak_s seconds; with `graph`, each step is a replay of
    the captured step.  Returns (max-over-ranks ms, per-step op events, launches)."""
    from FlagOS_mhc import _C
    step = (lambda: graph.replay()) if graph is not None else (
        lambda: run_step(M, inp, world, x_scaled=x_scaled, reducer=reducer))
    if clocks is not None:
        clocks.mark_load()
    # soak: the same number of steps on every rank (each step holds a collective), about
    # soak_s seconds' worth as timed from one step
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    step()
    torch.cuda.synchronize()
    n = torch.tensor([int(soak_s / max(time.perf_counter() - t0, 1e-4))], device=dev)
    if world > 1:
        dist.all_reduce(n, op=dist.ReduceOp.MAX)
    for _ in range(min(int(n.item()), 20000)):
        step()
    torch.cuda.synchronize()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    n0 = _C.lib().mhc_kernel_launches()
    if clocks is not None:
        clocks.mark_start()
    start.record()
    for k in range(K):
        step()
    stop.record()
    torch.cuda.synchronize()
    if clocks is not None:
        clocks.mark_stop()
    launches = _C.lib().mhc_kernel_launches() - n0 + (graph_launches * K if graph else 0)
    if world > 1:
        dist.barrier()
    ms_total = start.elapsed_time(stop)
    if world > 1:
        t = torch.tensor([ms_total], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_total = float(t.item())
    # the per-operator split comes from separate eager steps (an event between two
    # operators stops the next one's launch from overlapping the previous kernel's tail,
    # ~3 us each); two untimed ones first, so that allocations made outside a captured
    # graph's memory pool are not timed
    for _ in range(2):
        run_step(M, inp, world, x_scaled=x_scaled, reducer=reducer)
    torch.cuda.synchronize()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(6)] for _ in range(K)]
    for k in range(K):
        run_step(M, inp, world, evs[k], x_scaled=x_scaled, reducer=reducer)
    torch.cuda.synchronize()
    return ms_total, evs, launches


def grad_sum_bench(MD, dist, dev, world, rank, K, W):
    """Back-to-back calls of the cross-GPU sum of the packed C3 parameter gradients
    (24 x 28672 + 27 fp32): the fused peer-memory kernel against NCCL's all-reduce.
    Device time per call, max over ranks."""
    n = 24 * 28672 + 27
    buf = torch.randn(n, device=dev)
    red = MD.PeerGradReducer(n, dev)
    res = {}
    for name, fn in (("fused_peer_kernel", red.reduce_),
                     ("nccl_all_reduce", lambda b: dist.all_reduce(b))):
        reps = max(K, 50)
        for _ in range(max(W, 5)):
            fn(buf)
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            fn(buf)
        e1.record()
        torch.cuda.synchronize()
        t = torch.tensor([e0.elapsed_time(e1) / reps * 1e3], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        res[name] = {"us_per_call": float(t.item()), "calls": reps}
    red.close()
    if rank == 0:
        print(json.dumps({"grad_sum_bench": res, "n_gpus": world, "floats": n,
                          "bytes": 4 * n}), flush=True)
    dist.barrier()
    dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=500,
                    help="timed steps (default: a timed region of >= 2 s at N=1)")
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--global-tokens", type=int, default=T_TOK,
                    help="tokens of the whole job, split evenly over the ranks (strong scaling)")
    ap.add_argument("--tokens", type=int, default=None,
                    help="tokens per GPU instead (weak scaling)")
    ap.add_argument("--soak-s", type=float, default=1.0,
                    help="untimed steps right before the timed region (clock sampling under load)")
    ap.add_argument("--e2e-steps", type=int, default=None, help="default: --steps")
    ap.add_argument("--collective", default="fused", choices=["fused", "nccl"],
                    help="cross-GPU gradient sum: the library's peer-memory kernel or NCCL")
    ap.add_argument("--grad-sum-bench", action="store_true",
                    help="N>1: time only the cross-GPU gradient sum (fused kernel vs NCCL)")
    ap.add_argument("--no-weak", action="store_true",
                    help="N>1: skip the secondary weak-scaling measurement")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-other-configs", action="store_true",
                    help="skip the C1 / C4 measurements reported beside the headline")
    ap.add_argument("--configs-only", action="store_true",
                    help="run only the C1 / C4 measurements (--steps / --warmup apply)")
    ap.add_argument("--configs", default=None,
                    help="with --configs-only: comma-separated groups (C1, pre_dtypes, "
                         "C3_boundary, C4); default all")
    ap.add_argument("--eager", action="store_true",
                    help="time the step as eager calls instead of replays of its CUDA graph")
    ap.add_argument("--skip-x-scaled", action="store_true",
                    help="opt-in variant: the forward does not write the fp32 x_scaled "
                         "(not the reference contract; the default keeps it)")
    args = ap.parse_args()

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return reference_arm(args, rank, world)

    import torch.distributed as dist
    import FlagOS_mhc as M
    from FlagOS_mhc import distributed as MD
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", device_id=dev)

    if args.grad_sum_bench:
        return grad_sum_bench(MD, dist, dev, world, rank, args.steps, args.warmup)

    if args.configs_only:
        peak, peak_kind = hbm_peak()
        only = set(args.configs.split(",")) if args.configs else None
        print(json.dumps({"other_configs": other_configs(M, dev, peak, steps=args.steps,
                                                         warmup=args.warmup, only=only),
                          "peak_kind": peak_kind}), flush=True)
        return 0

    N, D = N_HC, D_HID
    if args.tokens is not None:
        T, T_global, scaling = args.tokens, args.tokens * world, "weak"
    else:
        a, b = MD.token_range(args.global_tokens, rank, world)
        T, T_global, scaling = b - a, args.global_tokens, "strong"
    xs_on = not args.skip_x_scaled
    K = args.steps
    inp = make_inputs(T, N, D, seed=1000 + rank, dev=dev)
    reducer = None
    if world > 1:
        reducer = (MD.PeerGradReducer(inp["phi"].numel() + 3 + inp["base"].numel(), dev)
                   if args.collective == "fused" else MD.allreduce_pre_grads)
    torch.cuda.synchronize()
    for _ in range(max(args.warmup, 0)):
        run_step(M, inp, world, x_scaled=xs_on, reducer=reducer)
    torch.cuda.synchronize()

    # the step as a CUDA graph (the library's calls and the cross-GPU sum captured once,
    # replayed each step); every rank must have captured it, else all run eagerly
    graph, glaunch, graph_note = None, 0, "eager (--eager)"
    if not args.eager:
        graph, glaunch = capture_step(M, inp, world, xs_on, reducer, dev)
        ok = torch.tensor([1 if graph is not None else 0], device=dev)
        if world > 1:
            dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        if graph is None or int(ok.item()) == 0:
            graph_note = f"eager (capture failed: {glaunch})" if graph is None else \
                "eager (capture failed on another rank)"
            graph, glaunch = None, 0
        else:
            graph_note = "cuda_graph"
    clocks = ClockSampler(local)
    clocks.start()
    ms_total, evs, launches = timed_steps(M, inp, world, K, xs_on, reducer, dist, dev,
                                          args.soak_s, clocks, graph=graph,
                                          graph_launches=glaunch)
    ck = clocks.stop()
    ms_step = ms_total / K
    eager_ms = None
    if graph is not None:  # the same K steps as eager calls, for reference
        eager_ms = timed_steps(M, inp, world, K, xs_on, reducer, dist, dev, 0.0)[0] / K
    value = T_global * K / (ms_total / 1e3)

    names = ["pre_fwd", "post_fwd", "post_bwd", "pre_bwd", "grad_sum"]
    op_ms = {n: statistics.mean(evs[k][i].elapsed_time(evs[k][i + 1]) for k in range(K))
             for i, n in enumerate(names)}
    ab = algorithmic_bytes(T, N, D, x_scaled=xs_on)
    peak, peak_kind = hbm_peak()
    step_bytes = sum(ab.values())
    ops = {n: {"ms": op_ms[n], "GB/s": ab[n] / (op_ms[n] / 1e3) / 1e9,
               "frac_of_" + peak_kind + "_peak": ab[n] / (op_ms[n] / 1e3) / 1e9 / peak}
           for n in ab}
    # roofline of one kernel measured live: post_bwd is a single launch between its two
    # events (the pre ops run several kernels) and the largest share of the step in the
    # ncu launch list
    dom = "post_bwd"
    tr = ncu_traffic().get(dom + "_per_token")
    traffic = tr * T if tr else None
    achieved = ab[dom] / (op_ms[dom] / 1e3) / 1e9

    weak = None
    if world > 1 and scaling == "strong" and not args.no_weak:
        inp_w = make_inputs(T_TOK, N, D, seed=2000 + rank, dev=dev)
        ms_w, _, _ = timed_steps(M, inp_w, world, K, xs_on, reducer, dist, dev, 0.2)
        weak = {"tokens_per_gpu": T_TOK, "global_tokens": T_TOK * world, "steps": K,
                "ms_per_step": ms_w / K, "value": world * T_TOK * K / (ms_w / 1e3)}
        del inp_w
        torch.cuda.empty_cache()

    e2e_steps = K if args.e2e_steps is None else args.e2e_steps
    e2e = None
    if e2e_steps > 0:
        e2e = e2e_measure(M, inp, world, e2e_steps, xs_on, reducer, dist, dev)

    others = None
    if rank == 0 and world == 1 and not args.no_other_configs:
        del inp
        torch.cuda.empty_cache()
        others = other_configs(M, dev, peak)

    cpu_base = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rate, times = cpu_ref_rate(256, budget_s=15.0, warmup=1)
        cpu_base = {"value": rate, "unit": "tokens/s", "cores": torch.get_num_threads(),
                    "kind": "port",
                    "sample": f"{len(times)} steps of a 256-token slice of the same workload "
                              "through the *_ref path; " + REF_SAMPLE_NOTE,
                    "c0": cpu_c0()}

    if rank == 0:
        coll = {"fused": "one library kernel over NVLink peer memory (rank-order sum)",
                "nccl": "packed NCCL all-reduce"}[args.collective]
        line = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": K,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": scaling, "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": WORKLOAD, "tokens_per_gpu": T, "global_tokens": T_global,
                       "N": N, "D": D, "hcMix": N * (N + 2), "clamp": [-10.0, 10.0],
                       "iter_times": 20,
                       "x_scaled": "written (reference contract)" if xs_on
                       else "skipped (opt-in materialize_x_scaled=False)",
                       "parallelism": f"dp{world} token-sharded"
                       + (f", gradient sum: {coll}" if world > 1 else ""),
                       "l2": "no flush: each step streams >= 2.6 GB per GPU (x alone "
                             f"{T * N * D * 2 / 1e6:.0f} MB) through the 126 MB L2"},
            "hbm_frac_step": step_bytes / (ms_step / 1e3) / 1e9 / peak,
            "roofline": {"bound": "hbm", "kernel": "post_bwd_n4x2_kernel", "achieved": achieved,
                         "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                         "frac": achieved / peak, "algorithmic_bytes": ab[dom],
                         "traffic": traffic,
                         "traffic_source": ncu_traffic().get("source")},
            "step_mode": graph_note, "eager_ms_per_step": eager_ms,
            "ops": ops, "grad_sum_ms": op_ms["grad_sum"],
            "gpu_launches": int(launches),
            "clocks": ck, "e2e": e2e, "cpu_baseline": cpu_base,
            "weak_scaling": weak, "other_configs": others,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        if reducer is not None and hasattr(reducer, "close"):
            reducer.close()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
