"""Benchmark of the mHC residual layer on B200 (BASELINE.json metric).

Default workload: one full mHC layer forward, batch 16 x
seq 2048 tokens per GPU, C = 768, n = 4 streams, bf16 activations, fp32
coefficient math, 20 Sinkhorn iterations, phi ~ N(0, 0.02), alpha = 0.01,
biases 0.  A step is one pass of the hot path over the batch: the coefficient
kernel (RMS + projection + gates + Sinkhorn) with the pre-aggregate, then the
post / res merge.  The sublayer f (a random-init SwiGLU 768 -> 2048 -> 768 in
torch) is outside the metric: it is evaluated once on the batch before the
timed region and its output is the merge's f input on every step.

Timing: W untimed warm-up steps, then K steps bracketed by a barrier and a
device synchronise, CUDA events on the launching stream, max over ranks.  x is
201 MB per GPU (larger than the 126 MB L2), so every step streams from HBM.

Multi-GPU: one process per GPU (torchrun), tokens sharded (weak scaling): every
rank runs its own 16 x 2048 tokens with no collective on the data path.

``--impl reference`` times the reference's pure-PyTorch CPU path of the same
layer (the oracle restatement in oracle/mhc_oracle.py, fp32, f = identity) on
the host cores with all threads, rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "minimind-mhc_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

METRIC = "mHC layer tokens/s"
NOMINAL_HBM_GBS = 8000.0


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def _time_backward(L, nat, x, ps, with_res, iters, z, h_post, h_res, inv_rms, mixes, f_out, t, n, c, fd, dev,
                   sptr, stream, steps, peak_of):
    """Backward of one layer through the C-ABI: mhc_post_bwd (merge) then
    mhc_pre_bwd (coefficients, Sinkhorn by recompute, RMSNorm, dphi / dalpha /
    dbias reductions).  dz stands in for the sublayer's input gradient.
    Algorithmic bytes per token s*(6nC + 3C)."""
    gen = torch.Generator(device=dev).manual_seed(99)
    dout = torch.randn(t, n * c, device=dev, dtype=torch.bfloat16, generator=gen)
    dz = torch.randn(t, c, device=dev, dtype=torch.bfloat16, generator=gen)
    dx_post = torch.empty_like(x)
    dx = torch.empty_like(x)
    dh_res = torch.empty(t, n * n, device=dev) if with_res else None
    dh_post = torch.empty(t, n, device=dev)
    df = torch.empty_like(f_out)
    gps = [torch.empty_like(p, dtype=torch.float32) for p in ps]
    g_res = (gps[5], gps[6]) if with_res else (None, None)
    a_res, b_res = (ps[5], ps[6]) if with_res else (None, None)
    ws = nat.workspace(L.mhc_pre_bwd_workspace(t, n, c, int(with_res), int(with_res), iters), dev)

    def step():
        st = L.mhc_post_bwd(nat.ptr(dout), nat.ptr(x), nat.BF16, nat.ptr(h_res), nat.F32, nat.ptr(h_post),
                            nat.F32, nat.ptr(f_out), nat.BF16, nat.ptr(dx_post), nat.ptr(dh_res), nat.ptr(dh_post),
                            nat.ptr(df), t, n, c, sptr)
        nat.check(st, "mhc_post_bwd")
        st = L.mhc_pre_bwd(nat.ptr(x), nat.BF16, t, n, c, nat.ptr(ps[0]), nat.ptr(ps[1]), nat.ptr(ps[2]),
                           nat.ptr(ps[3]), nat.ptr(ps[4]), nat.ptr(a_res), nat.ptr(b_res), nat.F32,
                           int(with_res), int(with_res), iters, 2.0, 1e-6, 1e-6, 1e-6, nat.ptr(inv_rms),
                           nat.ptr(mixes), nat.ptr(dz), None, nat.ptr(dh_post), nat.ptr(dh_res), nat.F32,
                           nat.ptr(dx_post), nat.ptr(dx), nat.ptr(gps[0]), nat.ptr(gps[1]), nat.ptr(gps[2]),
                           nat.ptr(gps[3]), nat.ptr(gps[4]), nat.ptr(g_res[0]), nat.ptr(g_res[1]), nat.ptr(ws),
                           ws.numel(), sptr)
        nat.check(st, "mhc_pre_bwd")

    for _ in range(3):
        step()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    torch.cuda.synchronize(dev)
    for e0, e1 in ev:
        e0.record(stream)
        step()
        e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = sorted(e0.elapsed_time(e1) for e0, e1 in ev)[len(ev) // 2]
    bytes_tok = 2 * (6 * n * c + 3 * c)
    peak, kind = peak_of()
    gbs = bytes_tok * t / (ms / 1e3) / 1e9
    return {"ms_per_step": ms, "tokens_per_s": t / (ms / 1e3), "algorithmic_bytes_per_token": bytes_tok,
            "gbs": gbs, "frac_of_measured": gbs / peak, "steps": steps,
            "calls": "mhc_post_bwd + mhc_pre_bwd (median step, CUDA events)"}


def _profiled_traffic(kernel, n, c, t, with_res):
    """DRAM bytes (read + write) per launch of the dominant kernel, from the
    committed ncu summary of this exact workload (profiles/*.md carries a line
    `traffic_bytes_per_launch: <int>`); None for other workloads."""
    if (n, c, t, bool(with_res)) != (4, 768, 32768, True):
        return None
    name = {"pre": "pre_tc_kernel_config2.md", "post": "post_fwd_kernel_config2.md"}[kernel]
    path = os.path.join(ROOT, "profiles", name)
    try:
        with open(path) as f:
            for line in f:
                if line.startswith("traffic_bytes_per_launch:"):
                    return int(line.split(":", 1)[1]), "ncu dram__bytes_read.sum + dram__bytes_write.sum, profiles/" + name
    except OSError:
        pass
    return None


def _layer_bytes(n, c, s, with_res):
    """Algorithmic bytes per token of the forward layer: read x twice (pre and
    post), write z, read f, write x' -> s * (3nC + 2C)."""
    return s * (3 * n * c + 2 * c)


class ClockSampler:
    """SM clock and throttle reasons of the benchmarked GPU, polled through NVML
    every millisecond from a background thread while the timed region runs
    (read-only queries)."""

    # NVML clocks-event-reason bits
    BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20,
            "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80}

    def __init__(self, device):
        self.device = device
        self.samples = []
        self.handle = None
        self._stop = threading.Event()
        try:
            import pynvml
            self.nv = pynvml
            pynvml.nvmlInit()
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            for cand in (uuid, "GPU-" + uuid):
                try:
                    self.handle = pynvml.nvmlDeviceGetHandleByUUID(cand)
                    break
                except Exception:
                    continue
            if self.handle is None:
                self.handle = pynvml.nvmlDeviceGetHandleByIndex(device.index or 0)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.handle = None

    def _poll(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(self.handle, nv.NVML_CLOCK_SM)
                try:
                    r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                except Exception:
                    r = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.handle)
                self.samples.append((sm, r))
            except Exception:
                pass
            time.sleep(0.001)

    def start(self):
        if self.handle is None:
            return
        self.t = threading.Thread(target=self._poll, daemon=True)
        self.t.start()

    def stop(self):
        if self.handle is None:
            return None
        self._stop.set()
        self.t.join(timeout=2)
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "samples": 0, "reasons": []}
        reasons = set()
        for _, r in self.samples:
            for nm, bit in self.BITS.items():
                if r & bit:
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(s for s, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "samples": len(self.samples), "reasons": sorted(reasons)}


def _cpu_reference(n, c, tokens, budget_s, min_runs, max_runs):
    """The reference's pure-PyTorch path (oracle restatement), fp32, f = identity."""
    from oracle import mhc_oracle as O
    torch.set_num_threads(os.cpu_count() or 1)
    gen = torch.Generator().manual_seed(0)
    x = torch.randn(1, tokens, n * c, generator=gen)
    p = O.make_full_params(n, c, generator=gen)
    with torch.no_grad():
        O.full_forward(x, p, lambda z: z, n, c, 20)  # warm-up
        times = []
        t_end = time.perf_counter() + budget_s
        while len(times) < max_runs and (len(times) < min_runs or time.perf_counter() < t_end):
            t0 = time.perf_counter()
            O.full_forward(x, p, lambda z: z, n, c, 20)
            times.append(time.perf_counter() - t0)
    return times


def run_reference(args, rank, world):
    if rank != 0:
        return
    n, c = 4, 768
    tokens = args.cpu_tokens
    step_times = []
    from oracle import mhc_oracle as O
    torch.set_num_threads(os.cpu_count() or 1)
    gen = torch.Generator().manual_seed(0)
    x = torch.randn(1, tokens, n * c, generator=gen)
    p = O.make_full_params(n, c, generator=gen)
    with torch.no_grad():
        for i in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            O.full_forward(x, p, lambda z: z, n, c, 20)
            dt = time.perf_counter() - t0
            if i >= args.warmup:
                step_times.append(dt)
    tot = sum(step_times)
    value = tokens * len(step_times) / tot
    sample = f"{tokens} tokens (C=768, n=4, fp32, f=identity, 20 Sinkhorn iters) per step"
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * tot / len(step_times), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "config2 mHC layer forward (reference pure-PyTorch CPU path)",
                   "tokens_per_step": tokens},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": torch.get_num_threads(),
                         "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args, rank, world, local_rank):
    import torch.distributed as dist
    import torch.nn.functional as F

    from model import _native as nat
    from model.mhc_fused import _params

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    n, c = 4, 768
    with_res = args.variant == "full"
    if args.variant == "nohres" and args.C:
        c = args.C
    t = args.tokens
    iters = 20 if with_res else 0
    fd = 2 * n + (n * n if with_res else 0)
    torch.manual_seed(1234 + rank)
    x = torch.randn(t, n * c, device=dev, dtype=torch.bfloat16)
    phi = torch.randn(n * c, fd, device=dev) * 0.02
    a = torch.tensor(0.01, device=dev)
    bn = torch.zeros(n, device=dev)
    ps = [phi, a, bn, a.clone(), bn.clone()] + ([a.clone(), torch.zeros(n, n, device=dev)] if with_res else [])
    ps = _params(*ps)
    # sublayer f = SwiGLU 768 -> 2048 -> 768 (torch), evaluated once outside the timed region
    w_gate = torch.randn(2048, c, device=dev, dtype=torch.bfloat16) * 0.02
    w_up = torch.randn(2048, c, device=dev, dtype=torch.bfloat16) * 0.02
    w_down = torch.randn(c, 2048, device=dev, dtype=torch.bfloat16) * 0.02

    z = torch.empty(t, c, device=dev, dtype=torch.bfloat16)
    h_post = torch.empty(t, n, device=dev)
    h_res = torch.empty(t, n, n, device=dev) if with_res else None
    inv_rms = torch.empty(t, device=dev)
    mixes = torch.empty(t, fd, device=dev)
    out = torch.empty_like(x)
    ws = nat.workspace(nat.lib().mhc_pre_fwd_workspace(t, n, c, int(with_res)), dev)
    stream = torch.cuda.current_stream(dev)
    sptr = stream.cuda_stream
    L = nat.lib()
    a_res, b_res = (ps[5], ps[6]) if with_res else (None, None)

    # the module's forward path: the coefficient kernel (with Sinkhorn-Knopp and
    # the pre-aggregate fused in), then the res / post merge
    def pre(xin):
        st = L.mhc_pre_fwd(nat.ptr(xin), nat.BF16, t, n, c, nat.ptr(ps[0]), nat.ptr(ps[1]), nat.ptr(ps[2]),
                           nat.ptr(ps[3]), nat.ptr(ps[4]), nat.ptr(a_res), nat.ptr(b_res), nat.F32,
                           int(with_res), int(with_res), iters, 2.0, 1e-6, 1e-6, 1e-6, nat.ptr(z), None,
                           nat.ptr(h_post), nat.ptr(h_res), nat.F32, nat.ptr(inv_rms), nat.ptr(mixes),
                           nat.ptr(ws), ws.numel(), sptr)
        nat.check(st, "mhc_pre_fwd")

    def post(xin, f, o):
        st = L.mhc_post_fwd(nat.ptr(xin), nat.BF16, nat.ptr(h_res), nat.F32, nat.ptr(h_post), nat.F32,
                            nat.ptr(f), nat.BF16, nat.ptr(o), t, n, c, 0, 0, 0.0, None, sptr)
        nat.check(st, "mhc_post_fwd")

    pre(x)
    f_out = (F.silu(z @ w_gate.t()) * (z @ w_up.t())) @ w_down.t()
    post(x, f_out, out)
    torch.cuda.synchronize(dev)

    fused = bool(L.mhc_last_path())
    launches_per_step = 2 if fused else 3  # fused coefficient+aggregate (or 2 generic kernels), merge
    bytes_tok = _layer_bytes(n, c, 2, with_res)
    pre_bytes = 2 * (n * c + c)
    post_bytes = 2 * (2 * n * c + c)

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        pre(x)
        post(x, f_out, out)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
           torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    sampler = ClockSampler(dev)
    barrier()
    torch.cuda.synchronize(dev)
    sampler.start()
    t_start = torch.cuda.Event(enable_timing=True)
    t_stop = torch.cuda.Event(enable_timing=True)
    # per-kernel events on the launching stream inside the timed region give
    # each kernel's live duration (the roofline figure below)
    t_start.record(stream)
    for i in range(args.steps):
        e0, e1, e2 = ev[i]
        e0.record(stream)
        pre(x)
        e1.record(stream)
        post(x, f_out, out)
        e2.record(stream)
    t_stop.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    clocks = sampler.stop()
    total_ms = t_start.elapsed_time(t_stop)
    pre_ms = [e0.elapsed_time(e1) for e0, e1, _ in ev]
    post_ms = [e1.elapsed_time(e2) for _, e1, e2 in ev]
    if world > 1:
        tt = torch.tensor([total_ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        total_ms = tt.item()

    # ---- backward of the layer (training config), reported beside the forward --
    bwd = None
    if not args.no_bwd:
        bwd = _time_backward(L, nat, x, ps, with_res, iters, z, h_post, h_res, inv_rms, mixes, f_out,
                             t, n, c, fd, dev, sptr, stream, max(3, min(args.steps, 20)), peak_of=_peaks)

    # ---- end to end through the public API with host buffers -------------------
    e2e = None
    if not args.no_e2e:
        x_h = x.cpu().pin_memory()
        f_h = f_out.cpu().pin_memory()
        o_h = torch.empty_like(x_h).pin_memory()
        x_d = torch.empty_like(x)
        f_d = torch.empty_like(f_out)

        def e2e_step():
            x_d.copy_(x_h, non_blocking=True)
            f_d.copy_(f_h, non_blocking=True)
            pre(x_d)
            post(x_d, f_d, out)
            o_h.copy_(out, non_blocking=True)

        for _ in range(max(1, args.warmup)):
            e2e_step()
        barrier()
        torch.cuda.synchronize(dev)
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        k_e2e = max(1, min(args.steps, 5))
        for _ in range(k_e2e):
            e2e_step()
        s1.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        e_ms = s0.elapsed_time(s1)
        if world > 1:
            tt = torch.tensor([e_ms], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            e_ms = tt.item()
        e2e = {"value": world * t * k_e2e / (e_ms / 1e3), "unit": "tokens/s",
               "h2d_bytes_per_step": int(x_h.numel() * 2 + f_h.numel() * 2),
               "d2h_bytes_per_step": int(o_h.numel() * 2), "steps": k_e2e,
               "ms_per_step": e_ms / k_e2e}

    if rank != 0:
        return
    peak, peak_kind = _peaks()
    step_ms = total_ms / args.steps
    value = world * t * args.steps / (total_ms / 1e3)
    pre_avg = sum(pre_ms) / len(pre_ms)
    post_avg = sum(post_ms) / len(post_ms)
    calls = {"pre": (pre_avg, pre_bytes * t), "post": (post_avg, post_bytes * t)}
    dom = max(calls, key=lambda k: calls[k][0])
    d_ms, d_bytes = calls[dom]
    achieved = d_bytes / (d_ms / 1e3) / 1e9
    layer_gbs = bytes_tok * t / (step_ms / 1e3) / 1e9  # per GPU, whole step
    traffic = _profiled_traffic(dom, n, c, t, with_res)

    cpu = None
    if not args.no_cpu_baseline:
        times = _cpu_reference(n, c, args.cpu_tokens, args.cpu_budget, 2, 50)
        cpu = {"value": args.cpu_tokens / statistics.median(times), "unit": "tokens/s",
               "cores": torch.get_num_threads(), "kind": "port",
               "sample": f"{args.cpu_tokens} tokens x {len(times)} runs (median), C=768, n=4, fp32, "
                         f"f=identity, 20 Sinkhorn iters; oracle restatement of _forward_ref"}

    line = {
        "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": step_ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": {
            "workload": ("config2: full mHC layer forward" if with_res else "config3: no-H_res mHC layer forward")
                        + f", {t} tokens/GPU (16x2048), C={c}, n={n}, bf16 activations, fp32 coefficients"
                        + (", 20 Sinkhorn iterations" if with_res else ""),
            "tokens_per_gpu": t, "global_tokens": world * t, "parallelism": f"dp{world} (token-sharded)",
            "sublayer": "SwiGLU 768-2048-768 in torch, outside the metric (evaluated once before timing)",
            "l2": "inputs larger than L2 (x = %.0f MB per GPU)" % (x.numel() * 2 / 1e6),
        },
        "hbm_gbs": layer_gbs,
        "hbm_frac_of_8tbs": layer_gbs / NOMINAL_HBM_GBS,
        "hbm_frac_of_measured": layer_gbs / peak,
        "algorithmic_bytes_per_token": bytes_tok,
        "per_call_ms": {"pre (coef+sinkhorn+aggregate)": pre_avg, "post (merge)": post_avg},
        "pre_path": "fused sm_100a cluster kernel (TMA + tcgen05 + DSMEM)" if fused else "generic CUDA-core kernels",
        "roofline": {"kernel": dom, "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_kind": peak_kind,
                     "traffic": traffic[0] if traffic else None,
                     "traffic_source": traffic[1] if traffic else None,
                     "algorithmic_bytes_per_launch": d_bytes},
        "cpu_baseline": cpu,
        "backward": bwd,
        "e2e": e2e,
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--variant", choices=["full", "nohres"], default="full")
    ap.add_argument("--C", type=int, default=0, help="stream width for --variant nohres (768 or 1024)")
    ap.add_argument("--tokens", type=int, default=16 * 2048)
    ap.add_argument("--cpu-tokens", type=int, default=4096)
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-bwd", action="store_true", help="skip the backward measurement")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        run_reference(args, rank, world)
        return

    if world > 1:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
