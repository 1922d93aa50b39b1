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

The same JSON line also carries, measured in the same run:
  * "backward": the layer backward (merge backward + coefficient backward);
  * "pre_other_kernel": the other fused forward kernel on the same inputs;
  * "e2e": the layer through the C-ABI from pinned host buffers, with the
    host link's copy-only ceiling;
  * "sweep": configs[1]'s token sweep, 4K to 256K tokens per GPU (L2 flushed
    between steps where the inputs would fit in it);
  * "nohres_c768", "nohres_c1024": configs[2], the no-H_res layer, forward and
    backward;
  * "fp32_stream": the layer with an fp32 residual stream and a bf16 sublayer
    output, the setting of the reference's bf16-autocast trainers;
  * "train_step": configs[4], the MoE + mHC training step (8 x 2048 tokens per
    GPU), with the NCCL gradient all-reduce timed on its own;
  * "post_pre": the step between two sublayers (merge of one, coefficient
    pass of the next, optionally its input RMSNorm) as two kernels and as the
    fused merge + coefficient kernel.

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


def _layer_bytes(n, c, s, with_res):
    """Algorithmic bytes per token of the forward layer: read x twice (pre and
    post), write z, read f, write x' -> s * (3nC + 2C)."""
    return s * (3 * n * c + 2 * c)


def _fwd_bytes(n, c, sx, sf):
    """Forward bytes per token with x (and z, x') of sx bytes and f of sf bytes:
    pre reads x and writes z, post reads x and f and writes x'."""
    return sx * (3 * n * c + c) + sf * c


def _bwd_bytes(n, c, sx, sf):
    """Backward bytes per token: the merge backward reads dx', x, f and writes
    dx_post, df; the coefficient backward reads x, dz, dx_post and writes dx."""
    return sx * (6 * n * c + c) + sf * 2 * c


def _profiled_traffic(kernel, n, c, t, with_res, pre_path=1):
    """DRAM bytes (read + write) per launch of the dominant kernel from the
    committed ncu summary of this exact workload (profiles/*.md carries a line
    `traffic_bytes_per_launch: <int>` and the commit the capture was made at);
    None for other workloads.  This is a profiled figure, not measured in this
    run."""
    if (n, c, t, bool(with_res)) != (4, 768, 32768, True):
        return None
    pre_name = "pre_sr_kernel_config2.md" if pre_path == 2 else "pre_tc_kernel_config2.md"
    name = {"pre": pre_name, "post": "post_fwd_kernel_config2.md"}[kernel]
    path = os.path.join(ROOT, "profiles", name)
    out = {}
    try:
        with open(path) as f:
            for line in f:
                for key in ("traffic_bytes_per_launch", "captured_at_commit"):
                    if line.startswith(key + ":"):
                        out[key] = line.split(":", 1)[1].strip()
    except OSError:
        return None
    if "traffic_bytes_per_launch" not in out:
        return None
    return (int(out["traffic_bytes_per_launch"]),
            f"profiled: ncu dram__bytes_read.sum + dram__bytes_write.sum, profiles/{name}, "
            f"captured at commit {out.get('captured_at_commit', 'unknown')}")


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


def _cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def _cpu_reference(n, c, tokens, budget_s, min_runs, max_runs, dtype=torch.float32):
    """The reference's pure-PyTorch path (oracle restatement), f = identity,
    on a bounded token sample; returns the per-run wall times."""
    from oracle import mhc_oracle as O
    torch.set_num_threads(os.cpu_count() or 1)
    gen = torch.Generator().manual_seed(0)
    x = torch.randn(1, tokens, n * c, generator=gen).to(dtype)
    p = O.make_full_params(n, c, generator=gen, dtype=dtype)
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


class LayerBench:
    """One mHC layer's buffers and its C-ABI calls: the forward (mhc_pre_fwd,
    then mhc_post_fwd) and the backward (mhc_post_bwd, then mhc_pre_bwd),
    launched on `stream`.  x ~ N(0, 1) in `x_dtype`, phi ~ N(0, 0.02), all
    alpha = 0.01, biases 0, 20 Sinkhorn iterations when the layer has H_res;
    the sublayer output f is a random-init SwiGLU C -> 2048 -> C of z in torch
    (bf16 weights, output in `f_dtype`), evaluated once before timing."""

    def __init__(self, t, n, c, with_res, x_dtype, f_dtype, dev, stream, seed):
        import torch.nn.functional as F

        from model import _native as nat
        from model.mhc_fused import _params
        self.nat, self.L = nat, nat.lib()
        self.t, self.n, self.c, self.with_res = t, n, c, with_res
        self.iters = 20 if with_res else 0
        self.fd = 2 * n + (n * n if with_res else 0)
        self.sptr = stream.cuda_stream
        self.xc, self.fc = nat.dtype_code(x_dtype), nat.dtype_code(f_dtype)
        g = torch.Generator(device=dev).manual_seed(seed)
        self.x = torch.randn(t, n * c, device=dev, generator=g).to(x_dtype)
        a = torch.tensor(0.01, device=dev)
        bn = torch.zeros(n, device=dev)
        ps = [torch.randn(n * c, self.fd, device=dev, generator=g) * 0.02, a, bn, a.clone(), bn.clone()]
        if with_res:
            ps += [a.clone(), torch.zeros(n, n, device=dev)]
        self.ps = _params(*ps)
        self.z = torch.empty(t, c, device=dev, dtype=x_dtype)
        self.h_post = torch.empty(t, n, device=dev)
        self.h_res = torch.empty(t, n, n, device=dev) if with_res else None
        self.inv = torch.empty(t, device=dev)
        self.mix = torch.empty(t, self.fd, device=dev)
        self.out = torch.empty_like(self.x)
        self.ws = nat.workspace(self.L.mhc_pre_fwd_workspace(t, n, c, int(with_res)), dev)
        self.pre()
        w1 = torch.randn(2048, c, device=dev, dtype=torch.bfloat16, generator=g) * 0.02
        w2 = torch.randn(2048, c, device=dev, dtype=torch.bfloat16, generator=g) * 0.02
        w3 = torch.randn(c, 2048, device=dev, dtype=torch.bfloat16, generator=g) * 0.02
        zb = self.z.to(torch.bfloat16)
        self.f = ((F.silu(zb @ w1.t()) * (zb @ w2.t())) @ w3.t()).to(f_dtype)
        self.pre_path = self.L.mhc_last_path()
        self._bwd_ready = False

    def pre(self, x=None):
        nat, ps = self.nat, self.ps
        a_res, b_res = (ps[5], ps[6]) if self.with_res else (None, None)
        st = self.L.mhc_pre_fwd(nat.ptr(self.x if x is None else x), self.xc, self.t, self.n, self.c,
                                nat.ptr(ps[0]), nat.ptr(ps[1]), nat.ptr(ps[2]), nat.ptr(ps[3]), nat.ptr(ps[4]),
                                nat.ptr(a_res), nat.ptr(b_res), nat.F32, int(self.with_res), int(self.with_res),
                                self.iters, 2.0, 1e-6, 1e-6, 1e-6, nat.ptr(self.z), None, nat.ptr(self.h_post),
                                nat.ptr(self.h_res), nat.F32, nat.ptr(self.inv), nat.ptr(self.mix),
                                nat.ptr(self.ws), self.ws.numel(), self.sptr)
        nat.check(st, "mhc_pre_fwd")

    def post(self):
        nat = self.nat
        st = self.L.mhc_post_fwd(nat.ptr(self.x), self.xc, nat.ptr(self.h_res), nat.F32, nat.ptr(self.h_post),
                                 nat.F32, nat.ptr(self.f), self.fc, nat.ptr(self.out), self.t, self.n, self.c,
                                 0, 0, 0.0, None, self.sptr)
        nat.check(st, "mhc_post_fwd")

    def _bwd_buffers(self):
        dev = self.x.device
        g = torch.Generator(device=dev).manual_seed(99)
        self.dout = torch.randn(self.x.shape, device=dev, generator=g).to(self.x.dtype)
        self.dz = torch.randn(self.z.shape, device=dev, generator=g).to(self.z.dtype)
        self.dx_post = torch.empty_like(self.x)
        self.dx = torch.empty_like(self.x)
        self.dh_res = torch.empty(self.t, self.n * self.n, device=dev) if self.with_res else None
        self.dh_post = torch.empty(self.t, self.n, device=dev)
        self.df = torch.empty_like(self.f)
        self.gps = [torch.empty_like(p, dtype=torch.float32) for p in self.ps]
        self.bws = self.nat.workspace(self.L.mhc_pre_bwd_workspace(self.t, self.n, self.c, int(self.with_res),
                                                                   int(self.with_res), self.iters), dev)
        self._bwd_ready = True

    def bwd(self):
        if not self._bwd_ready:
            self._bwd_buffers()
        nat, ps, gps = self.nat, self.ps, self.gps
        a_res, b_res = (ps[5], ps[6]) if self.with_res else (None, None)
        g_res = (gps[5], gps[6]) if self.with_res else (None, None)
        st = self.L.mhc_post_bwd(nat.ptr(self.dout), nat.ptr(self.x), self.xc, nat.ptr(self.h_res), nat.F32,
                                 nat.ptr(self.h_post), nat.F32, nat.ptr(self.f), self.fc, nat.ptr(self.dx_post),
                                 nat.ptr(self.dh_res), nat.ptr(self.dh_post), nat.ptr(self.df), self.t, self.n,
                                 self.c, self.sptr)
        nat.check(st, "mhc_post_bwd")
        st = self.L.mhc_pre_bwd(nat.ptr(self.x), self.xc, self.t, self.n, self.c, nat.ptr(ps[0]), nat.ptr(ps[1]),
                                nat.ptr(ps[2]), nat.ptr(ps[3]), nat.ptr(ps[4]), nat.ptr(a_res), nat.ptr(b_res),
                                nat.F32, int(self.with_res), int(self.with_res), self.iters, 2.0, 1e-6, 1e-6, 1e-6,
                                nat.ptr(self.inv), nat.ptr(self.mix), nat.ptr(self.dz), None, nat.ptr(self.dh_post),
                                nat.ptr(self.dh_res), nat.F32, nat.ptr(self.dx_post), nat.ptr(self.dx),
                                nat.ptr(gps[0]), nat.ptr(gps[1]), nat.ptr(gps[2]), nat.ptr(gps[3]),
                                nat.ptr(gps[4]), nat.ptr(g_res[0]), nat.ptr(g_res[1]), nat.ptr(self.bws),
                                self.bws.numel(), self.sptr)
        nat.check(st, "mhc_pre_bwd")

    def input_bytes(self):
        return self.x.numel() * self.x.element_size()


L2_FLUSH_BYTES = 256 << 20  # twice the B200's 126 MB L2


def _time_steps(fns, steps, warmup, stream, flush=None):
    """Per-step device time of calling `fns` in order, CUDA events on `stream`
    around each step (and around each fn).  With `flush`, a buffer larger than
    L2 is rewritten between steps, outside the events.  Returns (median step
    ms, mean ms per fn)."""
    for _ in range(warmup):
        for fn in fns:
            fn()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(len(fns) + 1)] for _ in range(steps)]
    torch.cuda.synchronize()
    for i in range(steps):
        if flush is not None:
            flush.add_(1)
        ev[i][0].record(stream)
        for k, fn in enumerate(fns):
            fn()
            ev[i][k + 1].record(stream)
    torch.cuda.synchronize()
    step = sorted(e[0].elapsed_time(e[-1]) for e in ev)[steps // 2]
    per = [sum(e[k].elapsed_time(e[k + 1]) for e in ev) / steps for k in range(len(fns))]
    return step, per


def _max_over_ranks(v, world, dev):
    if world <= 1:
        return v
    import torch.distributed as dist
    tt = torch.tensor([float(v)], device=dev)
    dist.all_reduce(tt, op=dist.ReduceOp.MAX)
    return float(tt.item())


def _layer_entry(lb, world, dev, steps, warmup, stream, peak, flush, with_bwd, sx, sf):
    """Forward (and backward) throughput of one LayerBench, whole job."""
    fl = flush if lb.input_bytes() < L2_FLUSH_BYTES else None
    f_ms, (pre_ms, post_ms) = _time_steps([lb.pre, lb.post], steps, warmup, stream, fl)
    f_ms = _max_over_ranks(f_ms, world, dev)
    n, c, t = lb.n, lb.c, lb.t
    fb = _fwd_bytes(n, c, sx, sf)
    alt_pre = None
    if lb.pre_path == 1 and sx == 2:
        prev = lb.L.mhc_set_path_policy(lb.nat.PATH_SINGLE_READ)
        _, (p_ms,) = _time_steps([lb.pre], steps, warmup, stream, fl)
        if lb.L.mhc_last_path() == 2:
            alt_pre = p_ms
        lb.L.mhc_set_path_policy(prev)
    gen_pre = None
    if lb.pre_path == lb.nat.RAN_FP32_STREAM:
        # the fp32-stream tensor-core kernel ran: the generic CUDA-core pre beside it
        prev = lb.L.mhc_set_path_policy(lb.nat.PATH_GENERIC)
        _, (p_ms,) = _time_steps([lb.pre], steps, warmup, stream, fl)
        if lb.L.mhc_last_path() == 0:
            gen_pre = p_ms
        lb.L.mhc_set_path_policy(prev)
    e = {"tokens_per_gpu": t, "tokens_per_s": world * t / (f_ms / 1e3), "ms_per_step": f_ms,
         "pre_single_read_ms": alt_pre, "pre_generic_ms": gen_pre,
         "algorithmic_bytes_per_token": fb, "hbm_gbs_per_gpu": fb * t / (f_ms / 1e3) / 1e9,
         "frac_of_measured": fb * t / (f_ms / 1e3) / 1e9 / peak,
         "per_call_ms": {"pre": pre_ms, "post": post_ms}, "pre_path": lb.pre_path,
         "l2": "flushed between steps" if fl is not None else "inputs larger than L2"}
    if with_bwd:
        b_ms, _ = _time_steps([lb.bwd], max(5, steps // 2), 3, stream, fl)
        b_ms = _max_over_ranks(b_ms, world, dev)
        bb = _bwd_bytes(n, c, sx, sf)
        e["backward"] = {"ms_per_step": b_ms, "tokens_per_s": world * t / (b_ms / 1e3),
                         "algorithmic_bytes_per_token": bb,
                         "frac_of_measured": bb * t / (b_ms / 1e3) / 1e9 / peak,
                         "bwd_path": lb.L.mhc_last_path()}
    return e


class PostPreBench:
    """The step between two consecutive sublayers on a LayerBench's buffers:
    the merge of this sublayer (x, f, H_res, H_post -> x') followed by the
    coefficient pass of the next (same parameters) on x', either as the two
    kernels (mhc_post_fwd, mhc_pre_fwd; plus torch's rms_norm on z for the
    next sublayer's input norm) or as one mhc_post_pre_fwd call under
    MHC_PATH_FUSED_POST_PRE (the fused merge + coefficient kernel, with the
    norm in the same kernel)."""

    def __init__(self, lb):
        self.lb = lb
        c = lb.c
        self.x2 = torch.empty_like(lb.x)
        self.z2 = torch.empty_like(lb.z)
        self.y = torch.empty_like(lb.z)
        self.hp2 = torch.empty_like(lb.h_post)
        self.hr2 = torch.empty_like(lb.h_res) if lb.with_res else None
        self.inv2 = torch.empty_like(lb.inv)
        self.mix2 = torch.empty_like(lb.mix)
        self.nw = torch.ones(c, device=lb.x.device)
        self.nw_b = self.nw.to(lb.z.dtype)

    def pair(self):
        self.lb.post()
        self.lb.pre(self.lb.out)

    def pair_norm(self):
        self.pair()
        torch.nn.functional.rms_norm(self.lb.z, (self.lb.c,), self.nw_b, 1e-6)

    def fused(self, norm=False, policy=None):
        lb, nat = self.lb, self.lb.nat
        ps = lb.ps
        prev = lb.L.mhc_set_path_policy(nat.PATH_FUSED_POST_PRE if policy is None else policy)
        a_res, b_res = (ps[5], ps[6]) if lb.with_res else (None, None)
        st = lb.L.mhc_post_pre_fwd(
            nat.ptr(lb.x), lb.xc, nat.ptr(lb.h_res), nat.ptr(lb.h_post), nat.F32, nat.ptr(lb.f), lb.fc,
            nat.ptr(self.x2), lb.t, lb.n, lb.c, nat.ptr(ps[0]), nat.ptr(ps[1]), nat.ptr(ps[2]), nat.ptr(ps[3]),
            nat.ptr(ps[4]), nat.ptr(a_res), nat.ptr(b_res), nat.F32, int(lb.with_res), int(lb.with_res), lb.iters,
            2.0, 1e-6, 1e-6, 1e-6, nat.ptr(self.z2), None, nat.ptr(self.hp2), nat.ptr(self.hr2), nat.F32,
            nat.ptr(self.inv2), nat.ptr(self.mix2), nat.ptr(self.nw) if norm else None, nat.F32, 1e-6,
            nat.ptr(self.y) if norm else None, nat.ptr(lb.ws), lb.ws.numel(), lb.sptr)
        lb.L.mhc_set_path_policy(prev)
        nat.check(st, "mhc_post_pre_fwd")

    def fused_norm(self):
        self.fused(True)

    def call(self):
        """mhc_post_pre_fwd under the default policy (merge kernel, the fastest
        coefficient kernel, no norm)."""
        self.fused(False, self.lb.nat.PATH_AUTO)

    def call_norm(self):
        """mhc_post_pre_fwd under the default policy with the input norm (merge
        kernel, the fastest coefficient kernel, the row RMSNorm kernel)."""
        self.fused(True, self.lb.nat.PATH_AUTO)


def _post_pre_entry(lb, world, dev, steps, warmup, stream, peak):
    """Two-kernel pair vs the fused merge + coefficient kernel, without and
    with the next sublayer's input RMSNorm (whole job, median step)."""
    pb = PostPreBench(lb)
    n, c, t = lb.n, lb.c, lb.t
    out = {"tokens_per_gpu": t, "n": n, "C": c, "with_res": lb.with_res}
    pair_b = 2 * (3 * n * c + 2 * c)
    fused_b = 2 * (2 * n * c + 2 * c)
    for key, fns, nbytes in (("pair", [pb.pair], pair_b), ("pair_norm", [pb.pair_norm], pair_b + 2 * 2 * c),
                             ("fused", [pb.fused], fused_b), ("fused_norm", [pb.fused_norm], fused_b + 2 * c),
                             ("call", [pb.call], pair_b), ("call_norm", [pb.call_norm], pair_b + 2 * 2 * c)):
        ms, _ = _time_steps(fns, steps, warmup, stream)
        ms = _max_over_ranks(ms, world, dev)
        gbs = nbytes * t / (ms / 1e3) / 1e9
        out[key] = {"ms": ms, "tokens_per_s": world * t / (ms / 1e3), "algorithmic_bytes_per_token": nbytes,
                    "gbs": gbs, "frac_of_measured": gbs / peak}
        if key.startswith("fused") or key.startswith("call"):
            out[key]["path"] = lb.L.mhc_last_path()
    out["speedup"] = out["pair"]["ms"] / out["fused"]["ms"]
    out["speedup_with_norm"] = out["pair_norm"]["ms"] / out["fused_norm"]["ms"]
    out["call_norm_speedup"] = out["pair_norm"]["ms"] / out["call_norm"]["ms"]
    out["calls"] = ("pair: mhc_post_fwd + mhc_pre_fwd (+ torch rms_norm on z); fused: one mhc_post_pre_fwd "
                    "under MHC_PATH_FUSED_POST_PRE (+ the norm in the same kernel); call: one mhc_post_pre_fwd "
                    "under the default policy (merge kernel, fastest coefficient kernel, row RMSNorm kernel)")
    return out


def run_post_pre(args, rank, world, local_rank):
    """--workload post_pre: config 2's step between two sublayers (merge of one,
    coefficient pass and input RMSNorm of the next), as the two-kernel pair and
    as the fused merge + coefficient kernel, K steps each after W warm-ups."""
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    peak, peak_kind = _peaks()
    lb = LayerBench(args.tokens, 4, 768, args.variant == "full", torch.bfloat16, torch.bfloat16, dev, stream,
                    66 + rank)
    e = _post_pre_entry(lb, world, dev, args.steps, args.warmup, stream, peak)
    if rank != 0:
        return
    ms = e["fused"]["ms"]
    print(json.dumps({"metric": "mHC post+pre step tokens/s", "value": e["fused"]["tokens_per_s"],
                      "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                      "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                      "dtype": "bf16", "data": "synthetic",
                      "config": {"workload": f"post_pre: merge of sublayer l + coefficient pass of l+1, "
                                             f"{args.tokens} tokens/GPU, C=768, n=4, {args.variant}",
                                 "l2": "inputs larger than L2" if args.tokens >= 16384 else "inputs fit in L2"},
                      "peak_kind": peak_kind, "post_pre": e}))


def run_fp32_stream(args, rank, world, local_rank):
    """--workload fp32_stream: the layer with an fp32 residual stream and a bf16
    sublayer output (the reference trainers' bf16-autocast setting), forward
    and backward, K steps each after W warm-ups, at --tokens per GPU."""
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    peak, peak_kind = _peaks()
    c = args.C or 768
    lb = LayerBench(args.tokens, 4, c, args.variant == "full", torch.float32, torch.bfloat16, dev, stream, 77 + rank)
    flush = torch.empty(L2_FLUSH_BYTES // 4, device=dev)
    e = _layer_entry(lb, world, dev, args.steps, args.warmup, stream, peak, flush, not args.no_bwd, 4, 2)
    if rank != 0:
        return
    print(json.dumps({"metric": "mHC layer tokens/s", "value": e["tokens_per_s"], "unit": "tokens/s",
                      "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": e["ms_per_step"],
                      "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
                      "data": "synthetic",
                      "config": {"workload": f"fp32 stream: x fp32, f bf16, {args.tokens} tokens/GPU, C={c}, n=4, "
                                             f"{args.variant}", "l2": e["l2"]},
                      "peak_kind": peak_kind, "fp32_stream": e}))


def run_ours(args, rank, world, local_rank):
    import torch.distributed as dist

    from model import _native as nat

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    peak, peak_kind = _peaks()
    n, c = 4, 768
    with_res = args.variant == "full"
    if args.variant == "nohres" and args.C:
        c = args.C
    t = args.tokens
    torch.manual_seed(1234 + rank)
    lb = LayerBench(t, n, c, with_res, torch.bfloat16, torch.bfloat16, dev, stream, 1234 + rank)
    L = lb.L
    x, out = lb.x, lb.out
    fused_path = lb.pre_path
    launches_per_step = 2 if fused_path else 3  # fused coefficient+aggregate (or 2 generic kernels), merge
    bytes_tok = _layer_bytes(n, c, 2, with_res)
    pre_bytes = 2 * (n * c + c)
    post_bytes = 2 * (2 * n * c + c)

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        lb.pre()
        lb.post()
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
        lb.pre()
        e1.record(stream)
        lb.post()
        e2.record(stream)
    t_stop.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    clocks = sampler.stop()
    total_ms = _max_over_ranks(t_start.elapsed_time(t_stop), world, dev)
    pre_ms = [e0.elapsed_time(e1) for e0, e1, _ in ev]
    post_ms = [e1.elapsed_time(e2) for _, e1, e2 in ev]

    # ---- the other fused forward kernel on the same inputs, for comparison -----
    alt = None
    if fused_path in (1, 2):
        other = nat.PATH_SINGLE_READ if fused_path == 1 else nat.PATH_TWO_READ
        prev = L.mhc_set_path_policy(other)
        _, (alt_pre,) = _time_steps([lb.pre], max(10, args.steps // 4), 3, stream)
        alt_path = L.mhc_last_path()
        L.mhc_set_path_policy(prev)
        lb.pre()
        if alt_path != fused_path:
            alt = {"pre_ms": alt_pre, "path": alt_path,
                   "kernel": {2: "single-read (x read from HBM once, kept in TMEM)",
                              1: "two-read (x read from HBM, then again from L2)"}.get(alt_path, "generic")}

    # ---- backward of the layer (training config), reported beside the forward --
    bwd = None
    if not args.no_bwd:
        b_ms, _ = _time_steps([lb.bwd], max(3, min(args.steps, 20)), 3, stream)
        b_ms = _max_over_ranks(b_ms, world, dev)
        bb = _bwd_bytes(n, c, 2, 2)
        gbs = bb * t / (b_ms / 1e3) / 1e9
        bwd = {"ms_per_step": b_ms, "tokens_per_s": world * t / (b_ms / 1e3), "algorithmic_bytes_per_token": bb,
               "gbs": gbs, "frac_of_measured": gbs / peak, "bwd_path": L.mhc_last_path(),
               "calls": "mhc_post_bwd + mhc_pre_bwd (median step, CUDA events)"}

    # ---- end to end through the public API with host buffers -------------------
    # A step copies x and f from pinned host memory, runs mhc_pre_fwd and
    # mhc_post_fwd through the C-ABI and copies x' back.  The batch goes in
    # E2E_CHUNKS token chunks rotated over E2E_STREAMS streams, so one chunk's
    # host-to-device copy overlaps another's device-to-host copy (separate copy
    # engines) and the kernels; every byte is still copied inside the step.  The
    # same copies without the kernels give the host link's ceiling.
    e2e = None
    if not args.no_e2e:
        e2e = _e2e(lb, args, world, dev, stream, barrier)

    # ---- sub-measurements of the other BASELINE configurations ----------------
    extra = {}
    if not args.no_extra and args.variant == "full" and t == 16 * 2048:
        flush = torch.empty(L2_FLUSH_BYTES // 4, device=dev)
        del lb
        torch.cuda.empty_cache()
        sweep = {}
        for ts in (4096, 16384, 65536, 262144):
            lbs = LayerBench(ts, n, c, True, torch.bfloat16, torch.bfloat16, dev, stream, 77 + rank)
            sweep[str(ts)] = _layer_entry(lbs, world, dev, 20, 3, stream, peak, flush, False, 2, 2)
            del lbs
            torch.cuda.empty_cache()
        extra["sweep"] = sweep
        lbs = LayerBench(t, n, c, True, torch.bfloat16, torch.bfloat16, dev, stream, 66 + rank)
        extra["post_pre"] = _post_pre_entry(lbs, world, dev, 20, 3, stream, peak)
        del lbs
        torch.cuda.empty_cache()
        for cc in (768, 1024):
            lbs = LayerBench(t, n, cc, False, torch.bfloat16, torch.bfloat16, dev, stream, 88 + rank)
            extra[f"nohres_c{cc}"] = _layer_entry(lbs, world, dev, 20, 3, stream, peak, flush, True, 2, 2)
            del lbs
            torch.cuda.empty_cache()
        lbs = LayerBench(t, n, c, True, torch.float32, torch.bfloat16, dev, stream, 99 + rank)
        extra["fp32_stream"] = _layer_entry(lbs, world, dev, 20, 3, stream, peak, flush, True, 4, 2)
        extra["fp32_stream"]["setting"] = ("x fp32, f bf16: the residual stream under the reference trainers' "
                                           "bf16 autocast with fp32 weights")
        del lbs, flush
        torch.cuda.empty_cache()
        if not args.no_train:
            extra["train_step"] = _train_step_entry(args, rank, world, dev)

    if rank != 0:
        return
    step_ms = total_ms / args.steps
    value = world * t * args.steps / (total_ms / 1e3)
    pre_avg = sum(pre_ms) / len(pre_ms)
    post_avg = sum(post_ms) / len(post_ms)
    calls = {"pre": (pre_avg, pre_bytes * t), "post": (post_avg, post_bytes * t)}
    dom = max(calls, key=lambda k: calls[k][0])
    d_ms, d_bytes = calls[dom]
    achieved = d_bytes / (d_ms / 1e3) / 1e9
    layer_gbs = bytes_tok * t / (step_ms / 1e3) / 1e9  # per GPU, whole step
    traffic = _profiled_traffic(dom, n, c, t, with_res, fused_path)

    cpu = None
    if not args.no_cpu_baseline:
        times = _cpu_reference(n, c, args.cpu_tokens, args.cpu_budget, 2, 50)
        cpu = {"value": args.cpu_tokens / statistics.median(times), "unit": "tokens/s",
               "cores": torch.get_num_threads(), "kind": "port", "cpu_model": _cpu_model(),
               "sample": f"{args.cpu_tokens} tokens x {len(times)} runs (median), C=768, n=4, fp32, "
                         f"f=identity, 20 Sinkhorn iters; oracle restatement of _forward_ref"}
        # [2, 512, 4, 512] fp32 on the CPU, and the config-2
        # shape in bf16 (bounded samples)
        t1 = _cpu_reference(4, 512, 1024, 3.0, 2, 20)
        cpu["config1_fp32"] = {"value": 1024 / statistics.median(t1), "unit": "tokens/s",
                               "sample": f"[2,512,4,512] fp32 x {len(t1)} runs (median)"}
        tb = _cpu_reference(n, c, 1024, 5.0, 2, 10, dtype=torch.bfloat16)
        cpu["config2_bf16"] = {"value": 1024 / statistics.median(tb), "unit": "tokens/s",
                               "sample": f"1024 tokens, C=768, n=4, bf16 x {len(tb)} runs (median)"}

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
        "pre_path": {2: "single-read sm_100a cluster kernel (TMA + tcgen05 + TMEM retention + DSMEM)",
                     1: "two-read sm_100a cluster kernel (TMA + tcgen05 + DSMEM, second read from L2)",
                     0: "generic CUDA-core kernels"}[fused_path],
        "pre_other_kernel": alt,
        "roofline": {"kernel": dom, "bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_kind": peak_kind,
                     "traffic": traffic[0] if traffic else None,
                     "traffic_kind": traffic[1] if traffic else None,
                     "algorithmic_bytes_per_launch": d_bytes},
        "cpu_baseline": cpu,
        "backward": bwd,
        "e2e": e2e,
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks,
    }
    line.update(extra)
    print(json.dumps(line), flush=True)


def _e2e(lb, args, world, dev, stream, barrier):
    nat, L = lb.nat, lb.L
    n, c, t, with_res, iters, fd = lb.n, lb.c, lb.t, lb.with_res, lb.iters, lb.fd
    ps = lb.ps
    a_res, b_res = (ps[5], ps[6]) if with_res else (None, None)
    E2E_CHUNKS, E2E_STREAMS = 8, 3
    x_h = lb.x.cpu().pin_memory()
    f_h = lb.f.cpu().pin_memory()
    o_h = torch.empty_like(x_h).pin_memory()
    bounds = [t * i // E2E_CHUNKS for i in range(E2E_CHUNKS + 1)]
    cmax = max(bounds[i + 1] - bounds[i] for i in range(E2E_CHUNKS))
    streams = [torch.cuda.Stream(dev) for _ in range(E2E_STREAMS)]
    slots = []
    for _ in range(E2E_STREAMS):
        slots.append(dict(
            x=torch.empty(cmax, n * c, device=dev, dtype=torch.bfloat16),
            f=torch.empty(cmax, c, device=dev, dtype=torch.bfloat16),
            o=torch.empty(cmax, n * c, device=dev, dtype=torch.bfloat16),
            z=torch.empty(cmax, c, device=dev, dtype=torch.bfloat16),
            hp=torch.empty(cmax, n, device=dev), hr=torch.empty(cmax, n, n, device=dev) if with_res else None,
            inv=torch.empty(cmax, device=dev), mix=torch.empty(cmax, fd, device=dev),
            ws=nat.workspace(L.mhc_pre_fwd_workspace(cmax, n, c, int(with_res)), dev)))

    def kernels_on(sl, m, sp):
        r = L.mhc_pre_fwd(nat.ptr(sl["x"]), nat.BF16, m, n, c, nat.ptr(ps[0]), nat.ptr(ps[1]), nat.ptr(ps[2]),
                          nat.ptr(ps[3]), nat.ptr(ps[4]), nat.ptr(a_res), nat.ptr(b_res), nat.F32,
                          int(with_res), int(with_res), iters, 2.0, 1e-6, 1e-6, 1e-6, nat.ptr(sl["z"]), None,
                          nat.ptr(sl["hp"]), nat.ptr(sl["hr"]), nat.F32, nat.ptr(sl["inv"]), nat.ptr(sl["mix"]),
                          nat.ptr(sl["ws"]), sl["ws"].numel(), sp)
        nat.check(r, "mhc_pre_fwd")
        r = L.mhc_post_fwd(nat.ptr(sl["x"]), nat.BF16, nat.ptr(sl["hr"]), nat.F32, nat.ptr(sl["hp"]), nat.F32,
                           nat.ptr(sl["f"]), nat.BF16, nat.ptr(sl["o"]), m, n, c, 0, 0, 0.0, None, sp)
        nat.check(r, "mhc_post_fwd")

    def chunk(k, kernels):
        lo, hi = bounds[k], bounds[k + 1]
        m = hi - lo
        st = streams[k % E2E_STREAMS]
        sl = slots[k % E2E_STREAMS]
        sp = st.cuda_stream
        with torch.cuda.stream(st):
            sl["x"][:m].copy_(x_h[lo:hi], non_blocking=True)
            sl["f"][:m].copy_(f_h[lo:hi], non_blocking=True)
        if kernels:
            kernels_on(sl, m, sp)
        with torch.cuda.stream(st):
            o_h[lo:hi].copy_(sl["o"][:m], non_blocking=True)

    def e2e_step(kernels=True):
        go = torch.cuda.Event()
        go.record(stream)
        for st in streams:
            st.wait_event(go)
        for k in range(E2E_CHUNKS):
            chunk(k, kernels)
        for st in streams:
            done = torch.cuda.Event()
            done.record(st)
            stream.wait_event(done)

    def timed(kernels, k_steps):
        for _ in range(max(1, args.warmup)):
            e2e_step(kernels)
        barrier()
        torch.cuda.synchronize(dev)
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        for _ in range(k_steps):
            e2e_step(kernels)
        s1.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        return _max_over_ranks(s0.elapsed_time(s1), world, dev)

    k_e2e = max(1, min(args.steps, 5))
    copy_ms = timed(False, k_e2e)
    e_ms = timed(True, k_e2e)
    # check every copied-back chunk: bit for bit against the same per-chunk
    # calls on device-resident inputs, and against the full-batch device step
    # to one bf16 rounding (a 4K-token chunk may run a different fused kernel
    # than the whole batch, with a different summation order)
    ref = torch.empty_like(lb.out)
    sl = slots[0]
    for k in range(E2E_CHUNKS):
        lo, hi = bounds[k], bounds[k + 1]
        sl["x"][:hi - lo].copy_(lb.x[lo:hi])
        sl["f"][:hi - lo].copy_(lb.f[lo:hi])
        kernels_on(sl, hi - lo, stream.cuda_stream)
        ref[lo:hi].copy_(sl["o"][:hi - lo])
    lb.pre()
    lb.post()
    torch.cuda.synchronize(dev)
    got = o_h.to(dev)
    e2e_ok = bool(torch.equal(got, ref))
    e2e_close = bool((got.float() - lb.out.float()).abs().max().item()
                     <= 2 ** -7 * lb.out.float().abs().max().item())
    value = world * t * k_e2e / (e_ms / 1e3)
    ceiling = world * t * k_e2e / (copy_ms / 1e3)
    return {"value": value, "unit": "tokens/s",
            "h2d_bytes_per_step": int(x_h.numel() * 2 + f_h.numel() * 2),
            "d2h_bytes_per_step": int(o_h.numel() * 2), "steps": k_e2e, "ms_per_step": e_ms / k_e2e,
            "pipeline": f"{E2E_CHUNKS} token chunks over {E2E_STREAMS} streams (H2D / kernels / D2H overlap)",
            "result_matches_device_step": e2e_ok,
            "result_matches_full_batch_to_bf16": e2e_close,
            "host_link_ceiling": {"tokens_per_s": ceiling, "ms_per_step": copy_ms / k_e2e,
                                  "note": "the same pinned H2D + D2H copies without the kernels, all ranks at once"},
            "frac_of_host_link_ceiling": value / ceiling}


def _train_step_entry(args, rank, world, dev):
    """BASELINE configs[4] inside the default line: the MoE + mHC training step
    at 8 x 2048 tokens per GPU (global 64 x 2048 at 8 GPUs), with the gradient
    all-reduce timed on its own."""
    import torch.nn.functional as F
    torch.manual_seed(1234 + rank)
    model = _build_decoder(moe=True, dev=dev)
    batch, seq = 8, 2048
    gen = torch.Generator(device=dev).manual_seed(77 + rank)
    ids = torch.randint(0, 6400, (batch, seq), device=dev, generator=gen)
    labels = torch.randint(0, 6400, (batch, seq), device=dev, generator=gen)
    params = list(model.parameters())
    opt = torch.optim.AdamW(params, lr=1e-4, fused=True)
    stream = torch.cuda.current_stream(dev)
    buckets = GradBuckets(params, world) if world > 1 else None
    ar = []

    def step(timed):
        logits = model(ids)
        loss = F.cross_entropy(logits.view(-1, logits.shape[-1]).float(), labels.view(-1)) + model.aux_loss()
        loss.backward()
        if buckets is not None:
            # the buckets were all-reduced during backward as they completed;
            # what remains on the stream after backward is the exposed part
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            buckets.finish()
            e1.record(stream)
            if timed:
                ar.append((e0, e1))
        opt.step()
        if buckets is not None:
            buckets.zero()
        else:
            opt.zero_grad(set_to_none=True)

    for _ in range(3):
        step(False)
    torch.cuda.synchronize(dev)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    k = 5
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record(stream)
    for _ in range(k):
        step(True)
    s1.record(stream)
    torch.cuda.synchronize(dev)
    ms = _max_over_ranks(s0.elapsed_time(s1) / k, world, dev)
    ar_ms = _max_over_ranks(sum(a.elapsed_time(b) for a, b in ar) / k, world, dev) if ar else 0.0
    del model, opt
    torch.cuda.empty_cache()
    return {"tokens_per_s": world * batch * seq / (ms / 1e3), "ms_per_step": ms, "tokens_per_gpu": batch * seq,
            "global_batch": f"{world * batch} x {seq}", "allreduce_exposed_ms_per_step": ar_ms,
            "allreduce_exposed_share": ar_ms / ms if ms else 0.0,
            "allreduce": "bucketed (32 MB), launched from gradient hooks during backward, fixed bucket order; "
                         "exposed = the time from the end of backward to the last bucket's completion",
            "model": "MiniMind MoE (8 experts, top-2) + mHC on every sublayer: hidden 768, 8 layers, vocab 6400, "
                     "n=4, 20 Sinkhorn iterations; fwd + bwd + gradient all-reduce + AdamW"}


# ---------------------------------------------------------------------------
# Model-level workloads
# ---------------------------------------------------------------------------

def _build_decoder(moe: bool, dev, n=4, hidden=768, layers=8, heads=8, kv_heads=4, inter=2048, vocab=6400,
                   experts=8, topk=2, moe_inter=None, theta=1e6, eps=1e-6, iters=20, use_mhc=1, chain=False,
                   aux_coef=5e-4, dtype=torch.bfloat16):
    """The reference's model with this build's mHC modules: a module tree whose
    state_dict keys, shapes and forward math are those of the reference's
    ``MiniMindForCausalLM`` with ``use_mhc`` 1 or 2 (``model/model_minimind.py``:
    ``Attention`` :163-250, ``FeedForward`` / ``MOEFeedForward`` :252-293,
    ``MiniMindBlock`` :295-340, ``MiniMindModel`` :353-403, tied ``lm_head``
    :405-415), so a reference checkpoint loads with ``strict=True``
    (``tests/test_gpu_model.py`` loads the reference's own weights and matches
    its logits and mHC gradients).  Attention runs through torch SDPA (causal,
    GQA), the reference's CUDA path minus the optional flash-attn library.  The
    MoE layer computes the same routing (softmax, top-k, renormalised) and
    auxiliary loss as the reference but groups each expert's rows with one sort
    instead of a mask per expert.  Random init N(0, 0.02) for the matrices."""
    import torch.nn as nn
    import torch.nn.functional as F

    from model.mhc_common import MHCHead, StreamExpand
    from model.mhc_fused import MHCConnection_Fused
    from model.mhc_fused_no_hres import MHCConnection_FusedNoHres

    hd = hidden // heads
    moe_inter = moe_inter or inter

    class Attention(nn.Module):
        def __init__(self):
            super().__init__()
            self.q_proj = nn.Linear(hidden, heads * hd, bias=False)
            self.k_proj = nn.Linear(hidden, kv_heads * hd, bias=False)
            self.v_proj = nn.Linear(hidden, kv_heads * hd, bias=False)
            self.o_proj = nn.Linear(heads * hd, hidden, bias=False)
            self.q_norm = nn.RMSNorm(hd, eps=eps)
            self.k_norm = nn.RMSNorm(hd, eps=eps)

        def forward(self, x, cos, sin):
            b, l, _ = x.shape
            q = self.q_norm(self.q_proj(x).view(b, l, heads, hd))
            k = self.k_norm(self.k_proj(x).view(b, l, kv_heads, hd))
            v = self.v_proj(x).view(b, l, kv_heads, hd)

            def rope(t):
                h = t.shape[-1] // 2
                rot = torch.cat((-t[..., h:], t[..., :h]), dim=-1)
                return (t * cos + rot * sin).to(t.dtype)

            q, k = rope(q), rope(k)
            o = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2),
                                               is_causal=True, enable_gqa=True)
            return self.o_proj(o.transpose(1, 2).reshape(b, l, heads * hd))

    class FeedForward(nn.Module):
        def __init__(self, width):
            super().__init__()
            self.gate_proj = nn.Linear(hidden, width, bias=False)
            self.down_proj = nn.Linear(width, hidden, bias=False)
            self.up_proj = nn.Linear(hidden, width, bias=False)

        def forward(self, x):
            return self.down_proj(F.silu(self.gate_proj(x)) * self.up_proj(x))

    class MOEFeedForward(nn.Module):
        """Softmax router, top-k experts, weights renormalised over the k."""
        def __init__(self):
            super().__init__()
            self.gate = nn.Linear(hidden, experts, bias=False)
            self.experts = nn.ModuleList([FeedForward(moe_inter) for _ in range(experts)])
            self.aux_loss = None

        def forward(self, x):
            shape = x.shape
            xf = x.reshape(-1, hidden)
            scores = torch.softmax(self.gate(xf), dim=-1)
            w, idx = scores.topk(topk, dim=-1)
            w = w / (w.sum(dim=-1, keepdim=True) + 1e-20)
            flat = idx.flatten()
            order = flat.argsort()
            tok = order // topk
            counts = torch.bincount(flat, minlength=experts).tolist()
            xs = xf.index_select(0, tok)
            # each expert's rows are zero-padded to a multiple of 1024, so the
            # GEMM shapes come from a small set (new shapes every step would
            # send the GEMM library back to its host-side selection each time)
            outs = []
            for e, c in zip(self.experts, xs.split(counts)):
                if c.shape[0] == 0:
                    continue
                pad = (-c.shape[0]) % 1024
                outs.append(e(F.pad(c, (0, 0, 0, pad)))[:c.shape[0]] if pad else e(c))
            ys = torch.cat(outs) if outs else xs[:0]
            ys = ys * w.flatten()[order].unsqueeze(1).to(ys.dtype)
            if self.training and aux_coef > 0:
                load = F.one_hot(idx, experts).float().mean(0)
                self.aux_loss = (load * scores.float().mean(0)).sum() * experts * aux_coef
            else:
                self.aux_loss = scores.new_zeros(())
            return torch.zeros_like(xf).index_add_(0, tok, ys.to(xf.dtype)).view(shape)

    conn = MHCConnection_Fused if use_mhc == 1 else MHCConnection_FusedNoHres

    class MiniMindBlock(nn.Module):
        def __init__(self):
            super().__init__()
            self.self_attn = Attention()
            self.mlp = MOEFeedForward() if moe else FeedForward(inter)
            self.attn_in_norm = nn.RMSNorm(hidden, eps=eps)
            self.ffn_in_norm = nn.RMSNorm(hidden, eps=eps)
            self.attn_mhc = conn(n, hidden, eps=eps)
            self.mlp_mhc = conn(n, hidden, eps=eps)
            if use_mhc == 1:
                # MiniMindBlock passes no sinkhorn_iters (module default 10); the
                # benchmark configs set it after construction
                self.attn_mhc.sinkhorn_iters = iters
                self.mlp_mhc.sinkhorn_iters = iters

        def forward(self, h, cos, sin):
            h = self.attn_mhc(h, lambda z: self.self_attn(self.attn_in_norm(z), cos, sin))
            return self.mlp_mhc(h, lambda z: self.mlp(self.ffn_in_norm(z)))

    class MiniMindModel(nn.Module):
        def __init__(self):
            super().__init__()
            self.embed_tokens = nn.Embedding(vocab, hidden)
            self.embed_up_norm = nn.Sequential(nn.RMSNorm(hidden, eps=eps), StreamExpand(n, hidden))
            self.layers = nn.ModuleList([MiniMindBlock() for _ in range(layers)])
            self.norm = nn.Sequential(MHCHead(n, hidden, eps=eps), nn.RMSNorm(hidden, eps=eps))
            self.use_chain = chain

        def forward(self, ids):
            l = ids.shape[1]
            pos = torch.arange(l, device=ids.device, dtype=torch.float32)
            inv = 1.0 / (theta ** (torch.arange(0, hd, 2, device=ids.device, dtype=torch.float32) / hd))
            ang = torch.outer(pos, inv)
            cos = torch.cat([ang.cos(), ang.cos()], dim=-1)[None, :, None, :]
            sin = torch.cat([ang.sin(), ang.sin()], dim=-1)[None, :, None, :]
            h = self.embed_up_norm(self.embed_tokens(ids))
            if self.use_chain:
                # every sublayer through the block-level API: the merge of one
                # sublayer, the coefficient pass and the input norm of the next
                # in one mhc_post_pre_fwd call (model/mhc_block.py)
                from model.mhc_block import mhc_chain
                steps = []
                for blk in self.layers:
                    steps.append((blk.attn_mhc, lambda y, blk=blk: blk.self_attn(y, cos, sin), blk.attn_in_norm))
                    steps.append((blk.mlp_mhc, blk.mlp, blk.ffn_in_norm))
                h = mhc_chain(h, steps)
            else:
                for blk in self.layers:
                    h = blk(h, cos, sin)
            return self.norm(h)

    class MiniMindForCausalLM(nn.Module):
        def __init__(self):
            super().__init__()
            self.model = MiniMindModel()
            self.lm_head = nn.Linear(hidden, vocab, bias=False)
            self.model.embed_tokens.weight = self.lm_head.weight

        def forward(self, ids):
            return self.lm_head(self.model(ids))

        def aux_loss(self):
            losses = [blk.mlp.aux_loss for blk in self.model.layers
                      if isinstance(blk.mlp, MOEFeedForward) and blk.mlp.aux_loss is not None]
            return sum(losses) if losses else None

    m = MiniMindForCausalLM()
    with torch.no_grad():
        for name, p in m.named_parameters():
            if p.dim() >= 2 and "mhc" not in name and "norm.0" not in name:
                p.normal_(0.0, 0.02)
    m = m.to(dev, dtype)
    # mHC parameters and their gradients stay fp32 (fp32 coefficient math)
    for mod in m.modules():
        if isinstance(mod, (MHCConnection_Fused, MHCConnection_FusedNoHres, MHCHead)):
            mod.float()
    return m


def allreduce_grads(params, world):
    """Average the gradients of `params` over the ranks: one flat bucket per
    parameter dtype (the fp32 mHC parameters, the bf16 rest), one NCCL
    all_reduce each.  Every rank reduces every parameter in the same order; a
    parameter that got no gradient on this rank (an expert no token was routed
    to) counts as zeros and receives the average, so the buckets, and the
    collective sequence, are identical on all ranks."""
    import torch.distributed as dist

    for dt in (torch.float32, torch.bfloat16):
        ps = [p for p in params if p.dtype == dt]
        if not ps:
            continue
        flat = torch.cat([(p.grad if p.grad is not None else torch.zeros_like(p)).reshape(-1) for p in ps])
        dist.all_reduce(flat)
        flat.div_(world)
        off = 0
        for p in ps:
            g = flat[off:off + p.numel()].view_as(p)
            if p.grad is None:
                p.grad = g.clone()
            else:
                p.grad.copy_(g)
            off += p.numel()


class GradBuckets:
    """Gradient all-reduce overlapped with backward (what DDP does with
    gradient_as_bucket_view): each parameter's .grad is a view into a
    persistent flat buffer per dtype, cut into buckets of about `bucket_mb` in
    reverse creation order (backward produces gradients roughly in that
    order).  A post-accumulate hook counts a bucket's gradients; a bucket is
    launched as an asynchronous all_reduce once it is complete and every
    earlier bucket has been launched, so all ranks issue the same collectives
    in the same order.  finish() launches what backward left incomplete (a
    parameter that got no gradient on this rank, such as an expert no local
    token was routed to, contributes its zeroed view), waits, and averages.
    zero() clears the buffers in place; the views stay attached."""

    def __init__(self, params, world, bucket_mb=32):
        import torch.distributed as dist
        self.dist, self.world = dist, world
        self.params = [p for p in params if p.requires_grad]
        self.flat = {}
        self.buckets = []      # [dtype, start, end, [param ids], seen]
        self.owner = {}
        by_dtype = {}
        for p in reversed(self.params):
            by_dtype.setdefault(p.dtype, []).append(p)
        cap = int(bucket_mb * (1 << 20))
        for dt, ps in by_dtype.items():
            total = sum(p.numel() for p in ps)
            buf = torch.zeros(total, dtype=dt, device=ps[0].device)
            self.flat[dt] = buf
            off, cur = 0, None
            for p in ps:
                n = p.numel()
                if cur is None or (cur[2] - cur[1]) * buf.element_size() >= cap:
                    cur = [dt, off, off, [], 0]
                    self.buckets.append(cur)
                p.grad = buf[off:off + n].view_as(p)
                cur[2] = off + n
                cur[3].append(id(p))
                self.owner[id(p)] = cur
                off += n
        self.index = {id(b): i for i, b in enumerate(self.buckets)}
        self.handles = []
        self.next = 0
        self.hooks = [p.register_post_accumulate_grad_hook(self._ready) for p in self.params]

    def _ready(self, p):
        b = self.owner[id(p)]
        b[4] += 1
        while self.next < len(self.buckets) and self.buckets[self.next][4] == len(self.buckets[self.next][3]):
            self._launch(self.buckets[self.next])

    def _launch(self, b):
        dt, a, e = b[0], b[1], b[2]
        self.handles.append((self.dist.all_reduce(self.flat[dt][a:e], async_op=True), b))
        self.next += 1

    def finish(self):
        while self.next < len(self.buckets):
            self._launch(self.buckets[self.next])
        for h, b in self.handles:
            h.wait()
            self.flat[b[0]][b[1]:b[2]].div_(self.world)
        self.handles = []
        self.next = 0
        for b in self.buckets:
            b[4] = 0

    def zero(self):
        for buf in self.flat.values():
            buf.zero_()


def run_model(args, rank, world, local_rank):
    """configs[3] (--workload c4): forward of the 8-layer decoder, 32 x 2048
    tokens per GPU.  configs[4] (--workload c5): training step (forward,
    backward, one NCCL all-reduce of all gradients in a flat bucket, AdamW) of
    the MoE variant, 8 x 2048 tokens per GPU (global 64 x 2048 at 8 GPUs).
    Weak scaling; token ids uniform over the vocabulary; CUDA-event timing,
    max over ranks."""
    import torch.nn.functional as F

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    train = args.workload == "c5"
    torch.manual_seed(1234 + rank)
    model = _build_decoder(moe=train, dev=dev, chain=args.chain)
    batch = 8 if train else 32
    seq = 2048
    gen = torch.Generator(device=dev).manual_seed(77 + rank)
    ids = torch.randint(0, 6400, (batch, seq), device=dev, generator=gen)
    labels = torch.randint(0, 6400, (batch, seq), device=dev, generator=gen)
    params = [p for p in model.parameters()]
    opt = torch.optim.AdamW(params, lr=1e-4, fused=True) if train else None
    dist = None
    if world > 1:
        import torch.distributed as dist
    buckets = GradBuckets(params, world) if (train and world > 1 and not args.flat_allreduce) else None

    def step():
        if not train:
            with torch.no_grad():
                model(ids)
            return
        logits = model(ids)
        loss = F.cross_entropy(logits.view(-1, logits.shape[-1]).float(), labels.view(-1))
        aux = model.aux_loss()
        if aux is not None:
            loss = loss + aux  # the trainers' loss (trainer/train_pretrain.py:37)
        loss.backward()
        if buckets is not None:
            buckets.finish()
        elif world > 1:
            allreduce_grads(params, world)
        opt.step()
        if buckets is not None:
            buckets.zero()
        else:
            opt.zero_grad(set_to_none=True)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(dev)
    sampler.start()
    e0.record()
    for _ in range(args.steps):
        step()
    e1.record()
    torch.cuda.synchronize(dev)
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
    if rank != 0:
        return
    tokens = batch * seq
    value = world * tokens * args.steps / (ms / 1e3)
    line = {
        "metric": "model training tokens/s" if train else "model forward tokens/s", "value": value,
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic (token ids uniform over the vocabulary, random-init weights)",
        "config": {
            "workload": ("config5: MiniMind MoE (8 experts, top-2) + mHC training step (fwd + bwd + grad "
                         "all-reduce + AdamW)" if train else
                         "config4: dense MiniMind-3-style decoder + mHC forward"),
            "model": "hidden 768, 8 layers, 8 q / 4 kv heads, RoPE 1e6, SwiGLU 2048, vocab 6400, n=4, "
                     "20 Sinkhorn iterations",
            "global_batch": world * batch, "seq_len": seq, "parallelism": f"dp{world}",
            "mhc_api": "block-level mhc_chain (merge + next coefficient pass + input norm per call)"
                       if args.chain else "drop-in modules, input norms in the closures",
        },
        "clocks": clocks,
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["layer", "c4", "c5", "post_pre", "fp32_stream"], default="layer",
                    help="layer: configs[1] mHC layer (the headline); c4 / c5: model-level configs[3] / [4]; "
                         "post_pre: the step between two sublayers, two kernels against the fused kernel; "
                         "fp32_stream: the layer with an fp32 residual stream (forward and backward)")
    ap.add_argument("--variant", choices=["full", "nohres"], default="full")
    ap.add_argument("--C", type=int, default=0, help="stream width for --variant nohres (768 or 1024)")
    ap.add_argument("--tokens", type=int, default=16 * 2048)
    ap.add_argument("--cpu-tokens", type=int, default=4096)
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-bwd", action="store_true", help="skip the backward measurement")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the token sweep, config-3 and fp32-stream sub-measurements")
    ap.add_argument("--no-train", action="store_true", help="skip the config-5 training-step sub-measurement")
    ap.add_argument("--chain", action="store_true",
                    help="c4 / c5: run the decoder's sublayers through the block-level mhc_chain API")
    ap.add_argument("--flat-allreduce", action="store_true",
                    help="c5: one flat all-reduce per dtype after backward instead of the overlapped buckets")
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
        if args.workload == "layer":
            run_ours(args, rank, world, local_rank)
        elif args.workload == "post_pre":
            run_post_pre(args, rank, world, local_rank)
        elif args.workload == "fp32_stream":
            run_fp32_stream(args, rank, world, local_rank)
        else:
            run_model(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
